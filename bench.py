"""Benchmark of the B200 INT8 convrot linear (one JSON line on rank 0).

Step (every N): the config-2 linear set of one attention block on this rank's tokens -- q, k, v and out convrot
linears, K = N = 5120, rank-32 low-rank correction and bias, q/k/v sharing one quantisation -- with, for N > 1, the
Ulysses seq<->head exchange of q, k, v ([M/P, 40 heads, 128] bf16) around an identity attention (o = v) and back,
fused into the kernels over peer memory (``--transport peer``, the default) or as NCCL all-to-alls (``nccl``).
M = 32768 token rows per rank (weak scaling; N = 4 is config 4's 131072 tokens; ``--rows`` changes it).

  value       INT8 TOPS of the whole job (4 GEMMs x 2*M*K*N per rank, all ranks) over the device-timed steps
  e2e         the same metric through the public module API with host buffers: each step copies x from pinned
              host memory and reads the out projection back to pinned host memory inside the timed region; the
              copies run on their own streams, double-buffered, overlapping the neighbouring steps' compute
  roofline    the tcgen05 GEMM (dominant kernel): 2*M*N*K INT8 ops per launch over its CUDA-event duration in the
              timed region, against the INT8 peak measured here (torch._int_mm = cuBLASLt, 8192^3)
  extras      (N = 1) config 2's single linear (TOPS), config 3's DiT-block linear set (ms), its FFN chain with and
              without the fused SwiGLU, its AdaLN prologue, the whole block fused and unfused, rotate+quantise GB/s
  cpu_baseline the reference's CPU path (_forward_torch, int8.py:173-179) as ported in oracle/ (numpy/BLAS),
              on a bounded row sample, rank 0 at N = 1

``--impl reference`` times that CPU port alone on the same metric (rank 0; other ranks exit at once).
Inputs are seeded synthetic tensors (hyperflow_h3_flash_b200.synthetic); the per-step activations (335 MB) are larger
than L2 (126 MB), so no L2 flush is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_DIM = N_DIM = 5120
RANK = 32
HEADS, HEAD_DIM = 40, 128
GROUP = 256
SPEC_INT8_TOPS = 4500.0


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=32768, help="token rows per rank")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--transport", choices=["peer", "nccl"], default="peer",
                    help="Ulysses exchange for N > 1: fused into the kernels over peer memory, or NCCL all-to-all")
    ap.add_argument("--peer-copies", default="",
                    help="peer transport: projections (of q, k, v) written locally and moved by the copy engines "
                         "while the next GEMM runs; the others store into the other GPUs' buffers from the epilogue")
    ap.add_argument("--pull-chunks", type=int, default=0,
                    help="peer transport: the copy engines pull the out projection's input in this many row chunks, "
                         "each overlapping the previous chunk's out projection (0: the rotate kernel gathers it)")
    ap.add_argument("--case", choices=["gemm", "gemm_plain", "gemm_ffn_up", "rotate", "rotate_adaln", "rotate_ffn_down",
                                       "down", "step"],
                    default=None,
                    help="run one kernel alone (for ncu captures): --rows rows, K=N=5120, 3 warm-up + 3 launches; "
                         "'step': --warmup + --steps steps of the config-2 linear set and nothing else (launch lists)")
    return ap.parse_args()


# --------------------------------------------------------------------------------------------------- clocks


class ClockSampler:
    """SM clock and throttle reasons sampled every 5 ms during the timed region, through NVML (read-only queries;
    nvidia-smi's own fields: clocks.sm, clocks.max.sm, clocks_event_reasons.*).  A background thread samples from
    before the region starts (the first sample is taken before __enter__ returns) until it ends."""

    PERIOD_S = float(os.environ.get("HF_CLOCK_PERIOD_MS", "5")) / 1000.0
    # NVML clocks-event-reason bits (nvml.h: nvmlClocksEventReason*)
    REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
               "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, int, float]] = []
        self.mem_mhz: list[float] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def _run(self, nvml, handle):
        while True:
            try:
                mhz = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                reasons = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                watts = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                self.samples.append((float(mhz), int(reasons), watts))
                self.mem_mhz.append(float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_MEM)))
            except Exception:  # noqa: BLE001 - a failed read is a missing sample, not an error of the bench
                pass
            if self._stop.wait(self.PERIOD_S):
                return

    def __enter__(self):
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.index]) if visible else self.index
            handle = nvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, args=(nvml, handle), daemon=True)
            self._thread.start()
            deadline = time.time() + 2.0
            while not self.samples and time.time() < deadline:
                time.sleep(0.001)
        except Exception:  # noqa: BLE001 - no NVML: the line reports no clock samples
            self._thread = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            time.sleep(2 * self.PERIOD_S)
            self._stop.set()
            self._thread.join(timeout=5)
        return False

    def summary(self) -> dict:
        sm = [mhz for mhz, _, _ in self.samples]
        reasons = sorted(name for name, bit in self.REASONS.items() if any(r & bit for _, r, _ in self.samples))
        watts = [w for _, _, w in self.samples]
        mx = self.max_mhz
        loaded = [v for v in sm if mx and v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx, "reasons": reasons,
                "mem_mhz": statistics.median(self.mem_mhz) if self.mem_mhz else None,
                "power_w": statistics.median(watts) if watts else None, "samples": len(sm),
                "source": f"NVML, every {self.PERIOD_S * 1000:g} ms during the timed region"}


# --------------------------------------------------------------------------------------------------- CPU arm


def host_threads() -> int:
    """Every core this process may run on, set as the thread count of torch and of numpy's BLAS: torchrun exports
    OMP_NUM_THREADS=1 to its children, which would otherwise leave the CPU arm on one core."""
    cores = len(os.sched_getaffinity(0))
    import torch

    torch.set_num_threads(cores)
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(limits=cores)
    except Exception:  # noqa: BLE001 - numpy then keeps its own default
        pass
    return cores


def load_reference_int8():
    """The reference's int8 module from its installed copy (baseline/_ref), loaded by file path: the package's
    __init__ imports diffusers, which this path does not need.  Returns (module, None) or (None, why)."""
    import importlib.util

    path = os.path.join(ROOT, "baseline", "_ref", "hyperflow_h3_flash", "int8.py")
    if not os.path.exists(path):
        return None, "the reference is not installed under baseline/_ref"
    try:
        spec = importlib.util.spec_from_file_location("hyperflow_h3_flash_ref_int8", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001 - reported as the reason
        return None, f"loading baseline/_ref int8.py failed: {type(e).__name__}: {e}"
    return mod, None


def reference_layers(ref, torch, dev, K: int, N: int, rank: int, count: int, seed0: int = 0):
    """`count` of the reference's own Int8RotLinear modules with the synthetic weights of this bench, plus their bias
    and LowRankLinear factors (transformer.py:48-58: two bias-free bf16 nn.Linear), on `dev`."""
    from hyperflow_h3_flash_b200 import synthetic

    out = []
    for i in range(count):
        w = synthetic.linear_weights(K, N, rank=rank, bias=True, group=GROUP, seed_offset=seed0 + i)
        layer = ref.Int8RotLinear(K, N, GROUP)
        layer.qweight.data.copy_(w.qweight)
        layer.wscale.data.copy_(w.wscale)
        down = torch.nn.Linear(K, rank, bias=False, dtype=torch.bfloat16)
        up = torch.nn.Linear(rank, N, bias=False, dtype=torch.bfloat16)
        down.weight.data.copy_(w.down)
        up.weight.data.copy_(w.up)
        out.append((layer.to(dev), w.bias.to(dev), down.to(dev), up.to(dev)))
    return out


def reference_linear(x, parts):
    """The reference's modules composed as this path computes: Int8RotLinear(x) + bias + up(down(x)), bf16 ops."""
    layer, bias, down, up = parts
    return layer(x) + bias + up(down(x))


def cpu_linear_set(rows: int, steps: int, warmup: int) -> dict:
    """The reference's CPU path for the linear set on `rows` token rows, on every host core: its own
    Int8RotLinear on CPU tensors (_forward_torch, int8.py:173-179) from the installed copy, plus bias and
    up(down(x)); the numpy/BLAS port in oracle/ when the copy is absent.  Median seconds per step."""
    import torch

    from hyperflow_h3_flash_b200 import synthetic

    cores = host_threads()
    ref, why = load_reference_int8()
    x = synthetic.activations(rows, K_DIM)
    if ref is not None:
        kind = "reference"
        parts = reference_layers(ref, torch, torch.device("cpu"), K_DIM, N_DIM, RANK, 4)

        def step():
            with torch.inference_mode():
                q, k, v = (reference_linear(x, parts[i]) for i in range(3))
                return reference_linear(v, parts[3])

        what = ("the reference's Int8RotLinear.forward on CPU tensors (_forward_torch, int8.py:173-179, from "
                "baseline/_ref) + bias + LowRankLinear, torch")
    else:
        import numpy as np

        from oracle import oracle as O

        kind = "port"
        xb = x.view(torch.int16).numpy().view(np.uint16)
        layers = [synthetic.linear_weights(K_DIM, N_DIM, rank=RANK, bias=True, group=GROUP, seed_offset=i)
                  for i in range(4)]
        h = O.regular_hadamard(GROUP)

        def linear(xv, w):
            bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
            y = O.bf16_to_f32(O.forward_cpu_port(xv, w.qweight.numpy(), w.wscale.numpy(), GROUP, h))
            y = O.bf16_to_f32(O.f32_to_bf16(y + O.bf16_to_f32(bits(w.bias))[None, :]))
            xa = O.f32_to_bf16(O.bf16_to_f32(xv) @ O.bf16_to_f32(bits(w.down)).T)
            lr = O.f32_to_bf16(O.bf16_to_f32(xa) @ O.bf16_to_f32(bits(w.up)).T)
            return O.f32_to_bf16(y + O.bf16_to_f32(lr))

        def step():
            q, k, v = (linear(xb, layers[i]) for i in range(3))
            return linear(v, layers[3])

        what = f"numpy/BLAS port of _forward_torch (oracle/) + bias + up(down(x)) ({why})"

    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    ops = 4 * 2.0 * rows * K_DIM * N_DIM
    t = statistics.median(times)
    return {"value": ops / t / 1e12, "unit": "TOPS", "cores": cores, "kind": kind,
            "sample": f"{rows} token rows of the linear set (4 linears {K_DIM}x{N_DIM}, r={RANK}, bias; q/k/v on x, "
                      f"out on v), median of {steps} steps after {warmup} warm-up, {cores} threads: {what}",
            "seconds_per_step": t, "mean_seconds_per_step": statistics.mean(times)}


#: The CPU sample of both arms: rows per step (about 0.5 s of CPU work per step on 32 cores) and warm-up steps.
CPU_ROWS, CPU_WARMUP = 1024, 1


METRIC = 'INT8 convrot linear TOPS & % dense-INT8 peak; DiT-block linear-set ms at 1/2/4/8 B200'
METRIC_DETAIL = ("value: INT8 TOPS of the config-2 linear set (the config-2 convrot layer, M=32768 rows per rank, "
                 "K=N=5120, r=32, bias, as to_q, to_k, to_v and to_out, q/k/v sharing one quantisation as the "
                 "reference's keep_input does), whole job; ms_per_step is that set's time; the single config-2 "
                 "linear is the single_linear extra and the config-3 block set the block_set_cfg3 extra")
DATA = "synthetic (seeded, random-init weights)"


def workload_config(rows: int, world: int, transport: str, peer_copies: str = "", pull_chunks: int = 0) -> dict:
    """The `config` object of both arms' lines (the reference arm times a row sample of this same workload)."""
    exchange = world > 1 and transport == "peer"
    return {"workload": "config-2 linear set per rank: q,k,v (shared quantisation), out; "
                        f"M={rows} rows/rank, K=N={K_DIM}, r={RANK}, bias, group {GROUP}"
                        + (f"; Ulysses all-to-all of q,k,v [M/P,{HEADS},{HEAD_DIM}] around identity attention"
                           + ((" (over peer memory: " + (", ".join(peer_copies) + " written locally and moved by the "
                                                          "copy engines, " if peer_copies else "")
                               + "the rest stored by the GEMM epilogue; "
                               + (f"pulled back by the copy engines in {pull_chunks} row chunks overlapping the out "
                                  "projection)" if pull_chunks > 0 else "gathered by the out projection's rotate kernel)"))
                              if exchange else " (NCCL)")
                           if world > 1 else ""),
            "rows_per_rank": rows, "total_rows": rows * world, "K": K_DIM, "N": N_DIM, "rank": RANK,
            "group": GROUP, "parallelism": f"ulysses{world}" if world > 1 else "single",
            "transport": transport if world > 1 else None,
            "l2": "inputs larger than L2 (x is 335 MB per step), no flush"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    res = cpu_linear_set(CPU_ROWS, args.steps, max(CPU_WARMUP, args.warmup))
    line = {
        "metric": METRIC, "metric_detail": METRIC_DETAIL, "value": res["value"],
        "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": DATA, "impl": "reference",
        "config": workload_config(args.rows, args.gpus, args.transport, args.peer_copies),
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------------- GPU arm


def measure_int8_peak(torch, dev) -> dict:
    """cuBLASLt INT8 (torch._int_mm) at 8192^3: best of 10 (burst) and a ~1.5 s loop (sustained)."""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b.t())
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b.t())
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, int(1500 / max(best, 1e-3)))
    s.record()
    for _ in range(reps):
        torch._int_mm(a, b.t())
    e.record()
    e.synchronize()
    ops = 2.0 * n**3
    return {"burst_tops": ops / best / 1e9, "sustained_tops": ops * reps / s.elapsed_time(e) / 1e9}


class KernelTimer:
    """Counts this library's kernel launches and brackets GEMM / rotate launches with CUDA events on the launching
    stream, by wrapping the module's kernel namespace."""

    def __init__(self, torch, kernels):
        self.torch = torch
        self.kernels = kernels
        self.saved = {}
        self.launches = 0
        self.active = False
        self.gemm_events, self.rq_events = [], []
        self.gemm_shapes, self.rq_shapes = [], []
        self.by_kind: dict[str, list] = {}  # per kernel kind (local / scatter GEMM, rotate, gather, down, flag wait)

    def _wrap(self, name, kind, n_launch):
        fn = getattr(self.kernels, name)
        self.saved[name] = fn
        torch = self.torch

        def wrapped(*a, **k):
            if not self.active:
                return fn(*a, **k)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*a, **k)
            e.record()
            self.launches += n_launch
            sub = {"gemm": "gemm_scatter" if k.get("out_ptrs") else "gemm_local",
                   "rq": "rotate_gather" if name == "rotate_quant_gather" else "rotate"}.get(kind, kind)
            self.by_kind.setdefault(sub, []).append((s, e))
            if kind == "gemm":
                self.gemm_events.append((s, e))
                self.gemm_shapes.append((a[0].shape[0], a[1].shape[0], a[0].shape[1]))
            elif kind == "rq":
                self.rq_events.append((s, e))
                self.rq_shapes.append(tuple(getattr(a[0], "shape", ())))
            return out

        setattr(self.kernels, name, wrapped)

    def __enter__(self):
        self._wrap("convrot_matmul", "gemm", 1)
        self._wrap("rotate_quant", "rq", 1)
        self._wrap("rotate_quant_torch_rounding", "rq", 1)
        self._wrap("lowrank_down", "down", 1)
        self._wrap("rotate_quant_packed", "rq", 1)
        self._wrap("lowrank_down_packed", "down", 1)
        self._wrap("rotate_quant_gather", "rq", 1)
        return self

    def __exit__(self, *exc):
        for k, v in self.saved.items():
            setattr(self.kernels, k, v)
        return False

    def reset(self):
        self.launches = 0
        self.gemm_events, self.rq_events, self.gemm_shapes, self.rq_shapes = [], [], [], []
        self.by_kind = {}

    def wrap_exchange(self, exchange) -> None:
        """Brackets the exchange's flag waits with events too (kind "flag_wait")."""
        if exchange is None:
            return
        wait = exchange.wait
        torch = self.torch

        def timed_wait(phase):
            if not self.active:
                return wait(phase)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            wait(phase)
            e.record()
            self.by_kind.setdefault("flag_wait", []).append((s, e))

        exchange.wait = timed_wait

    def breakdown(self, steps: int) -> dict:
        """Per kind: launches and ms per step (sum of its CUDA-event durations / steps)."""
        return {kind: {"launches": len(ev), "ms_per_step": sum(s.elapsed_time(e) for s, e in ev) / steps,
                       "avg_launch_ms": sum(s.elapsed_time(e) for s, e in ev) / max(len(ev), 1)}
                for kind, ev in sorted(self.by_kind.items())}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic, ulysses

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        bind_to_gpu_cpus(local)  # before any pinned host buffer is allocated (first touch picks its NUMA node)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    M = args.rows

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- the linear set of one attention block
    def make_layer(i, K, N, rank_lr, bias=True):
        w = synthetic.linear_weights(K, N, rank=rank_lr, bias=bias, group=GROUP, seed_offset=i)
        layer = I.Int8RotLinear(K, N, GROUP, bias=bias, rank=rank_lr)
        synthetic.load_into(layer, w)
        return layer.to(dev)

    to_q, to_k, to_v, to_out = (make_layer(i, K_DIM, N_DIM, RANK) for i in range(4))
    to_q.keep_input = to_k.keep_input = True
    I.share_lowrank(to_q, to_k, to_v)
    x_host = synthetic.activations(M, K_DIM, seed=rank).pin_memory()
    x = x_host.to(dev)
    y_host = torch.empty(M, N_DIM, dtype=torch.bfloat16).pin_memory()

    exchange = None
    if world > 1 and args.transport == "peer":
        # every rank must agree on the transport: a rank whose mapping fails tells the others through an all-reduce
        try:
            exchange = ulysses.PeerExchange(M, N_DIM, HEADS, device=dev, copy_names=tuple(args.peer_copies),
                                            pull_chunks=args.pull_chunks)
            failed = 0
        except Exception as e:  # noqa: BLE001 - reported, and the NCCL transport is used instead
            print(f"peer-memory exchange unavailable on rank {rank}: {e}; using NCCL all-to-all", file=sys.stderr)
            failed = 1
        flag = torch.tensor([failed], device=dev)
        dist.all_reduce(flag)
        if flag.item():
            if exchange is not None:
                exchange.close()
            exchange = None
            args.transport = "nccl"

    def step(inp):
        return ulysses.attention_block_linears(inp, to_q, to_k, to_v, to_out, HEADS, exchange=exchange)

    kernels = I._kernels()
    timer = KernelTimer(torch, kernels)
    timer.wrap_exchange(exchange)
    with torch.inference_mode(), timer:
        # Untimed steps for SETTLE_S seconds before the warm-up steps: without them, single runs on a fresh box were
        # 15-20 % slower, once 2.9x (GEMM 1.87 ms against 0.56 ms), while runs after 0.3 s of load were steady.
        settled = settle(torch, dist, world, dev, lambda: step(x), SETTLE_S)
        # device-timed steps, inputs resident in HBM
        for _ in range(args.warmup):
            step(x)
        torch.cuda.synchronize()
        barrier()
        timer.active = True
        timer.reset()
        exchange_launches = exchange.kernel_launches if exchange else 0
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            torch.cuda.synchronize()
            barrier()
            start.record()
            for _ in range(args.steps):
                out = step(x)
            end.record()
            torch.cuda.synchronize()
            barrier()
        timer.active = False
        breakdown = timer.breakdown(args.steps)
        ms = start.elapsed_time(end)
        gemm_ms = [s.elapsed_time(e) for s, e in timer.gemm_events]
        rq_ms = [s.elapsed_time(e) for s, e in timer.rq_events]
        launches = timer.launches + (exchange.kernel_launches - exchange_launches if exchange else 0)
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())

        # e2e through the module API with host buffers: every step copies its x from pinned host memory and reads
        # its out projection back to pinned host memory.  Copies run on their own streams, double-buffered, so the
        # upload of step i+1 and the download of step i-1 overlap the compute of step i (PCIe is full duplex).
        e2e_ms = pipelined_e2e(torch, dev, step, x_host, y_host, args, barrier)
        te = torch.tensor([e2e_ms], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item())
        barrier()
        copies = copy_bound(torch, dev, x_host, y_host)  # all ranks at once, as in the e2e steps
        barrier()

        # correctness of the whole step, exchange included: rows of this rank's output against the same layers run
        # on those rows alone on this GPU (no exchange; attention is identity, so out = to_out(to_v(x))).  1056
        # rows keep the down projection on its unsplit K order, as at full size; the 2-SM GEMM is pinned for both.
        check = verify_rows(torch, I, out, x, to_q, to_k, to_v, to_out, min(1056, M))
        ok = torch.tensor([1 if check["bitwise_equal"] else 0], device=dev)
        if world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        check["all_ranks_bitwise_equal"] = bool(ok.item())

        # config 4 as stated: 131072 tokens in total, split over the N ranks (strong scaling)
        strong = strong_scaling_cfg4(torch, dist, synthetic, ulysses, dev, rank, world, args, to_q, to_k, to_v,
                                     to_out, barrier)

    ops_step = 4 * 2.0 * M * K_DIM * N_DIM
    value = world * ops_step * args.steps / (ms_max * 1e-3) / 1e12
    e2e_value = world * ops_step * args.steps / (e2e_ms * 1e-3) / 1e12

    extras = {}
    peak = None
    with torch.inference_mode():
        peak = measure_int8_peak(torch, dev)  # every rank, on its own GPU: the roofline denominator
        if world == 1 and not args.no_extras:
            extras = run_extras(torch, I, synthetic, dev, args, x)
    gemm_avg = statistics.mean(gemm_ms) if gemm_ms else None
    gemm_ops = 2.0 * M * K_DIM * N_DIM
    achieved = gemm_ops / (gemm_avg * 1e-3) / 1e12 if gemm_avg else None
    # Denominator: the dense INT8 rate of B200 is twice its bf16 rate, so the peak is 2 x the driver-measured bf16
    # burst (MEASURED_PEAKS.json; the spec 4.5 POPS when that file is absent).  cuBLASLt's own INT8 rate, measured
    # in this run, is reported beside it.
    bf16_burst = measured_peak("bf16_tflops")
    peak_tops = 2.0 * bf16_burst if bf16_burst else SPEC_INT8_TOPS
    roofline = {
        "kernel": "convrot_gemm2sm_kernel (tcgen05 kind::i8, cta_group::2, 256x256 pair tiles, fused "
                  "dequant + bias + low-rank epilogue, TMA-store output)",
        "bound": "tensor", "unit": "TFLOP/s", "achieved": achieved, "peak": peak_tops,
        "frac": (achieved / peak_tops) if achieved else None,
        "peak_source": ("of measured: 2 x MEASURED_PEAKS.json bf16_tflops (dense INT8 = 2 x dense bf16 on B200); "
                        "INT8 ops, so the unit reads tera-ops") if bf16_burst else "spec dense INT8 4.5 POPS (fallback)",
        "frac_of_spec_4500": achieved / SPEC_INT8_TOPS if achieved else None,
        "cublaslt_int8_burst_tops": peak["burst_tops"] if peak else None,
        "frac_of_cublaslt_burst": (achieved / peak["burst_tops"]) if (achieved and peak) else None,
        "per_launch_ops": gemm_ops, "avg_launch_ms": gemm_avg, "launches_timed": len(gemm_ms),
        "traffic": load_traffic("gemm"),
    }
    if peak:
        roofline["cublaslt_int8_sustained_tops"] = peak["sustained_tops"]
    bf16_sustained = measured_peak("bf16_tflops_sustained")
    if bf16_sustained and achieved:
        # the power-capped steady state: 2 x the seconds-long bf16 loop of MEASURED_PEAKS.json
        roofline["peak_sustained"] = 2.0 * bf16_sustained
        roofline["frac_of_sustained"] = achieved / (2.0 * bf16_sustained)
    rq_avg = statistics.mean(rq_ms) if rq_ms else None
    rq_bytes = M * K_DIM * 3 + 4 * M
    per_rank = [None] * world
    if world > 1:
        dist.all_gather_object(per_rank, breakdown)
    else:
        per_rank = [breakdown]
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_extras:
            cpu = cpu_linear_set(CPU_ROWS, 5, CPU_WARMUP)
            cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line = {
            "metric": METRIC,
            "metric_detail": METRIC_DETAIL,
            "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": DATA,
            "config": workload_config(M, world, args.transport, args.peer_copies, args.pull_chunks),
            "e2e": {"value": e2e_value, "unit": "TOPS", "ms_per_step": e2e_ms / args.steps,
                    "h2d_bytes_per_step": M * K_DIM * 2, "d2h_bytes_per_step": M * N_DIM * 2,
                    "pipelining": "H2D / compute / D2H on three streams, double-buffered",
                    "copy_floor": copies,
                    "frac_of_copy_floor": copies["floor_ms_per_step"] / (e2e_ms / args.steps)},
            "gpu_launches": launches,
            "settle": {"seconds": SETTLE_S, "steps": settled,
                       "what": "untimed steps before the warm-up steps, until SETTLE_S seconds have passed on rank 0"},
            "roofline": roofline,
            "rotate_quant": {"bound": "hbm", "avg_launch_ms": rq_avg, "bytes_per_launch": rq_bytes,
                             "achieved_gbs": rq_bytes / (rq_avg * 1e-3) / 1e9 if rq_avg else None,
                             "peak_gbs": measured_peak("hbm_gbs"),
                             "traffic": load_traffic("rotate_quant")},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "kernel_breakdown_per_rank": per_rank,
            "correctness": check,
            "strong_cfg4": strong,
        }
        if line["rotate_quant"]["achieved_gbs"] and line["rotate_quant"]["peak_gbs"]:
            line["rotate_quant"]["frac"] = line["rotate_quant"]["achieved_gbs"] / line["rotate_quant"]["peak_gbs"]
        line.update(extras)
        if "block_set_cfg3" in extras:
            # config 3 headline: the DiT block's four linears at M = 32760, r = 64 (and with the fused SwiGLU chain)
            b = extras["block_set_cfg3"]
            line["block_set_cfg3_ms"] = b["ms"]
            line["block_set_cfg3_frac"] = b["tops"] / peak_tops
            line["block_set_cfg3_target_ms"] = 6.6
            line["block_set_cfg3_swiglu_ms"] = extras["block_set_cfg3_swiglu"]["ms"]
        print(json.dumps(line), flush=True)
    if exchange is not None:
        exchange.close()
    if world > 1:
        dist.destroy_process_group()


def verify_rows(torch, I, out, x, to_q, to_k, to_v, to_out, rows: int) -> dict:
    """Rows [0, rows) of the last step's output against to_out(to_v(x[:rows])) computed on this GPU alone (q, k
    and v with the step's sharing), bitwise; the 2-SM GEMM is pinned for the recomputation as for the full size."""
    from hyperflow_h3_flash_b200 import _lib

    L = _lib.lib()
    _lib.check(L.convrot_set_gemm_mode(2), "gemm mode")
    try:
        xs = x[:rows].clone()
        to_q(xs)
        to_k(xs)
        ref = to_out(to_v(xs))
    finally:
        L.convrot_set_gemm_mode(0)
    got = out.reshape(-1, ref.shape[-1])[:rows]
    torch.cuda.synchronize()
    return {"rows_checked": rows, "bitwise_equal": bool(torch.equal(got, ref)),
            "mismatching_values": int((got != ref).sum()),
            "what": "rows of the out projection after the full step (exchange included) against the same layers "
                    "on those rows alone, no exchange, identity attention"}


def strong_scaling_cfg4(torch, dist, synthetic, ulysses, dev, rank, world, args, to_q, to_k, to_v, to_out,
                        barrier) -> dict:
    """Config 4 as BASELINE states it: 131072 tokens in total split evenly over the N ranks, the same linear set
    and exchange; device-timed steps (max over ranks)."""
    total = 131072
    rows = total // world
    xs = synthetic.activations(rows, K_DIM, seed=100 + rank).to(dev)
    exchange = None
    if world > 1 and args.transport == "peer":
        exchange = ulysses.PeerExchange(rows, N_DIM, HEADS, device=dev, copy_names=tuple(args.peer_copies),
                                        pull_chunks=args.pull_chunks)

    def step():
        return ulysses.attention_block_linears(xs, to_q, to_k, to_v, to_out, HEADS, exchange=exchange)

    steps = max(3, args.steps // 2)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    barrier()
    t = torch.tensor([s.elapsed_time(e) / steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if exchange is not None:
        exchange.close()
    ms = float(t.item())
    ops = 4 * 2.0 * total * K_DIM * N_DIM
    return {"total_rows": total, "rows_per_rank": rows, "steps": steps, "ms_per_step": ms,
            "tops": ops / (ms * 1e-3) / 1e12, "scaling": "strong",
            "what": "config-2 linear set (q, k, v, out; Ulysses exchange for N > 1) on 131072 tokens in total"}


def bind_to_gpu_cpus(local_rank: int) -> None:
    """Pins this rank to the CPU cores NVML reports as closest to its GPU (within the cores it may use), so its
    pinned host buffers live on the GPU's NUMA node and eight ranks' PCIe copies do not all cross one socket.
    A read-only NVML query; without NVML or an overlap the affinity is left as it is."""
    try:
        import pynvml as nvml

        nvml.nvmlInit()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        index = int(visible.split(",")[local_rank]) if visible else local_rank
        handle = nvml.nvmlDeviceGetHandleByIndex(index)
        words = nvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        near = {64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        allowed = os.sched_getaffinity(0) & near
        if allowed:
            os.sched_setaffinity(0, allowed)
    except Exception:  # noqa: BLE001 - an optimisation only
        pass


SETTLE_S = float(os.environ.get("HF_SETTLE_S", "0.3"))


def settle(torch, dist, world: int, dev, fn, seconds: float) -> int:
    """Run fn in batches of 10 until `seconds` have passed on rank 0; every rank runs the same batches (rank 0's
    decision is broadcast), so the exchange's collectives and flags stay in step.  Returns the calls made."""
    t0 = time.time()
    n = 0
    while True:
        for _ in range(10):
            fn()
        n += 10
        torch.cuda.synchronize()
        go = torch.tensor([1 if time.time() - t0 < seconds else 0], device=dev)
        if world > 1:
            dist.broadcast(go, 0)
        if not int(go.item()):
            return n


def pipelined_e2e(torch, dev, step, x_host, y_host, args, barrier) -> float:
    """Milliseconds for args.steps pipelined steps: H2D(x) -> linear set -> D2H(out), all inside the timed region."""
    compute = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    x_dev = [torch.empty_like(x_host, device=dev) for _ in range(2)]
    y_pin = [y_host, torch.empty_like(y_host).pin_memory()]
    y_dev = [None, None]
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(computed[b])  # step i-2 no longer reads x_dev[b]
                x_dev[b].copy_(x_host, non_blocking=True)
                uploaded[b].record(up)
            compute.wait_event(uploaded[b])
            # (each step writes a fresh output tensor; record_stream below keeps the allocator from reusing one
            # before its download ends, so compute never waits for the download of an earlier step)
            y_dev[b] = step(x_dev[b])
            computed[b].record(compute)
            with torch.cuda.stream(down):
                down.wait_event(computed[b])
                y_pin[b].copy_(y_dev[b], non_blocking=True)
                y_dev[b].record_stream(down)  # the allocator must not recycle it before the download ends
        compute.wait_stream(down)
        compute.wait_stream(up)

    run(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    run(args.steps)
    end.record(compute)
    torch.cuda.synchronize()
    barrier()
    return start.elapsed_time(end)


def copy_bound(torch, dev, x_host, y_host, reps: int = 3) -> dict:
    """The PCIe floor under the e2e number: the step's upload (x) and download (out) between the same pinned host
    buffers and device memory, timed alone and both at once on two streams (best of `reps`, CUDA events)."""
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xd = torch.empty_like(x_host, device=dev)
    yd = torch.empty_like(y_host, device=dev)

    def timed(fn) -> float:
        best = None
        for _ in range(reps):
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            best = s.elapsed_time(e) if best is None else min(best, s.elapsed_time(e))
        return best

    def both():
        cur = torch.cuda.current_stream(dev)
        up.wait_stream(cur)
        down.wait_stream(cur)
        with torch.cuda.stream(up):
            xd.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(down):
            y_host.copy_(yd, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)

    h2d = timed(lambda: xd.copy_(x_host, non_blocking=True))
    d2h = timed(lambda: y_host.copy_(yd, non_blocking=True))
    duplex = timed(both)
    nx, ny = x_host.numel() * x_host.element_size(), y_host.numel() * y_host.element_size()
    return {"h2d_ms": h2d, "h2d_gbs": nx / (h2d * 1e-3) / 1e9, "d2h_ms": d2h, "d2h_gbs": ny / (d2h * 1e-3) / 1e9,
            "both_at_once_ms": duplex, "floor_ms_per_step": max(h2d, d2h, duplex)}


def reference_gpu_path(torch, I, dev, x, steps: int) -> dict:
    """The reference's own B200 path beside this one, on the same seeded config-2 inputs (N = 1):

    * parity: its Triton rotate_quant kernels (factored, the pipeline default, pipeline.py:232; and dense,
      int8.py:194-262) against this library's codes and scales; torch._int_mm's int32 accumulator (its B200 GEMM,
      int8.py:353-364) and its int8_matmul output (cuBLASLt + Triton rescale) against this library's on the same
      codes;
    * time: its linear set (Int8RotLinear with the q/k/v keep_input sharing, + bias + LowRankLinear in bf16 torch
      ops) and its parts, CUDA events over `steps` calls after 3 warm-up calls.
    """
    ref, why = load_reference_int8()
    if ref is None:
        return {"unavailable": why}
    try:
        kernels = ref._kernels()
    except Exception as e:  # noqa: BLE001 - reported
        return {"unavailable": f"the reference's _kernels() failed: {type(e).__name__}: {e}"}
    if kernels is None:
        return {"unavailable": "Triton is not importable, so the reference has no CUDA kernels (int8.py:182-188)"}
    M = x.shape[0]
    out = {"source": "baseline/_ref/hyperflow_h3_flash/int8.py loaded by file path; kernel options as "
                     "load_pipeline's defaults (int8_gemm auto -> cublas on sm_100, rotate_quant factored) unless named",
           "resolved_int8_gemm": ref.resolve_int8_gemm(dev)}
    parts = reference_layers(ref, torch, dev, K_DIM, N_DIM, RANK, 4)
    layer0 = parts[0][0]
    q, s = I.rotate_quant(x, GROUP)
    parity = {}
    for opt in ("factored", "dense"):
        ref.set_kernel_options(rotate_quant=opt)
        qr, sr = kernels.rotate_quant(x, GROUP)
        torch.cuda.synchronize()
        dq = (qr.to(torch.int16) - q.to(torch.int16)).abs()
        su, sru = s.view(torch.int32).long(), sr.view(torch.int32).long()
        parity[f"rotate_quant_{opt}"] = {
            "codes_equal_frac": float((dq == 0).double().mean()), "codes_max_abs_diff": int(dq.max()),
            "codes_differing": int((dq != 0).sum()), "codes_total": dq.numel(),
            "scales_equal_frac": float((su == sru).double().mean()),
            "scales_max_ulp_diff": int((su - sru).abs().max()),
        }
        del qr, sr, dq
    acc_ours = I.int8_mm_acc(q, layer0.qweight)
    acc_ref = torch._int_mm(q, layer0.qweight.t())
    parity["int32_accumulator_bitwise_equal"] = bool(torch.equal(acc_ours, acc_ref))
    del acc_ours, acc_ref
    y_ours = I.int8_matmul(q, layer0.qweight, s, layer0.wscale)
    y_ref = kernels.int8_matmul(q, layer0.qweight, s, layer0.wscale)
    parity["int8_matmul_output_bitwise_equal"] = bool(torch.equal(y_ours, y_ref))
    del y_ours, y_ref
    out["parity_cfg2"] = parity

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(steps):
            fn()
        en.record()
        en.synchronize()
        return st.elapsed_time(en) / steps

    to_q, to_k = parts[0][0], parts[1][0]

    def linear_set():
        to_q.keep_input = to_k.keep_input = True
        q_, k_, v_ = (reference_linear(x, parts[i]) for i in range(3))
        return reference_linear(v_, parts[3])

    ops = 4 * 2.0 * M * K_DIM * N_DIM
    times = {}
    with torch.inference_mode():
        for opt in ("factored", "dense"):
            ref.set_kernel_options(rotate_quant=opt)
            ms = timed(linear_set)
            times[f"linear_set_{opt}"] = {"ms": ms, "tops": ops / (ms * 1e-3) / 1e12}
            times[f"rotate_quant_{opt}_ms"] = timed(lambda: kernels.rotate_quant(x, GROUP))
        ref.set_kernel_options(rotate_quant="factored")
        times["int8_matmul_ms"] = timed(lambda: kernels.int8_matmul(q, layer0.qweight, s, layer0.wscale))
        down, up = parts[0][2], parts[0][3]
        times["lowrank_up_down_ms"] = timed(lambda: up(down(x)))
    to_q.keep_input = to_k.keep_input = False
    ref.Int8RotLinear._last_input.clear()
    out["time_cfg2"] = times
    out["ms_per_step"] = times["linear_set_factored"]["ms"]
    out["tops"] = times["linear_set_factored"]["tops"]
    return out


def run_extras(torch, I, synthetic, dev, args, x) -> dict:
    """Config 2's single linear, config 3's block set, rotate+quantise bandwidth (N = 1 only)."""
    out = {}

    def timed(fn, steps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / steps

    def timed_ab(fns: dict, steps: int, rounds: int = 4) -> dict:
        """Per-call ms of each variant, median over rounds that alternate the variants (order reversed every
        other round). Seconds of INT8 GEMMs push the GPU onto its 1 kW power cap and its clock drifts down; timing
        one variant after the other would charge the drift to the later one."""
        names = list(fns)
        samples = {n: [] for n in names}
        for r in range(rounds):
            for n in (names if r % 2 == 0 else names[::-1]):
                samples[n].append(timed(fns[n], steps))
        return {n: sorted(v)[len(v) // 2] for n, v in samples.items()}

    M = args.rows
    out["reference_gpu"] = reference_gpu_path(torch, I, dev, x, args.steps)
    w = synthetic.linear_weights(K_DIM, N_DIM, rank=RANK, bias=True, group=GROUP, seed_offset=7)
    layer = I.Int8RotLinear(K_DIM, N_DIM, GROUP, bias=True, rank=RANK)
    synthetic.load_into(layer, w)
    layer = layer.to(dev)
    ms = timed(lambda: layer(x), args.steps)
    out["single_linear"] = {"config": f"config 2: M={M}, K=N={K_DIM}, r={RANK}, bias", "ms": ms,
                            "tops": 2.0 * M * K_DIM * N_DIM / (ms * 1e-3) / 1e12}
    ms = timed(lambda: I.rotate_quant(x, GROUP), args.steps)
    nbytes = M * K_DIM * 3 + 4 * M
    out["rotate_quant_cfg2"] = {"ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9, "bytes": nbytes}
    # config 3: DiT-block linear set at M = 32760, rank 64
    Mb = 32760
    xb = synthetic.activations(Mb, K_DIM, seed=1).to(dev)
    hb = synthetic.activations(Mb, 13824, seed=2).to(dev)
    shapes = [("qkv", K_DIM, 15360), ("out", K_DIM, K_DIM), ("ffn_up", K_DIM, 2 * 13824), ("ffn_down", 13824, K_DIM)]
    layers = {}
    for i, (name, K, N) in enumerate(shapes):
        wl = synthetic.linear_weights(K, N, rank=64, bias=True, group=GROUP, seed_offset=20 + i)
        ly = I.Int8RotLinear(K, N, GROUP, bias=True, rank=64)
        synthetic.load_into(ly, wl)
        layers[name] = ly.to(dev)
        del wl

    def block():
        layers["qkv"](xb)
        layers["out"](xb)
        layers["ffn_up"](xb)
        layers["ffn_down"](hb)

    ops = sum(2.0 * Mb * K * N for _, K, N in shapes)

    # the same block with the feed-forward's real dataflow: FFN-down reads the SwiGLU of FFN-up's output, either
    # unfused (projection [M, 27648] -> a * silu(g) in torch -> down) or fused into the FFN-up epilogue
    from hyperflow_h3_flash_b200 import ffn

    swiglu_up = ffn.SwiGLUInt8(layers["ffn_up"])

    def chain_unfused():
        return layers["ffn_down"](ffn.swiglu_reference(layers["ffn_up"](xb)))

    def chain_fused():
        return layers["ffn_down"](swiglu_up(xb))

    def block_fused():
        layers["qkv"](xb)
        layers["out"](xb)
        chain_fused()

    steps_b = max(3, args.steps // 4)
    t = timed_ab({"block": block, "block_fused": block_fused}, steps_b)
    ms, ms_block = t["block"], t["block_fused"]
    out["block_set_cfg3"] = {"config": "config 3: M=32760, r=64, QKV 5120->15360, out 5120->5120, "
                                       "FFN-up 5120->27648, FFN-down 13824->5120 (bias, low-rank)",
                             "ms": ms, "tops": ops / (ms * 1e-3) / 1e12}
    t = timed_ab({"unfused": chain_unfused, "fused": chain_fused}, steps_b)
    ms_unfused, ms_fused = t["unfused"], t["fused"]
    out["ffn_chain_cfg3"] = {"config": "M=32760: FFN-up 5120->27648 (r=64, bias) -> a*silu(g) -> FFN-down "
                                       "13824->5120 (r=64, bias)",
                             "ms_unfused": ms_unfused, "ms_fused_swiglu": ms_fused}
    out["block_set_cfg3_swiglu"] = {"config": "config 3 with FFN-down reading the fused SwiGLU of FFN-up",
                                    "ms": ms_block, "tops": ops / (ms_block * 1e-3) / 1e12}

    # the block's AdaLN prologue before q/k/v (chunk_block): h = LN(x) * (1 + scale[idx]) + shift[idx], quantised
    import torch.nn.functional as F

    frames = 8
    gen = torch.Generator().manual_seed(9)
    mod_scale = (torch.randn(frames, K_DIM, generator=gen) * 0.1).to(torch.bfloat16).to(dev)
    mod_shift = (torch.randn(frames, K_DIM, generator=gen) * 0.1).to(torch.bfloat16).to(dev)
    mod_idx = (torch.arange(Mb, device=dev) * frames // Mb).to(torch.int32)

    def adaln_unfused():
        hh = F.layer_norm(xb, (K_DIM,), eps=1e-6)
        hh = hh * (1.0 + mod_scale.index_select(0, mod_idx)) + mod_shift.index_select(0, mod_idx)
        return I.rotate_quant(hh, GROUP), hh

    def adaln_fused():
        return I.rotate_quant_adaln(xb, GROUP, mod_scale, mod_shift, mod_idx)

    out["adaln_prologue_cfg3"] = {"config": "M=32760, K=5120, 8 modulation rows: LayerNorm + modulate + "
                                            "rotate+quantise",
                                  **{f"ms_{k}": v for k, v in timed_ab({"unfused": adaln_unfused,
                                                                        "fused": adaln_fused}, args.steps).items()}}

    # the whole block as chunk_block runs it (transformer.py:339-380), attention replaced by identity (o = v):
    # AdaLN -> QKV -> out + gated residual -> AdaLN -> FFN-up -> SwiGLU -> FFN-down + gated residual
    mods = [(torch.randn(frames, K_DIM, generator=gen) * 0.1).to(torch.bfloat16).to(dev) for _ in range(6)]
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mods
    idx_l = mod_idx.long()

    def block_unfused():
        hh = F.layer_norm(xb, (K_DIM,), eps=1e-6)
        hh = hh * (1.0 + scale_msa.index_select(0, idx_l)) + shift_msa.index_select(0, idx_l)
        o = layers["qkv"](hh)[:, 2 * K_DIM:]
        h2 = xb + gate_msa.index_select(0, idx_l) * layers["out"](o)
        n = F.layer_norm(h2, (K_DIM,), eps=1e-6)
        n = n * (1.0 + scale_mlp.index_select(0, idx_l)) + shift_mlp.index_select(0, idx_l)
        f = layers["ffn_down"](ffn.swiglu_reference(layers["ffn_up"](n)))
        return h2 + gate_mlp.index_select(0, idx_l) * f

    def block_fused():
        hh = I.adaln_modulate_quantize(xb, scale_msa, shift_msa, mod_idx, GROUP)
        o = layers["qkv"](hh)[:, 2 * K_DIM:]
        h2 = layers["out"](o, residual=xb, gate=gate_msa, gate_index=mod_idx)
        n = I.adaln_modulate_quantize(h2, scale_mlp, shift_mlp, mod_idx, GROUP)
        return layers["ffn_down"](swiglu_up(n), residual=h2, gate=gate_mlp, gate_index=mod_idx)

    # config 5: cross-attention K/V projections on text tokens (4096 -> 5120, r = 32), eager and as a CUDA graph
    from hyperflow_h3_flash_b200.graphs import CapturedCall

    kv_layers = []
    for i in range(2):
        wl = synthetic.linear_weights(4096, K_DIM, rank=RANK, bias=True, group=GROUP, seed_offset=80 + i)
        ly = I.Int8RotLinear(4096, K_DIM, GROUP, bias=True, rank=RANK)
        synthetic.load_into(ly, wl)
        kv_layers.append(ly.to(dev))
    kv_layers[0].keep_input = True

    def kv(t):
        return kv_layers[0](t), kv_layers[1](t)

    from hyperflow_h3_flash_b200.grouped import GroupedInt8RotLinear

    kv_group = GroupedInt8RotLinear(*kv_layers)
    # the reference's own modules on the same weights (its Triton and cuBLASLt kernels, eager as it runs)
    ref, _ = load_reference_int8()
    ref_kv = None
    if ref is not None and ref._kernels() is not None:
        ref.set_kernel_options(rotate_quant="factored", int8_gemm="auto")
        ref_parts = reference_layers(ref, torch, dev, 4096, K_DIM, RANK, 2, seed0=80)

        def ref_kv(t):
            ref_parts[0][0].keep_input = True
            return reference_linear(t, ref_parts[0]), reference_linear(t, ref_parts[1])

    cfg5 = {}
    for rows in (256, 333):
        xt = synthetic.activations(rows, 4096, seed=rows).to(dev)
        graphed = CapturedCall(kv, xt)
        graphed_group = CapturedCall(kv_group, xt)
        variants = {"eager": lambda: kv(xt), "graph": lambda: graphed(xt), "grouped_graph": lambda: graphed_group(xt)}
        if ref_kv is not None:
            variants["reference_eager"] = lambda: ref_kv(xt)
        t = timed_ab(variants, args.steps * 5)
        cfg5[f"M{rows}"] = {f"{k}_us": v * 1e3 for k, v in t.items()}
    if ref is not None:
        ref.Int8RotLinear._last_input.clear()
    out["cross_attention_kv_cfg5"] = {"config": "config 5: K and V projections 4096 -> 5120 (r=32, bias, shared "
                                                "quantisation) on 256 / 333 text tokens, per call; grouped = one "
                                                "quantisation, one down projection and one GEMM launch for both; "
                                                "reference_eager = the reference's own Int8RotLinear (Triton "
                                                "factored rotate, cuBLASLt + rescale) + bias + LowRankLinear",
                                      **cfg5}

    # config 2's q / k / v as three layers (shared quantisation and down projection) or as one grouped launch
    qkv_layers = []
    for i in range(3):
        wl = synthetic.linear_weights(K_DIM, N_DIM, rank=RANK, bias=True, group=GROUP, seed_offset=60 + i)
        ly = I.Int8RotLinear(K_DIM, N_DIM, GROUP, bias=True, rank=RANK)
        synthetic.load_into(ly, wl)
        qkv_layers.append(ly.to(dev))
    I.share_lowrank(*qkv_layers)
    qkv_layers[0].keep_input = qkv_layers[1].keep_input = True
    qkv_group = GroupedInt8RotLinear(*qkv_layers)
    t = timed_ab({"separate": lambda: [ly(x) for ly in qkv_layers], "grouped": lambda: qkv_group(x)}, args.steps)
    out["qkv_cfg2"] = {"config": f"config 2's q, k, v (M={M}, K=N={K_DIM}, r={RANK}, bias): three layers sharing "
                                 "quantisation and down projection, or one grouped GEMM launch",
                       "separate_ms": t["separate"], "grouped_ms": t["grouped"]}

    t = timed_ab({"unfused": block_unfused, "fused": block_fused}, steps_b)
    ms_bu, ms_bf = t["unfused"], t["fused"]
    out["dit_block_cfg3"] = {"config": "config 3 block dataflow (chunk_block with identity attention): AdaLN, QKV, "
                                       "out + gated residual, AdaLN, FFN-up, SwiGLU, FFN-down + gated residual",
                             "ms_unfused": ms_bu, "ms_fused": ms_bf, "int8_ops": ops,
                             "tops_fused": ops / (ms_bf * 1e-3) / 1e12}
    return out


def measured_peak(key: str):
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


def load_traffic(kind: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), when present."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(kind)
    except (OSError, ValueError):
        return None


def run_case(args) -> None:
    """One kernel alone on a small case, for `ncu -k regex:<kernel> -s 3 -c 1`; prints its CUDA-event time."""
    import torch

    from hyperflow_h3_flash_b200 import int8 as I
    from hyperflow_h3_flash_b200 import synthetic

    dev = torch.device("cuda", 0)
    M = args.rows
    if args.case == "step":  # the bench's step alone (1 GPU): its kernels' launch list, no extras or baselines
        from hyperflow_h3_flash_b200 import ulysses

        layers = []
        for i in range(4):
            w = synthetic.linear_weights(K_DIM, N_DIM, rank=RANK, bias=True, group=GROUP, seed_offset=i)
            layer = I.Int8RotLinear(K_DIM, N_DIM, GROUP, bias=True, rank=RANK)
            synthetic.load_into(layer, w)
            layers.append(layer.to(dev))
        layers[0].keep_input = layers[1].keep_input = True
        I.share_lowrank(*layers[:3])
        x = synthetic.activations(M, K_DIM).to(dev)
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.inference_mode():
            for i in range(args.warmup + args.steps):
                if i == args.warmup:
                    torch.cuda.synchronize()
                    st.record()
                ulysses.attention_block_linears(x, *layers, HEADS)
            en.record()
            en.synchronize()
        print(json.dumps({"case": "step", "rows": M, "ms_per_step": st.elapsed_time(en) / max(args.steps, 1)}),
              flush=True)
        return
    x = synthetic.activations(M, K_DIM).to(dev)
    w = synthetic.linear_weights(K_DIM, N_DIM, rank=RANK, bias=True, group=GROUP).to(dev)
    q, s = I.rotate_quant(x, GROUP)
    xa = I.lowrank_down(x, w.down)
    if args.case == "gemm_ffn_up":  # config 3's FFN-up with the fused SwiGLU: B (141 MB) is larger than L2
        from hyperflow_h3_flash_b200 import ffn

        wf = synthetic.linear_weights(K_DIM, 2 * 13824, rank=64, bias=True, group=GROUP, seed_offset=22)
        perm = ffn.interleave_rows(2 * 13824)
        wf = synthetic.LinearWeights(wf.qweight[perm], wf.wscale[perm], wf.bias[perm], wf.down, wf.up[perm]).to(dev)
        xa64 = I.lowrank_down(x, wf.down)
    if args.case == "rotate_adaln":  # the AdaLN prologue of a block: 8 modulation rows, frames of tokens
        gen = torch.Generator().manual_seed(9)
        mod_sc = (torch.randn(8, K_DIM, generator=gen) * 0.1).to(torch.bfloat16).to(dev)
        mod_sh = (torch.randn(8, K_DIM, generator=gen) * 0.1).to(torch.bfloat16).to(dev)
        mod_idx = (torch.arange(M, device=dev) * 8 // M).to(torch.int32)
    if args.case == "rotate_ffn_down":  # config 3's FFN-down input (K = 13824: the one-column kernel)
        h = synthetic.activations(M, 13824, seed=2).to(dev)
    fns = {
        "rotate_ffn_down": lambda: I.rotate_quant(h, GROUP),
        "rotate_adaln": lambda: I.rotate_quant_adaln(x, GROUP, mod_sc, mod_sh, mod_idx),
        "gemm_ffn_up": lambda: I.convrot_matmul(q, wf.qweight, s, wf.wscale, bias=wf.bias, xa=xa64, up=wf.up,
                                                swiglu=True),
        "gemm": lambda: I.convrot_matmul(q, w.qweight, s, w.wscale, bias=w.bias, xa=xa, up=w.up),
        "gemm_plain": lambda: I.int8_matmul(q, w.qweight, s, w.wscale),
        "rotate": lambda: I.rotate_quant(x, GROUP),
        "down": lambda: I.lowrank_down(x, w.down),
    }
    fn = fns[args.case]
    times = []
    for i in range(6):
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        fn()
        en.record()
        en.synchronize()
        if i >= 3:
            times.append(st.elapsed_time(en))
    print(json.dumps({"case": args.case, "rows": M, "ms": times}), flush=True)


def main() -> None:
    args = parse()
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
