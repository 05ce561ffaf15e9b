"""Generates the golden fixtures in this folder from the reference implementation itself.

Run once, where the reference source is available (it is not on the GPU machines):

    python tests/golden/make_golden.py /path/to/hyperflow-h3-flash

Nothing here is imported by the tests; they only read the ``.npz`` files written below.

What is captured, all on CPU:

* ``hadamard.npz``: ``regular_hadamard(g)`` for g = 4..256, ``hadamard_factors`` for 256/1024/4096/16/64
  (src/hyperflow_h3_flash/int8.py:100-119), and which sizes raise.
* ``cpu_forward.npz``: ``Int8RotLinear`` forwards on CPU tensors, i.e. the reference's torch path
  ``_forward_torch`` (int8.py:161-179), for the recipe of tests/test_int8.py:51-63 (group 16, fp32 input) and a small
  ``layer_and_input``-style case (tests/test_int8.py:93-102: group 256, bf16 input with ``x[:, ::97] *= 30``), with
  the checkpoint recipe ``quantize`` (tests/test_int8.py:31-36) imported from the reference's test module.
* ``triton_kernels.npz``: the reference's own Triton kernels (int8.py:194-324) executed by Triton's CPU
  interpreter (``TRITON_INTERPRET=1``). Three interpreter defects are patched in this harness, none in the kernels:
  ``tl.dot`` on bf16 multiplied the raw uint16 bit patterns, fp32->bf16 casts truncated instead of rounding to
  nearest even, and ``libdevice.rint`` has no interpreter binding (numpy's ``rint`` rounds half to even, as the
  device ``rint`` does). Two dot models are recorded for the rotation kernels:
  ``exact``: each ``tl.dot`` formed in float64 (exact for these inputs) and rounded once to fp32, the ideal fp32
  accumulator; ``fp32``: numpy's float32 matmul, an inexact accumulation like a tensor core's.
  The int8 GEMM kernel (with its ``(acc * sa) * sb`` epilogue) and the rescale kernel are exact integer/fp32 work
  and are recorded once.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    spec = importlib.util.spec_from_file_location("hyperflow_h3_flash.int8",
                                                  os.path.join(root, "src/hyperflow_h3_flash/int8.py"))
    int8 = importlib.util.module_from_spec(spec)
    package = types.ModuleType("hyperflow_h3_flash")
    package.int8 = int8
    sys.modules["hyperflow_h3_flash"] = package
    sys.modules["hyperflow_h3_flash.int8"] = int8
    spec.loader.exec_module(int8)
    tspec = importlib.util.spec_from_file_location("ref_test_int8", os.path.join(root, "tests/test_int8.py"))
    test_int8 = importlib.util.module_from_spec(tspec)
    tspec.loader.exec_module(test_int8)
    return int8, test_int8


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def patch_interpreter(dot_model: str) -> None:
    import triton.language as tl
    import triton.language.extra.cuda.libdevice as libdevice
    import triton.runtime.interpreter as TI
    from triton.runtime.interpreter import TensorHandle

    def rint(x, _semantic=None):
        return tl.core.tensor(TensorHandle(np.rint(x.handle.data), x.handle.dtype), x.type)

    libdevice.rint = rint

    def as_f32(h):
        if h.dtype == tl.bfloat16:
            return (h.data.astype(np.uint32) << 16).view(np.float32)
        return h.data

    orig_dot = getattr(TI.InterpreterBuilder, "_golden_orig_dot", TI.InterpreterBuilder.create_dot)
    TI.InterpreterBuilder._golden_orig_dot = orig_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype == tl.bfloat16 or b.dtype == tl.bfloat16:
            a32, b32 = as_f32(a), as_f32(b)
            if dot_model == "exact":
                prod = np.matmul(a32.astype(np.float64), b32.astype(np.float64))
                out = (prod + d.data.astype(np.float64)).astype(np.float32)
            else:
                out = np.matmul(a32, b32, dtype=np.float32) + d.data
            return TensorHandle(out.astype(np.float32), d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    TI.InterpreterBuilder.create_dot = create_dot

    orig_cast = getattr(TI.InterpreterBuilder, "_golden_orig_cast", TI.InterpreterBuilder.cast_impl)
    TI.InterpreterBuilder._golden_orig_cast = orig_cast

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            t = torch.from_numpy(np.ascontiguousarray(src.data, dtype=np.float32)).to(torch.bfloat16)
            return TensorHandle(t.view(torch.int16).numpy().view(np.uint16), dst_type.scalar)
        return orig_cast(self, src, dst_type)

    TI.InterpreterBuilder.cast_impl = cast_impl


def hadamard_fixture(int8) -> None:
    out = {}
    for g in (4, 16, 64, 256):
        out[f"h{g}"] = int8.regular_hadamard(g).numpy()
    rejects = []
    for g in (2, 8, 32, 128, 512):
        try:
            int8.regular_hadamard(g)
        except ValueError:
            rejects.append(g)
    out["rejected"] = np.array(rejects)
    groups = [16, 64, 256, 1024, 4096]
    out["factor_groups"] = np.array(groups)
    out["factors"] = np.array([int8.hadamard_factors(g) or (0, 0) for g in groups])
    np.savez_compressed(os.path.join(HERE, "hadamard.npz"), **out)


def cpu_forward_fixture(int8, test_int8) -> None:
    out = {}
    # tests/test_int8.py:51-63 recipe, group 16, fp32 input.
    torch.manual_seed(0)
    weight = torch.randn(96, 128) * 0.05
    x = torch.randn(5, 7, 128)
    layer = int8.Int8RotLinear(128, 96, group=16)
    qw, ws = test_int8.quantize(weight, 16)
    layer.qweight.copy_(qw)
    layer.wscale.copy_(ws)
    with torch.no_grad():
        y = layer(x)
    out.update(a_weight=weight.numpy(), a_x=x.numpy(), a_qweight=qw.numpy(), a_wscale=ws.numpy(), a_y=y.numpy())
    # layer_and_input recipe (tests/test_int8.py:93-102) at a CPU-sized shape, group 256, bf16 input.
    torch.manual_seed(0)
    weight = torch.randn(256, 1024) * 0.02
    layer = int8.Int8RotLinear(1024, 256, group=256)
    qw, ws = test_int8.quantize(weight, 256)
    layer.qweight.copy_(qw)
    layer.wscale.copy_(ws)
    x = torch.randn(40, 1024, dtype=torch.bfloat16)
    x[:, ::97] *= 30
    with torch.no_grad():
        y = layer(x)
    out.update(b_x=bits(x), b_qweight=qw.numpy(), b_wscale=ws.numpy(), b_y=bits(y))
    # The checkpoint recipe at group 256 on a small weight (the weight itself is stored for the recipe pin).
    torch.manual_seed(3)
    weight = torch.randn(24, 512) * 0.02
    qw, ws = test_int8.quantize(weight, 256)
    out.update(c_weight=weight.numpy(), c_qweight=qw.numpy(), c_wscale=ws.numpy())
    np.savez_compressed(os.path.join(HERE, "cpu_forward.npz"), **out)


def triton_fixture(int8) -> None:
    import triton

    out = {}
    gen = torch.Generator().manual_seed(7)
    M, K = 70, 1024  # 70 rows: a full 64-row block and a ragged one
    x = torch.randn(M, K, dtype=torch.bfloat16, generator=gen)
    x[:, ::97] *= 30
    x[3] = 0  # an all-zero row: the 1e-12 floor of the scale
    x[5, :256] = 0  # an all-zero group
    out["x"] = bits(x)
    for model in ("exact", "fp32"):
        patch_interpreter(model)
        kernels = int8._kernels.__wrapped__()
        for g in (16, 64, 256):
            q = torch.empty(M, K, dtype=torch.int8)
            s = torch.empty(M, dtype=torch.float32)
            bn = min(128, g)
            kernels.jit.rotate_quant[(triton.cdiv(M, 64),)](
                x, int8.regular_hadamard(g).to(torch.bfloat16), q, s, M, K, x.stride(0), q.stride(0),
                G=g, BM=64, BN=bn, num_warps=8, num_stages=1)
            out[f"dense_{model}_g{g}_q"] = q.numpy()
            out[f"dense_{model}_g{g}_s"] = s.numpy()
        q = torch.empty(M, K, dtype=torch.int8)
        s = torch.empty(M, dtype=torch.float32)
        h16 = int8.regular_hadamard(16).to(torch.bfloat16)
        kernels.jit.rotate_quant_factored[(triton.cdiv(M, 16),)](
            x, h16, h16, q, s, M, K, x.stride(0), q.stride(0), GA=16, GB=16, BM=16, num_warps=4, num_stages=4)
        out[f"factored_{model}_g256_q"] = q.numpy()
        out[f"factored_{model}_g256_s"] = s.numpy()

    # The GEMM kernel with its epilogue, and the rescale epilogue, on exact int8 codes.
    patch_interpreter("exact")
    kernels = int8._kernels.__wrapped__()
    gen = torch.Generator().manual_seed(11)
    Mg, Ng, Kg = 70, 96, 512
    a = torch.randint(-127, 128, (Mg, Kg), dtype=torch.int8, generator=gen)
    b = torch.randint(-127, 128, (Ng, Kg), dtype=torch.int8, generator=gen)
    sa = (torch.rand(Mg, generator=gen) * 0.1 + 1e-3).float()
    sb = (torch.rand(Ng, generator=gen) * 1e-3 + 1e-5).float()
    c = torch.empty(Mg, Ng, dtype=torch.bfloat16)
    m_bucket = 1 << max(Mg - 1, 1).bit_length()
    kernels.jit.int8_mm.fn[(triton.cdiv(Mg, 64) * triton.cdiv(Ng, 64),)](
        a, b, c, sa, sb, Mg, Ng, Kg, m_bucket, a.stride(0), b.stride(0), c.stride(0),
        BM=64, BN=64, BK=64, GROUP_M=8)
    acc = a.int() @ b.int().t()
    c2 = torch.empty(Mg, Ng, dtype=torch.bfloat16)
    kernels.jit.rescale[(triton.cdiv(Mg, 64), triton.cdiv(Ng, 128))](acc, sa, sb, c2, Mg, Ng, BM=64, BN=128,
                                                                     num_warps=8)
    out.update(gemm_a=a.numpy(), gemm_b=b.numpy(), gemm_sa=sa.numpy(), gemm_sb=sb.numpy(), gemm_out=bits(c),
               rescale_acc=acc.numpy(), rescale_out=bits(c2))
    np.savez_compressed(os.path.join(HERE, "triton_kernels.npz"), **out)


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HYPERFLOW_REFERENCE", "")
    if not root or not os.path.isdir(root):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    int8, test_int8 = load_reference(root)
    hadamard_fixture(int8)
    cpu_forward_fixture(int8, test_int8)
    triton_fixture(int8)
    for name in sorted(os.listdir(HERE)):
        if name.endswith(".npz"):
            print(name, os.path.getsize(os.path.join(HERE, name)))


if __name__ == "__main__":
    main()
