// C ABI of the B200 INT8 convrot linear (declarations and contracts: include/convrot.h).
//
// One translation unit holds every kernel, so the device error word is a plain file-scope __device__ variable.
// Host side: argument validation (shape, alignment, group), TMA tensor-map encoding through the driver entry
// point (no libcuda link dependency), per-device lazy state (SM count, compute capability), and dispatch to the
// template instances of rotate_quant_kernel and convrot_gemm_kernel.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/convrot.h"
#include "gemm_sm100.cuh"
#include "gemm_sm100_2sm.cuh"
#include "peer.cuh"
#include "rotate_quant.cuh"

namespace convrot {

__device__ int g_error_word;  // CONVROT_ERR_TIMEOUT after a bounded wait expired; cleared by convrot_poll_error

// Scratch of convrot_linear_noalloc: the codes, scales and low-rank input of one call live here instead of in a
// caller allocation.  It is part of the library's device image, so every GPU that loads the library holds these
// CONVROT_NOALLOC_SCRATCH_BYTES until the process exits.  In host code the name is only a host-side stand-in:
// its device address comes from cudaGetSymbolAddress (see noalloc_scratch below), never from the name itself.
static __device__ __align__(256) uint8_t g_noalloc_scratch[CONVROT_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local int t_last_cuda_error = 0;
uint64_t g_wait_limit_ns = 2000000000ull;
int g_gemm_mode = 0;  // 0 auto, 1 one-SM kernel, 2 two-SM kernel
int g_rq_variant = 0;  // G = 256 rotation: 0 two-column team kernel, 1 one-column kernel
int g_rq_stages = 0, g_rq_blocks = 0;  // rotation tuning overrides (0 = automatic)
std::atomic<int64_t> g_split_fallbacks{0};  // split-K down projections that ran unsplit (cluster not placeable)

struct DeviceState {
  bool ready = false;
  int status = CONVROT_OK;
  int sms = 0;
  int* error_word = nullptr;
  uint8_t* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch on this device (first no-alloc call)
};

constexpr int kMaxDevices = 64;
DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn g_address_range = nullptr;

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return CONVROT_ERR_CUDA;
}

// Per-device lazy set-up: architecture check, SM count, the address of the error word, the driver entry point.
int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return CONVROT_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& st = g_devices[dev];
  if (!st.ready) {
    int major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) return cuda_fail(e);
    if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) return cuda_fail(e);
    if ((e = cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return cuda_fail(e);
    st.status = (major == 10 && minor == 0) ? CONVROT_OK : CONVROT_ERR_ARCH;
    if (st.status == CONVROT_OK) {
      if ((e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.error_word), g_error_word)) != cudaSuccess)
        return cuda_fail(e);
      if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if ((e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q)) != cudaSuccess)
          return cuda_fail(e);
        if (q != cudaDriverEntryPointSuccess || !fn) return CONVROT_ERR_CUDA;
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
      }
      if (!g_address_range) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if ((e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q)) != cudaSuccess)
          return cuda_fail(e);
        if (q != cudaDriverEntryPointSuccess || !fn) return CONVROT_ERR_CUDA;
        g_address_range = reinterpret_cast<AddressRangeFn>(fn);
      }
    }
    st.ready = true;
  }
  if (st.status != CONVROT_OK) return st.status;
  *out = &st;
  return CONVROT_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D K-major tensor map: rows x cols elements of `elem` bytes, row pitch ld elements, box box_rows x box_cols,
// swizzle matching box_cols * elem (128 or 64 bytes).
int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem, int64_t rows, int64_t cols,
             int64_t ld, int box_rows, int box_cols) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const int inner = box_cols * elem;
  CUtensorMapSwizzle sw = inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return CONVROT_ERR_CUDA;
  }
  return CONVROT_OK;
}

// Per-(device, kernel) launch facts computed once: the shared-memory opt-in and the resident CTAs / clusters.
// Keyed by the kernel's address; a handful of instances exist, so a small linear table suffices.
struct LaunchCache {
  const void* fn;
  int dev;
  int resident;
};
constexpr int kLaunchCacheSize = 256;
LaunchCache g_launch_cache[kLaunchCacheSize];
int g_launch_cache_n = 0;

int cached_resident(const void* fn, int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  std::lock_guard<std::mutex> lock(g_mutex);
  for (int i = 0; i < g_launch_cache_n; ++i)
    if (g_launch_cache[i].fn == fn && g_launch_cache[i].dev == dev) {
      *out = g_launch_cache[i].resident;
      return CONVROT_OK;
    }
  *out = -1;
  return CONVROT_OK;
}

void store_resident(const void* fn, int resident) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_launch_cache_n < kLaunchCacheSize) {
    LaunchCache& c = g_launch_cache[g_launch_cache_n++];
    c.fn = fn;
    c.dev = dev;
    c.resident = resident;
  }
}

// 3-D map over "chunked rows": element (m, k) at base + (k / W) * S + m * L + k % W, i.e. dims (W, M, K / W) with
// byte strides (L * elem, S * elem); box box_cols x box_rows x 1, swizzle as make_map.
int make_map3(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem, int64_t rows, int64_t W,
              int64_t chunks, int64_t L, int64_t S, int box_rows, int box_cols) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(chunks)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(L * elem),
                           static_cast<cuuint64_t>((chunks > 1 ? S : L * rows) * elem)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const int inner = box_cols * elem;
  CUtensorMapSwizzle sw = inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return CONVROT_ERR_CUDA;
  }
  return CONVROT_OK;
}

template <class Cfg, int KIND, int EPI, int LR_ATOM, int LR_ATOMS>
int launch_gemm(const DeviceState& st, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& txa,
                const CUtensorMap& tup, const GemmParams& p, cudaStream_t stream) {
  auto kernel = convrot_gemm_kernel<Cfg, KIND, EPI, LR_ATOM, LR_ATOMS>;
  int resident = -1;
  int rc = cached_resident(reinterpret_cast<const void*>(kernel), &resident);
  if (rc) return rc;
  cudaError_t e;
  if (resident < 0) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e);
    store_resident(reinterpret_cast<const void*>(kernel), 1);
  }
  // Kernels whose shared memory and TMEM leave room run two CTAs per SM (the low-rank down projection is
  // HBM-bound with few tiles: two per SM keeps every tile of a 32k-row input in flight at once).
  const int per_sm = (Cfg::kSmemBytes <= 113 * 1024 && Cfg::kTmemCols <= 256) ? 2 : 1;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + Cfg::kBN - 1) / Cfg::kBN);
  bool split = p.split_k > 1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr = {};
  if (split) {  // clusters of split_k CTAs, one tile per cluster (EPI_BF16 split K)
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * p.split_k), 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(p.split_k);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    // Whether the GPU can place one such cluster at all, asked once per (kernel, split) and cached under a key of
    // its own (the kernel's address offset by the split, which no other entry uses).
    const void* key = reinterpret_cast<const char*>(kernel) + p.split_k;
    int placeable = -1;
    if ((rc = cached_resident(key, &placeable))) return rc;
    if (placeable < 0) {
      int clusters = 0;
      if ((e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg)) != cudaSuccess) return cuda_fail(e);
      placeable = clusters > 0 ? 1 : 0;
      store_resident(key, placeable);
    }
    if (placeable) {
      e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, txa, tup, p);
      return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
    }
    // The unsplit kernel below instead (counted: its K order, and so possibly the last bit of xa, differs).
    g_split_fallbacks.fetch_add(1, std::memory_order_relaxed);
  }
  GemmParams q = p;
  q.split_k = 1;
  const int grid = tiles < per_sm * st.sms ? tiles : per_sm * st.sms;
  kernel<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, txa, tup, q);
  e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

template <class Cfg, int EPI, int LR_ATOM, int LR_ATOMS>
int launch_gemm2(const DeviceState& st, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& txa,
                 const CUtensorMap& tup, const OutMaps& ty, const GemmParams& p, cudaStream_t stream) {
  auto kernel = convrot_gemm2sm_kernel<Cfg, EPI, LR_ATOM, LR_ATOMS>;
  const int pair_tiles = ((p.M + 2 * kBM - 1) / (2 * kBM)) * ((p.N + Cfg::kBN - 1) / Cfg::kBN);
  int clusters = -1;
  int rc = cached_resident(reinterpret_cast<const void*>(kernel), &clusters);
  if (rc) return rc;
  cudaError_t e;
  if (clusters < 0) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * st.sms, 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);
    if (e != cudaSuccess) return cuda_fail(e);
    if (clusters < 1) clusters = st.sms / 2;
    store_resident(reinterpret_cast<const void*>(kernel), clusters);
  }
  const int pairs = pair_tiles < clusters ? pair_tiles : clusters;
  kernel<<<2 * pairs, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, txa, tup, ty, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

// ---------------------------------------------------------------------------------------------- GEMM dispatch

using CfgI8 = GemmCfg<KIND_I8, 256, 4, EPI_DEQUANT, 0, 0>;
using CfgI8LR32 = GemmCfg<KIND_I8, 256, 4, EPI_DEQUANT, 64, 1>;
using CfgI8LR64 = GemmCfg<KIND_I8, 256, 3, EPI_DEQUANT, 128, 1>;
using CfgRaw = GemmCfg<KIND_I8, 256, 4, EPI_RAW_I32, 0, 0>;
using Cfg2 = Gemm2Cfg<5, 0, 0>;
using Cfg2LR32 = Gemm2Cfg<5, 64, 1>;
using Cfg2LR64 = Gemm2Cfg<5, 128, 1>;

struct ResidualArgs {
  const void* res;
  int64_t ld_res;
  const void* gate;
  int64_t ld_gate;
  const int32_t* gate_index;
};

// n_chunks > 1 writes the bf16 output in column chunks of N / n_chunks: chunk j as [M, ldo] rows at chunks[j] (the
// Ulysses send layout, or the receive buffers of the other GPUs); `out` is then ignored.
int gemm_i8(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
            const void* bias, const void* xa, int64_t ldxa, const void* up, int64_t ld_up, int64_t r, int64_t M,
            int64_t N, int64_t K, void* out, int64_t ldo, bool raw, cudaStream_t stream,
            void* const* chunks = nullptr, int n_chunks = 1, bool swiglu = false,
            const ResidualArgs* residual = nullptr, int lr_segments = 1) {
  if (n_chunks < 1 || n_chunks > kMaxChunks || (n_chunks > 1 && !chunks)) return CONVROT_ERR_ARG;
  if (lr_segments < 1 || lr_segments > kMaxChunks) return CONVROT_ERR_ARG;
  if (swiglu && (raw || n_chunks > 1)) return CONVROT_ERR_ARG;
  if (residual) {
    if (raw || swiglu || n_chunks > 1 || !residual->res) return CONVROT_ERR_ARG;
    if (residual->ld_res < N || (residual->gate && residual->ld_gate < N)) return CONVROT_ERR_SHAPE;
    if (residual->ld_res % 8 || !aligned16(residual->res)) return CONVROT_ERR_ALIGN;
    if (residual->gate && (residual->ld_gate % 8 || !aligned16(residual->gate))) return CONVROT_ERR_ALIGN;
  }
  if (swiglu && N % 64) return CONVROT_ERR_SHAPE;
  int64_t out_chunk = swiglu ? N / 2 : N;
  if (n_chunks > 1) {
    if (raw || N % n_chunks || (N / n_chunks) % 32) return CONVROT_ERR_SHAPE;
    out_chunk = N / n_chunks;
    for (int j = 0; j < n_chunks; ++j) {
      if (!chunks[j]) return CONVROT_ERR_ARG;
      if (!aligned16(chunks[j])) return CONVROT_ERR_ALIGN;
    }
    out = chunks[0];
  }
  if (M < 0 || N <= 0 || K <= 0) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || N > (1 << 24)) return CONVROT_ERR_SHAPE;
  if (!q || !w || !out) return CONVROT_ERR_ARG;
  if (!raw && (!sx || !ws)) return CONVROT_ERR_ARG;
  const bool has_lr = !raw && xa && up && r > 0;
  if (!raw && (xa || up) && !has_lr) return CONVROT_ERR_ARG;
  if (has_lr && r > 256) return CONVROT_ERR_SHAPE;
  if (K % 16 || ldq < K || ldw < K || ldo < out_chunk) return CONVROT_ERR_SHAPE;
  if (ldq % 16 || ldw % 16 || !aligned16(q) || !aligned16(w)) return CONVROT_ERR_ALIGN;
  if (raw ? (ldo % 4 || !aligned16(out)) : (ldo % 8 || !aligned16(out))) return CONVROT_ERR_ALIGN;
  if (!raw && (!aligned16(ws) || (bias && !aligned16(bias)))) return CONVROT_ERR_ALIGN;
  if (has_lr && (ldxa < r * lr_segments || ld_up < r || ldxa % 8 || ld_up % 8 || !aligned16(xa) || !aligned16(up)))
    return ldxa < r * lr_segments || ld_up < r ? CONVROT_ERR_SHAPE : CONVROT_ERR_ALIGN;
  // Segments (layers stacked along N): whole 256-column tiles per segment, and each segment's xa columns start on a
  // 16-byte boundary (the TMA load's inner coordinate).
  if (lr_segments > 1 && (!has_lr || N % lr_segments || (N / lr_segments) % 256 || r % 8 || swiglu || residual))
    return has_lr && !swiglu && !residual ? CONVROT_ERR_SHAPE : CONVROT_ERR_ARG;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;

  // Both kernels do the same work per SM and tile (128 rows x 256 columns) and give identical bits.  Automatic mode
  // takes the one with fewer waves of tiles, and the 1-SM kernel whenever its tiles fit one wave (it skips the
  // pair's cluster start-up: 31-32 against 33-49 us on B200 for single-wave shapes at M = 200-500); otherwise the
  // 2-SM kernel, whose halved B traffic per SM makes each tile cheaper at full load.
  bool two_sm = g_gemm_mode == 2;
  if (g_gemm_mode == 0 && M > kBM) {
    const int64_t n_tiles = (N + 255) / 256;
    const int64_t sms = st->sms > 1 ? st->sms : 2;
    const int64_t waves1 = ((M + kBM - 1) / kBM * n_tiles + sms - 1) / sms;
    const int64_t waves2 = ((M + 2 * kBM - 1) / (2 * kBM) * n_tiles + sms / 2 - 1) / (sms / 2);
    two_sm = !(waves1 <= 1 || waves1 < waves2);
  }
  const int b_rows = two_sm ? 128 : 256;  // B rows per CTA tile
  CUtensorMap ta, tb, txa, tup;
  memset(&txa, 0, sizeof(txa));
  memset(&tup, 0, sizeof(tup));
  // A: 2-D for the 2-SM kernel, a one-chunk 3-D map for the 1-SM kernel (which also serves chunked bf16 inputs)
  if (two_sm) {
    if ((rc = make_map(&ta, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, ldq, kBM, 128))) return rc;
  } else if ((rc = make_map3(&ta, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, 1, ldq, 0, kBM, 128))) {
    return rc;
  }
  if ((rc = make_map(&tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, ldw, b_rows, 128))) return rc;
  const int lr_atom = r <= 32 ? 64 : 128;
  if (has_lr) {
    if ((rc = make_map(&txa, xa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, r * lr_segments, ldxa, kBM, lr_atom / 2)))
      return rc;
    // up rows per load: one 128-column half of the tile (1-SM), or the 2-SM CTA's 64-row share of one half
    const int up_rows = two_sm ? 64 : 128;
    if ((rc = make_map(&tup, up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, r, ld_up, up_rows, lr_atom / 2))) return rc;
  }
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = sx;
  p.sb = ws;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.out = out;
  for (int j = 0; j < kMaxChunks; ++j) p.out_chunks[j] = j < n_chunks ? (n_chunks > 1 ? chunks[j] : out) : nullptr;
  p.ldo = ldo;
  p.out_chunk = static_cast<int>(out_chunk);
  p.swiglu = swiglu ? 1 : 0;
  if (residual) {
    p.res = static_cast<const __nv_bfloat16*>(residual->res);
    p.ld_res = residual->ld_res;
    p.gate = static_cast<const __nv_bfloat16*>(residual->gate);
    p.ld_gate = residual->ld_gate;
    p.gate_index = residual->gate_index;
  }
  p.a_chunk = static_cast<int>(K);
  p.r = has_lr ? static_cast<int>(r) : 0;
  p.lr_seg_n = lr_segments > 1 ? static_cast<int>(N / lr_segments) : 0;
  p.wait_limit_ns = g_wait_limit_ns;
  p.error_word = st->error_word;
  // Weights above 64 MB do not stay in L2 between tile groups next to the streaming output, so every group reads
  // them from HBM again: 16 M blocks per group halve that, while a group's A rows (16 x 256 x K bytes) stay at most
  // 32 MB.  Measured at M = 32760-32768 on one box each, 16 against 8: FFN-up with SwiGLU (141.6 MB) 3.08-3.12
  // against 3.16-3.18 ms, QKV (78.6 MB) 1.657-1.663 against 1.703-1.704 ms; FFN-down (70.8 MB, K = 13824: 57 MB of
  // A per group) 1.496-1.498 against 1.475-1.480 ms (and 1.61-1.62 ms with 4), so it keeps 8.  Weights of at most
  // 32 MB stay in L2 anyway; there 4 M blocks per group measured 0.9 % faster than 8 (config 2, 26 MB, alternating
  // runs on one box: 0.5695-0.5829 against 0.5760-0.5840 ms).
  const int64_t b_bytes = static_cast<int64_t>(N) * K;
  p.group_m = b_bytes <= (32LL << 20) ? 4 : b_bytes > (64LL << 20) && K <= 8192 ? 16 : 0;
  if (two_sm) {
    // bf16 output, one map per chunk: 32 x 64 boxes when every chunk (and so the whole output) is a multiple of 64
    // columns wide, else 32 x 32
    OutMaps ty;
    memset(&ty, 0, sizeof(ty));
    p.wide_store = out_chunk % 64 == 0 ? 1 : 0;
    const int box_cols = p.wide_store ? 64 : 32;
    for (int j = 0; j < n_chunks && !raw; ++j)
      if ((rc = make_map(&ty.m[j], p.out_chunks[j], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, out_chunk, ldo, 32,
                         box_cols)))
        return rc;
    if (raw) return launch_gemm2<Cfg2, EPI_RAW_I32, 0, 0>(*st, ta, tb, txa, tup, ty, p, stream);
    if (!has_lr) return launch_gemm2<Cfg2, EPI_DEQUANT, 0, 0>(*st, ta, tb, txa, tup, ty, p, stream);
    if (lr_atom == 64) return launch_gemm2<Cfg2LR32, EPI_DEQUANT, 64, 1>(*st, ta, tb, txa, tup, ty, p, stream);
    return launch_gemm2<Cfg2LR64, EPI_DEQUANT, 128, 1>(*st, ta, tb, txa, tup, ty, p, stream);
  }
  if (raw) return launch_gemm<CfgRaw, KIND_I8, EPI_RAW_I32, 0, 0>(*st, ta, tb, txa, tup, p, stream);
  if (!has_lr) return launch_gemm<CfgI8, KIND_I8, EPI_DEQUANT, 0, 0>(*st, ta, tb, txa, tup, p, stream);
  if (lr_atom == 64) return launch_gemm<CfgI8LR32, KIND_I8, EPI_DEQUANT, 64, 1>(*st, ta, tb, txa, tup, p, stream);
  return launch_gemm<CfgI8LR64, KIND_I8, EPI_DEQUANT, 128, 1>(*st, ta, tb, txa, tup, p, stream);
}

// x . down^T -> bf16 [M, r] on kind::f16 tensor cores.
template <int BN, int STAGES>
using CfgDown = GemmCfg<KIND_BF16, BN, STAGES, EPI_BF16, 0, 0>;

// x in chunked rows (W = x_chunk, S = x_chunk_stride; plain rows: x_chunk = K).
int lowrank_down(const void* x, int64_t ldx, const void* down, int64_t ld_down, int64_t M, int64_t K, int64_t r,
                 void* xa, int64_t ldxa, cudaStream_t stream, int64_t x_chunk = 0, int64_t x_chunk_stride = 0) {
  if (x_chunk <= 0) x_chunk = K;
  if (K % x_chunk || (x_chunk != K && (x_chunk % 64 || x_chunk_stride % 8))) return CONVROT_ERR_SHAPE;
  if (M < 0 || K <= 0 || r <= 0) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  if (M > INT32_MAX || K > INT32_MAX || r > 256) return CONVROT_ERR_SHAPE;
  if (!x || !down || !xa) return CONVROT_ERR_ARG;
  if (K % 8 || ldx < x_chunk || ld_down < K || ldxa < r) return CONVROT_ERR_SHAPE;
  if (ldx % 8 || ld_down % 8 || ldxa % 8 || !aligned16(x) || !aligned16(down) || !aligned16(xa))
    return CONVROT_ERR_ALIGN;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const int bn = r <= 32 ? 32 : r <= 64 ? 64 : r <= 128 ? 128 : 256;
  CUtensorMap ta, tb, tz;
  memset(&tz, 0, sizeof(tz));
  if ((rc = make_map3(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, x_chunk, K / x_chunk, ldx, x_chunk_stride,
                      kBM, 64)))
    return rc;
  if ((rc = make_map(&tb, down, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, r, K, ld_down, bn, 64))) return rc;
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(r);
  p.K = static_cast<int>(K);
  p.out = xa;
  p.out_chunks[0] = xa;
  p.ldo = ldxa;
  p.out_chunk = static_cast<int>(r);
  p.a_chunk = static_cast<int>(x_chunk);
  p.wait_limit_ns = g_wait_limit_ns;
  p.error_word = st->error_word;
  // Few row tiles (M <= 1024): split K over a cluster of up to 8 CTAs per tile, so the serial K loop of each tile is
  // shared instead of running on one SM.  The split depends on M and K only, so layers that share an input compute
  // each xa column with the same additions whether their down projections run stacked or one by one.
  const int64_t nkb = (K + 63) / 64;
  if (M <= 8 * kBM && nkb >= 4) {
    int split = 1;
    while (split * 2 <= 8 && split * 2 <= nkb / 2) split *= 2;
    p.split_k = split;
  }
  switch (bn) {
    case 32: return launch_gemm<CfgDown<32, 5>, KIND_BF16, EPI_BF16, 0, 0>(*st, ta, tb, tz, tz, p, stream);
    case 64: return launch_gemm<CfgDown<64, 4>, KIND_BF16, EPI_BF16, 0, 0>(*st, ta, tb, tz, tz, p, stream);
    case 128: return launch_gemm<CfgDown<128, 3>, KIND_BF16, EPI_BF16, 0, 0>(*st, ta, tb, tz, tz, p, stream);
    default: return launch_gemm<CfgDown<256, 4>, KIND_BF16, EPI_BF16, 0, 0>(*st, ta, tb, tz, tz, p, stream);
  }
}

// ---------------------------------------------------------------------------------------------- rotate+quant

using RotQuantKernel = void (*)(const RotQuantParams);

// The instance of a rotate kernel for a rounding mode (CONVROT_ROUND_KERNEL / _TORCH / _TRITON).
RotQuantKernel by_rounding(int rounding, RotQuantKernel kernel_mode, RotQuantKernel torch_mode,
                           RotQuantKernel triton_mode) {
  return rounding == CONVROT_ROUND_TORCH ? torch_mode : rounding == CONVROT_ROUND_TRITON ? triton_mode : kernel_mode;
}

template <int G>
int launch_rq(const DeviceState& st, const RotQuantParams& p, cudaStream_t stream) {
  const int nslots = p.K / 16;
  int slots = 1;
  while ((nslots + slots - 1) / slots > 512) slots *= 2;
  if (slots > 4) return CONVROT_ERR_SHAPE;
  int threads = (nslots + slots - 1) / slots;
  threads = (threads + 31) / 32 * 32;
  RotQuantParams q = p;
  cudaError_t e;
  void (*kernel)(const RotQuantParams) = nullptr;
  switch (slots) {
    case 1: kernel = by_rounding(p.rounding, rotate_quant_kernel<G, 1, 0>, rotate_quant_kernel<G, 1, 1>,
                                 rotate_quant_kernel<G, 1, 2>); break;
    case 2: kernel = by_rounding(p.rounding, rotate_quant_kernel<G, 2, 0>, rotate_quant_kernel<G, 2, 1>,
                                 rotate_quant_kernel<G, 2, 2>); break;
    default: kernel = by_rounding(p.rounding, rotate_quant_kernel<G, 4, 0>, rotate_quant_kernel<G, 4, 1>,
                                  rotate_quant_kernel<G, 4, 2>); break;
  }
  int regs = -1;  // the kernel's registers per thread, cached with the shared-memory opt-in
  int rc = cached_resident(reinterpret_cast<const void*>(kernel), &regs);
  if (rc) return rc;
  if (regs < 0) {
    if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)) != cudaSuccess)
      return cuda_fail(e);
    cudaFuncAttributes attr;
    if ((e = cudaFuncGetAttributes(&attr, kernel)) != cudaSuccess) return cuda_fail(e);
    regs = attr.numRegs > 0 ? attr.numRegs : 128;
    store_resident(reinterpret_cast<const void*>(kernel), regs);
  }
  // Resident CTAs first (from the kernel's registers, allocated per warp in units of 8 per thread), then the
  // deepest row ring that fits beside them: the per-row chain is latency-bound, so CTAs beat ring depth (measured
  // on B200 for K = 13824: 2 CTAs x 1 row buffer 0.57 ms, 1 CTA x 6 buffers 0.69 ms).  The grid is
  // oversubscribed 4x so that the last rows spread evenly.
  const int regs_alloc = (regs + 7) / 8 * 8;
  int resident = 65536 / (threads * regs_alloc);
  if (resident > 2048 / threads) resident = 2048 / threads;
  if (resident < 1) resident = 1;
  while (resident > 1 && static_cast<size_t>(resident) * (rq_smem_bytes(p.K, threads, 1) + 1024) > 228 * 1024)
    --resident;
  int stages = 1;
  for (int st_try = 2; st_try <= kRQMaxStages; ++st_try) {
    const size_t sm = rq_smem_bytes(p.K, threads, st_try);
    if (sm > 227 * 1024 || static_cast<size_t>(resident) * (sm + 1024) > 228 * 1024) break;
    stages = st_try;
  }
  int best_blocks = 4 * resident;
  if (g_rq_stages > 0) stages = g_rq_stages;
  if (g_rq_blocks > 0) best_blocks = g_rq_blocks;
  q.stages = stages;
  const size_t smem = rq_smem_bytes(p.K, threads, stages);
  if (smem > 227 * 1024) return CONVROT_ERR_SHAPE;
  int64_t grid = static_cast<int64_t>(st.sms) * best_blocks;
  if (grid > p.M) grid = p.M;
  kernel<<<static_cast<int>(grid), threads, smem, stream>>>(q);
  e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

// G = 256: the two-column team kernel (8 threads per group).
int launch_rq256(const DeviceState& st, const RotQuantParams& p, cudaStream_t stream) {
  const int ngroups = p.K / 256;
  // One group per thread up to 256 threads (K = 8192), two groups per thread beyond (up to 512 threads)
  const int slots = ngroups * 8 <= 256 ? 1 : 2;
  if ((ngroups * 8 + slots - 1) / slots > 512) return CONVROT_ERR_SHAPE;
  int threads = (ngroups * 8 + slots - 1) / slots;
  threads = (threads + 31) / 32 * 32;
  RotQuantParams q = p;
  const bool chunked = p.x_chunk != p.K;
  const bool adaln = p.mod_scale != nullptr;
  if (adaln && (chunked || slots != 1)) return CONVROT_ERR_SHAPE;
  if (chunked && slots == 1 && threads > kRQ256ChunkedThreads) return launch_rq<256>(st, p, stream);
  void (*kernel)(const RotQuantParams) = nullptr;
  if (adaln)
    kernel = by_rounding(p.rounding, rotate_quant256_kernel<1, 0, false, true>,
                         rotate_quant256_kernel<1, 1, false, true>, rotate_quant256_kernel<1, 2, false, true>);
  else if (slots == 1 && !chunked)
    kernel = by_rounding(p.rounding, rotate_quant256_kernel<1, 0, false>, rotate_quant256_kernel<1, 1, false>,
                         rotate_quant256_kernel<1, 2, false>);
  else if (slots == 1)
    kernel = by_rounding(p.rounding, rotate_quant256_kernel<1, 0, true>, rotate_quant256_kernel<1, 1, true>,
                         rotate_quant256_kernel<1, 2, true>);
  else if (!chunked)
    kernel = by_rounding(p.rounding, rotate_quant256_kernel<2, 0, false>, rotate_quant256_kernel<2, 1, false>,
                         rotate_quant256_kernel<2, 2, false>);
  else
    kernel = by_rounding(p.rounding, rotate_quant256_kernel<2, 0, true>, rotate_quant256_kernel<2, 1, true>,
                         rotate_quant256_kernel<2, 2, true>);
  int regs = -1;  // the kernel's registers per thread, cached with the shared-memory opt-in
  int rc = cached_resident(reinterpret_cast<const void*>(kernel), &regs);
  if (rc) return rc;
  cudaError_t e;
  if (regs < 0) {
    if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)) != cudaSuccess)
      return cuda_fail(e);
    cudaFuncAttributes attr;
    if ((e = cudaFuncGetAttributes(&attr, kernel)) != cudaSuccess) return cuda_fail(e);
    regs = attr.numRegs > 0 ? attr.numRegs : 128;
    store_resident(reinterpret_cast<const void*>(kernel), regs);
  }
  // The per-row work is a serial chain (exact rotation, block-wide amax, quantise), so throughput comes from
  // resident CTAs: fill the SM with as many CTAs as its registers hold (allocated per warp in units of 8 per
  // thread), then give each the deepest row ring that still fits (measured on B200: K = 5120 -> 4 CTAs x 3 row
  // buffers).
  const int regs_alloc = (regs + 7) / 8 * 8;
  int best_blocks = 65536 / (threads * regs_alloc);
  if (best_blocks > 2048 / threads) best_blocks = 2048 / threads;
  if (best_blocks < 1) best_blocks = 1;
  int best_stages = 1;
  for (int stages = 2; stages <= kRQMaxStages; ++stages) {
    const size_t sm = rq256_smem_bytes(p.K, threads, stages, chunked, adaln);
    if (sm > 227 * 1024 || static_cast<size_t>(best_blocks) * (sm + 1024) > 228 * 1024) break;
    best_stages = stages;
  }
  if (best_stages < 2) best_stages = 2;
  q.stages = best_stages;
  if (g_rq_stages > 0) q.stages = g_rq_stages;
  if (g_rq_blocks > 0) best_blocks = g_rq_blocks;
  const size_t smem = rq256_smem_bytes(p.K, threads, q.stages, chunked, adaln);
  if (smem > 227 * 1024) return CONVROT_ERR_SHAPE;
  int64_t grid = static_cast<int64_t>(st.sms) * best_blocks;
  if (grid > p.M) grid = p.M;
  kernel<<<static_cast<int>(grid), threads, smem, stream>>>(q);
  e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

// Row m of x is the concatenation of chunk j's row m over j (n_chunks chunks of K / n_chunks columns, rows ldx
// apart); one chunk is plain row-major x.  x_out (optional, chunked input only) receives each gathered row.
int rotate_quant(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding, int8_t* q, int64_t ldq,
                 float* s, cudaStream_t stream, const void* const* chunks = nullptr, int n_chunks = 1,
                 void* x_out = nullptr, int64_t ld_out = 0) {
  if (n_chunks < 1 || n_chunks > kMaxChunks || (n_chunks > 1 && !chunks)) return CONVROT_ERR_ARG;
  if (M < 0 || K <= 0) return CONVROT_ERR_SHAPE;
  const int64_t x_chunk = K / n_chunks;
  if (n_chunks > 1) {
    if (K % n_chunks || x_chunk % 128) return CONVROT_ERR_SHAPE;
    for (int j = 0; j < n_chunks; ++j) {
      if (!chunks[j]) return CONVROT_ERR_ARG;
      if (!aligned16(chunks[j])) return CONVROT_ERR_ALIGN;
    }
    x = chunks[0];
  } else if (x_out) {
    return CONVROT_ERR_ARG;  // a plain row-major x is already what x_out would hold
  }
  if (group != 4 && group != 16 && group != 64 && group != 256) return CONVROT_ERR_GROUP;
  if (rounding != CONVROT_ROUND_KERNEL && rounding != CONVROT_ROUND_TORCH && rounding != CONVROT_ROUND_TRITON)
    return CONVROT_ERR_ARG;
  if (K % group || K % 16 || K > 32768 || ldx < x_chunk || ldq < K || M > INT32_MAX) return CONVROT_ERR_SHAPE;
  if (x_out && ld_out < K) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  if (!x || !q || !s) return CONVROT_ERR_ARG;
  if (ldx % 8 || ldq % 16 || !aligned16(x) || !aligned16(q)) return CONVROT_ERR_ALIGN;
  if (x_out && (ld_out % 8 || !aligned16(x_out))) return CONVROT_ERR_ALIGN;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  RotQuantParams p;
  memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(x);
  for (int j = 0; j < n_chunks; ++j)
    p.xs[j] = static_cast<const __nv_bfloat16*>(n_chunks > 1 ? chunks[j] : x);
  p.ldx = ldx;
  p.x_chunk = static_cast<int>(x_chunk);
  p.x_out = static_cast<__nv_bfloat16*>(x_out);
  p.ld_out = ld_out;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.q = q;
  p.ldq = ldq;
  p.s = s;
  p.rounding = rounding;
  p.stages = kRQMaxStages;
  p.wait_limit_ns = g_wait_limit_ns;
  p.error_word = st->error_word;
  switch (group) {
    case 4: return launch_rq<4>(*st, p, stream);
    case 16: return launch_rq<16>(*st, p, stream);
    case 64: return launch_rq<64>(*st, p, stream);
    default: {
      // The two-column kernel up to K = 16384 (two groups per thread above K = 8192: at K = 13824 0.545 ms against
      // 0.568 ms for the one-column kernel, and 0.80 ms for one group per thread); the one-column kernel beyond.
      const bool two_col = g_rq_variant == 0 && (K / 256) * 8 <= 512;
      if (g_rq_variant == 2) return launch_rq256(*st, p, stream);
      return two_col ? launch_rq256(*st, p, stream) : launch_rq<256>(*st, p, stream);
    }
  }
}

// The AdaLN-modulated rotate+quantise: the rotated row is h = modulate(LayerNorm(x)) (RotQuantParams), and h is
// also stored to h_out when given.  The two-column kernel only (group 256, K <= 8192, plain rows).
int rotate_quant_adaln(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding, const void* scale,
                       const void* shift, const int32_t* index, int64_t ld_mod, float eps, int8_t* q, int64_t ldq,
                       float* s, void* h_out, int64_t ld_h, cudaStream_t stream) {
  if (group != 256) return CONVROT_ERR_GROUP;
  if (M < 0 || K <= 0 || K % 256 || K > 8192 || ldx < K || ldq < K || ld_mod < K || M > INT32_MAX)
    return CONVROT_ERR_SHAPE;
  if (rounding != CONVROT_ROUND_KERNEL && rounding != CONVROT_ROUND_TORCH && rounding != CONVROT_ROUND_TRITON)
    return CONVROT_ERR_ARG;
  if (!(eps >= 0.0f)) return CONVROT_ERR_ARG;
  if (h_out && ld_h < K) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  if (!x || !q || !s || !scale || !shift || !index) return CONVROT_ERR_ARG;
  if (ldx % 8 || ldq % 16 || ld_mod % 8 || !aligned16(x) || !aligned16(q) || !aligned16(scale) || !aligned16(shift))
    return CONVROT_ERR_ALIGN;
  if (h_out && (ld_h % 8 || !aligned16(h_out))) return CONVROT_ERR_ALIGN;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  RotQuantParams p;
  memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.xs[0] = p.x;
  p.ldx = ldx;
  p.x_chunk = static_cast<int>(K);
  p.x_out = static_cast<__nv_bfloat16*>(h_out);
  p.ld_out = ld_h;
  p.mod_scale = static_cast<const __nv_bfloat16*>(scale);
  p.mod_shift = static_cast<const __nv_bfloat16*>(shift);
  p.mod_index = index;
  p.ld_mod = ld_mod;
  p.norm_eps = eps;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.q = q;
  p.ldq = ldq;
  p.s = s;
  p.rounding = rounding;
  p.stages = kRQMaxStages;
  p.wait_limit_ns = g_wait_limit_ns;
  p.error_word = st->error_word;
  return launch_rq256(*st, p, stream);
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// Bytes convrot_linear needs for q (int8 [M, ldq]), s (fp32 [M]) and xa (bf16 [M, ldxa]), each 256-byte aligned.
size_t linear_workspace_need(int64_t M, int64_t K, int64_t r) {
  const int64_t ldxa = (r + 7) / 8 * 8;
  const int64_t ldq = (K + 15) / 16 * 16;
  return align256(static_cast<size_t>(M) * ldq) + align256(static_cast<size_t>(M) * 4) +
         align256(static_cast<size_t>(M) * ldxa * 2);
}

// Device address of the no-alloc scratch on the current device, looked up once per device (with that device
// current) and kept in the device state.  cudaGetSymbolAddress allocates nothing.
int noalloc_scratch(uint8_t** out) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!st->noalloc_scratch) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    if (!ptr || (reinterpret_cast<uintptr_t>(ptr) & 255u)) return CONVROT_ERR_CUDA;
    st->noalloc_scratch = static_cast<uint8_t*>(ptr);
  }
  *out = st->noalloc_scratch;
  return CONVROT_OK;
}

}  // namespace
}  // namespace convrot

using namespace convrot;

extern "C" {

int convrot_rotate_quant(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding, int8_t* q_out,
                         int64_t ldq, float* s_out, const void* lr_down, int64_t ld_down, int64_t r, void* xa_out,
                         int64_t ldxa, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = rotate_quant(x, ldx, M, K, group, rounding, q_out, ldq, s_out, s);
  if (rc || !lr_down) return rc;
  return lowrank_down(x, ldx, lr_down, ld_down, M, K, r, xa_out, ldxa, s);
}

int convrot_rotate_quant_packed(const void* x, int64_t chunk_cols, int64_t M, int64_t K, int group, int rounding,
                                int8_t* q_out, int64_t ldq, float* s_out, void* stream) {
  if (chunk_cols <= 0 || M < 0 || K % chunk_cols || K / chunk_cols > kMaxChunks) return CONVROT_ERR_SHAPE;
  if (!x) return CONVROT_ERR_ARG;
  const void* chunks[kMaxChunks];
  const int n = static_cast<int>(K / chunk_cols);
  for (int j = 0; j < n; ++j) chunks[j] = static_cast<const uint8_t*>(x) + j * M * chunk_cols * 2;
  return rotate_quant(x, chunk_cols, M, K, group, rounding, q_out, ldq, s_out, static_cast<cudaStream_t>(stream),
                      chunks, n);
}

int convrot_rotate_quant_adaln(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding,
                               const void* mod_scale, const void* mod_shift, const int32_t* mod_index, int64_t ld_mod,
                               float eps, int8_t* q_out, int64_t ldq, float* s_out, void* h_out, int64_t ld_h,
                               void* stream) {
  return rotate_quant_adaln(x, ldx, M, K, group, rounding, mod_scale, mod_shift, mod_index, ld_mod, eps, q_out, ldq,
                            s_out, h_out, ld_h, static_cast<cudaStream_t>(stream));
}

int convrot_rotate_quant_gather(const void* const* x_chunks, int n_chunks, int64_t ldx, int64_t M, int64_t K,
                                int group, int rounding, int8_t* q_out, int64_t ldq, float* s_out, void* x_out,
                                int64_t ld_out, void* stream) {
  if (n_chunks < 2) return CONVROT_ERR_ARG;
  return rotate_quant(nullptr, ldx, M, K, group, rounding, q_out, ldq, s_out, static_cast<cudaStream_t>(stream),
                      x_chunks, n_chunks, x_out, ld_out);
}

int convrot_lowrank_down_packed(const void* x, int64_t chunk_cols, const void* lr_down, int64_t ld_down, int64_t M,
                                int64_t K, int64_t r, void* xa_out, int64_t ldxa, void* stream) {
  if (chunk_cols <= 0 || M < 0) return CONVROT_ERR_SHAPE;
  return lowrank_down(x, chunk_cols, lr_down, ld_down, M, K, r, xa_out, ldxa, static_cast<cudaStream_t>(stream),
                      chunk_cols, M * chunk_cols);
}

int convrot_gemm_packed(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                        const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                        int64_t M, int64_t N, int64_t K, void* y, int64_t chunk_cols, void* stream) {
  if (chunk_cols <= 0 || M < 0 || N % chunk_cols || N / chunk_cols > kMaxChunks) return CONVROT_ERR_SHAPE;
  if (!y) return CONVROT_ERR_ARG;
  void* chunks[kMaxChunks];
  const int n = static_cast<int>(N / chunk_cols);
  for (int j = 0; j < n; ++j) chunks[j] = static_cast<uint8_t*>(y) + j * M * chunk_cols * 2;
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, xa, ldxa, lr_up, ld_up, r, M, N, K, y, chunk_cols, false,
                 static_cast<cudaStream_t>(stream), chunks, n);
}

int convrot_gemm_residual(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx,
                          const float* ws, const void* bias, const void* xa, int64_t ldxa, const void* lr_up,
                          int64_t ld_up, int64_t r, int64_t M, int64_t N, int64_t K, const void* res, int64_t ld_res,
                          const void* gate, int64_t ld_gate, const int32_t* gate_index, void* y, int64_t ldy,
                          void* stream) {
  const ResidualArgs args{res, ld_res, gate, ld_gate, gate_index};
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, xa, ldxa, lr_up, ld_up, r, M, N, K, y, ldy, false,
                 static_cast<cudaStream_t>(stream), nullptr, 1, false, &args);
}

int convrot_gemm_swiglu(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                        const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                        int64_t M, int64_t N, int64_t K, void* h, int64_t ldh, void* stream) {
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, xa, ldxa, lr_up, ld_up, r, M, N, K, h, ldh, false,
                 static_cast<cudaStream_t>(stream), nullptr, 1, true);
}

int convrot_gemm_grouped(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                         const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                         int64_t M, int64_t N, int64_t K, int segments, void* const* y_chunks, int64_t ldy,
                         void* stream) {
  if (segments < 2 || segments > kMaxChunks || !y_chunks) return CONVROT_ERR_ARG;
  if (r > 0 && (!xa || !lr_up)) return CONVROT_ERR_ARG;
  // without a low-rank term the segments need no xa offsets: the chunked output alone separates the layers
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, r > 0 ? xa : nullptr, ldxa, r > 0 ? lr_up : nullptr, ld_up, r, M, N, K,
                 nullptr, ldy, false, static_cast<cudaStream_t>(stream), y_chunks, segments, false, nullptr,
                 r > 0 ? segments : 1);
}

int convrot_silu(const void* x, void* y, int64_t n, void* stream) {
  if (n < 0) return CONVROT_ERR_SHAPE;
  if (n == 0) return CONVROT_OK;
  if (!x || !y) return CONVROT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 1) return CONVROT_ERR_ALIGN;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4 * static_cast<int64_t>(st->sms)) blocks = 4 * static_cast<int64_t>(st->sms);
  silu_bf16_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

int convrot_gemm_scatter(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                         const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                         int64_t M, int64_t N, int64_t K, void* const* y_chunks, int n_chunks, int64_t ldy,
                         void* stream) {
  if (n_chunks < 2) return CONVROT_ERR_ARG;
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, xa, ldxa, lr_up, ld_up, r, M, N, K, nullptr, ldy, false,
                 static_cast<cudaStream_t>(stream), y_chunks, n_chunks);
}

int convrot_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return CONVROT_ERR_ARG;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = g_address_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return CONVROT_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e);
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return CONVROT_OK;
}

int convrot_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return CONVROT_ERR_ARG;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

int convrot_ipc_close(void* base) {
  if (!base) return CONVROT_ERR_ARG;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

int convrot_peer_signal(uint32_t* const* slots, int n, uint32_t epoch, void* stream) {
  if (n < 1 || n > kMaxChunks || !slots) return CONVROT_ERR_ARG;
  PeerSlots ps;
  memset(&ps, 0, sizeof(ps));
  for (int j = 0; j < n; ++j) {
    if (!slots[j] || (reinterpret_cast<uintptr_t>(slots[j]) & 3u)) return CONVROT_ERR_ARG;
    ps.slot[j] = slots[j];
  }
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  peer_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(ps, n, epoch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

int convrot_peer_wait(const uint32_t* flags, int n, uint32_t epoch, void* stream) {
  if (n < 1 || n > kMaxChunks || !flags || (reinterpret_cast<uintptr_t>(flags) & 3u)) return CONVROT_ERR_ARG;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, n, epoch, g_wait_limit_ns,
                                                                   st->error_word);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CONVROT_OK : cuda_fail(e);
}

int convrot_copy_blocks(void* const* dst, const void* const* src, const size_t* bytes, int n, void* stream) {
  if (n < 0 || n > 64 || (n > 0 && (!dst || !src || !bytes))) return CONVROT_ERR_ARG;
  for (int j = 0; j < n; ++j)
    if ((!dst[j] || !src[j]) && bytes[j]) return CONVROT_ERR_ARG;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  // One plain cudaMemcpyAsync per block (copy engines; no batched-copy API).
  for (int j = 0; j < n; ++j) {
    if (!bytes[j]) continue;
    const cudaError_t e = cudaMemcpyAsync(dst[j], src[j], bytes[j], cudaMemcpyDeviceToDevice,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return CONVROT_OK;
}

int convrot_lowrank_down(const void* x, int64_t ldx, const void* lr_down, int64_t ld_down, int64_t M, int64_t K,
                         int64_t r, void* xa_out, int64_t ldxa, void* stream) {
  return lowrank_down(x, ldx, lr_down, ld_down, M, K, r, xa_out, ldxa, static_cast<cudaStream_t>(stream));
}

int convrot_gemm(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                 const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                 int64_t M, int64_t N, int64_t K, void* y, int64_t ldy, void* stream) {
  return gemm_i8(q, ldq, w, ldw, sx, ws, bias, xa, ldxa, lr_up, ld_up, r, M, N, K, y, ldy, false,
                 static_cast<cudaStream_t>(stream));
}

int convrot_gemm_acc(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                     int32_t* acc, int64_t ldc, void* stream) {
  return gemm_i8(q, ldq, w, ldw, nullptr, nullptr, nullptr, nullptr, 0, nullptr, 0, 0, M, N, K, acc, ldc, true,
                 static_cast<cudaStream_t>(stream));
}

size_t convrot_workspace_size(int64_t M, int64_t K, int64_t r) {
  if (M < 0 || K < 0 || r < 0) return 0;
  // exactly what convrot_linear checks: q rows padded to 16 bytes, xa rows to 8 elements (16 bytes)
  return linear_workspace_need(M, K, r);
}

int convrot_linear(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* ws, const void* bias,
                   const void* lr_down, int64_t ld_down, const void* lr_up, int64_t ld_up, int64_t r, int64_t M,
                   int64_t N, int64_t K, int group, void* workspace, size_t workspace_bytes, void* y, int64_t ldy,
                   void* stream) {
  if (M < 0 || K <= 0 || r < 0) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  const bool has_lr = lr_down && lr_up && r > 0;
  if ((lr_down || lr_up) && !has_lr) return CONVROT_ERR_ARG;
  const int64_t rr = has_lr ? r : 0;
  const int64_t ldxa = (rr + 7) / 8 * 8;
  const int64_t ldq = (K + 15) / 16 * 16;
  const size_t need = linear_workspace_need(M, K, rr);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return CONVROT_ERR_ARG;
  uint8_t* ws_bytes = static_cast<uint8_t*>(workspace);
  int8_t* q = reinterpret_cast<int8_t*>(ws_bytes);
  float* sx = reinterpret_cast<float*>(ws_bytes + align256(static_cast<size_t>(M) * ldq));
  void* xa = ws_bytes + align256(static_cast<size_t>(M) * ldq) + align256(static_cast<size_t>(M) * 4);
  int rc = convrot_rotate_quant(x, ldx, M, K, group, CONVROT_ROUND_KERNEL, q, ldq, sx, has_lr ? lr_down : nullptr,
                                ld_down, rr, xa, ldxa, stream);
  if (rc) return rc;
  return convrot_gemm(q, ldq, w, ldw, sx, ws, bias, has_lr ? xa : nullptr, ldxa, has_lr ? lr_up : nullptr, ld_up, rr,
                      M, N, K, y, ldy, stream);
}

int convrot_linear_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* ws,
                           const void* bias, const void* lr_down, int64_t ld_down, const void* lr_up, int64_t ld_up,
                           int64_t r, int64_t M, int64_t N, int64_t K, int group, void* y, int64_t ldy,
                           void* stream) {
  if (M < 0 || K <= 0 || r < 0) return CONVROT_ERR_SHAPE;
  if (M == 0) return CONVROT_OK;
  const bool has_lr = lr_down && lr_up && r > 0;
  if (linear_workspace_need(M, K, has_lr ? r : 0) > CONVROT_NOALLOC_SCRATCH_BYTES) return CONVROT_ERR_SCRATCH;
  uint8_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // The same two launches as convrot_linear, with the built-in scratch as the workspace.  Both kernels write their
  // part of the scratch completely before anything reads it, so no part needs clearing between calls.
  return convrot_linear(x, ldx, w, ldw, ws, bias, lr_down, ld_down, lr_up, ld_up, r, M, N, K, group, scratch,
                        CONVROT_NOALLOC_SCRATCH_BYTES, y, ldy, stream);
}

const char* convrot_status_string(int status) {
  switch (status) {
    case CONVROT_OK: return "ok";
    case CONVROT_ERR_SHAPE: return "unsupported or inconsistent shape";
    case CONVROT_ERR_GROUP: return "unsupported Hadamard group (4, 16, 64 or 256)";
    case CONVROT_ERR_ALIGN: return "pointer or leading dimension breaks the 16-byte alignment rules";
    case CONVROT_ERR_CUDA: return "CUDA call failed";
    case CONVROT_ERR_ARCH: return "device is not sm_100 (B200)";
    case CONVROT_ERR_TIMEOUT: return "a kernel's bounded wait expired";
    case CONVROT_ERR_ARG: return "missing pointer or unknown option";
    case CONVROT_ERR_SCRATCH: return "problem needs more than the built-in scratch of convrot_linear_noalloc";
    default: return "unknown status";
  }
}

int convrot_last_cuda_error(void) { return t_last_cuda_error; }

int convrot_poll_error(void* stream) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int word = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&word, g_error_word, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e);
  if (word) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_error_word, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return word;
}

void convrot_set_wait_limit_ns(uint64_t ns) { g_wait_limit_ns = ns ? ns : 2000000000ull; }

int convrot_set_rotate_tuning(int stages, int ctas_per_sm) {
  if (stages < 0 || stages > kRQMaxStages || ctas_per_sm < 0 || ctas_per_sm > 32) return CONVROT_ERR_ARG;
  g_rq_stages = stages;
  g_rq_blocks = ctas_per_sm;
  return CONVROT_OK;
}

int convrot_set_rotate_variant(int variant) {
  if (variant < 0 || variant > 2) return CONVROT_ERR_ARG;
  g_rq_variant = variant;
  return CONVROT_OK;
}

int convrot_set_gemm_mode(int mode) {
  if (mode < 0 || mode > 2) return CONVROT_ERR_ARG;
  g_gemm_mode = mode;
  return CONVROT_OK;
}

int convrot_version(void) { return 100; }

int64_t convrot_split_k_fallbacks(void) { return g_split_fallbacks.load(std::memory_order_relaxed); }

}  // extern "C"
