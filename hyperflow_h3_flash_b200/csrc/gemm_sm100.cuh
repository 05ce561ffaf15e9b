// Persistent warp-specialised tcgen05 GEMM for sm_100a, with the convrot epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T, both operands K-major (row-major with K contiguous), staged by TMA in 128-byte
//   SWIZZLE_128B rows, accumulated in TMEM (two accumulator buffers so the epilogue of one tile overlaps the
//   main loop of the next).
//
//   KIND_I8  : int8 x int8 -> int32 (tcgen05.mma kind::i8, K = 32 per instruction, 128 K per stage)
//   KIND_BF16: bf16 x bf16 -> fp32  (tcgen05.mma kind::f16, K = 16 per instruction, 64 K per stage)
//
// Warp roles (one CTA per SM, CTAs stride over output tiles in row-major tile order):
//   warp 0      TMA producer of the A/B ring
//   warp 1      TMEM allocator; lane 0 issues every MMA and commit
//   warps 2..5  epilogue: TMEM -> registers -> global, one 32-lane TMEM quadrant each
//   warp 6      (low-rank only) TMA producer of the low-rank operand tiles
//
// Epilogues:
//   EPI_DEQUANT   y = bf16((float(acc) * sa[m]) * sb[n] [+ bias[n]] [+ xa[m,:] . up[n,:]])   (int8.py:311, 324)
//                 The low-rank term is a second, kind::f16 MMA (A = xa tile, B = up tile) that accumulates onto
//                 the dequantised fp32 values the epilogue writes back into the same TMEM buffer.
//   EPI_RAW_I32   acc as int32 (accumulator parity tests)
//   EPI_BF16      y = bf16(acc_f32) (the low-rank down projection x . down^T)
//
// Every wait is bounded by a %globaltimer deadline; on expiry the CTA records CONVROT_ERR_TIMEOUT in a device
// error word, drains its own TMA loads and MMAs (again bounded), frees its TMEM and returns.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace convrot {

enum { KIND_I8 = 0, KIND_BF16 = 1 };
enum { EPI_DEQUANT = 0, EPI_RAW_I32 = 1, EPI_BF16 = 2 };

// Operand / output layout "chunked rows": element (m, k) at base + (k / W) * S + m * L + k % W.  Plain row-major
// storage is the one-chunk case W = K (L = leading dimension); the Ulysses all-to-all buffers are W = K / P,
// L = W, S = M * W (all tokens of head block j, then block j + 1, ...).
struct GemmParams {
  int M, N, K;
  const float* sa;      // [M]   (EPI_DEQUANT)
  const float* sb;      // [N]   (EPI_DEQUANT)
  const __nv_bfloat16* bias;  // [N] or null
  void* out;            // bf16 [M, N] or int32 [M, N] (plain rows)
  void* out_chunks[kMaxChunks];  // bf16 output in column chunks of out_chunk: chunk j is [M, ldo] rows at [j]
  int64_t ldo;          // elements (row pitch of the output, or of each chunk)
  int out_chunk;        // columns per chunk (N for plain rows, out_chunks[0] == out)
  int swiglu;           // 1: the B rows are a SwiGLU projection interleaved in 32-row blocks (a0 g0 a1 g1 ...);
                        //    the bf16 output is h = a * silu(g), [M, N / 2]
  // Gated residual (res != null): out = bf16(res + bf16(gate[idx] * bf16(y))), idx = gate_index[row] (0 without an
  // index), and out = bf16(res + bf16(y)) without a gate.
  const __nv_bfloat16* res;
  int64_t ld_res;
  const __nv_bfloat16* gate;
  int64_t ld_gate;
  const int32_t* gate_index;
  int a_chunk;          // W of operand A along K (K for plain rows); its TMA map is 3-D (W, M, K / W)
  int r;                // low-rank width (0 = none)
  int lr_seg_n;         // > 0: output columns [s lr_seg_n, (s + 1) lr_seg_n) read xa columns [s r, (s + 1) r)
  int split_k;          // > 1 (the bf16 down projection only): clusters of split_k CTAs split K, one tile each
  int wide_store;       // 2-SM epilogue: 1 = stores leave as 32 x 64 boxes (128-byte rows), 0 = 32 x 32 boxes
  int group_m;          // tile order: M blocks per group (0: kGroupM)
  uint64_t wait_limit_ns;
  int* error_word;
};

// Pointer to output column n (a multiple of 32 inside one chunk) of row `row`.
template <class T>
__device__ __forceinline__ T* out_ptr(const GemmParams& p, int row, int n) {
  const int j = n / p.out_chunk;
  return reinterpret_cast<T*>(select_chunk(p.out_chunks, j)) + static_cast<int64_t>(row) * p.ldo +
         (n - j * p.out_chunk);
}

constexpr int kBM = 128;

// Tile order of the persistent GEMMs: groups of kGroupM M blocks, and inside a group the M block varies fastest, then
// the N block.  The tiles in flight at once (one per CTA or CTA pair) then cover a few M blocks times a few N blocks,
// so the A rows and B rows they read stay in L2 even when B (the weights: 141 MB for a 5120 -> 27648 projection) is
// larger than L2.  In plain row-major order every M block would stream all of B from HBM again.  kGroupM is the
// default; a launch sets GemmParams::group_m by the size of B (4, 8 or 16 M blocks per group).
constexpr int kGroupM = 8;

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb, int& nb) {
  const int gm = group_m > 0 ? group_m : kGroupM;
  const int group_tiles = gm * num_n;
  const int g = tile / group_tiles;
  const int first = g * gm;
  const int rows = num_m - first < gm ? num_m - first : gm;
  const int in = tile - g * group_tiles;
  mb = first + in % rows;
  nb = in / rows;
}
constexpr int kRowBytes = 128;  // bytes of K per stage row (one SWIZZLE_128B atom)

__host__ __device__ constexpr int tmem_cols_for(int bn) {
  return (2 * bn) <= 32 ? 32 : (2 * bn) <= 64 ? 64 : (2 * bn) <= 128 ? 128 : (2 * bn) <= 256 ? 256 : 512;
}

// LR_ATOM: bytes of K per low-rank operand row atom (64 -> SWIZZLE_64B, 128 -> SWIZZLE_128B); LR_ATOMS atoms.
template <int KIND, int BN, int STAGES, int EPI, int LR_ATOM, int LR_ATOMS>
struct GemmCfg {
  static constexpr int kBN = BN;
  static constexpr int kStages = STAGES;
  static constexpr bool kHasLR = (LR_ATOMS > 0);
  static constexpr int kABytes = kBM * kRowBytes;
  static constexpr int kBBytes = BN * kRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kLRXaBytes = kHasLR ? kBM * LR_ATOM * LR_ATOMS : 0;
  // The low-rank term runs per half of the tile's columns: one half's up rows at a time.
  static constexpr int kLRUpRows = BN / 2;
  static constexpr int kLRUpBytes = kHasLR ? kLRUpRows * LR_ATOM * LR_ATOMS : 0;
  static constexpr int kMmaPerStage = 4;  // 32 bytes of K per MMA
  static constexpr int kTmemCols = tmem_cols_for(BN);
  static constexpr int kThreads = kHasLR ? 224 : 192;
  // barriers: full[S], empty[S], tmem_full[2], tmem_empty[2], epi_ready[2 x 2], lr_done[2 x 2], lr_full, lr_empty,
  // drain, lr_drain (epi_ready and lr_done per accumulator buffer and half of the columns)
  static constexpr int kNumBars = 2 * STAGES + 12 + 4;
  static constexpr int kBarBytes = ((kNumBars * 8 + 16 + 127) / 128) * 128;
  static constexpr int kSmemBytes = 1024 /*alignment slack*/ + STAGES * kStageBytes + kLRXaBytes + kLRUpBytes +
                                    kBarBytes;
  static constexpr uint32_t kIdesc = KIND == KIND_I8 ? make_idesc_i8(kBM, BN) : make_idesc_bf16(kBM, BN);
  static constexpr uint32_t kIdescLR = make_idesc_bf16(kBM, BN / 2);  // one half of the columns per low-rank MMA
};

__device__ __forceinline__ void record_error(int* word, int code) {
  if (word) atomicCAS(word, 0, code);
}

// Dequantise 32 accumulator columns [n, n + 32) of one row: t = fp32(fp32(float(acc) * sa) * sb[n]) [+ bias[n]],
// each product rounded to fp32 without FMA contraction (int8.py:311, 324).  Columns at or beyond N give 0.
__device__ __forceinline__ void dequant_chunk(const uint32_t (&v)[32], float sa, const float* __restrict__ sbv,
                                              const __nv_bfloat16* __restrict__ biasv, int n, int N, float (&t)[32]) {
  float sb[32], bias[32];
  if (n + 32 <= N) {
    const float4* s4 = reinterpret_cast<const float4*>(sbv + n);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 f = __ldg(s4 + j);
      sb[4 * j] = f.x;
      sb[4 * j + 1] = f.y;
      sb[4 * j + 2] = f.z;
      sb[4 * j + 3] = f.w;
    }
    if (biasv) {
      const uint4* b4 = reinterpret_cast<const uint4*>(biasv + n);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = __ldg(b4 + j);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          bias[8 * j + 2 * h] = __uint_as_float(w[h] << 16);
          bias[8 * j + 2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const bool in = n + j < N;
      sb[j] = in ? __ldg(sbv + n + j) : 0.0f;
      bias[j] = (in && biasv) ? __bfloat162float(biasv[n + j]) : 0.0f;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float x = __fmul_rn(__int2float_rn(static_cast<int>(v[j])), sa);
    x = __fmul_rn(x, sb[j]);
    if (biasv) x = __fadd_rn(x, bias[j]);
    t[j] = x;
  }
}

// Round 32 fp32 values to bf16 (nearest even) and store them at dst[0..32) (columns n.. of a row, N columns).
__device__ __forceinline__ void store_bf16_chunk(__nv_bfloat16* dst, const float (&t)[32], int n, int N) {
  if (n + 32 <= N) {
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * j], t[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n + j < N) dst[j] = __float2bfloat16_rn(t[j]);
  }
}

// The gated residual on 32 output columns [n, n + 32) of one row (row < M): t holds the linear's fp32 values and
// becomes bf16(res + bf16(gate * bf16(t))) -- the bf16 tensor ops `res + gate * linear(x)` -- columns at or beyond
// N give 0 (they are not stored).
__device__ __forceinline__ void gated_residual(float (&t)[32], const GemmParams& p, int row, int n) {
  const __nv_bfloat16* rrow = p.res + static_cast<int64_t>(row) * p.ld_res + n;
  const __nv_bfloat16* grow = nullptr;
  if (p.gate) grow = p.gate + static_cast<int64_t>(p.gate_index ? __ldg(p.gate_index + row) : 0) * p.ld_gate + n;
  uint32_t r[16], g[16];
  if (n + 32 <= p.N) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(rrow) + j);
      r[4 * j] = u.x;
      r[4 * j + 1] = u.y;
      r[4 * j + 2] = u.z;
      r[4 * j + 3] = u.w;
      if (grow) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(grow) + j);
        g[4 * j] = v.x;
        g[4 * j + 1] = v.y;
        g[4 * j + 2] = v.z;
        g[4 * j + 3] = v.w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const bool in0 = n + 2 * j < p.N, in1 = n + 2 * j + 1 < p.N;
      const uint32_t r0 = in0 ? __bfloat16_as_ushort(rrow[2 * j]) : 0u;
      const uint32_t r1 = in1 ? __bfloat16_as_ushort(rrow[2 * j + 1]) : 0u;
      r[j] = r0 | (r1 << 16);
      if (grow) {
        const uint32_t g0 = in0 ? __bfloat16_as_ushort(grow[2 * j]) : 0u;
        const uint32_t g1 = in1 ? __bfloat16_as_ushort(grow[2 * j + 1]) : 0u;
        g[j] = g0 | (g1 << 16);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int sh = (j & 1) ? 0 : 16;
    const float rj = __uint_as_float((r[j >> 1] << sh) & 0xffff0000u);
    float v = __bfloat162float(__float2bfloat16_rn(t[j]));
    if (grow) v = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__uint_as_float((g[j >> 1] << sh) & 0xffff0000u), v)));
    t[j] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(rj, v)));
  }
}

// silu on a bf16 input g: bf16(g / (1 + expf(-g))), the bits torch's F.silu gives a bf16 tensor (fp32 arithmetic,
// IEEE division).  It depends on the 16 bits of g alone, so a table of it is exact: the 2-SM epilogue reads it from
// shared memory for the magnitudes [2^-19, 32) of both signs (24 binades of 128 mantissas, filled once per CTA by
// this same function) and evaluates the function itself for every other input (zeros, tiny or large magnitudes,
// inf, NaN).
constexpr uint32_t kSiluExpLo = 108;                    // bf16 exponent field of 2^-19
constexpr uint32_t kSiluPerSign = 24 * 128;             // table entries per sign
constexpr int kSiluTableBytes = 2 * kSiluPerSign * 2;   // 12 KB

__device__ __forceinline__ float silu_bf16(float g) {  // g holds a bf16 value
  return __bfloat162float(__float2bfloat16_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g)))));
}

// Entries [first, 2 * kSiluPerSign) in steps of `step`: positive magnitudes first, then negative.
__device__ __forceinline__ void silu_table_fill(uint16_t* tab, int first, int step) {
  for (int i = first; i < static_cast<int>(2 * kSiluPerSign); i += step) {
    const uint32_t sign = i >= static_cast<int>(kSiluPerSign) ? 0x8000u : 0u;
    const uint32_t bits = sign | ((static_cast<uint32_t>(i) % kSiluPerSign) + (kSiluExpLo << 7));
    tab[i] = static_cast<uint16_t>(__float_as_uint(silu_bf16(__uint_as_float(bits << 16))) >> 16);
  }
}

// silu_bf16 of the bf16 value with bits b (< 2^16), from the table; sets `miss` when b lies outside it.
__device__ __forceinline__ float silu_lookup(const uint16_t* tab, uint32_t b, bool& miss) {
  const uint32_t off = (b & 0x7fffu) - (kSiluExpLo << 7);
  const bool in = off < kSiluPerSign;
  miss = miss || !in;
  return __uint_as_float(static_cast<uint32_t>(tab[in ? off + (b >> 15) * kSiluPerSign : 0u]) << 16);
}

// SwiGLU over the interleaved projection, one 32-column block at a time (c = the block's first column in the tile):
// an `a` block (c / 32 even) is kept as bf16 in ya; on the `g` block that follows, t becomes the pair's 32 outputs
//   h = bf16( float(bf16(a)) * silu_bf16(float(bf16(t))) ),
// the bf16 composition that `a * silu(g)` evaluates on the bf16 outputs of the projection (the product of two bf16
// values is exact in fp32, so the caller's bf16 store rounds it once).  `tab` is the silu table in shared memory,
// or null to evaluate silu_bf16 directly.  Returns whether t holds outputs to store.
__device__ __forceinline__ bool swiglu_block(float (&t)[32], int c, uint32_t (&ya)[16], const uint16_t* tab) {
  if (((c >> 5) & 1) == 0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * j], t[2 * j + 1]);
      ya[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    return false;
  }
  float sg[32];
  bool miss = tab == nullptr;
  if (tab) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * j], t[2 * j + 1]);
      const uint32_t gb = *reinterpret_cast<uint32_t*>(&h);
      sg[2 * j] = silu_lookup(tab, gb & 0xffffu, miss);
      sg[2 * j + 1] = silu_lookup(tab, gb >> 16, miss);
    }
  }
  if (miss) {  // no table, or an input outside it: the function itself for the whole block
#pragma unroll
    for (int j = 0; j < 32; ++j) sg[j] = silu_bf16(__bfloat162float(__float2bfloat16_rn(t[j])));
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float a = __uint_as_float((j & 1) ? (ya[j >> 1] & 0xffff0000u) : (ya[j >> 1] << 16));
    t[j] = __fmul_rn(a, sg[j]);
  }
  return true;
}

// The epilogue's silu alone, elementwise over n bf16 values (convrot_silu): the same table and the same fallback.
__global__ void __launch_bounds__(256) silu_bf16_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n) {
  __shared__ uint16_t tab[2 * kSiluPerSign];
  silu_table_fill(tab, threadIdx.x, blockDim.x);
  __syncthreads();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t b = __bfloat16_as_ushort(x[i]);
    bool miss = false;
    float v = silu_lookup(tab, b, miss);
    if (miss) v = silu_bf16(__uint_as_float(b << 16));
    y[i] = __float2bfloat16_rn(v);
  }
}

template <class Cfg, int KIND, int EPI, int LR_ATOM, int LR_ATOMS>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    convrot_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_xa, const __grid_constant__ CUtensorMap tmap_up,
                        const GemmParams p) {
  constexpr int BN = Cfg::kBN;
  constexpr int S = Cfg::kStages;
  constexpr bool HAS_LR = Cfg::kHasLR;
  extern __shared__ __align__(1024) uint8_t gemm_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* lr_xa = ring + S * Cfg::kStageBytes;
  uint8_t* lr_up = lr_xa + Cfg::kLRXaBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(lr_up + Cfg::kLRUpBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tmem_full = bars + 2 * S;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* epi_ready = tmem_full + 4;  // [buf * 2 + half]
  uint64_t* lr_done = tmem_full + 8;    // [buf * 2 + half]
  uint64_t* lr_full = tmem_full + 12;
  uint64_t* lr_empty = tmem_full + 13;
  uint64_t* drain = tmem_full + 14;
  uint64_t* lr_drain = tmem_full + 15;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // The low-rank term streams through its operand buffers in rank chunks of LR_ATOMS * LR_ATOM / 2 columns.
  const int lr_chunks = HAS_LR ? (p.r + LR_ATOMS * (LR_ATOM / 2) - 1) / (LR_ATOMS * (LR_ATOM / 2)) : 0;
  const int nkb = (p.K * (KIND == KIND_I8 ? 1 : 2) + kRowBytes - 1) / kRowBytes;
  constexpr int kKPerStage = KIND == KIND_I8 ? 128 : 64;  // elements
  // Split K (EPI_BF16, few row tiles): the launch is clusters of ksplit CTAs with one tile per cluster; CTA s of a
  // cluster accumulates the K stages [s nkb / ksplit, (s + 1) nkb / ksplit), and the cluster sums the partial tiles
  // through distributed shared memory at the end of the kernel, in the order s = 0, 1, ... for every element.
  const int ksplit = EPI == EPI_BF16 && p.split_k > 1 ? p.split_k : 1;
  const int krank = ksplit > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int kb_begin = krank * nkb / ksplit, kb_end = (krank + 1) * nkb / ksplit;
  const int tile0 = static_cast<int>(blockIdx.x) / ksplit, tile_step = static_cast<int>(gridDim.x) / ksplit;
  constexpr int kPartStride = BN + 4;  // floats per row of a partial tile (16-byte pad: conflict-free rows)
  static_assert(KIND != KIND_BF16 || kBM * kPartStride * 4 <= S * Cfg::kStageBytes, "partial tile beyond the ring");

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 4);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&epi_ready[b], 4);
      mbar_init(&lr_done[b], 1);
    }
    mbar_init(lr_full, 1);
    mbar_init(lr_empty, 1);
    mbar_init(drain, 1);
    mbar_init(lr_drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (HAS_LR) {
      tma_prefetch_desc(&tmap_xa);
      tma_prefetch_desc(&tmap_up);
    }
  }
  if (warp == 1) {
    tmem_alloc<Cfg::kTmemCols>(tmem_holder);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;
  auto fail = [&]() {
    *abort_flag = 1;
    record_error(p.error_word, 6 /* CONVROT_ERR_TIMEOUT */);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (A/B ring)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;  // last load per stage, for draining after an abort
      bool ok = true;
      for (int tile = tile0; ok && tile < num_tiles; tile += tile_step) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
        const int m0 = mb * kBM;
        const int n0 = nb * BN;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, limit, abort_flag)) {
            fail();
            ok = false;
            break;
          }
          uint8_t* sa_ptr = ring + stage * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          {
            const int ka = kb * kKPerStage;  // A is a 3-D map (W, M, K / W): one chunk holds whole stage boxes
            const int ja = ka / p.a_chunk;
            tma_load_3d(sa_ptr, &tmap_a, &full[stage], ka - ja * p.a_chunk, m0, ja);
          }
          tma_load_2d(sa_ptr + Cfg::kABytes, &tmap_b, &full[stage], kb * kKPerStage, n0);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let every load this thread issued land before the CTA leaves
        volatile int never = 0;
        for (int s = 0; s < S; ++s)
          if (issued_mask >> s & 1) mbar_wait_bounded(&full[s], issued_parity >> s & 1, limit, &never);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      const uint32_t ring_base = smem_u32(ring);
      int i = 0;
      for (int tile = tile0; ok && tile < num_tiles; tile += tile_step, ++i) {
        const uint32_t buf = i & 1;
        if (!mbar_wait_bounded(&tmem_empty[buf], ((i >> 1) & 1) ^ 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, limit, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = ring_base + stage * Cfg::kStageBytes;
          const uint32_t b_addr = a_addr + Cfg::kABytes;
          const uint64_t ad = make_kmajor_desc(a_addr, kRowBytes);
          const uint64_t bd = make_kmajor_desc(b_addr, kRowBytes);
#pragma unroll
          for (int kk = 0; kk < Cfg::kMmaPerStage; ++kk) {
            // +32 bytes of K inside the 128-byte swizzle atom: +2 in the (addr >> 4) field
            if (KIND == KIND_I8)
              mma_i8(d, ad + 2 * kk, bd + 2 * kk, Cfg::kIdesc, kb != kb_begin || kk != 0);
            else
              mma_f16(d, ad + 2 * kk, bd + 2 * kk, Cfg::kIdesc, kb != kb_begin || kk != 0);
          }
          mma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tmem_full[buf]);
      }
      if (!ok) fail();
      // Make sure no MMA is still reading shared memory or writing TMEM when the CTA winds down.
      mma_commit(drain);
      volatile int never = 0;
      mbar_wait_bounded(drain, 0, limit, &never);
    }
  } else if (HAS_LR && warp == 6) {
    // ---------------------------------------------------------------- low-rank term: operand loads and MMAs
    // Issued from this warp so that the main loop's issuer never waits or polls for them (each thread's
    // tcgen05.commit tracks its own MMAs, and the two streams write different accumulator buffers).  Unit u =
    // (local tile i, half h of the columns, rank chunk c).
    if (lane == 0) {
      int u = 0;
      bool ok = true;
      const uint32_t xa_base = smem_u32(lr_xa);
      const uint32_t up_base = smem_u32(lr_up);
      int i = 0;
      for (int tile = tile0; ok && tile < num_tiles; tile += tile_step, ++i) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
        const int m0 = mb * kBM;
        const int xs = p.lr_seg_n ? (nb * BN / p.lr_seg_n) * p.r : 0;  // this tile's segment of xa
        for (int h = 0; ok && h < 2; ++h) {
          const int n0 = nb * BN + h * Cfg::kLRUpRows;
          for (int c = 0; c < lr_chunks; ++c, ++u) {
            // unit u reuses the operand buffers once the MMAs of unit u-1 (phase u-1 of lr_empty) are done
            if (!mbar_wait_bounded(lr_empty, (u & 1) ^ 1, limit, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(lr_full, Cfg::kLRXaBytes + Cfg::kLRUpBytes);
            for (int a = 0; a < LR_ATOMS; ++a) {
              const int x = (c * LR_ATOMS + a) * (LR_ATOM / 2);
              tma_load_2d(lr_xa + a * kBM * LR_ATOM, &tmap_xa, lr_full, x + xs, m0);
              tma_load_2d(lr_up + a * Cfg::kLRUpRows * LR_ATOM, &tmap_up, lr_full, x, n0);
            }
            // the operands have landed, and (first chunk) the epilogue has read the half's accumulator
            if (!mbar_wait_bounded(lr_full, u & 1, limit, abort_flag) ||
                (c == 0 && !mbar_wait_bounded(&epi_ready[(i & 1) * 2 + h], (i >> 1) & 1, limit, abort_flag))) {
              ok = false;
              break;
            }
            tc_fence_after();
            // The half's first MMA overwrites its accumulator columns (the epilogue holds the dequantised values in
            // registers); the half's last chunk tells the epilogue.
            const uint32_t d = tmem_base + (i & 1) * BN + h * Cfg::kLRUpRows;
            for (int a = 0; a < LR_ATOMS; ++a) {
              for (int off = 0; off < LR_ATOM; off += 32) {
                const uint64_t ad = make_kmajor_desc(xa_base + a * kBM * LR_ATOM + off, LR_ATOM);
                const uint64_t bd = make_kmajor_desc(up_base + a * Cfg::kLRUpRows * LR_ATOM + off, LR_ATOM);
                mma_f16(d, ad, bd, Cfg::kIdescLR, (c | a | off) != 0);
              }
            }
            if (c + 1 == lr_chunks) mma_commit(&lr_done[(i & 1) * 2 + h]);
            mma_commit(lr_empty);
          }
        }
      }
      if (!ok) {
        fail();
        // a load still in flight lands before the CTA leaves (bounded)
        volatile int never = 0;
        if (u > 0) mbar_wait_bounded(lr_full, (u - 1) & 1, limit, &never);
      }
      mma_commit(lr_drain);  // this thread's MMAs are done before the CTA may free its TMEM
      volatile int never = 0;
      mbar_wait_bounded(lr_drain, 0, limit, &never);
    }
  } else if (warp >= 2 && warp <= 5) {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    int i = 0;
    for (int tile = tile0; tile < num_tiles; tile += tile_step, ++i) {
      const uint32_t buf = i & 1;
      const uint32_t par = (i >> 1) & 1;
      int mb, nb;
      tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
      const int m0 = mb * kBM;
      const int n0 = nb * BN;
      if (!mbar_wait_bounded(&tmem_full[buf], par, limit, abort_flag)) {
        fail();
        break;
      }
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN;

      if (EPI == EPI_DEQUANT && HAS_LR) {
        // Per half of the columns: read the int32 accumulators and hold the dequantised values (+ bias) in
        // registers, tell the low-rank warp that the half's columns are free, and wait while its MMA writes
        // xa . up^T over them (accumulate = 0); then y = held + product, rounded once to bf16 on the way out.
        const float sa = row_ok ? __ldg(p.sa + row) : 0.0f;
        const int n_out = p.swiglu ? p.N >> 1 : p.N;
        uint32_t ya[16];  // SwiGLU: the bf16 `a` block awaiting its `g` block
        bool lr_ok = true;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          float hold[BN / 2];
#pragma unroll
          for (int cc = 0; cc < BN / 64; ++cc) {
            const int c = h * (BN / 2) + cc * 32;
            uint32_t v[32];
            tmem_ld_32x32b_x32(taddr + c, v);
            tmem_ld_wait();
            float t[32];
            dequant_chunk(v, sa, p.sb, p.bias, n0 + c, p.N, t);
#pragma unroll
            for (int j = 0; j < 32; ++j) hold[cc * 32 + j] = t[j];
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&epi_ready[buf * 2 + h]);
          if (!mbar_wait_bounded(&lr_done[buf * 2 + h], par, limit, abort_flag)) {
            lr_ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < BN / 64; ++cc) {
            const int c = h * (BN / 2) + cc * 32;
            uint32_t v[32];
            tmem_ld_32x32b_x32(taddr + c, v);
            tmem_ld_wait();
            if (!row_ok) continue;
            float t[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) t[j] = __fadd_rn(hold[cc * 32 + j], __uint_as_float(v[j]));
            if (!p.swiglu) {
              if (p.res) gated_residual(t, p, row, n0 + c);
              store_bf16_chunk(out_ptr<__nv_bfloat16>(p, row, n0 + c), t, n0 + c, p.N);
            } else if (swiglu_block(t, c, ya, nullptr)) {
              store_bf16_chunk(out_ptr<__nv_bfloat16>(p, row, (n0 + c - 32) >> 1), t, (n0 + c - 32) >> 1, n_out);
            }
          }
        }
        if (!lr_ok) {
          fail();
          break;
        }
      } else if (EPI == EPI_DEQUANT) {
        const float sa = row_ok ? __ldg(p.sa + row) : 0.0f;
        const int n_out = p.swiglu ? p.N >> 1 : p.N;
        uint32_t ya[16];  // SwiGLU: the bf16 `a` block awaiting its `g` block
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c, v);
          tmem_ld_wait();
          const int n = n0 + c;
          float t[32];
          dequant_chunk(v, sa, p.sb, p.bias, n, p.N, t);
          if (!p.swiglu) {
            if (row_ok) {
              if (p.res) gated_residual(t, p, row, n);
              store_bf16_chunk(out_ptr<__nv_bfloat16>(p, row, n), t, n, p.N);
            }
          } else if (swiglu_block(t, c, ya, nullptr) && row_ok) {
            store_bf16_chunk(out_ptr<__nv_bfloat16>(p, row, (n - 32) >> 1), t, (n - 32) >> 1, n_out);
          }
        }
      } else if (EPI == EPI_RAW_I32) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c, v);
          tmem_ld_wait();
          const int n = n0 + c;
          if (!row_ok) continue;
          int32_t* orow = reinterpret_cast<int32_t*>(p.out) + static_cast<int64_t>(row) * p.ldo + n;
          if (n + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n + j < p.N) orow[j] = static_cast<int32_t>(v[j]);
          }
        }
      } else {  // EPI_BF16
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c, v);
          tmem_ld_wait();
          const int n = n0 + c;
          if (ksplit > 1) {  // this CTA's partial row, into the operand ring (idle: the tile's loads are consumed)
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(ring) + row_in_tile * kPartStride + c);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                   __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            continue;
          }
          if (!row_ok) continue;
          float t[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = __uint_as_float(v[j]);
          store_bf16_chunk(reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo + n, t, n, p.N);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (ksplit > 1) {
    // Every CTA of the cluster reaches both barriers (the roles above return only through here).  Between them,
    // the epilogue warps of CTA s sum columns [s BN / ksplit, (s + 1) BN / ksplit) of the tile over the cluster's
    // partials, in rank order, and store them as bf16.
    cluster_sync();
    if (warp >= 2 && warp <= 5 && tile0 < num_tiles) {
      int mb, nb;
      tile_coords(tile0, num_m, num_n, p.group_m, mb, nb);
      const int row_in_tile = (warp & 3) * 32 + lane;
      const int row = mb * kBM + row_in_tile;
      const int cols = BN / ksplit;  // a multiple of 4
      const int c0 = krank * cols;
      const uint32_t mine = smem_u32(reinterpret_cast<float*>(ring) + row_in_tile * kPartStride);
      if (row < p.M) {
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.ldo;
        for (int c = c0; c < c0 + cols; c += 4) {
          const int n = nb * BN + c;
          if (n >= p.N) break;
          float4 acc = ld_shared_cluster_v4(mapa_shared(mine + c * 4, 0));
          for (int r = 1; r < ksplit; ++r) {
            const float4 t = ld_shared_cluster_v4(mapa_shared(mine + c * 4, r));
            acc.x = __fadd_rn(acc.x, t.x);
            acc.y = __fadd_rn(acc.y, t.y);
            acc.z = __fadd_rn(acc.z, t.z);
            acc.w = __fadd_rn(acc.w, t.w);
          }
          const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
          *reinterpret_cast<uint2*>(orow + n) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
        }
      }
    }
    cluster_sync();  // the partials stay in place until every CTA of the cluster has read them
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace convrot
