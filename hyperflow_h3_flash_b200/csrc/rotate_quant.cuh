// Fused online block-Hadamard rotation + per-token symmetric INT8 quantisation for sm_100a.
//
// Replaces the reference's `rotate_quant_kernel` / `rotate_quant_factored_kernel` (hyperflow_h3_flash,
// src/hyperflow_h3_flash/int8.py:194-262, wrapper :326-344), and its torch path for short inputs (:173-178).
//
// Arithmetic.  y = x . blockdiag(H_G), H_G = kron(H4/2, ..., H4/2) = 2^-L H', H' = kron(H4', ...) with the
// integer H4' = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]], H4' v = (v0+v1+v2+v3) - 2 reverse(v).
// Every butterfly runs in fp64 on integer-form sums, so each partial sum is exact while the bf16 exponents of a
// group span at most 45 - 2L binades (37 for G = 256, i.e. max|x| / min nonzero |x| < 2^37 inside a group):
// y is the exact dot, rounded ONCE (to fp32 in the kernel mode, to bf16 in the torch mode).  Then
//   kernel mode (int8.py:212-220): s = fp32(max(amax, 1e-12) / 127), inv = fp32(1 / s), q = rint(fp32(y * inv))
//   torch  mode (int8.py:177-178): s = fp32(max(amax, 1e-12) / 127),                  q = rint(fp32(y / s))
// with IEEE round-to-nearest divisions and products, rint = half to even, q clamped to +-127.
//
// Data flow (one CTA row at a time, rows striding by gridDim.x):
//   * thread 0 streams whole rows into a ring of shared-memory buffers with bulk copies (cp.async.bulk), several
//     rows ahead, so HBM sees deep queues without holding registers;
//   * a team of T = G/16 threads owns one group, viewed as a T x 16 matrix X[a][b] (channel a*16 + b); each thread
//     loads 16/T columns, applies H_T along a in registers, the team transposes through padded shared memory (fp64),
//     and each thread then applies H16 along b to one row: it ends up with 16 CONTIGUOUS output channels;
//   * row amax by warp shuffles + shared memory, then each thread quantises its 16 values and writes 16 bytes.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace convrot {

// x is read as "chunked rows": element (m, k) at xs[k / x_chunk] + m * ldx + k % x_chunk.  Plain row-major input is
// one chunk (x_chunk = K, xs[0] = x).  The Ulysses receive buffer [P, M, K / P] is P chunks of K / P columns; so is
// the same data left in the P senders' buffers, when the kernel gathers each row straight from the other GPUs.
struct RotQuantParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* xs[kMaxChunks];
  int64_t ldx;
  int x_chunk;
  __nv_bfloat16* x_out;  // optional: each gathered (or modulated) bf16 row is also stored to x_out + m * ld_out
  int64_t ld_out;
  // AdaLN prologue (two-column kernel, plain rows): the row that is rotated is
  //   h = bf16( bf16( bf16(LayerNorm(x)) * bf16(1 + scale[idx]) ) + shift[idx] ),  idx = mod_index[m]
  // with scale / shift rows of ld_mod elements; LayerNorm has no affine part and eps = norm_eps.
  const __nv_bfloat16* mod_scale;
  const __nv_bfloat16* mod_shift;
  const int32_t* mod_index;
  int64_t ld_mod;
  float norm_eps;
  int M, K;
  int8_t* q;
  int64_t ldq;
  float* s;
  int rounding;  // 0 = kernel semantics, 1 = torch-path semantics (selects the template instance)
  int stages;    // row buffers in flight, 1..kRQMaxStages
  uint64_t wait_limit_ns;
  int* error_word;
};

constexpr int kRQMaxStages = 8;
constexpr int kRQPadDoubles = 2;  // 16-byte pad per transpose row: conflict-free 128-bit reads

__device__ __forceinline__ void h4_int(double& a, double& b, double& c, double& d) {
  const double s = (a + b) + (c + d);
  const double na = fma(-2.0, d, s);
  const double nb = fma(-2.0, c, s);
  const double nc = fma(-2.0, b, s);
  const double nd = fma(-2.0, a, s);
  a = na;
  b = nb;
  c = nc;
  d = nd;
}

// H16' on 16 values (index = 4 * hi + lo): H4' over lo, then over hi.
__device__ __forceinline__ void h16_int(double (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 4; ++h) h4_int(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
#pragma unroll
  for (int l = 0; l < 4; ++l) h4_int(v[l], v[4 + l], v[8 + l], v[12 + l]);
}

// The per-token scale and its inverse from the row's amax (int8.py:212-214):
//   s = max(amax, 1e-12) / 127,  inv = 1 / s.
// Modes 0 (kernel) and 1 (torch path) divide with IEEE round-to-nearest, as the reference's source and its CPU path
// state.  Mode 2 divides with PTX div.full.f32, the full-range approximate division (within 2 ulp) that the
// reference's Triton kernels compile `/` to, so that codes and scales follow its B200 kernels bit for bit.
template <int ROUNDING>
__device__ __forceinline__ void scale_and_inverse(float amax, float& scale, float& inv) {
  if constexpr (ROUNDING == 2) {
    asm("div.full.f32 %0, %1, %2;" : "=f"(scale) : "f"(fmaxf(amax, 1e-12f)), "f"(127.0f));
    asm("div.full.f32 %0, %1, %2;" : "=f"(inv) : "f"(1.0f), "f"(scale));
  } else {
    scale = __fdiv_rn(fmaxf(amax, 1e-12f), 127.0f);
    inv = __fdiv_rn(1.0f, scale);
  }
}

__device__ __forceinline__ uint32_t pack4_codes(float a, float b, float c, float d) {
  // |a..d| < 127.5: adding 1.5 * 2^23 rounds to an integer (half to even) and leaves the two's-complement code in
  // the low byte.
  const uint32_t ua = __float_as_uint(__fadd_rn(a, 12582912.0f));
  const uint32_t ub = __float_as_uint(__fadd_rn(b, 12582912.0f));
  const uint32_t uc = __float_as_uint(__fadd_rn(c, 12582912.0f));
  const uint32_t ud = __float_as_uint(__fadd_rn(d, 12582912.0f));
  return __byte_perm(__byte_perm(ua, ub, 0x0040), __byte_perm(uc, ud, 0x0040), 0x5410);
}

__device__ __forceinline__ void record_error_rq(int* word) {
  if (word) atomicCAS(word, 0, 6 /* CONVROT_ERR_TIMEOUT */);
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Shared memory: `stages` row buffers of K bf16 | transpose rows (blockDim * (16 + pad) doubles) |
//                warp maxima (32 floats) | mbarriers.
__host__ __device__ inline size_t rq_smem_bytes(int K, int threads, int stages) {
  size_t rows = static_cast<size_t>(stages) * K * 2;
  rows = (rows + 127) / 128 * 128;
  size_t tr = static_cast<size_t>(threads) * (16 + kRQPadDoubles) * 8;
  return rows + tr + 32 * 4 + kRQMaxStages * 8 + 64;
}

// G: group size (4, 16, 64, 256).  SLOTS: 16-channel slots per thread; blockDim is a multiple of 32 with
// blockDim * SLOTS >= K / 16; threads whose slot lies beyond the row form whole idle teams.
template <int G, int SLOTS, int ROUNDING>
__global__ void __launch_bounds__(512) rotate_quant_kernel(const RotQuantParams p) {
  constexpr int T = G >= 16 ? G / 16 : 1;  // threads per group
  constexpr int CPT = 16 / T;              // columns per thread in the column phase
  constexpr int L = G == 4 ? 1 : G == 16 ? 2 : G == 64 ? 3 : 4;
  // y = 2^-L * Y with Y the integer-form sum.  fp32/bf16 rounding commutes with the power-of-two scale (results
  // below 2^-126, where it would not, can neither reach the 1e-12 floor of amax nor a nonzero code), so Y is
  // rounded and the 2^-L goes into the scale arithmetic: exact.
  constexpr float kScale = 1.0f / static_cast<float>(1 << L);

  extern __shared__ __align__(1024) uint8_t rq_smem_raw[];
  const int K = p.K;
  const int nthr = blockDim.x;
  const int stages = p.stages;
  const int nslots = K / 16;
  size_t rows_bytes = (static_cast<size_t>(stages) * K * 2 + 127) / 128 * 128;
  __nv_bfloat16* rows = reinterpret_cast<__nv_bfloat16*>(rq_smem_raw);
  double* tr = reinterpret_cast<double*>(rq_smem_raw + rows_bytes);
  float* warp_max = reinterpret_cast<float*>(tr + static_cast<size_t>(nthr) * (16 + kRQPadDoubles));
  uint64_t* bars = reinterpret_cast<uint64_t*>(warp_max + 32);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = nthr >> 5;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * 2;

  if (tid == 0) {
    for (int st = 0; st < stages; ++st) mbar_init(&bars[st], 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  // One bulk copy per chunk of the row (one for plain rows) into the stage's linear row buffer.
  auto issue_row_v1 = [&](int stage, int m) {
    mbar_arrive_expect_tx(&bars[stage], row_bytes);
    const int64_t roff = static_cast<int64_t>(m) * p.ldx;
    int j = 0;
    for (int k0 = 0; k0 < K; k0 += p.x_chunk, ++j)
      bulk_load(rows + static_cast<size_t>(stage) * K + k0, select_chunk(p.xs, j) + roff,
                static_cast<uint32_t>(p.x_chunk) * 2, &bars[stage]);
  };
  if (tid == 0) {
    for (int st = 0; st < stages; ++st) {
      const int m = blockIdx.x + st * gridDim.x;
      if (m >= p.M) break;
      issue_row_v1(st, m);
    }
  }

  const int team_thread = tid % T;  // position in the group team (for G >= 64)
  // Teams sync on their own lanes: a warp may hold one active and one idle team (slots beyond the row).
  const unsigned team_mask = T >= 32 ? 0xffffffffu : (((1u << T) - 1u) << (lane & ~(T - 1)));
  int it = 0;
  bool aborted = false;
  for (int m = blockIdx.x; m < p.M; m += gridDim.x, ++it) {
    const int st = it % stages;
    const uint32_t parity = (it / stages) & 1;
    volatile int never = 0;
    const bool arrived = mbar_wait_bounded(&bars[st], parity, p.wait_limit_ns, &never);
    const __nv_bfloat16* xr = rows + static_cast<size_t>(st) * K;
    if (tid == 0 && p.x_out && arrived) {  // the gathered row, as it landed
      bulk_store(p.x_out + static_cast<int64_t>(m) * p.ld_out, xr, row_bytes);
      bulk_commit_group();
    }

    float y[SLOTS][16];
    float amax = 0.0f;
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl) {
      const int slot = tid + sl * nthr;  // 16-channel slot: channels [16 slot, 16 slot + 16)
      if (slot >= nslots) {  // team-uniform: nslots and nthr are multiples of the team size
#pragma unroll
        for (int j = 0; j < 16; ++j) y[sl][j] = 0.0f;
        continue;
      }
      double v[16];
      if constexpr (G == 4 || G == 16) {
        const uint4* src = reinterpret_cast<const uint4*>(xr + slot * 16);
        const uint4 u0 = src[0], u1 = src[1];
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[2 * j] = static_cast<double>(__uint_as_float(w[j] << 16));
          v[2 * j + 1] = static_cast<double>(__uint_as_float(w[j] & 0xffff0000u));
        }
        if constexpr (G == 4) {
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) h4_int(v[4 * gq], v[4 * gq + 1], v[4 * gq + 2], v[4 * gq + 3]);
        } else {
          h16_int(v);
        }
      } else {
        // Column phase: this thread loads columns [team_thread * CPT, +CPT) of the T x 16 group matrix.
        const int group_base = (slot - team_thread) * 16;  // first channel of the group
        double c[T][CPT];
#pragma unroll
        for (int a = 0; a < T; ++a) {
          const __nv_bfloat16* src = xr + group_base + a * 16 + team_thread * CPT;
          if constexpr (CPT == 1) {
            c[a][0] = static_cast<double>(__bfloat162float(src[0]));
          } else {  // CPT == 4
            const uint2 u = *reinterpret_cast<const uint2*>(src);
            c[a][0] = static_cast<double>(__uint_as_float(u.x << 16));
            c[a][1] = static_cast<double>(__uint_as_float(u.x & 0xffff0000u));
            c[a][2] = static_cast<double>(__uint_as_float(u.y << 16));
            c[a][3] = static_cast<double>(__uint_as_float(u.y & 0xffff0000u));
          }
        }
        // H_T along a, per column
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
          if constexpr (T == 16) {
            double col[16];
#pragma unroll
            for (int a = 0; a < 16; ++a) col[a] = c[a][j];
            h16_int(col);
#pragma unroll
            for (int a = 0; a < 16; ++a) c[a][j] = col[a];
          } else {  // T == 4
            h4_int(c[0][j], c[1][j], c[2][j], c[3][j]);
          }
        }
        // Transpose through shared memory: each thread owns one padded row of the team's T x 16 block; it writes
        // its columns into every row, then reads back its own row.
        double* team_buf = tr + static_cast<size_t>(tid - team_thread) * (16 + kRQPadDoubles);
        __syncwarp(team_mask);
#pragma unroll
        for (int a = 0; a < T; ++a)
#pragma unroll
          for (int j = 0; j < CPT; ++j) team_buf[a * (16 + kRQPadDoubles) + team_thread * CPT + j] = c[a][j];
        __syncwarp(team_mask);
        const double2* rd = reinterpret_cast<const double2*>(team_buf + team_thread * (16 + kRQPadDoubles));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const double2 d2 = rd[j];
          v[2 * j] = d2.x;
          v[2 * j + 1] = d2.y;
        }
        __syncwarp(team_mask);
        h16_int(v);
      }
      // Round the exact sums once (to fp32, or to bf16 in the torch-path mode).
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float f;
        if constexpr (ROUNDING != 1)
          f = __double2float_rn(v[j]);
        else
          f = __bfloat162float(__double2bfloat16(v[j]));
        y[sl][j] = f;
        amax = fmaxf(amax, fabsf(f));
      }
    }

    // Row amax: warp shuffle, then across warps.  The barrier also agrees on a timed-out row copy.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (lane == 0) warp_max[warp] = amax;
    if (__syncthreads_or(!arrived)) {
      if (tid == 0) record_error_rq(p.error_word);
      aborted = true;
      break;
    }
    float rmax = 0.0f;
    for (int w = 0; w < nwarps; ++w) rmax = fmaxf(rmax, warp_max[w]);
    float scale, inv;
    scale_and_inverse<ROUNDING>(__fmul_rn(rmax, kScale), scale, inv);
    // y * inv = Yf * (inv * 2^-L) and y / s = Yf / (s * 2^L): the power-of-two factors are exact
    const float inv_y = __fmul_rn(inv, kScale);
    const float scale_y = __fdiv_rn(scale, kScale);
    int8_t* qrow = p.q + static_cast<int64_t>(m) * p.ldq;
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl) {
      const int slot = tid + sl * nthr;
      if (slot >= nslots) continue;
      // No clamp is needed: |y| <= amax gives |y * inv| <= 127 (1 + 2^-24) / (1 - 2^-24) < 127.5 (and likewise
      // |y / s| < 127.5), so rint never leaves [-127, 127] for finite inputs.
      float t[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if constexpr (ROUNDING != 1)
          t[j] = __fmul_rn(y[sl][j], inv_y);
        else
          t[j] = __fdiv_rn(y[sl][j], scale_y);
      }
      uint4 out;  // pack4_codes rounds half to even
      out.x = pack4_codes(t[0], t[1], t[2], t[3]);
      out.y = pack4_codes(t[4], t[5], t[6], t[7]);
      out.z = pack4_codes(t[8], t[9], t[10], t[11]);
      out.w = pack4_codes(t[12], t[13], t[14], t[15]);
      *reinterpret_cast<uint4*>(qrow + slot * 16) = out;
    }
    if (tid == 0) p.s[m] = scale;
    __syncthreads();  // the row buffer and warp maxima are free again
    if (tid == 0) {
      const int m_next = m + stages * gridDim.x;
      if (p.x_out) bulk_wait_group_read<0>();  // the row store has read this buffer
      if (m_next < p.M) issue_row_v1(st, m_next);
    }
  }
  if (tid == 0 && p.x_out) bulk_wait_group_all();
  if (aborted && tid == 0) {
    // Let the row copies still in flight land before the CTA leaves (bounded as well).
    volatile int never = 0;
    for (int k = 0; k < stages; ++k) {
      const int j = it + k;
      const int m = blockIdx.x + j * gridDim.x;
      if (m >= p.M) break;
      mbar_wait_bounded(&bars[j % stages], (j / stages) & 1, p.wait_limit_ns, &never);
    }
  }
}

// ------------------------------------------------------------------------------------------------------------------
// G = 256 kernel: a team of 8 threads per group, two columns per thread.
//
// The row lands in shared memory as it lies in HBM: one bulk copy per row (per chunk of a chunked row), groups at
// 512-byte strides.  Thread tt of a team loads the bf16 pair (columns 2tt, 2tt+1) of every row a of the 16 x 16 group
// matrix (16 32-bit loads for 32 values), applies H16 along a to both columns, and the team transposes through shared
// memory in two halves (rows 0-7, then 8-15; 128-bit stores and loads): thread tt ends up with rows tt and tt+8, i.e.
// channels [16 tt, 16 tt + 16) and [16 (tt+8), ...) of the group, applies H16 along b, and writes 2 x 16 contiguous
// codes.
//
// Bank order.  The four teams of a warp read four groups 512 bytes apart, i.e. the same banks for the same row a.
// Team j (0..3 within its warp) therefore loads row a ^ j into register a.  H4' has the entry -1 exactly where
// row ^ column == 3, so H4'[i ^ j][k] = H4'[i][k ^ j]: the column transform of the row-permuted input is the
// transform's output permuted the same way (register k holds output row k ^ j), and the transpose stores register
// 8h + a at row (8h + a) ^ j.  The operations are those of the unpermuted order up to commutation of the additions,
// so the results are bitwise the same, and the four teams' loads hit four different rows' banks.
constexpr int kSlotBytes = 512;        // one group of 256 bf16, unpadded (see "Bank order")
constexpr int kPaddedSlotBytes = 544;  // the AdaLN form's slot: 32 bytes of pad put the warp's four groups on
                                       // different banks without reordering the rows
constexpr int kTrRow = 16 + kRQPadDoubles;  // doubles per transpose row

// Threads of a chunked one-slot CTA at most (K <= 10240): bounding them lets the compiler keep that kernel within 96
// registers, four CTAs per SM at K = 5120, like the plain kernel.
constexpr int kRQ256ChunkedThreads = 320;

__host__ __device__ inline size_t rq256_smem_bytes(int K, int threads, int stages, bool chunked = false,
                                                   bool adaln = false) {
  const size_t slots = static_cast<size_t>(K / 256) * (adaln ? kPaddedSlotBytes : kSlotBytes);
  const size_t tr = static_cast<size_t>(threads / 8) * 8 * kTrRow * 8;  // per team: 8 rows of the half transpose
  (void)chunked;
  const size_t stats = 64 * 8;  // AdaLN: per-warp (sum, sum of squares) in fp64
  return static_cast<size_t>(stages) * slots + tr + 64 * 4 + kRQMaxStages * 8 + stats + 64;
}

// AdaLN on a pair of bf16 values (low half = even column): n = bf16((x - mean) * rstd) in fp32, then
// bf16(bf16(n * bf16(1 + scale)) + shift), each step rounded to bf16 as the unfused bf16 tensor ops round it.
// Two fp32 values rounded to bf16 in one paired conversion, returned as the packed pair and unpacked again.
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float bf16_lo(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t p) { return __uint_as_float(p & 0xffff0000u); }

__device__ __forceinline__ uint32_t adaln_pair(uint32_t w, uint32_t sc, uint32_t sh, float mean, float rstd) {
  // both halves step by step, each rounding done on the pair at once
  const uint32_t n = bf16x2_rn(__fmul_rn(__fsub_rn(bf16_lo(w), mean), rstd),
                               __fmul_rn(__fsub_rn(bf16_hi(w), mean), rstd));
  const uint32_t one_s = bf16x2_rn(__fadd_rn(1.0f, bf16_lo(sc)), __fadd_rn(1.0f, bf16_hi(sc)));
  // bf16 * bf16 is exact in fp32 (16 significant bits, same exponent range), so rounding the fp32 product to bf16
  // is one rounding of the exact product: what the packed bf16 multiply computes, in one instruction for the pair.
  __nv_bfloat162 nb, ob;
  memcpy(&nb, &n, 4);
  memcpy(&ob, &one_s, 4);
  const __nv_bfloat162 tb = __hmul2(nb, ob);
  uint32_t t;
  memcpy(&t, &tb, 4);
  return bf16x2_rn(__fadd_rn(bf16_lo(t), bf16_lo(sh)), __fadd_rn(bf16_hi(t), bf16_hi(sh)));
}

// CHUNKED selects the chunked-row input (the Ulysses layouts, in this GPU's memory or gathered from the others'):
// one bulk copy per chunk of each row (K / x_chunk of them, 1280 bytes each for K = 5120 over 8 GPUs), and x_out may
// receive each gathered row.  Plain rows (x_chunk == K) use the instantiation without it.  The launch sizes
// residency from the compiled register count; at K = 5120 (160 threads) both forms stay within 96 (plain 92 with no
// bound; chunked under its thread bound), so four CTAs fit an SM.
template <int SLOTS, int ROUNDING, bool CHUNKED, bool ADALN = false>
__global__ void __launch_bounds__(CHUNKED && SLOTS == 1 ? kRQ256ChunkedThreads : 512, CHUNKED && SLOTS == 1 ? 2 : 0)
    rotate_quant256_kernel(const RotQuantParams p) {
  extern __shared__ __align__(1024) uint8_t rq2_smem_raw[];
  const int K = p.K;
  const int ngroups = K / 256;
  const int nthr = blockDim.x;
  const int stages = p.stages;
  constexpr int kSlot = ADALN ? kPaddedSlotBytes : kSlotBytes;
  const size_t stage_bytes = static_cast<size_t>(ngroups) * kSlot;
  uint8_t* rows = rq2_smem_raw;
  double* tr = reinterpret_cast<double*>(rq2_smem_raw + stages * stage_bytes);
  // per-warp row maxima, two sets used by alternate rows (so plain rows need one block barrier per row)
  float* warp_max = reinterpret_cast<float*>(tr + static_cast<size_t>(nthr / 8) * 8 * kTrRow);
  uint64_t* bars = reinterpret_cast<uint64_t*>(warp_max + 64);
  double* stats = reinterpret_cast<double*>(bars + kRQMaxStages);  // ADALN: (sum, sum of squares) per warp

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = nthr >> 5;
  const int tt = tid & 7;                              // thread in team
  // team in warp: the row order a ^ jx (see "Bank order").  The AdaLN form keeps the plain order in padded slots:
  // its modulation operands, indexed by the row, would need per-row addresses, and the registers they take cost it a
  // CTA per SM.
  const int jx = ADALN ? 0 : (tid >> 3) & 3;
  const unsigned team_mask = 0xffu << (lane & ~7);     // the team's 8 lanes
  double* team_buf = tr + static_cast<size_t>(tid >> 3) * 8 * kTrRow;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * 2;
  constexpr float kScale = 1.0f / 16.0f;  // 2^-L, L = 4

  auto issue_row = [&](int stage, int m) {
    // the row as it lies in HBM: one bulk copy (one per chunk of a chunked row), completing on the stage's barrier
    mbar_arrive_expect_tx(&bars[stage], row_bytes);
    const int64_t roff = static_cast<int64_t>(m) * p.ldx;
    uint8_t* dst = rows + stage * stage_bytes;
    if constexpr (ADALN) {
      for (int g = 0; g < ngroups; ++g) bulk_load(dst + g * kSlot, p.x + roff + g * 256, 512, &bars[stage]);
    } else if constexpr (!CHUNKED) {
      bulk_load(dst, p.x + roff, row_bytes, &bars[stage]);
    } else {
      const uint32_t chunk_bytes = static_cast<uint32_t>(p.x_chunk) * 2;
      const int nchunks = K / p.x_chunk;
#pragma unroll 1
      for (int j = 0; j < nchunks; ++j) bulk_load(dst + j * chunk_bytes, select_chunk(p.xs, j) + roff, chunk_bytes,
                                                  &bars[stage]);
    }
  };

  if (tid == 0) {
    for (int st = 0; st < stages; ++st) mbar_init(&bars[st], 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int st = 0; st < stages; ++st) {
      const int m = blockIdx.x + st * gridDim.x;
      if (m >= p.M) break;
      issue_row(st, m);
    }

  int it = 0;
  bool aborted = false;
  for (int m = blockIdx.x; m < p.M; m += gridDim.x, ++it) {
    const int st = it % stages;
    volatile int never = 0;
    const bool arrived = mbar_wait_bounded(&bars[st], (it / stages) & 1, p.wait_limit_ns, &never);
    const uint8_t* xr = rows + st * stage_bytes;
    if constexpr (CHUNKED) {
      // the gathered row, as it landed, stored in one piece
      if (tid == 0 && p.x_out && arrived) {
        bulk_store(p.x_out + static_cast<int64_t>(m) * p.ld_out, xr, row_bytes);
        bulk_commit_group();
      }
    }

    // AdaLN: the row's mean and 1/sqrt(var + eps), from fp64 sums (exact for bf16 rows of moderate range),
    // each rounded once to fp32
    float mean_f = 0.0f, rstd_f = 0.0f;
    const uint32_t* scale_row = nullptr;
    const uint32_t* shift_row = nullptr;
    if constexpr (ADALN) {
      const int64_t idx = __ldg(p.mod_index + m);
      scale_row = reinterpret_cast<const uint32_t*>(p.mod_scale + idx * p.ld_mod);
      shift_row = reinterpret_cast<const uint32_t*>(p.mod_shift + idx * p.ld_mod);
      double s1 = 0.0, s2 = 0.0;
#pragma unroll
      for (int sl = 0; sl < SLOTS; ++sl) {
        const int g = (tid + sl * nthr) >> 3;
        if (g >= ngroups) continue;
        const uint32_t* col = reinterpret_cast<const uint32_t*>(xr + g * kSlot) + tt;
#pragma unroll
        for (int a = 0; a < 16; ++a) {
          const uint32_t w = col[a * 8];
          const double x0 = __uint_as_float(w << 16), x1 = __uint_as_float(w & 0xffff0000u);
          s1 += x0 + x1;
          s2 = fma(x0, x0, fma(x1, x1, s2));
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, off);
        s2 += __shfl_xor_sync(0xffffffffu, s2, off);
      }
      if (lane == 0) {
        stats[2 * warp] = s1;
        stats[2 * warp + 1] = s2;
      }
      __syncthreads();
      double t1 = 0.0, t2 = 0.0;
      for (int w = 0; w < nwarps; ++w) {
        t1 += stats[2 * w];
        t2 += stats[2 * w + 1];
      }
      const double mean = t1 / K;
      const double var = fmax(t2 / K - mean * mean, 0.0);
      mean_f = __double2float_rn(mean);
      rstd_f = __double2float_rn(1.0 / sqrt(var + static_cast<double>(p.norm_eps)));
    }

    float y[SLOTS][32];
    float amax = 0.0f;
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl) {
      const int g = (tid + sl * nthr) >> 3;  // group of this team (team-uniform)
      if (g >= ngroups) {
#pragma unroll
        for (int j = 0; j < 32; ++j) y[sl][j] = 0.0f;
        continue;
      }
      // column phase: columns 2tt and 2tt+1 of the 16 x 16 group matrix
      double c0[16], c1[16];
      const uint32_t* col = reinterpret_cast<const uint32_t*>(xr + g * kSlot) + tt;
      // a ^ jx = 4 (a >> 2) + ((a & 3) ^ jx): one base per a & 3, the rest an immediate offset
      const uint32_t* colr[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) colr[r] = col + (r ^ jx) * 8;
#pragma unroll
      for (int a = 0; a < 16; ++a) {
        // row a ^ jx, held in register a (the AdaLN form, in the plain order, addresses it directly: fewer registers)
        uint32_t* src = ADALN ? const_cast<uint32_t*>(col) + a * 8 : const_cast<uint32_t*>(colr[a & 3]) + (a >> 2) * 32;
        uint32_t w = *src;
        if constexpr (ADALN) {
          // element (a ^ jx, 2tt) of the group is column 256 g + 16 (a ^ jx) + 2 tt of the row
          const int ra = a ^ jx;
          w = adaln_pair(w, __ldg(scale_row + g * 128 + ra * 8 + tt), __ldg(shift_row + g * 128 + ra * 8 + tt),
                         mean_f, rstd_f);
          *src = w;  // h replaces x in the row buffer (stored to x_out below)
        }
        c0[a] = static_cast<double>(__uint_as_float(w << 16));
        c1[a] = static_cast<double>(__uint_as_float(w & 0xffff0000u));
      }
      h16_int(c0);
      h16_int(c1);
      // transpose in two halves: rows [8h, 8h + 8) go through the team buffer, thread tt takes row 8h + tt
      double v[2][16];
      double* tbr[4];  // row (a ^ jx) of the half buffer = tbr[a & 3] + 4 (a >> 2) rows
#pragma unroll
      for (int r = 0; r < 4; ++r) tbr[r] = team_buf + (r ^ jx) * kTrRow + 2 * tt;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        __syncwarp(team_mask);
#pragma unroll
        for (int a = 0; a < 8; ++a)  // register 8h + a holds row 8h + (a ^ jx)
          *reinterpret_cast<double2*>(tbr[a & 3] + (a >> 2) * 4 * kTrRow) = make_double2(c0[8 * h + a], c1[8 * h + a]);
        __syncwarp(team_mask);
        const double2* rd = reinterpret_cast<const double2*>(team_buf + tt * kTrRow);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const double2 d2 = rd[j];
          v[h][2 * j] = d2.x;
          v[h][2 * j + 1] = d2.y;
        }
      }
      h16_int(v[0]);
      h16_int(v[1]);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float f;
          if constexpr (ROUNDING != 1)
            f = __double2float_rn(v[h][j]);
          else
            f = __bfloat162float(__double2bfloat16(v[h][j]));
          y[sl][16 * h + j] = f;
          amax = fmaxf(amax, fabsf(f));
        }
    }

#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    float* row_max = warp_max + (it & 1) * 32;
    if (lane == 0) row_max[warp] = amax;
    if constexpr (ADALN) fence_proxy_async_smem();  // h in the row buffer, for the bulk stores below
    if constexpr (CHUNKED && !ADALN) {
      // the gathered row's store (issued when it landed) has read the buffer before the barrier below
      if (tid == 0 && p.x_out) bulk_wait_group_read<0>();
    }
    if (__syncthreads_or(!arrived)) {
      if (tid == 0) record_error_rq(p.error_word);
      aborted = true;
      break;
    }
    if constexpr (!ADALN) {
      // Every thread has read its part of the row buffer (column phase), and the gathered row's stores are done
      // reading it, so it is refilled now; the maxima of the next row go to the other set, so no second barrier is
      // needed before the next row.
      if (tid == 0) {
        const int m_next = m + stages * gridDim.x;
        if (m_next < p.M) issue_row(st, m_next);
      }
    }
    if constexpr (ADALN) {
      if (tt == 0 && p.x_out) {  // each team stores its groups of h (fenced by their writers before the barrier)
#pragma unroll 1
        for (int g = tid >> 3; g < ngroups; g += nthr >> 3)
          bulk_store(p.x_out + static_cast<int64_t>(m) * p.ld_out + g * 256, xr + g * kSlot, 512);
        bulk_commit_group();
      }
    }
    float rmax = 0.0f;
    for (int w = 0; w < nwarps; ++w) rmax = fmaxf(rmax, row_max[w]);
    float scale, inv;
    scale_and_inverse<ROUNDING>(__fmul_rn(rmax, kScale), scale, inv);
    const float inv_y = __fmul_rn(inv, kScale);
    const float scale_y = __fdiv_rn(scale, kScale);
    int8_t* qrow = p.q + static_cast<int64_t>(m) * p.ldq;
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl) {
      const int g = (tid + sl * nthr) >> 3;
      if (g >= ngroups) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float t[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if constexpr (ROUNDING != 1)
            t[j] = __fmul_rn(y[sl][16 * h + j], inv_y);
          else
            t[j] = __fdiv_rn(y[sl][16 * h + j], scale_y);
        }
        uint4 out;
        out.x = pack4_codes(t[0], t[1], t[2], t[3]);
        out.y = pack4_codes(t[4], t[5], t[6], t[7]);
        out.z = pack4_codes(t[8], t[9], t[10], t[11]);
        out.w = pack4_codes(t[12], t[13], t[14], t[15]);
        *reinterpret_cast<uint4*>(qrow + g * 256 + (8 * h + tt) * 16) = out;
      }
    }
    if (tid == 0) p.s[m] = scale;
    if constexpr (ADALN) {
      // the stores of h read this buffer until they are done, so it is refilled only after every team saw them
      if (tt == 0 && p.x_out) bulk_wait_group_read<0>();
      __syncthreads();
      if (tid == 0) {
        const int m_next = m + stages * gridDim.x;
        if (m_next < p.M) issue_row(st, m_next);
      }
    }
  }
  if constexpr (CHUNKED) {
    if (tid == 0 && p.x_out) bulk_wait_group_all();
  }
  if constexpr (ADALN) {
    if (tt == 0 && p.x_out) bulk_wait_group_all();
  }
  if (aborted && tid == 0) {
    volatile int never = 0;
    for (int k = 0; k < stages; ++k) {
      const int j = it + k;
      const int m = blockIdx.x + j * gridDim.x;
      if (m >= p.M) break;
      mbar_wait_bounded(&bars[j % stages], (j / stages) & 1, p.wait_limit_ns, &never);
    }
  }
}

}  // namespace convrot
