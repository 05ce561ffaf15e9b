// 2-SM (cta_group::2) tcgen05 INT8 GEMM for sm_100a: one CTA pair per 256 x 256 output tile.
//
// The pair shares the tensor-core instruction  D[256 x 256] (+)= A[256 x K] . B[256 x K]^T  (kind::i8, K = 32):
// CTA r of the pair holds A rows [128 r, 128 r + 128) and B rows (output columns) [128 r, 128 r + 128) in its own
// shared memory, and its own TMEM holds accumulator rows [128 r, 128 r + 128) x all 256 columns.  Per SM this moves
// half the B bytes of the 1-SM 128 x 256 tile for the same MACs, which is what keeps shared memory below its
// bandwidth limit.
//
// Roles per CTA (224 threads; warp 6 only with the low-rank term):
//   warp 0      TMA producer: this CTA's A tile and B half, signalling the LEADER's full barrier (cta_group::2 load)
//   warp 1      TMEM allocation for the pair; in the leader (rank 0), lane 0 issues the int8 main loop's MMAs
//   warps 2..5  epilogue over this CTA's 128 accumulator rows (as in the 1-SM kernel)
//   warp 6      TMA producer of this CTA's low-rank tiles (xa rows, up rows); in the leader, lane 0 also issues the
//               low-rank MMAs, so the main loop's issuer neither waits for nor polls anything of the low-rank term
//
// Cross-CTA signalling: TMA loads (never multicast: each CTA fetches its own bytes) complete on the leader's barrier
// through its cluster address, the leader signals MMA completion to both CTAs' barriers with one tcgen05.commit,
// and the peer's epilogue arrives on the leader's barriers remotely (mapa).  Every wait is bounded as in the 1-SM
// kernel.
//
// With the low-rank term the epilogue works per 128-column half of its accumulator: it reads and dequantises the
// half into registers, the leader then runs the half's kind::f16 MMA xa . up^T (M = 256, N = 128, accumulate = 0)
// over those TMEM columns, and the epilogue adds the product to the held values.  No fp32 value is written back to
// TMEM.
#pragma once

#include "gemm_sm100.cuh"

namespace convrot {

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking cluster-scope check (see mbar_test_wait).
__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait with cluster-scope acquire, for barriers that receive arrivals from the other CTA.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                                          volatile int* abort) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((spin & 63) == 63) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) return false;
    }
  }
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on a barrier that may live in the
// other CTA of the pair (cluster address).  No multicast: each CTA fetches its own bytes.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

template <int NCOLS>
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* holder_smem) {  // one warp in each CTA of the pair
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder_smem)),
               "n"(NCOLS)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int NCOLS>
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(NCOLS) : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the barrier at `cluster_addr` (this CTA's or the peer's) when the pair's MMAs so far are done.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

// The same arrival on the barrier at this shared-memory offset in BOTH CTAs of the pair, as one commit (an MMA
// completion signal, not a data copy).  Measured on B200: one commit per stage instead of two shortens the MMA
// issue of a 256 x 256 x 5120 tile from 23.8k to 22.1k cycles.
__device__ __forceinline__ void mma_commit_pair_both(uint32_t smem_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

template <int STAGES, int LR_ATOM, int LR_ATOMS>
struct Gemm2Cfg {
  static constexpr int kBN = 256;             // output columns per pair tile (= per CTA accumulator)
  static constexpr int kBHalf = 128;          // B rows per CTA
  static constexpr int kStages = STAGES;
  static constexpr bool kHasLR = LR_ATOMS > 0;
  static constexpr int kABytes = kBM * kRowBytes;      // 16 KB
  static constexpr int kBBytes = kBHalf * kRowBytes;   // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kLRXaBytes = kHasLR ? kBM * LR_ATOM * LR_ATOMS : 0;
  // The low-rank term runs per 128-column half of the tile: this CTA's share of one half's up rows is 64 rows.
  static constexpr int kLRUpRows = 64;
  static constexpr int kLRUpBytes = kHasLR ? kLRUpRows * LR_ATOM * LR_ATOMS : 0;
  static constexpr int kTmemCols = 512;
  static constexpr int kThreads = kHasLR ? 224 : 192;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], epi_ready[2 x 2], lr_done[2 x 2], lr_full, lr_empty, drain,
  // lr_drain (epi_ready and lr_done per accumulator buffer and 128-column half)
  static constexpr int kNumBars = 2 * STAGES + 12 + 4;
  static constexpr int kBarBytes = ((kNumBars * 8 + 16 + 127) / 128) * 128;
  // Output staging per epilogue warp: two 32 x 32 bf16 boxes (2 KB each, SWIZZLE_64B), or in their place one
  // 32 x 64 box (4 KB, SWIZZLE_128B) for wide stores; two wide boxes when shared memory has room for them, so that
  // a box is written while the previous one's store (over NVLink, for a scattered output) still reads the other.
  static constexpr int kStoreBoxBytes = 32 * 64;
  static constexpr int kWideBoxBytes = 32 * 128;
  static constexpr int kSmemNoStore =
      1024 + STAGES * kStageBytes + kLRXaBytes + kLRUpBytes + kBarBytes + kSiluTableBytes;
  static constexpr int kWideBoxes = kSmemNoStore + 4 * 2 * kWideBoxBytes <= 227 * 1024 ? 2 : 1;
  static constexpr int kStoreBytes = 4 * kWideBoxes * kWideBoxBytes;
  // After the barriers: the silu table of the SwiGLU epilogue (filled only by SwiGLU launches).
  static constexpr int kSmemBytes = kSmemNoStore + kStoreBytes;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory above the sm_100 per-CTA limit");
  static constexpr uint32_t kIdesc = make_idesc_i8(256, 256);
  static constexpr uint32_t kIdescLR = make_idesc_bf16(256, 128);  // one 128-column half per low-rank MMA
};

// One bf16 output map per column chunk (box 32 x 32): chunk j covers columns [j W, (j + 1) W) of the result.
struct OutMaps {
  CUtensorMap m[kMaxChunks];
};

template <class Cfg, int EPI, int LR_ATOM, int LR_ATOMS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::kThreads, 1)
    convrot_gemm2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_xa, const __grid_constant__ CUtensorMap tmap_up,
                           const __grid_constant__ OutMaps tmap_y, const GemmParams p) {
  constexpr int BN = Cfg::kBN;
  constexpr int S = Cfg::kStages;
  constexpr bool HAS_LR = Cfg::kHasLR;
  extern __shared__ __align__(1024) uint8_t gemm2_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm2_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* lr_xa = ring + S * Cfg::kStageBytes;
  uint8_t* lr_up = lr_xa + Cfg::kLRXaBytes;
  uint8_t* store_stage = lr_up + Cfg::kLRUpBytes;  // 1024-aligned: stage and tile sizes are multiples of 1 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(store_stage + Cfg::kStoreBytes);
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
  uint16_t* silu_tab = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(bars) + Cfg::kBarBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (p.M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // The low-rank term streams through its operand buffers in rank chunks of LR_ATOMS * LR_ATOM / 2 columns.
  const int lr_chunks = HAS_LR ? (p.r + LR_ATOMS * (LR_ATOM / 2) - 1) / (LR_ATOMS * (LR_ATOM / 2)) : 0;
  const int nkb = (p.K + kRowBytes - 1) / kRowBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&epi_ready[b], 8);
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
    tmem_alloc_pair<Cfg::kTmemCols>(tmem_holder);
    tmem_relinquish_pair();
  }
  if (p.swiglu) silu_table_fill(silu_tab, threadIdx.x, blockDim.x);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated for the pair, the silu table filled
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t limit = p.wait_limit_ns;
  auto fail = [&]() {
    *abort_flag = 1;
    record_error(p.error_word, 6 /* CONVROT_ERR_TIMEOUT */);
  };
  // Cluster addresses of the leader's barriers (targets of TMA transaction bytes and of the peer's arrivals).
  const uint32_t leader_full0 = mapa_shared(smem_u32(full), 0);
  const uint32_t leader_tmem_empty0 = mapa_shared(smem_u32(tmem_empty), 0);
  const uint32_t leader_epi_ready0 = mapa_shared(smem_u32(epi_ready), 0);
  const uint32_t leader_lr_full = mapa_shared(smem_u32(lr_full), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer: this CTA's A rows and B half
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += num_pairs) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
        const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int n0 = nb * BN + static_cast<int>(rank) * Cfg::kBHalf;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, limit, abort_flag)) {
            fail();
            ok = false;
            break;
          }
          uint8_t* st_ptr = ring + stage * Cfg::kStageBytes;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          const uint32_t bar = leader_full0 + stage * 8;
          tma_load_2d_pair(st_ptr, &tmap_a, bar, kb * 128, m0);
          tma_load_2d_pair(st_ptr + Cfg::kABytes, &tmap_b, bar, kb * 128, n0);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let loads in flight land before the CTA leaves (their barrier may be the peer's)
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer of the int8 main loop (leader only)
    if (lane == 0 && rank == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      const uint32_t ring_base = smem_u32(ring);
      const uint32_t empty_self = smem_u32(empty);
      const uint32_t tfull_self = smem_u32(tmem_full);
      int i = 0;
      for (int tile = pair; ok && tile < num_tiles; tile += num_pairs, ++i) {
        const uint32_t buf = i & 1;
        if (!mbar_wait_cluster_bounded(&tmem_empty[buf], ((i >> 1) & 1) ^ 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, limit, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = ring_base + stage * Cfg::kStageBytes;
          const uint64_t ad = make_kmajor_desc(a_addr, kRowBytes);
          const uint64_t bd = make_kmajor_desc(a_addr + Cfg::kABytes, kRowBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_i8_pair(d, ad + 2 * kk, bd + 2 * kk, Cfg::kIdesc, (kb | kk) != 0);
          mma_commit_pair_both(empty_self + stage * 8);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair_both(tfull_self + buf * 8);
      }
      if (!ok) fail();
      mma_commit_pair(smem_u32(drain));
      volatile int never = 0;
      mbar_wait_bounded(drain, 0, limit, &never);
    }
  } else if (HAS_LR && warp == 6) {
    // ------------------------------------------------------------ low-rank term: operand loads of this CTA, and in
    // the leader also the kind::f16 MMAs, issued from this warp so that the main loop's issuer never waits or polls
    // for them (each thread's tcgen05.commit tracks its own MMAs, and the two streams write different accumulator
    // buffers).  Unit u = (local tile i, 128-column half h, rank chunk c).
    if (lane == 0) {
      int u = 0;
      bool ok = true;
      const uint32_t xa_base = smem_u32(lr_xa);
      const uint32_t up_base = smem_u32(lr_up);
      const uint32_t lrdone_self = smem_u32(lr_done);
      const uint32_t lrempty_self = smem_u32(lr_empty);
      int i = 0;
      for (int tile = pair; ok && tile < num_tiles; tile += num_pairs, ++i) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
        const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int xs = p.lr_seg_n ? (nb * BN / p.lr_seg_n) * p.r : 0;  // this tile's segment of xa
        // Per half h, this CTA holds up rows [128 h + 64 rank, + 64) of the tile (the pair's N = 128 MMA splits its
        // B operand between the two CTAs), and the xa rows of its 128 accumulator rows.
        for (int h = 0; ok && h < 2; ++h) {
          const int n0 = nb * BN + h * (BN / 2) + static_cast<int>(rank) * Cfg::kLRUpRows;
          for (int c = 0; c < lr_chunks; ++c, ++u) {
            // unit u reuses the operand buffers once the MMAs of unit u-1 (phase u-1 of lr_empty) are done
            if (!mbar_wait_bounded(lr_empty, (u & 1) ^ 1, limit, abort_flag)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(lr_full, 2 * (Cfg::kLRXaBytes + Cfg::kLRUpBytes));
            for (int a = 0; a < LR_ATOMS; ++a) {
              const int x = (c * LR_ATOMS + a) * (LR_ATOM / 2);
              tma_load_2d_pair(lr_xa + a * kBM * LR_ATOM, &tmap_xa, leader_lr_full, x + xs, m0);
              tma_load_2d_pair(lr_up + a * Cfg::kLRUpRows * LR_ATOM, &tmap_up, leader_lr_full, x, n0);
            }
            if (rank != 0) continue;
            // both CTAs' operands have landed, and (first chunk) both epilogues have read the half's accumulator
            if (!mbar_wait_bounded(lr_full, u & 1, limit, abort_flag) ||
                (c == 0 && !mbar_wait_cluster_bounded(&epi_ready[(i & 1) * 2 + h], (i >> 1) & 1, limit, abort_flag))) {
              ok = false;
              break;
            }
            tc_fence_after();
            // The half's first MMA overwrites its accumulator columns (the epilogue holds the dequantised values in
            // registers), so the product lands in TMEM on its own; the half's last chunk tells both epilogues.
            const uint32_t d = tmem_base + (i & 1) * BN + h * (BN / 2);
            for (int a = 0; a < LR_ATOMS; ++a) {
              for (int off = 0; off < LR_ATOM; off += 32) {
                const uint64_t ad = make_kmajor_desc(xa_base + a * kBM * LR_ATOM + off, LR_ATOM);
                const uint64_t bd = make_kmajor_desc(up_base + a * Cfg::kLRUpRows * LR_ATOM + off, LR_ATOM);
                mma_f16_pair(d, ad, bd, Cfg::kIdescLR, (c | a | off) != 0);
              }
            }
            if (c + 1 == lr_chunks) mma_commit_pair_both(lrdone_self + ((i & 1) * 2 + h) * 8);
            mma_commit_pair_both(lrempty_self);
          }
        }
      }
      if (!ok) {
        fail();
        const uint64_t t0 = globaltimer_ns();  // let loads in flight land (their barrier may be the peer's)
        while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
      }
      if (rank == 0) {  // this thread's MMAs are done before the CTA may free its TMEM
        mma_commit_pair(smem_u32(lr_drain));
        volatile int never = 0;
        mbar_wait_bounded(lr_drain, 0, limit, &never);
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------ epilogue over this CTA's 128 rows
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    // bf16 results leave through shared memory and TMA stores, from this warp's 4 KB of staging:
    //  * wide (p.wide_store): one 32 x 64 box (128-byte rows, SWIZZLE_128B: 16-byte chunk c of row r at c ^ (r & 7)),
    //    filled by two consecutive 32-column chunks and stored once the second has landed.  Rows of 128 bytes
    //    leave for another GPU at a far higher rate than rows of 64 (measured on B200: a GEMM whose whole output
    //    goes to the other GPU, 0.84 -> 0.70 ms);
    //  * otherwise two alternating 32 x 32 boxes (64-byte rows, SWIZZLE_64B: chunk c of row r at c ^ ((r >> 1) & 3)),
    //    one store per chunk.
    uint8_t* my_boxes = store_stage + (warp - 2) * Cfg::kWideBoxes * Cfg::kWideBoxBytes;
    int box_sel = 0;   // narrow boxes: which of the two 2 KB boxes
    int wide_sel = 0;  // wide boxes: which of the kWideBoxes 4 KB boxes
    auto stage_and_store = [&](const float (&t)[32], int m_box, int n_col) {
      // A box wholly right of N has nothing to store; skipping it also keeps jy inside the maps that exist (with
      // one chunk of width N, n_col >= N would name chunk 1).  n_col is warp-uniform.
      if (n_col >= (p.swiglu ? p.N >> 1 : p.N)) return;
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * j], t[2 * j + 1]);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      if (p.wide_store) {
        const bool first = (n_col & 63) == 0;  // the box's left half (the output width is a multiple of 64)
        uint8_t* wbox = my_boxes + wide_sel * Cfg::kWideBoxBytes;
        if (first) {
          // the store that last used this box has read it (with two boxes, the latest store may still be reading
          // the other one)
          if (lane == 0) bulk_wait_group_read<Cfg::kWideBoxes - 1>();
          __syncwarp();
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int pc = ((first ? 0 : 4) + c) ^ (lane & 7);
          *reinterpret_cast<uint4*>(wbox + lane * 128 + pc * 16) =
              make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        }
        if (!first) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int n_box = n_col - 32;
            const int jy = n_box / p.out_chunk;  // a 64-column box sits in one chunk (chunk widths % 64 == 0)
            tma_store_2d(&tmap_y.m[jy], wbox, n_box - jy * p.out_chunk, m_box);
            bulk_commit_group();
          }
          if constexpr (Cfg::kWideBoxes == 2) wide_sel ^= 1;
        }
        return;
      }
      uint8_t* box = my_boxes + box_sel * Cfg::kStoreBoxBytes;
      if (lane == 0) bulk_wait_group_read<1>();  // the store that used this box two chunks ago has read it
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int pc = c ^ ((lane >> 1) & 3);
        *reinterpret_cast<uint4*>(box + lane * 64 + pc * 16) =
            make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int jy = n_col / p.out_chunk;  // one 2-D map per output chunk; a 32-column box sits in one chunk
        tma_store_2d(&tmap_y.m[jy], box, n_col - jy * p.out_chunk, m_box);
        bulk_commit_group();
      }
      box_sel ^= 1;
    };
    int i = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++i) {
      const uint32_t buf = i & 1;
      const uint32_t par = (i >> 1) & 1;
      int mb, nb;
      tile_coords(tile, num_m, num_n, p.group_m, mb, nb);
      const int m0 = mb * 2 * kBM + static_cast<int>(rank) * kBM;
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
        // Per 128-column half: read the int32 accumulators and hold the dequantised values (+ bias) in registers,
        // tell the MMA issuer that the half's columns are free, and wait while the low-rank MMA writes its product
        // xa . up^T over them (accumulate = 0); then y = held + product, rounded once to bf16 on the way out.
        const float sa = row_ok ? __ldg(p.sa + row) : 0.0f;
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
          if (lane == 0) mbar_arrive_remote(leader_epi_ready0 + (buf * 2 + h) * 8);
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
            float t[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) t[j] = __fadd_rn(hold[cc * 32 + j], __uint_as_float(v[j]));
            if (!p.swiglu) {
              if (p.res && row_ok) gated_residual(t, p, row, n0 + c);
              stage_and_store(t, m0 + quad * 32, n0 + c);  // rows beyond M are clipped by the TMA store
            } else if (swiglu_block(t, c, ya, silu_tab)) {
              stage_and_store(t, m0 + quad * 32, (n0 + c - 32) >> 1);
            }
          }
        }
        if (!lr_ok) {
          fail();
          break;
        }
      } else if (EPI == EPI_DEQUANT) {
        const float sa = row_ok ? __ldg(p.sa + row) : 0.0f;
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
            if (p.res && row_ok) gated_residual(t, p, row, n);
            stage_and_store(t, m0 + quad * 32, n);  // rows beyond M are clipped by the TMA store
          } else if (swiglu_block(t, c, ya, silu_tab)) {
            stage_and_store(t, m0 + quad * 32, (n - 32) >> 1);
          }
        }
      } else {  // EPI_RAW_I32
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
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(leader_tmem_empty0 + buf * 8);
    }
    if (lane == 0) bulk_wait_group_all();  // every output store has landed before the CTA leaves
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while the pair may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem_base);
  }
}

}  // namespace convrot
