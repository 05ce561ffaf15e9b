/*
 * convrot.h -- C ABI of the B200 (sm_100a) INT8 "convrot" linear.
 *
 * The functions replace the kernel namespace that the reference's `Int8RotLinear`
 * calls into (hyperflow_h3_flash, src/hyperflow_h3_flash/int8.py):
 *
 *   convrot_rotate_quant  <- `rotate_quant(x2, group) -> (q, s)`         int8.py:326-344
 *                            (kernels rotate_quant_kernel :194-221 and
 *                             rotate_quant_factored_kernel :223-262)
 *   convrot_gemm          <- `int8_matmul(a, b, sa, sb) -> bf16`         int8.py:376-390
 *                            (int8_mm_kernel :283-313, or torch._int_mm +
 *                             rescale_kernel :315-324, 353-364 on B200)
 *                            plus a bias and the `up` half of LowRankLinear
 *                            (transformer.py:48-58) fused into its epilogue
 *   convrot_lowrank_down  <- `LowRankLinear.down(x)`                     transformer.py:57-58
 *   convrot_linear        <- `Int8RotLinear.forward` kernel branch       int8.py:161-171
 *
 * Conventions
 *   - Every pointer is a device pointer; every matrix is row-major with an explicit
 *     leading dimension in ELEMENTS.  bf16 data is passed as `void*` (raw 16-bit
 *     bfloat16 values).  `stream` is a `cudaStream_t` (NULL = legacy default stream).
 *   - The caller allocates and owns every buffer.  The library keeps only a lazy
 *     per-device cache (SM count, driver entry point), built on first use.
 *   - Calls are stream-ordered and never synchronise the host.
 *   - Every function returns a status (CONVROT_OK = 0); none aborts or throws.
 *     `convrot_status_string` names a status.  CONVROT_ERR_CUDA carries the CUDA
 *     error in `convrot_last_cuda_error()` (per host thread).
 *   - M == 0 is a valid empty call: nothing is launched, CONVROT_OK is returned.
 */
#ifndef CONVROT_H_
#define CONVROT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CONVROT_OK 0
#define CONVROT_ERR_SHAPE 1       /* negative / too large M, N, K, r, or K % group != 0 */
#define CONVROT_ERR_GROUP 2       /* group is not a supported power of 4 (4, 16, 64, 256) */
#define CONVROT_ERR_ALIGN 3       /* a pointer or leading dimension breaks the 16-byte rules */
#define CONVROT_ERR_CUDA 4        /* a CUDA runtime / driver call failed */
#define CONVROT_ERR_ARCH 5        /* the current device is not sm_100 (B200 / GB200) */
#define CONVROT_ERR_TIMEOUT 6     /* a kernel's bounded wait expired (see convrot_poll_error) */
#define CONVROT_ERR_ARG 7         /* a required pointer is NULL or an option is unknown */
#define CONVROT_ERR_SCRATCH 8     /* convrot_linear_noalloc: the problem needs more than its built-in scratch */

/* Rotation arithmetic of convrot_rotate_quant. */
#define CONVROT_ROUND_KERNEL 0 /* reference CUDA path (int8.py:194-221): exact dot rounded once to fp32,
                                  q = rint(y * (1/scale)) */
#define CONVROT_ROUND_TORCH 1  /* reference torch path (int8.py:173-178), used there for M < 17 rows:
                                  exact dot rounded once to bf16, q = rint(y / scale) */
#define CONVROT_ROUND_TRITON 2 /* as CONVROT_ROUND_KERNEL, with both divisions (scale = amax / 127, inv = 1 / scale)
                                  done by PTX div.full.f32, the approximate division the reference's Triton
                                  kernels run on the GPU: its B200 codes and scales */

/*
 * Rotate + quantise (replaces int8.py:326-344).
 *   x      bf16 [M, K], leading dimension ldx (elements)
 *   q_out  int8 [M, K], leading dimension ldq; q = clamp(rint(y * inv), -127, 127)
 *   s_out  fp32 [M];    s = max(amax_k |y[m,k]|, 1e-12) / 127, inv = 1 / s
 * with y = x . blockdiag(H_group), H_group = kron(H4/2, ...) (int8.py:100-109).
 * group in {4, 16, 64, 256}; K % group == 0 and K % 16 == 0; ldx, ldq multiples of 8 / 16;
 * x, q_out 16-byte aligned.
 * Low-rank (optional): if lr_down != NULL, also xa_out[m, j] = bf16(sum_k x[m,k] * lr_down[j,k]),
 *   lr_down bf16 [r, K] (LowRankLinear.down.weight, leading dim ld_down), xa_out bf16 [M, r] (ldxa).
 */
int convrot_rotate_quant(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding,
                         int8_t* q_out, int64_t ldq, float* s_out,
                         const void* lr_down, int64_t ld_down, int64_t r, void* xa_out, int64_t ldxa,
                         void* stream);

/*
 * Low-rank down projection alone: xa[m, j] = bf16(sum_k x[m,k] * lr_down[j,k]) (transformer.py:57-58).
 * A tcgen05 bf16 GEMM with an fp32 accumulator; 1 <= r <= 256, K % 8 == 0, ldx / ld_down / ldxa multiples of 8.
 */
int convrot_lowrank_down(const void* x, int64_t ldx, const void* lr_down, int64_t ld_down,
                         int64_t M, int64_t K, int64_t r, void* xa_out, int64_t ldxa, void* stream);

/*
 * INT8 GEMM with the dequantising epilogue (replaces int8.py:376-390):
 *   y[m, n] = bf16( fp32(fp32(float(acc[m,n]) * sx[m]) * ws[n]) [+ bias[n]] [+ sum_j xa[m,j] * lr_up[n,j]] )
 *   acc[m, n] = sum_k q[m,k] * w[n,k] (exact int32)
 *   q int8 [M, K] (ldq), w int8 [N, K] (ldw, the reference's `qweight`), sx fp32 [M], ws fp32 [N] (`wscale`),
 *   bias bf16 [N] or NULL, xa bf16 [M, r] (ldxa) and lr_up bf16 [N, r] (ld_up, LowRankLinear.up.weight) or NULL,
 *   y bf16 [M, N] (ldy).
 * Without bias and low-rank the output is bitwise the reference's (int8.py:311, 324).
 * K % 16 == 0; ldq, ldw multiples of 16; ldy multiple of 8; 1 <= r <= 256 when present, with ldxa and ld_up
 * multiples of 8 (a rank that is not a multiple of 8 is read through padded rows; the padding is never read).
 */
int convrot_gemm(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                 const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                 int64_t M, int64_t N, int64_t K, void* y, int64_t ldy, void* stream);

/*
 * The raw int32 accumulator acc = q . w^T of the same tcgen05 GEMM (no epilogue arithmetic); for parity tests
 * of the accumulator (int8.py:306, 362: torch._int_mm).  acc int32 [M, N] (ldc multiple of 4).
 */
int convrot_gemm_acc(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, int64_t M, int64_t N,
                     int64_t K, int32_t* acc, int64_t ldc, void* stream);

/*
 * Packed layouts of the Ulysses all-to-all (no counterpart in the reference, whose all-to-all lives in diffusers;
 * call site distributed.py:88-96).  A packed bf16 matrix [M, C] with chunk_cols = W is stored as [C / W, M, W]:
 * element (m, c) at base[(c / W) * M * W + m * W + c % W] -- all M rows of column block 0, then block 1, ...
 * This is exactly the send buffer of all_to_all_single for seq -> head (block j goes to rank j) and the receive
 * buffer of head -> seq (block j came from rank j), so no pack or unpack copy is needed around the collective.
 *
 * convrot_gemm_packed         as convrot_gemm, writing y packed (N % chunk_cols == 0, chunk_cols % 32 == 0)
 * convrot_rotate_quant_packed as convrot_rotate_quant, reading x packed (K % chunk_cols == 0, chunk_cols % 128 == 0)
 * convrot_lowrank_down_packed as convrot_lowrank_down, reading x packed (chunk_cols % 64 == 0)
 */
int convrot_gemm_packed(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                        const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                        int64_t M, int64_t N, int64_t K, void* y, int64_t chunk_cols, void* stream);
int convrot_rotate_quant_packed(const void* x, int64_t chunk_cols, int64_t M, int64_t K, int group, int rounding,
                                int8_t* q_out, int64_t ldq, float* s_out, void* stream);
int convrot_lowrank_down_packed(const void* x, int64_t chunk_cols, const void* lr_down, int64_t ld_down, int64_t M,
                                int64_t K, int64_t r, void* xa_out, int64_t ldxa, void* stream);

/*
 * AdaLN modulation fused into the rotate+quantise prologue (no counterpart in the reference; its call site is
 * chunk_block, transformer.py:345-348, where the block computes h = norm1(x) * (1 + scale_msa[idx]) + shift_msa[idx]
 * in bf16 tensor ops before to_q / to_k / to_v).  The rotated and quantised row is
 *   h[m] = bf16( bf16( bf16(LN(x[m])) * bf16(1 + scale[idx[m]]) ) + shift[idx[m]] )
 * with LN a LayerNorm without affine parameters (mean and 1/sqrt(var + eps) from fp64 sums, each rounded once to
 * fp32; (x - mean) * rstd in fp32).  mod_scale / mod_shift are bf16 [T, K] (ld_mod), mod_index int32 [M] in [0, T).
 * h_out (optional, bf16 [M, K], ld_h) receives h for the low-rank down projection.  group 256, K % 256 == 0,
 * K <= 8192; other arguments as convrot_rotate_quant.
 */
int convrot_rotate_quant_adaln(const void* x, int64_t ldx, int64_t M, int64_t K, int group, int rounding,
                               const void* mod_scale, const void* mod_shift, const int32_t* mod_index, int64_t ld_mod,
                               float eps, int8_t* q_out, int64_t ldq, float* s_out, void* h_out, int64_t ld_h,
                               void* stream);

/*
 * A gated residual fused into the GEMM epilogue (no counterpart in the reference; its call sites are chunk_block's
 * `h = x + gate_msa[idx] * to_out(o)` and `out = h + gate_mlp[idx] * ff(n)`, transformer.py:374-378, bf16 tensor ops):
 *   y[m, n] = bf16( res[m, n] + bf16( gate[idx[m], n] * bf16(linear[m, n]) ) )
 * with linear[m, n] the convrot_gemm value (bias and low-rank included).  res bf16 [M, N] (ld_res); gate bf16 [T, N]
 * (ld_gate) or NULL (y = bf16(res + bf16(linear))); gate_index int32 [M] or NULL (row 0 of gate for every token).
 * y may be res (same leading dimension): each element is read before it is written.
 */
int convrot_gemm_residual(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx,
                          const float* ws, const void* bias, const void* xa, int64_t ldxa, const void* lr_up,
                          int64_t ld_up, int64_t r, int64_t M, int64_t N, int64_t K, const void* res, int64_t ld_res,
                          const void* gate, int64_t ld_gate, const int32_t* gate_index, void* y, int64_t ldy,
                          void* stream);

/*
 * The FFN's SwiGLU fused into the up projection's epilogue (no counterpart in the reference: diffusers' gated `net[0]`
 * runs `proj`, then `a, g = y.chunk(2, -1)`, then `a * silu(g)`; call site transformer.py:87-99).  The B operand is
 * the projection with its rows interleaved in 32-row blocks -- rows [64 j, 64 j + 32) are rows [32 j, 32 j + 32) of
 * the `a` half and rows [64 j + 32, 64 j + 64) those of the `g` half -- and ws, bias and lr_up are permuted alike.
 * N is the full projection width (a multiple of 64); h is bf16 [M, N / 2] with leading dimension ldh:
 *   h = bf16( bf16(a) * bf16( g / (1 + exp(-g)) ) ),  g = bf16(projection output), silu in fp32.
 */
int convrot_gemm_swiglu(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                        const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                        int64_t M, int64_t N, int64_t K, void* h, int64_t ldh, void* stream);

/*
 * Several linears that read one input (to_q / to_k / to_v, or a cross-attention's to_k / to_v), as ONE GEMM launch
 * (no counterpart in the reference: one convrot_gemm per layer).  Their weights are stacked along N: w, ws, bias and
 * lr_up hold `segments` layers of N / segments output columns each, and layer s writes y_chunks[s] ([M, N / segments],
 * leading dimension ldy).  Every layer has the same rank r (or none): xa is [M, segments * r] with layer s's down
 * projection in columns [s r, (s + 1) r) (what one down projection over the stacked down weights produces), and
 * lr_up's rows of layer s are its up weights.  With r > 0, N / segments must be a multiple of 256 (whole tiles per
 * layer) and r a multiple of 8; 2 <= segments <= 8.  Results are bitwise those of the separate convrot_gemm calls.
 */
int convrot_gemm_grouped(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                         const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                         int64_t M, int64_t N, int64_t K, int segments, void* const* y_chunks, int64_t ldy,
                         void* stream);

/*
 * The SwiGLU epilogue's silu alone, elementwise: y[i] = bf16( x[i] / (1 + exp(-x[i])) ) over n bf16 values, silu in
 * fp32 with IEEE division -- the bits torch's F.silu gives a bf16 CUDA tensor.  The epilogue reads these values from
 * a table over the bf16 inputs (exact: the function depends on the 16 input bits only) and evaluates the formula for
 * inputs outside it; this entry runs the same code, so one call over all 65536 bf16 patterns checks the epilogue's
 * silu against torch's.  x and y bf16 (2-byte aligned; y may be x).
 */
int convrot_silu(const void* x, void* y, int64_t n, void* stream);

/*
 * The Ulysses exchange fused into the kernels, over peer memory (no counterpart in the reference, whose all-to-all
 * is diffusers' NCCL call; call site distributed.py:88-96).  One process per GPU; every rank maps the others'
 * exchange buffers (convrot_ipc_*), so a chunk pointer below may name another GPU's memory.  At most 8 chunks.
 *
 * convrot_gemm_scatter        as convrot_gemm, writing output column chunk j (N / n_chunks columns, a multiple of
 *                             32) as [M, ldy] rows at y_chunks[j]: the seq -> head all-to-all done by the epilogue's
 *                             stores.  y_chunks is a host array of device pointers.
 * convrot_rotate_quant_gather as convrot_rotate_quant, reading row m as the concatenation over j of row m of
 *                             x_chunks[j] ([M, ldx] rows of K / n_chunks columns, a multiple of 128): the head ->
 *                             seq all-to-all done by the kernel's row copies.  x_out (optional, bf16 [M, ld_out])
 *                             receives each gathered row for the low-rank down projection.
 * convrot_ipc_handle          64-byte CUDA IPC handle of the allocation holding ptr, and ptr's offset in it.
 * convrot_ipc_open            maps another process's allocation (base address; add the offset); _close unmaps it.
 * convrot_peer_signal         stores `epoch` to each of the n flags slots[j] (host array of device pointers, usually
 *                             this rank's slot in rank j's flags) with release semantics at system scope, after the
 *                             work queued before it on the stream.
 * convrot_peer_wait           holds the stream until each of the n flags at `flags` has reached `epoch` (acquire at
 *                             system scope; compared modulo 2^32).  Bounded by the wait limit: on expiry the device
 *                             error word reads CONVROT_ERR_TIMEOUT (convrot_poll_error) and the stream continues.
 */
#define CONVROT_IPC_HANDLE_BYTES 64
int convrot_gemm_scatter(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* ws,
                         const void* bias, const void* xa, int64_t ldxa, const void* lr_up, int64_t ld_up, int64_t r,
                         int64_t M, int64_t N, int64_t K, void* const* y_chunks, int n_chunks, int64_t ldy,
                         void* stream);
int convrot_rotate_quant_gather(const void* const* x_chunks, int n_chunks, int64_t ldx, int64_t M, int64_t K,
                                int group, int rounding, int8_t* q_out, int64_t ldq, float* s_out, void* x_out,
                                int64_t ld_out, void* stream);
int convrot_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
int convrot_ipc_open(const void* handle, void** base_out);
int convrot_ipc_close(void* base);
int convrot_peer_signal(uint32_t* const* slots, int n, uint32_t epoch, void* stream);
int convrot_peer_wait(const uint32_t* flags, int n, uint32_t epoch, void* stream);

/*
 * n device-to-device block copies on `stream`, dst[j] <- src[j] (bytes[j] each, 0 skips), one cudaMemcpyAsync per
 * block so that the GPU's copy engines move them (no counterpart in the reference: exchange plumbing).  Used by the
 * peer exchange for layers whose output is written locally and then copied into the other GPUs' receive buffers
 * while the next GEMM runs on the SMs.  At most 64 blocks.
 */
int convrot_copy_blocks(void* const* dst, const void* const* src, const size_t* bytes, int n, void* stream);

/*
 * Workspace for convrot_linear: q (int8 [M, K] with rows padded to a multiple of 16 bytes), s (fp32 [M]) and xa
 * (bf16 [M, r] with rows padded to a multiple of 8 elements), each 256-byte aligned.  Exactly the size
 * convrot_linear requires; 0 for negative arguments.
 */
size_t convrot_workspace_size(int64_t M, int64_t K, int64_t r);

/*
 * The whole layer (int8.py:161-171 kernel branch + bias + low-rank): rotate+quantise into `workspace`
 * (convrot_workspace_size bytes, 256-byte aligned), then the GEMM.  Arguments as above.
 */
int convrot_linear(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* ws, const void* bias,
                   const void* lr_down, int64_t ld_down, const void* lr_up, int64_t ld_up, int64_t r,
                   int64_t M, int64_t N, int64_t K, int group, void* workspace, size_t workspace_bytes,
                   void* y, int64_t ldy, void* stream);

/*
 * The whole layer without any allocation (no counterpart in the reference): the same computation as
 * convrot_linear, with the workspace replaced by scratch built into the library.
 *
 * For callers that cannot allocate device memory on the call path: hosts that own all device memory and forbid
 * allocations once serving has started (a fixed arena planned at start-up), plugin-style interfaces whose enqueue
 * call hands over only the inputs, the outputs and a stream, and code that must not call cudaMalloc / cudaFree
 * because those can synchronise the device and stall every other stream.  This function calls no cudaMalloc,
 * cudaFree or allocating library routine.
 *
 * Limit: the codes, scales and low-rank input of one call must fit CONVROT_NOALLOC_SCRATCH_BYTES (16 MiB), i.e.
 * convrot_workspace_size(M, K, r) <= 16 MiB (for example M = 3072 rows at K = 5120);
 * larger problems return CONVROT_ERR_SCRATCH without launching anything.  The scratch is part of the library's
 * device image: every GPU that loads the library holds those 16 MiB until the process exits.
 *
 * Set-up: the first call on a device (with that device current) looks up the scratch's device address once;
 * make that first call before any stream capture.
 *
 * Sharing: all calls, on all streams, use the same scratch and it keeps the last call's contents.  Nothing in it
 * has to start at zero (each call writes its codes, scales and low-rank input before reading them), but calls
 * whose work overlaps on the GPU race on the scratch: order them on one stream, or otherwise make one finish
 * before the next starts.
 */
#define CONVROT_NOALLOC_SCRATCH_BYTES (16u << 20)
int convrot_linear_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* ws,
                           const void* bias, const void* lr_down, int64_t ld_down, const void* lr_up, int64_t ld_up,
                           int64_t r, int64_t M, int64_t N, int64_t K, int group, void* y, int64_t ldy,
                           void* stream);

/* Name of a status code. */
const char* convrot_status_string(int status);

/* The last CUDA error code seen by a call on this host thread (0 if none). */
int convrot_last_cuda_error(void);

/*
 * Device-side error word of the current device: nonzero after a kernel's bounded wait expired
 * (CONVROT_ERR_TIMEOUT); reading it synchronises `stream` and clears the word.
 */
int convrot_poll_error(void* stream);

/* Bounded-wait limit of the GEMM kernels, in nanoseconds of %globaltimer (default 2e9). */
void convrot_set_wait_limit_ns(uint64_t ns);

/*
 * Which INT8 GEMM kernel convrot_gemm / convrot_gemm_acc / convrot_linear launch: 0 = automatic (the 2-SM
 * cta_group::2 kernel with 256 x 256 tiles per CTA pair, unless the 1-SM 128 x 256 kernel's tiles fit one wave on
 * the GPU's SMs or need fewer waves than the pairs' tiles; M <= 128 always takes the 1-SM kernel),
 * 1 = always the 1-SM kernel, 2 = always the 2-SM kernel.  Both give bitwise identical results.
 * Process-wide; returns CONVROT_ERR_ARG for other values.
 */
int convrot_set_gemm_mode(int mode);

/*
 * Kernel for group 256 in convrot_rotate_quant: 0 = automatic (the two-column team kernel for K <= 8192, else the
 * one-column kernel used for the other groups), 1 = always one-column, 2 = always two-column.  All are bit-exact;
 * the switch exists so tests cover each kernel.
 */
int convrot_set_rotate_variant(int variant);

/*
 * Launch shape of convrot_rotate_quant: row buffers per CTA (1..8) and CTAs per SM (1..32); 0 keeps the automatic
 * choice.  Performance tuning only; results do not depend on it.
 */
int convrot_set_rotate_tuning(int stages, int ctas_per_sm);

/* Library version (major * 10000 + minor * 100 + patch). */
int convrot_version(void);

/*
 * How many low-rank down projections of this process ran without their K split (no counterpart in the reference).
 * Down projections with M <= 1024 split K over a cluster of 2-8 CTAs; if the GPU cannot place such a cluster the
 * launch runs the unsplit kernel instead, whose different fp32 summation order can change the last bf16 bit of xa
 * (and so of the low-rank term).  Any other launch error is returned as CONVROT_ERR_CUDA, never absorbed.
 */
int64_t convrot_split_k_fallbacks(void);

#ifdef __cplusplus
}
#endif

#endif /* CONVROT_H_ */
