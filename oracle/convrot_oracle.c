/*
 * CPU oracle for the INT8 "convrot" linear -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's hot path
 * (hyperflow_h3_flash, src/hyperflow_h3_flash/int8.py) so that the CUDA kernels of
 * this repository can be checked bit for bit.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it; the product path never does.
 *
 * Semantics restated ("kernel semantics", the reference's Triton path):
 *   - rotation  y = x . blockdiag(H_G), H_G = kron(H4/2, ..., H4/2)       int8.py:100-109
 *     with the dot accumulated exactly and rounded ONCE to fp32
 *     (int8.py:211,219: tl.dot of bf16 x and bf16 H into an fp32 accumulator);
 *   - scale = fp32(max(amax, 1e-12f) / 127), inv = fp32(1 / scale)        int8.py:212-214
 *     (IEEE round-to-nearest divisions);
 *   - q = clamp(rint(fp32(y * inv)), -127, 127), rint = half-to-even      int8.py:219-220
 *   - acc = sum_k q[m,k] * w[n,k] exactly (int32)                         int8.py:306, 362
 *   - out = bf16_rn(fp32(fp32(float(acc) * sa[m]) * sb[n]))               int8.py:311, 324
 * and the CPU path's variant (int8.py:173-179): the rotation rounded to bf16,
 * then q = clamp(rint(fp32(xr / sx)), -127, 127).
 *
 * Exactness: a group's exact dot is formed in 128-bit fixed point with a fast
 * Walsh-type transform (every partial sum is an integer multiple of the group's
 * smallest bf16 quantum); groups whose bf16 exponents span too far for 128 bits
 * go through a 320-bit super-accumulator instead.  Either way the sum is exact
 * and is rounded once, to nearest-even, including fp32/bf16 subnormal results.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, pthreads).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef __int128 i128;
typedef unsigned __int128 u128;

/* ---------------------------------------------------------------- helpers */

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* fp32 -> bf16, round to nearest even (what torch's .to(bfloat16) and the GPU's cvt.rn do). */
static inline uint16_t f32_to_bf16_rn(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* value = (-1)^neg * m * 2^E with m < 2^8; returns -1 for inf/NaN. */
static inline int bf16_split(uint16_t b, int* neg, uint32_t* m, int* E) {
  int e = (b >> 7) & 0xff;
  uint32_t f = b & 0x7fu;
  *neg = b >> 15;
  if (e == 0xff) return -1;
  if (e == 0) { *m = f; *E = -133; }           /* f/128 * 2^-126 */
  else { *m = 128u | f; *E = e - 134; }        /* (1 + f/128) * 2^(e-127) */
  return 0;
}

static inline int bitlen_u128(u128 v) {
  uint64_t hi = (uint64_t)(v >> 64), lo = (uint64_t)v;
  if (hi) return 128 - __builtin_clzll(hi);
  if (lo) return 64 - __builtin_clzll(lo);
  return 0;
}

/*
 * Round (-1)^neg * mag * 2^base to nearest-even in a binary format with a p-bit
 * significand whose smallest quantum is 2^qmin and whose largest finite value is
 * below 2^emax_excl.  `sticky` says that nonzero bits lie below mag's bit 0.
 * The result is returned as a double (exactly representable for p <= 24).
 */
static double round_fixed(int neg, u128 mag, int base, int sticky, int p, int qmin, int emax_excl) {
  if (mag == 0) return neg ? -0.0 : 0.0;
  int n = bitlen_u128(mag);
  int e_msb = base + n - 1;
  int q = e_msb - (p - 1);
  if (q < qmin) q = qmin;
  int shift = q - base;
  u128 M;
  if (shift <= 0) {
    M = mag << (-shift); /* exact; sticky bits are below half a quantum and cannot matter */
  } else if (shift > 127) {
    M = 0; /* everything is below half a quantum (mag < 2^127 <= 2^(shift-1)) */
  } else {
    M = mag >> shift;
    u128 rem = mag & ((((u128)1) << shift) - 1);
    u128 half = ((u128)1) << (shift - 1);
    if (rem > half || (rem == half && (sticky || (M & 1)))) M += 1;
  }
  double v = ldexp((double)M, q);
  if (v >= ldexp(1.0, emax_excl)) v = INFINITY;
  return neg ? -v : v;
}

static inline float round_to_f32(int neg, u128 mag, int base, int sticky) {
  return (float)round_fixed(neg, mag, base, sticky, 24, -149, 128);
}

static inline uint16_t round_to_bf16_bits(int neg, u128 mag, int base, int sticky) {
  double v = round_fixed(neg, mag, base, sticky, 8, -133, 128);
  float f = (float)v; /* exact: v has at most 8 significant bits */
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------- exact group rotation */

static int log4_of(int g) {
  int L = 0, n = 1;
  while (n < g) { n *= 4; L++; }
  return n == g ? L : -1;
}

/*
 * Signed exact sums W = H' x, H' = kron(H4', ..., H4') with the integer
 * H4' = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]] = 2 (H4/2).
 * H4' v = (v0+v1+v2+v3) - 2 reverse(v).  Returns the common base exponent, so
 * that y_j = W_j * 2^(base) with the 2^-L of H_G folded into base.
 * Returns INT32_MIN when the exponent span is too wide for 128 bits.
 */
static int group_fixed_i128(const uint16_t* x, int G, int L, i128* W, int* nonfinite) {
  int Emin = 1 << 20, Emax = -(1 << 20);
  *nonfinite = 0;
  for (int i = 0; i < G; i++) {
    int neg, E;
    uint32_t m;
    if (bf16_split(x[i], &neg, &m, &E)) { *nonfinite = 1; return 0; }
    if (m == 0) continue;
    if (E < Emin) Emin = E;
    if (E > Emax) Emax = E;
  }
  if (Emax < Emin) { /* all zeros */
    for (int i = 0; i < G; i++) W[i] = 0;
    return 0;
  }
  if (Emax - Emin > 100) return INT32_MIN;
  for (int i = 0; i < G; i++) {
    int neg, E;
    uint32_t m;
    bf16_split(x[i], &neg, &m, &E);
    i128 v = m ? ((i128)m << (E - Emin)) : 0;
    W[i] = neg ? -v : v;
  }
  for (int stride = 1; stride < G; stride *= 4) {
    for (int blk = 0; blk < G; blk += 4 * stride) {
      for (int j = 0; j < stride; j++) {
        i128* p = W + blk + j;
        i128 a = p[0], b = p[stride], c = p[2 * stride], d = p[3 * stride];
        i128 s = a + b + c + d;
        p[0] = s - 2 * d;
        p[stride] = s - 2 * c;
        p[2 * stride] = s - 2 * b;
        p[3 * stride] = s - 2 * a;
      }
    }
  }
  return Emin - L;
}

/* sign of H_G[i][j] (+1 or -1): product over base-4 digits of H4' entries. */
static inline int hsign(int i, int j, int L) {
  int s = 1;
  for (int d = 0; d < L; d++) {
    int a = (i >> (2 * d)) & 3, b = (j >> (2 * d)) & 3;
    if (a + b == 3) s = -s; /* H4' is -1 exactly on the anti-diagonal */
  }
  return s;
}

/*
 * Super-accumulator path: exact dense sum y_j = sum_i sign_ij x_i for groups whose
 * exponent span is too wide for 128 bits.  32-bit digits held in int64 cover
 * every bf16 quantum (2^-133) up to 2^160 with room for 2^20 terms.
 */
#define SA_DIGITS 10
#define SA_BIAS 133
static void group_slow_one(const uint16_t* x, int G, int L, int j, int* neg_out, u128* mag_out,
                           int* base_out, int* sticky_out) {
  int64_t acc[SA_DIGITS + 1];
  memset(acc, 0, sizeof(acc));
  for (int i = 0; i < G; i++) {
    int neg, E;
    uint32_t m;
    bf16_split(x[i], &neg, &m, &E);
    if (!m) continue;
    if (hsign(i, j, L) < 0) neg = !neg;
    int b = E + SA_BIAS;                 /* bit index of m's LSB, >= 0 */
    int d = b >> 5, r = b & 31;
    uint64_t t = (uint64_t)m << r;       /* < 2^39 */
    int64_t lo = (int64_t)(t & 0xffffffffu), hi = (int64_t)(t >> 32);
    if (neg) { lo = -lo; hi = -hi; }
    acc[d] += lo;
    acc[d + 1] += hi;
  }
  /* normalise to digits in [0, 2^32) with a signed top carry */
  for (int d = 0; d < SA_DIGITS; d++) {
    int64_t c = acc[d] >> 32; /* arithmetic shift = floor division */
    acc[d] -= c << 32;
    acc[d + 1] += c;
  }
  int neg = acc[SA_DIGITS] < 0;
  if (neg) { /* two's complement negate over the digit string */
    int64_t carry = 1;
    for (int d = 0; d < SA_DIGITS; d++) {
      int64_t v = (int64_t)(~(uint64_t)acc[d] & 0xffffffffu) + carry;
      acc[d] = v & 0xffffffff;
      carry = v >> 32;
    }
  }
  int top = SA_DIGITS - 1;
  while (top >= 0 && acc[top] == 0) top--;
  if (top < 0) { *neg_out = 0; *mag_out = 0; *base_out = 0; *sticky_out = 0; return; }
  /* take the top three digits (96 bits) as the window, OR the rest into sticky */
  u128 mag = 0;
  int lowest = top - 2 < 0 ? 0 : top - 2;
  for (int d = top; d >= lowest; d--) mag = (mag << 32) | (u128)(uint64_t)acc[d];
  int sticky = 0;
  for (int d = 0; d < lowest; d++) sticky |= acc[d] != 0;
  *neg_out = neg;
  *mag_out = mag;
  *base_out = lowest * 32 - SA_BIAS - L;
  *sticky_out = sticky;
}

/*
 * Rotate one row (K = n_groups * G bf16 values) exactly.  out_f32 receives the
 * fp32-rounded values (kernel semantics), out_bf16 (if non-null) the bf16-rounded
 * ones (CPU-path semantics).  Returns the number of groups that needed the slow path,
 * or -1 on a non-finite input.
 */
static int rotate_row(const uint16_t* x, int K, int G, int L, float* out_f32, uint16_t* out_bf16, i128* W) {
  int slow = 0;
  for (int g0 = 0; g0 < K; g0 += G) {
    int nonfinite = 0;
    int base = group_fixed_i128(x + g0, G, L, W, &nonfinite);
    if (nonfinite) return -1;
    if (base == INT32_MIN) {
      slow++;
      for (int j = 0; j < G; j++) {
        int neg, sticky, b;
        u128 mag;
        group_slow_one(x + g0, G, L, j, &neg, &mag, &b, &sticky);
        out_f32[g0 + j] = round_to_f32(neg, mag, b, sticky);
        if (out_bf16) out_bf16[g0 + j] = round_to_bf16_bits(neg, mag, b, sticky);
      }
      continue;
    }
    for (int j = 0; j < G; j++) {
      i128 w = W[j];
      int neg = w < 0;
      u128 mag = neg ? (u128)(-w) : (u128)w;
      out_f32[g0 + j] = round_to_f32(neg, mag, base, 0);
      if (out_bf16) out_bf16[g0 + j] = round_to_bf16_bits(neg, mag, base, 0);
    }
  }
  return slow;
}

/* ------------------------------------------------------- parallel-for */

#include <pthread.h>
#include <unistd.h>

typedef void (*range_fn)(void* ctx, int begin, int end);
typedef struct { range_fn fn; void* ctx; int begin, end; } range_job;

static void* range_thread(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

static int oracle_threads = 0; /* 0 = all online CPUs */

void oracle_set_threads(int n) { oracle_threads = n; }

int oracle_get_threads(void) {
  if (oracle_threads > 0) return oracle_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* Runs fn over [0, n) split into contiguous chunks, one per thread; returns when all are done. */
static void par_for(int n, range_fn fn, void* ctx) {
  int T = oracle_get_threads();
  if (T > n) T = n;
  if (T <= 1) { if (n > 0) fn(ctx, 0, n); return; }
  pthread_t th[256];
  range_job jobs[256];
  if (T > 256) T = 256;
  for (int t = 0; t < T; t++) {
    jobs[t].fn = fn;
    jobs[t].ctx = ctx;
    jobs[t].begin = (int)((int64_t)n * t / T);
    jobs[t].end = (int)((int64_t)n * (t + 1) / T);
  }
  int started = 0;
  for (int t = 1; t < T; t++) {
    if (pthread_create(&th[t], NULL, range_thread, &jobs[t]) != 0) break;
    started = t;
  }
  fn(ctx, jobs[0].begin, jobs[0].end);
  for (int t = started + 1; t < T; t++) fn(ctx, jobs[t].begin, jobs[t].end); /* threads that failed to start */
  for (int t = 1; t <= started; t++) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------- public API */

typedef struct {
  const uint16_t* x; int64_t ldx; int K, G, L;
  float* y_f32; uint16_t* y_bf16;
  int8_t* q; int64_t ldq; float* s;
  int mode; /* 0 = rotate only, 1 = kernel-semantics quant, 2 = CPU-path quant */
  pthread_mutex_t mu; int bad, slow;
} rot_ctx;

static void rot_range(void* p, int begin, int end) {
  rot_ctx* c = (rot_ctx*)p;
  int K = c->K;
  i128* W = (i128*)malloc(sizeof(i128) * (size_t)c->G);
  float* y = (float*)malloc(sizeof(float) * (size_t)K);
  uint16_t* yb = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)K);
  int bad = 0, slow = 0;
  for (int m = begin; m < end; m++) {
    const uint16_t* xr = c->x + (int64_t)m * c->ldx;
    if (c->mode == 0) {
      int r = rotate_row(xr, K, c->G, c->L, c->y_f32 + (int64_t)m * K, c->y_bf16 ? c->y_bf16 + (int64_t)m * K : NULL, W);
      if (r < 0) bad = 1; else slow += r;
      continue;
    }
    int r = rotate_row(xr, K, c->G, c->L, y, c->mode == 2 ? yb : NULL, W);
    if (r < 0) { bad = 1; continue; }
    slow += r;
    int8_t* qrow = c->q + (int64_t)m * c->ldq;
    float amax = 0.0f;
    if (c->mode == 1) {
      for (int k = 0; k < K; k++) amax = fmaxf(amax, fabsf(y[k]));
      float scale = (float)((double)fmaxf(amax, 1e-12f) / 127.0); /* IEEE fp32 division */
      float inv = (float)(1.0 / (double)scale);                   /* IEEE fp32 division */
      c->s[m] = scale;
      for (int k = 0; k < K; k++) {
        float v = y[k] * inv; /* fp32 multiply, RN */
        float r8 = rintf(v);  /* half to even */
        if (r8 > 127.0f) r8 = 127.0f;
        if (r8 < -127.0f) r8 = -127.0f;
        qrow[k] = (int8_t)r8;
      }
    } else {
      for (int k = 0; k < K; k++) amax = fmaxf(amax, fabsf(bf16_to_f32(yb[k])));
      float sx = (float)((double)fmaxf(amax, 1e-12f) / 127.0);
      c->s[m] = sx;
      for (int k = 0; k < K; k++) {
        float v = (float)((double)bf16_to_f32(yb[k]) / (double)sx); /* IEEE fp32 division */
        float r8 = rintf(v);
        if (r8 > 127.0f) r8 = 127.0f;
        if (r8 < -127.0f) r8 = -127.0f;
        qrow[k] = (int8_t)r8;
      }
    }
  }
  free(W); free(y); free(yb);
  pthread_mutex_lock(&c->mu);
  c->bad |= bad;
  c->slow += slow;
  pthread_mutex_unlock(&c->mu);
}

static int rot_run(rot_ctx* c, int M) {
  c->L = log4_of(c->G);
  if (c->L < 0 || c->K % c->G) return -2;
  pthread_mutex_init(&c->mu, NULL);
  c->bad = 0;
  c->slow = 0;
  par_for(M, rot_range, c);
  pthread_mutex_destroy(&c->mu);
  return c->bad ? -1 : c->slow;
}

/* Rotated activations only: fp32 (kernel semantics) and, if y_bf16 is non-null, bf16 (CPU semantics).
 * Returns the number of groups that took the wide-span path, -1 on non-finite input, -2 on bad shape. */
int oracle_rotate(const uint16_t* x, int64_t ldx, int M, int K, int G, float* y_f32, uint16_t* y_bf16) {
  rot_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x; c.ldx = ldx; c.K = K; c.G = G; c.y_f32 = y_f32; c.y_bf16 = y_bf16; c.mode = 0;
  return rot_run(&c, M);
}

/* Kernel-semantics rotate + per-token quantisation (int8.py:194-221). */
int oracle_rotate_quant(const uint16_t* x, int64_t ldx, int M, int K, int G, int8_t* q, int64_t ldq, float* s) {
  rot_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x; c.ldx = ldx; c.K = K; c.G = G; c.q = q; c.ldq = ldq; c.s = s; c.mode = 1;
  return rot_run(&c, M);
}

/* CPU-path semantics (int8.py:173-178): bf16-rounded rotation, q = rint(xr / sx). */
int oracle_rotate_quant_cpu(const uint16_t* x, int64_t ldx, int M, int K, int G, int8_t* q, int64_t ldq, float* s) {
  rot_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x; c.ldx = ldx; c.K = K; c.G = G; c.q = q; c.ldq = ldq; c.s = s; c.mode = 2;
  return rot_run(&c, M);
}

typedef struct {
  const int8_t* a; int64_t lda; const int8_t* b; int64_t ldb; int N, K; int32_t* acc; int64_t ldc;
  volatile int overflow;
} gemm_ctx;

static void gemm_range(void* p, int begin, int end) {
  gemm_ctx* c = (gemm_ctx*)p;
  for (int m = begin; m < end; m++) {
    const int8_t* ar = c->a + (int64_t)m * c->lda;
    for (int n = 0; n < c->N; n++) {
      const int8_t* br = c->b + (int64_t)n * c->ldb;
      int64_t s = 0;
      for (int k = 0; k < c->K; k++) s += (int32_t)ar[k] * (int32_t)br[k];
      if (s > INT32_MAX || s < INT32_MIN) c->overflow = 1;
      c->acc[(int64_t)m * c->ldc + n] = (int32_t)s;
    }
  }
}

/* acc[m,n] = sum_k a[m,k] * b[n,k] exactly (int8.py:306, 362); returns -3 if a sum leaves int32. */
int oracle_int8_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int M, int N, int K, int32_t* acc,
                     int64_t ldc) {
  gemm_ctx c = {a, lda, b, ldb, N, K, acc, ldc, 0};
  par_for(M, gemm_range, &c);
  return c.overflow ? -3 : 0;
}

typedef struct {
  const int32_t* acc; int64_t ldc; const float* sa; const float* sb; const uint16_t* bias;
  const uint16_t* xa; int64_t ldxa; const uint16_t* B; int64_t ldb; int r, N; uint16_t* out; int64_t ldo;
} epi_ctx;

static void epi_range(void* p, int begin, int end) {
  epi_ctx* c = (epi_ctx*)p;
  for (int m = begin; m < end; m++) {
    for (int n = 0; n < c->N; n++) {
      float t = (float)c->acc[(int64_t)m * c->ldc + n] * c->sa[m];
      t = t * c->sb[n];
      if (c->bias) t = t + bf16_to_f32(c->bias[n]);
      if (c->xa && c->B && c->r > 0) {
        float lr = 0.0f;
        for (int k = 0; k < c->r; k++)
          lr = fmaf(bf16_to_f32(c->xa[(int64_t)m * c->ldxa + k]), bf16_to_f32(c->B[(int64_t)k * c->ldb + n]), lr);
        t = t + lr;
      }
      c->out[(int64_t)m * c->ldo + n] = f32_to_bf16_rn(t);
    }
  }
}

/*
 * Epilogue (int8.py:311, 324): t = fp32(fp32(float(acc) * sa[m]) * sb[n]) -> bf16 (RNE).
 * With bias (bf16 [N]) and/or the low-rank term (xa bf16 [M,r], B bf16 [r,N]):
 * out = bf16_rn((t + bias[n]) + lr), lr = sum_k xa[m,k] * B[k,n] as fp32 fma in order k = 0..r-1.
 * The bias / low-rank part has no reference counterpart; tests compare it with a tolerance.
 */
void oracle_epilogue(const int32_t* acc, int64_t ldc, const float* sa, const float* sb, const uint16_t* bias,
                     const uint16_t* xa, int64_t ldxa, const uint16_t* B, int64_t ldb, int r, int M, int N,
                     uint16_t* out, int64_t ldo) {
  epi_ctx c = {acc, ldc, sa, sb, bias, xa, ldxa, B, ldb, r, N, out, ldo};
  par_for(M, epi_range, &c);
}

typedef struct {
  const uint16_t* x; int64_t ldx; const uint16_t* A; int64_t lda; int K, r; uint16_t* xa; int64_t ldxa;
} down_ctx;

static void down_range(void* p, int begin, int end) {
  down_ctx* c = (down_ctx*)p;
  for (int m = begin; m < end; m++) {
    for (int k = 0; k < c->r; k++) {
      double s = 0.0;
      for (int i = 0; i < c->K; i++)
        s += (double)bf16_to_f32(c->x[(int64_t)m * c->ldx + i]) * (double)bf16_to_f32(c->A[(int64_t)i * c->lda + k]);
      c->xa[(int64_t)m * c->ldxa + k] = f32_to_bf16_rn((float)s);
    }
  }
}

/* Low-rank down projection xa = bf16_rn(x . A) (transformer.py:57-58, `down` of LowRankLinear), summed in fp64. */
void oracle_lowrank_down(const uint16_t* x, int64_t ldx, const uint16_t* A, int64_t lda, int M, int K, int r,
                         uint16_t* xa, int64_t ldxa) {
  down_ctx c = {x, ldx, A, lda, K, r, xa, ldxa};
  par_for(M, down_range, &c);
}

/* fp32 -> bf16 bits, round to nearest even. */
void oracle_f32_to_bf16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = f32_to_bf16_rn(x[i]);
}

int oracle_version(void) { return 1; }
