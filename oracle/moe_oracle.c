/*
 * C restatement of the com.microsoft MoE / QMoE CPU path -- TEST INFRASTRUCTURE ONLY.
 *
 * Used as the timed CPU baseline of bench.py (kind "port") and cross-checked against
 * oracle/moe_oracle.py by the CPU tests.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it; the product path never does.
 *
 * PARITY UNPINNED: the arithmetic of this path is defined by the ONNX Runtime 1.26.0
 * CPU EP (commit 8c546c37b43caaca1fa25db430dab94b901cf277, an un-vendored submodule of
 * the reference, third_party/README.md:5-6), whose source is not available here.  The
 * contract restated is documented in oracle/moe_oracle.py; this file follows it with
 * fp32 storage and fp32 (vectorised) accumulation, multi-threaded with pthreads over
 * output columns the way a CPU GEMM library would be (thread count: oracle_set_threads,
 * default = online cores).
 *
 * Routing follows musa/ep/src/kernels/math/topk_impl.mu:46-65 (ties -> lower index)
 * and the softmax of musa/ep/src/kernels/math/softmax_impl.mu:49-84.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <unistd.h>
#include <stdlib.h>
#include <string.h>

enum { ACT_RELU = 0, ACT_GELU = 1, ACT_SILU = 2, ACT_IDENTITY = 3, ACT_SWIGLU = 4 };

static float act1(int act, float x) {
  switch (act) {
    case ACT_RELU: return x > 0.f ? x : 0.f;
    case ACT_GELU: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
    case ACT_SILU: return x / (1.f + expf(-x));
    default: return x;
  }
}

/* ------------------------------------------------------------ parallel for */
static int g_threads = 0;

void oracle_set_threads(int n) { g_threads = n; }
int oracle_get_threads(void) {
  if (g_threads <= 0) {
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    g_threads = c > 0 ? (int)c : 1;
  }
  return g_threads;
}

typedef void (*range_fn)(int64_t begin, int64_t end, void* ctx);
typedef struct { range_fn fn; void* ctx; int64_t begin, end; } range_job;

static void* run_range(void* p) {
  range_job* j = (range_job*)p;
  if (j->begin < j->end) j->fn(j->begin, j->end, j->ctx);
  return NULL;
}

/* Splits [0, n) into contiguous ranges, one per thread. */
static void parallel_for(int64_t n, range_fn fn, void* ctx) {
  int nt = oracle_get_threads();
  if (nt > 256) nt = 256;
  if (n < nt) nt = n > 0 ? (int)n : 1;
  if (nt <= 1) { fn(0, n, ctx); return; }
  pthread_t th[256];
  range_job jobs[256];
  for (int i = 0; i < nt; ++i) {
    jobs[i].fn = fn; jobs[i].ctx = ctx;
    jobs[i].begin = n * i / nt; jobs[i].end = n * (i + 1) / nt;
  }
  for (int i = 1; i < nt; ++i) pthread_create(&th[i], NULL, run_range, &jobs[i]);
  run_range(&jobs[0]);
  for (int i = 1; i < nt; ++i) pthread_join(th[i], NULL);
}

/* Routing of one row: top-k with ties to the lower index, weights per the
 * normalize_routing_weights rule.  Returns nothing; fills idx[k], w[k]. */
static void route_row(const float* l, int E, int k, int normalize, int32_t* idx, float* w) {
  unsigned char taken[1024];
  memset(taken, 0, (size_t)E);
  double m = -INFINITY;
  for (int e = 0; e < E; ++e) if (l[e] > m) m = l[e];
  for (int r = 0; r < k; ++r) {
    int bi = -1;
    float bv = -INFINITY;
    for (int e = 0; e < E; ++e) {
      if (taken[e]) continue;
      float v = l[e] != l[e] ? -INFINITY : l[e];
      if (bi < 0 || v > bv) { bi = e; bv = v; }
    }
    taken[bi] = 1;
    idx[r] = bi;
  }
  double s = 0.0;
  if (normalize) {
    double top = l[idx[0]];
    for (int r = 0; r < k; ++r) s += exp((double)l[idx[r]] - top);
    for (int r = 0; r < k; ++r) w[r] = (float)(exp((double)l[idx[r]] - top) / s);
  } else {
    for (int e = 0; e < E; ++e) s += exp((double)l[e] - m);
    for (int r = 0; r < k; ++r) w[r] = (float)(exp((double)l[idx[r]] - m) / s);
  }
}

typedef struct { const float* logits; int E, k, normalize; int32_t* idx; float* w; } route_ctx;

static void route_range(int64_t b, int64_t e, void* p) {
  route_ctx* c = (route_ctx*)p;
  for (int64_t t = b; t < e; ++t)
    route_row(c->logits + t * c->E, c->E, c->k, c->normalize, c->idx + t * c->k, c->w + t * c->k);
}

void oracle_route(const float* logits, int64_t T, int E, int k, int normalize, int32_t* idx,
                  float* w) {
  route_ctx c = {logits, E, k, normalize, idx, w};
  parallel_for(T, route_range, &c);
}

/* C[m][n] = sum_k A[m][k] * B[n][k] (+ bias[n]); A [M,K], B [N,K], C [M,N].
 *
 * Cache-blocked and register-tiled the way a CPU GEMM library blocks it: each thread
 * owns a range of 16-column panels of C; per KC-deep slice of K it packs a panel of B
 * transposed ([KC][16], L1-resident) and sweeps all rows of A in 6-row micro-tiles,
 * whose 6x16 accumulators stay in registers (12 8-wide vectors) over the slice.  The
 * A slice [M, KC] is reused from L2 across the thread's panels.  Sums run in ascending
 * k within and across slices (fp32). */
typedef float v8 __attribute__((vector_size(32)));
enum { GEMM_MR = 6, GEMM_NR = 16, GEMM_KC = 256 };

typedef struct { const float *A, *B, *bias; float* C; int64_t M, N, K; } gemm_ctx;

/* acc[MR][NR] = sum over kc of a[r][k] * bp[k][0..NR) for the MR rows a[r]. */
static void gemm_micro(int64_t kc, const float* const* a, const float* bp, float* acc) {
  v8 c0[GEMM_MR], c1[GEMM_MR];
  for (int r = 0; r < GEMM_MR; ++r) { c0[r] = (v8){0}; c1[r] = (v8){0}; }
  for (int64_t k = 0; k < kc; ++k) {
    v8 b0, b1;
    memcpy(&b0, bp + k * GEMM_NR, sizeof(v8));
    memcpy(&b1, bp + k * GEMM_NR + 8, sizeof(v8));
    for (int r = 0; r < GEMM_MR; ++r) {
      const float av = a[r][k];
      c0[r] += av * b0;
      c1[r] += av * b1;
    }
  }
  for (int r = 0; r < GEMM_MR; ++r) {
    memcpy(acc + r * GEMM_NR, &c0[r], sizeof(v8));
    memcpy(acc + r * GEMM_NR + 8, &c1[r], sizeof(v8));
  }
}

/* The same micro-tile on AVX-512 hosts: 12 rows of 16 accumulators, one 16-wide vector
 * each (selected at run time; the library itself is built for AVX2). */
typedef float v16 __attribute__((vector_size(64)));
enum { GEMM_MR16 = 12 };

__attribute__((target("avx512f"))) static void gemm_micro16(int64_t kc, const float* const* a,
                                                              const float* bp, float* acc) {
  v16 c[GEMM_MR16];
  for (int r = 0; r < GEMM_MR16; ++r) c[r] = (v16){0};
  for (int64_t k = 0; k < kc; ++k) {
    v16 b;
    memcpy(&b, bp + k * GEMM_NR, sizeof(v16));
    for (int r = 0; r < GEMM_MR16; ++r) c[r] += a[r][k] * b;
  }
  for (int r = 0; r < GEMM_MR16; ++r) memcpy(acc + r * GEMM_NR, &c[r], sizeof(v16));
}

static int use_avx512(void) {
  static int v = -1;
  if (v < 0) v = __builtin_cpu_supports("avx512f") ? 1 : 0;
  return v;
}

static void gemm_range(int64_t p_begin, int64_t p_end, void* p) {
  gemm_ctx* g = (gemm_ctx*)p;
  const float *A = g->A, *B = g->B, *bias = g->bias;
  float* C = g->C;
  const int64_t M = g->M, N = g->N, K = g->K;
  float* bp = (float*)aligned_alloc(64, sizeof(float) * GEMM_KC * GEMM_NR);
  float* zero = (float*)calloc((size_t)(K > 0 ? K : 1), sizeof(float));
  float acc[GEMM_MR16 * GEMM_NR];
  const int wide = use_avx512();
  const int64_t mr = wide ? GEMM_MR16 : GEMM_MR;
  for (int64_t k0 = 0; k0 < K; k0 += GEMM_KC) {
    const int64_t kc = K - k0 < GEMM_KC ? K - k0 : GEMM_KC;
    for (int64_t pn = p_begin; pn < p_end; ++pn) {
      const int64_t n0 = pn * GEMM_NR;
      const int64_t nn = N - n0 < GEMM_NR ? N - n0 : GEMM_NR;
      for (int64_t j = 0; j < GEMM_NR; ++j) {  /* pack B[n0+j][k0..k0+kc) as bp[k][j] */
        const float* b = j < nn ? B + (n0 + j) * K + k0 : zero;
        for (int64_t k = 0; k < kc; ++k) bp[k * GEMM_NR + j] = b[k];
      }
      for (int64_t m0 = 0; m0 < M; m0 += mr) {
        const float* a[GEMM_MR16];
        const int64_t mm = M - m0 < mr ? M - m0 : mr;
        for (int r = 0; r < GEMM_MR16; ++r) a[r] = r < mm ? A + (m0 + r) * K + k0 : zero;
        if (wide) gemm_micro16(kc, a, bp, acc);
        else gemm_micro(kc, a, bp, acc);
        for (int64_t r = 0; r < mm; ++r) {
          float* c = C + (m0 + r) * N + n0;
          const float* s = acc + r * GEMM_NR;
          if (k0 == 0) for (int64_t j = 0; j < nn; ++j) c[j] = s[j];
          else for (int64_t j = 0; j < nn; ++j) c[j] += s[j];
        }
      }
    }
  }
  if (K == 0)
    for (int64_t m = 0; m < M; ++m)
      for (int64_t n = p_begin * GEMM_NR; n < N && n < p_end * GEMM_NR; ++n) C[m * N + n] = 0.f;
  if (bias)
    for (int64_t m = 0; m < M; ++m)
      for (int64_t n = p_begin * GEMM_NR; n < N && n < p_end * GEMM_NR; ++n) C[m * N + n] += bias[n];
  free(zero);
  free(bp);
}

static void gemm_nt(const float* A, const float* B, const float* bias, float* C, int64_t M,
                    int64_t N, int64_t K) {
  if (M <= 0 || N <= 0) return;
  gemm_ctx g = {A, B, bias, C, M, N, K};
  parallel_for((N + GEMM_NR - 1) / GEMM_NR, gemm_range, &g);
}

/* One expert FFN over its gathered rows xe [M,H] -> ye [M,H].
 * w1: [N1,H] (N1 = I, or 2I for fused swiglu); w3: [I,H] or NULL; w2: [H,I]. */
static void expert_ffn(const float* xe, int64_t M, int64_t H, int64_t I, int act, int fusion,
                       float alpha, float beta, float limit, const float* w1, const float* b1,
                       const float* w3, const float* b3, const float* w2, const float* b2,
                       float* h, float* u, float* a, float* ye) {
  const int fused = act == ACT_SWIGLU && fusion != 0;
  const int64_t N1 = fused ? 2 * I : I;
  gemm_nt(xe, w1, b1, h, M, N1, H);
  if (w3) gemm_nt(xe, w3, b3, u, M, I, H);
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t c = 0; c < I; ++c) {
      float g, l = 0.f;
      if (fused && fusion == 1) { g = h[m * N1 + 2 * c]; l = h[m * N1 + 2 * c + 1]; }
      else if (fused) { g = h[m * N1 + c]; l = h[m * N1 + I + c]; }
      else { g = h[m * N1 + c]; if (w3) l = u[m * I + c]; }
      float v;
      if (act == ACT_SWIGLU) {
        g = g < limit ? g : limit;
        l = l < -limit ? -limit : (l > limit ? limit : l);
        v = g / (1.f + expf(-alpha * g)) * (l + beta);
      } else {
        v = act1(act, g);
        if (w3) v *= l;
      }
      a[m * I + c] = v;
    }
  }
  gemm_nt(a, w2, b2, ye, M, H, I);
}

/* Dequantises rows [N, K] of one expert (codes with zero point 2^(bits-1)). */
typedef struct { const uint8_t* q; const float* scales; int64_t K; int bits, block_size; float* out; } dq_ctx;

static void dequant_range(int64_t n0, int64_t n1, void* p) {
  dq_ctx* d = (dq_ctx*)p;
  const uint8_t* q = d->q;
  const float* scales = d->scales;
  const int64_t K = d->K;
  const int bits = d->bits, block_size = d->block_size;
  float* out = d->out;
  const int64_t row_bytes = bits == 4 ? (K + 1) / 2 : K;
  const int64_t nb = block_size ? (K + block_size - 1) / block_size : 1;
  for (int64_t n = n0; n < n1; ++n)
    for (int64_t c = 0; c < K; ++c) {
      int code;
      if (bits == 4) {
        const uint8_t b = q[n * row_bytes + c / 2];
        code = ((c & 1) ? (b >> 4) : (b & 0xF)) - 8;
      } else {
        code = (int)q[n * row_bytes + c] - 128;
      }
      const float s = block_size ? scales[n * nb + c / block_size] : scales[n];
      out[n * K + c] = (float)code * s;
    }
}

static void dequant_rows(const uint8_t* q, const float* scales, int64_t N, int64_t K, int bits,
                         int block_size, float* out) {
  dq_ctx d = {q, scales, K, bits, block_size, out};
  parallel_for(N, dequant_range, &d);
}

/* One MoE (bits == 0, weights fp32) or QMoE (bits 4/8: w* are uint8 codes and s*
 * fp32 scales) layer call.  Returns 0 on success. */
int oracle_moe(int64_t T, int64_t H, int64_t I, int64_t E, int k, int normalize, int act,
               int fusion, float alpha, float beta, float limit, int bits, int block_size,
               const float* x, const float* logits, const void* w1, const float* s1,
               const float* b1, const void* w2, const float* s2, const float* b2,
               const void* w3, const float* s3, const float* b3, float* out) {
  const int fused = act == ACT_SWIGLU && fusion != 0;
  const int64_t N1 = fused ? 2 * I : I;
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * T * k);
  float* w = (float*)malloc(sizeof(float) * T * k);
  int64_t* rows = (int64_t*)malloc(sizeof(int64_t) * T);
  int32_t* slots = (int32_t*)malloc(sizeof(int32_t) * T);
  float* xe = (float*)malloc(sizeof(float) * T * H);
  float* ye = (float*)malloc(sizeof(float) * T * H);
  float* h = (float*)malloc(sizeof(float) * T * N1);
  float* u = (float*)malloc(sizeof(float) * T * I);
  float* a = (float*)malloc(sizeof(float) * T * I);
  float *d1 = NULL, *d2 = NULL, *d3 = NULL;
  if (bits) {
    d1 = (float*)malloc(sizeof(float) * N1 * H);
    d2 = (float*)malloc(sizeof(float) * H * I);
    d3 = w3 ? (float*)malloc(sizeof(float) * I * H) : NULL;
  }
  if (!idx || !w || !rows || !slots || !xe || !ye || !h || !u || !a ||
      (bits && (!d1 || !d2 || (w3 && !d3))))
    return 1;
  oracle_route(logits, T, (int)E, k, normalize, idx, w);
  memset(out, 0, sizeof(float) * T * H);
  const int64_t nb = block_size ? (H + block_size - 1) / block_size : 1;
  const int64_t nbi = block_size ? (I + block_size - 1) / block_size : 1;
  const int64_t hb = bits == 4 ? (H + 1) / 2 : H, ib = bits == 4 ? (I + 1) / 2 : I;
  for (int64_t e = 0; e < E; ++e) {
    int64_t M = 0;
    for (int64_t t = 0; t < T; ++t)
      for (int j = 0; j < k; ++j)
        if (idx[t * k + j] == e) { rows[M] = t; slots[M] = j; ++M; }
    if (M == 0) continue;
    for (int64_t m = 0; m < M; ++m) memcpy(xe + m * H, x + rows[m] * H, sizeof(float) * H);
    const float *W1, *W2, *W3 = NULL;
    if (bits) {
      dequant_rows((const uint8_t*)w1 + e * N1 * hb, s1 + e * N1 * nb, N1, H, bits, block_size, d1);
      dequant_rows((const uint8_t*)w2 + e * H * ib, s2 + e * H * nbi, H, I, bits, block_size, d2);
      if (w3) dequant_rows((const uint8_t*)w3 + e * I * hb, s3 + e * I * nb, I, H, bits, block_size, d3);
      W1 = d1; W2 = d2; W3 = w3 ? d3 : NULL;
    } else {
      W1 = (const float*)w1 + e * N1 * H;
      W2 = (const float*)w2 + e * H * I;
      W3 = w3 ? (const float*)w3 + e * I * H : NULL;
    }
    expert_ffn(xe, M, H, I, act, fusion, alpha, beta, limit, W1, b1 ? b1 + e * N1 : NULL, W3,
               b3 ? b3 + e * I : NULL, W2, b2 ? b2 + e * H : NULL, h, u, a, ye);
    for (int64_t m = 0; m < M; ++m) {
      const float wt = w[rows[m] * k + slots[m]];
      float* o = out + rows[m] * H;
      const float* y = ye + m * H;
      for (int64_t c = 0; c < H; ++c) o[c] += wt * y[c];
    }
  }
  free(idx); free(w); free(rows); free(slots); free(xe); free(ye); free(h); free(u); free(a);
  free(d1); free(d2); free(d3);
  return 0;
}
