/* oracle.c - TEST INFRASTRUCTURE ONLY: a plain-C restatement of the reference's CPU
 * path for the dense-contraction hot path, used as the parity checker of the CUDA
 * kernels (never as the product; the library does not link or load it).
 *
 * Each function cites the reference function (StableDiffusion-cpp, src/...) whose
 * arithmetic it restates. Summation orders follow the reference so that, compiled
 * with the same floating-point contraction (gnu11: `a += x * y` fused to an FMA, as
 * g++ does for the reference's C++), results agree with the reference bit for bit
 * on the same host; the parity tests pin this
 * against the reference compiled from its own sources and against committed golden
 * vectors. Outer loops run on a pthreads parallel-for, which does not change any
 * per-output arithmetic.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

#define MIN(a, b) ((a) < (b) ? (a) : (b))
#define MAX(a, b) ((a) > (b) ? (a) : (b))

/* ---- parallel-for over item indices (pthreads + an atomic counter, like the
 * reference's pool, tensor.cpp:149-265); per-item arithmetic is unaffected. ---- */
static int g_threads = 0; /* 0 = all online CPUs */
void orc_set_num_threads(int n) { g_threads = n; }
int orc_num_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
typedef void (*item_fn)(int64_t i, void* ctx);
typedef struct {
  item_fn fn;
  void* ctx;
  int64_t n;
  atomic_llong next;
} job_t;
static void* worker(void* arg) {
  job_t* j = (job_t*)arg;
  int64_t i;
  while ((i = atomic_fetch_add(&j->next, 1)) < j->n) j->fn(i, j->ctx);
  return NULL;
}
static void par_for(int64_t n, item_fn fn, void* ctx) {
  if (n <= 0) return;
  int T = orc_num_threads();
  if (T > n) T = (int)n;
  job_t j;
  j.fn = fn;
  j.ctx = ctx;
  j.n = n;
  atomic_init(&j.next, 0);
  if (T <= 1) {
    worker(&j);
    return;
  }
  pthread_t th[256];
  if (T > 256) T = 256;
  for (int t = 1; t < T; ++t) pthread_create(&th[t], NULL, worker, &j);
  worker(&j);
  for (int t = 1; t < T; ++t) pthread_join(th[t], NULL);
}

/* tensor.cpp:114-121 f32_to_bf16: round to nearest even, inf/NaN truncated. */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  if ((bits & 0x7F800000u) == 0x7F800000u) return (uint16_t)(bits >> 16);
  bits += 0x7FFFu + ((bits >> 16) & 1u);
  return (uint16_t)(bits >> 16);
}
/* tensor.h:137-142 bf16_to_f32: widen by a 16-bit shift. */
static inline float bf16_to_f32(uint16_t h) {
  uint32_t b = (uint32_t)h << 16;
  float f;
  memcpy(&f, &b, 4);
  return f;
}
void orc_f32_to_bf16_array(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_f32_to_bf16(x[i]);
}
void orc_bf16_to_f32_array(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = bf16_to_f32(x[i]);
}

/* ------------------------------------------------------------------------------ */
/* GEMM: C = A * B^T (tensor.cpp:296-406)                                           */
/* ------------------------------------------------------------------------------ */
static inline float hsum4(const float* v) { return (v[0] + v[1]) + (v[2] + v[3]); }

/* tensor.cpp:301-312 dot(): two 4-lane accumulators over 8-wide steps, scalar tail. */
static float dot_ref(const float* a, const float* b, int64_t K) {
  float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
  int64_t k = 0;
  for (; k + 8 <= K; k += 8)
    for (int l = 0; l < 4; ++l) {
      acc0[l] += a[k + l] * b[k + l];
      acc1[l] += a[k + 4 + l] * b[k + 4 + l];
    }
  float s = hsum4(acc0) + hsum4(acc1);
  for (; k < K; ++k) s += a[k] * b[k];
  return s;
}

/* tensor.cpp:314-343 micro_4x4(): 16 outputs, each a 4-lane vector dot product over
 * 4-wide K steps, horizontal sum, scalar K tail, then added to C. */
static void micro_4x4(int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc) {
  float acc[4][4][4];
  memset(acc, 0, sizeof acc);
  int64_t k = 0;
  for (; k + 4 <= K; k += 4)
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 4; ++j)
        for (int l = 0; l < 4; ++l) acc[i][j][l] += A[i * lda + k + l] * B[j * ldb + k + l];
  float s[4][4];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) s[i][j] = hsum4(acc[i][j]);
  for (; k < K; ++k)
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 4; ++j) s[i][j] += A[i * lda + k] * B[j * ldb + k];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) C[i * ldc + j] += s[i][j];
}

static void micro_edge(int64_t mr, int64_t nr, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                       float* C, int64_t ldc) {
  for (int64_t i = 0; i < mr; ++i)
    for (int64_t j = 0; j < nr; ++j) C[i * ldc + j] += dot_ref(A + i * lda, B + j * ldb, K);
}

typedef struct {
  int64_t M, N, K, lda, ldb, ldc, nblocks;
  const float* A;
  const float* B;       /* fp32 B (gemm_nt) */
  const uint16_t* Bh;   /* bf16 B (gemm_nt_bf16) */
  float* C;
  const float* bias;
  int accumulate;
} gemm_job;

static void seed_tile(const gemm_job* g, int64_t m0, int64_t m1, int64_t n0, int64_t n1) {
  for (int64_t i = m0; i < m1; ++i) {
    float* c = g->C + i * g->ldc;
    if (!g->accumulate) {
      if (g->bias)
        memcpy(c + n0, g->bias + n0, (size_t)(n1 - n0) * sizeof(float));
      else
        memset(c + n0, 0, (size_t)(n1 - n0) * sizeof(float));
    } else if (g->bias) {
      for (int64_t j = n0; j < n1; ++j) c[j] += g->bias[j];
    }
  }
}

static void gemm_tile(int64_t t, void* ctx) {
  const gemm_job* g = (const gemm_job*)ctx;
  const int64_t MB = 64, NB = 128, KB = 128;
  const int64_t m0 = (t / g->nblocks) * MB, m1 = MIN(g->M, m0 + MB);
  const int64_t n0 = (t % g->nblocks) * NB, n1 = MIN(g->N, n0 + NB);
  seed_tile(g, m0, m1, n0, n1);
  for (int64_t k0 = 0; k0 < g->K; k0 += KB) {
    const int64_t kc = MIN(KB, g->K - k0);
    for (int64_t i = m0; i < m1; i += 4) {
      const int64_t mr = MIN(4, m1 - i);
      for (int64_t j = n0; j < n1; j += 4) {
        const int64_t nr = MIN(4, n1 - j);
        const float* a = g->A + i * g->lda + k0;
        const float* b = g->B + j * g->ldb + k0;
        float* c = g->C + i * g->ldc + j;
        if (mr == 4 && nr == 4)
          micro_4x4(kc, a, g->lda, b, g->ldb, c, g->ldc);
        else
          micro_edge(mr, nr, kc, a, g->lda, b, g->ldb, c, g->ldc);
      }
    }
  }
}

/* tensor.cpp:354-406 gemm_nt (built-in kernel; the Accelerate branch is macOS-only):
 * 64 x 128 output tiles, C seeded with bias / zero / kept (accumulate), K walked in
 * 128-wide slices with the 4x4 micro-kernel and the edge fallback. */
void orc_gemm_nt(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                 int64_t ldc, const float* bias, int accumulate) {
  if (M <= 0 || N <= 0) return;
  gemm_job g = {M, N, K, lda, ldb, ldc, (N + 127) / 128, A, B, NULL, C, bias, accumulate};
  par_for(((M + 63) / 64) * g.nblocks, gemm_tile, &g);
}

/* tensor.cpp:412-474 gemm_nt_bf16: per tile, each 128-wide K slice of B is widened to
 * fp32 exactly (bf16 -> fp32 is a shift), then the same micro-kernels run; A stays
 * exact fp32. Arithmetically identical to gemm_nt on the widened B. */
static void gemm_bf16_tile(int64_t t, void* ctx) {
  const gemm_job* g = (const gemm_job*)ctx;
  const int64_t MB = 64, NB = 128, KB = 128;
  static __thread float pack[128 * 128];
  const int64_t m0 = (t / g->nblocks) * MB, m1 = MIN(g->M, m0 + MB);
  const int64_t n0 = (t % g->nblocks) * NB, n1 = MIN(g->N, n0 + NB);
  seed_tile(g, m0, m1, n0, n1);
  for (int64_t k0 = 0; k0 < g->K; k0 += KB) {
    const int64_t kc = MIN(KB, g->K - k0);
    for (int64_t j = n0; j < n1; ++j) {
      const uint16_t* src = g->Bh + j * g->ldb + k0;
      float* dst = pack + (j - n0) * KB;
      for (int64_t k = 0; k < kc; ++k) dst[k] = bf16_to_f32(src[k]);
    }
    for (int64_t i = m0; i < m1; i += 4) {
      const int64_t mr = MIN(4, m1 - i);
      for (int64_t j = n0; j < n1; j += 4) {
        const int64_t nr = MIN(4, n1 - j);
        const float* a = g->A + i * g->lda + k0;
        const float* bp = pack + (j - n0) * KB;
        float* c = g->C + i * g->ldc + j;
        if (mr == 4 && nr == 4)
          micro_4x4(kc, a, g->lda, bp, KB, c, g->ldc);
        else
          micro_edge(mr, nr, kc, a, g->lda, bp, KB, c, g->ldc);
      }
    }
  }
}

void orc_gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                      float* C, int64_t ldc, const float* bias, int accumulate) {
  if (M <= 0 || N <= 0) return;
  gemm_job g = {M, N, K, lda, ldb, ldc, (N + 127) / 128, A, NULL, B, C, bias, accumulate};
  par_for(((M + 63) / 64) * g.nblocks, gemm_bf16_tile, &g);
}

/* ------------------------------------------------------------------------------ */
/* Attention (tensor.cpp:752-810)                                                   */
/* ------------------------------------------------------------------------------ */
/* tensor.cpp:752-769 softmax_rows_: scaled max-subtracted softmax, causal rows keep
 * r + 1 entries and zero the rest. */
typedef struct {
  float* x;
  int64_t cols;
  float scale;
  int causal;
} softmax_job;
static void softmax_row(int64_t r, void* ctx) {
  const softmax_job* s = (const softmax_job*)ctx;
  const int64_t cols = s->cols;
  const float scale = s->scale;
  const int causal = s->causal;
  {
    float* p = s->x + r * cols;
    const int64_t valid = causal ? MIN(cols, r + 1) : cols;
    float m = -INFINITY;
    for (int64_t j = 0; j < valid; ++j) m = fmaxf(m, p[j] * scale);
    float sum = 0.0f;
    for (int64_t j = 0; j < valid; ++j) {
      p[j] = expf(p[j] * scale - m);
      sum += p[j];
    }
    const float inv = 1.0f / sum;
    for (int64_t j = 0; j < valid; ++j) p[j] *= inv;
    for (int64_t j = valid; j < cols; ++j) p[j] = 0.0f;
  }
}
void orc_softmax_rows(float* x, int64_t rows, int64_t cols, float scale, int causal) {
  softmax_job s = {x, cols, scale, causal};
  par_for(rows, softmax_row, &s);
}

/* tensor.cpp:776-810 attention: per (sample, head) the full score matrix
 * S = Q_h K_h^T (gemm_nt), softmax with 1/sqrt(d), V_h transposed, O_h = P V_h
 * (gemm_nt). Query head h uses kv head h / (heads / kv_heads). */
void orc_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                   int heads, int kv_heads, int64_t d, int causal) {
  const int64_t inner = heads * d, kv_inner = kv_heads * d, group = heads / kv_heads;
  const float scale = 1.0f / sqrtf((float)d);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(Sq * Skv));
  float* vT = (float*)malloc(sizeof(float) * (size_t)(d * Skv));
  for (int64_t n = 0; n < N; ++n)
    for (int h = 0; h < heads; ++h) {
      const float* qh = q + n * Sq * inner + h * d;
      const float* kh = k + n * Skv * kv_inner + (h / group) * d;
      const float* vh = v + n * Skv * kv_inner + (h / group) * d;
      orc_gemm_nt(Sq, Skv, d, qh, inner, kh, kv_inner, scores, Skv, NULL, 0);
      orc_softmax_rows(scores, Sq, Skv, scale, causal);
      for (int64_t s = 0; s < Skv; ++s)
        for (int64_t j = 0; j < d; ++j) vT[j * Skv + s] = vh[s * kv_inner + j];
      orc_gemm_nt(Sq, d, Skv, scores, Skv, vT, Skv, out + n * Sq * inner + h * d, inner, NULL, 0);
    }
  free(scores);
  free(vT);
}

/* ------------------------------------------------------------------------------ */
/* Norms, rotary embedding, gated activations (tensor.cpp:588-748, :813-917)        */
/* ------------------------------------------------------------------------------ */
/* tensor.cpp:660-679 rms_norm: double sum of squares, fp32 rstd. */
typedef struct {
  const float* x;
  float* y;
  int64_t C;
  const float* gamma;
  const float* beta;
  float eps;
} norm_job;
static void rms_row(int64_t r, void* ctx) {
  const norm_job* j = (const norm_job*)ctx;
  const int64_t C = j->C;
  const float* p = j->x + r * C;
  float* q = j->y + r * C;
  double ss = 0;
  for (int64_t i = 0; i < C; ++i) ss += (double)p[i] * p[i];
  const float rstd = (float)(1.0 / sqrt(ss / C + j->eps));
  for (int64_t i = 0; i < C; ++i) q[i] = p[i] * rstd * (j->gamma ? j->gamma[i] : 1.0f);
}
void orc_rms_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, float eps) {
  norm_job j = {x, y, C, gamma, NULL, eps};
  par_for(rows, rms_row, &j);
}
/* tensor.cpp:628-658 layer_norm: two-pass mean / variance in double. */
static void layer_row(int64_t r, void* ctx) {
  const norm_job* j = (const norm_job*)ctx;
  const int64_t C = j->C;
  const float* gamma = j->gamma;
  const float* beta = j->beta;
  const float eps = j->eps;
  {
    const float* p = j->x + r * C;
    float* q = j->y + r * C;
    double sum = 0;
    for (int64_t i = 0; i < C; ++i) sum += p[i];
    const float mean = (float)(sum / C);
    double var = 0;
    for (int64_t i = 0; i < C; ++i) {
      const float dd = p[i] - mean;
      var += (double)dd * dd;
    }
    const float rstd = (float)(1.0 / sqrt(var / C + eps));
    for (int64_t i = 0; i < C; ++i) {
      float v = (p[i] - mean) * rstd;
      if (gamma) v *= gamma[i];
      if (beta) v += beta[i];
      q[i] = v;
    }
  }
}
void orc_layer_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta,
                    float eps) {
  norm_job j = {x, y, C, gamma, beta, eps};
  par_for(rows, layer_row, &j);
}
/* tensor.cpp:681-699 rms_norm_heads_ (in place, per group of dim values). */
void orc_rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps) {
  norm_job j = {x, x, dim, gamma, NULL, eps};
  par_for(groups, rms_row, &j);
}
/* tensor.cpp:701-730 rope_ (in place): interleaved pairs (2i, 2i+1) or rotate_half
 * pairs (i, i + dim/2); tables [S, dim]. */
void orc_rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cs, const float* sn,
              int interleaved) {
  const int64_t heads = inner / dim, half = dim / 2;
  for (int64_t ns = 0; ns < N * S; ++ns) {
    const int64_t s = ns % S;
    const float* c = cs + s * dim;
    const float* sv = sn + s * dim;
    for (int64_t h = 0; h < heads; ++h) {
      float* p = x + ns * inner + h * dim;
      if (interleaved) {
        for (int64_t i = 0; i < dim; i += 2) {
          const float a = p[i], b = p[i + 1];
          p[i] = a * c[i] - b * sv[i];
          p[i + 1] = b * c[i] + a * sv[i];
        }
      } else {
        for (int64_t i = 0; i < half; ++i) {
          const float a = p[i], b = p[i + half];
          p[i] = a * c[i] - b * sv[i];
          p[i + half] = b * c[i + half] + a * sv[i + half];
        }
      }
    }
  }
}
/* tensor.cpp:732-748 swiglu: g / (1 + e^-g) * u. */
void orc_swiglu(const float* g, const float* u, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}
/* tensor.cpp:813-835 geglu: first half value, second half gate; a * 0.5 g (1 + erf(g/sqrt2)). */
void orc_geglu(const float* x, float* y, int64_t rows, int64_t D) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* a = x + r * 2 * D;
    const float* g = a + D;
    float* o = y + r * D;
    for (int64_t i = 0; i < D; ++i) {
      const float gg = g[i];
      o[i] = a[i] * 0.5f * gg * (1.0f + erff(gg * 0.70710678118654752f));
    }
  }
}
/* tensor.cpp:889-901 mul_rows_: x[r, :] *= v. */
void orc_mul_rows(float* x, const float* v, int64_t rows, int64_t dim) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t i = 0; i < dim; ++i) x[r * dim + i] *= v[i];
}
/* tensor.cpp:903-917 add_rows_scaled_: x[r, :] += g * y[r, :]. */
void orc_add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t i = 0; i < dim; ++i) x[r * dim + i] += g[i] * y[r * dim + i];
}
/* tensor.cpp:588-626 group_norm: mean and variance in double per (sample, group). */
void orc_group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                    const float* beta, float eps) {
  const int64_t cg = C / groups, len = cg * HW;
  for (int64_t t = 0; t < N * groups; ++t) {
    const int64_t n = t / groups, g = t % groups;
    const float* p = x + (n * C + g * cg) * HW;
    float* q = y + (n * C + g * cg) * HW;
    double sum = 0;
    for (int64_t i = 0; i < len; ++i) sum += p[i];
    const double mean = sum / len;
    double var = 0;
    for (int64_t i = 0; i < len; ++i) {
      const double dd = p[i] - mean;
      var += dd * dd;
    }
    const float rstd = (float)(1.0 / sqrt(var / len + eps));
    for (int64_t c = 0; c < cg; ++c) {
      const int64_t ch = g * cg + c;
      const float a = rstd * gamma[ch];
      const float bb = beta[ch] - (float)mean * a;
      for (int64_t i = 0; i < HW; ++i) q[c * HW + i] = p[c * HW + i] * a + bb;
    }
  }
}
/* tensor.cpp:529-586 conv2d: im2col in pixel chunks of at most 2^24 floats, then
 * gemm_nt(Cout, P, K) into the NCHW output, bias seeded first. */
void orc_conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out) {
  const int64_t Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
  const int64_t K = Cin * kh * kw, HW = Ho * Wo;
  if (bias) {
    for (int64_t n = 0; n < N; ++n)
      for (int64_t co = 0; co < Cout; ++co)
        for (int64_t i = 0; i < HW; ++i) out[(n * Cout + co) * HW + i] = bias[co];
  }
  const int64_t chunk = MAX(1, MIN(HW, ((int64_t)1 << 24) / K));
  float* cols = (float*)malloc(sizeof(float) * (size_t)(chunk * K));
  for (int64_t n = 0; n < N; ++n) {
    const float* xin = x + n * Cin * H * W;
    for (int64_t p0 = 0; p0 < HW; p0 += chunk) {
      const int64_t P = MIN(chunk, HW - p0);
      for (int64_t p = 0; p < P; ++p) {
        const int64_t oy = (p0 + p) / Wo, ox = (p0 + p) % Wo;
        float* row = cols + p * K;
        for (int64_t ci = 0; ci < Cin; ++ci)
          for (int64_t ky = 0; ky < kh; ++ky) {
            const int64_t iy = oy * stride - pad + ky;
            float* r = row + (ci * kh + ky) * kw;
            for (int64_t kx = 0; kx < kw; ++kx) {
              const int64_t ix = ox * stride - pad + kx;
              r[kx] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xin[(ci * H + iy) * W + ix] : 0.0f;
            }
          }
      }
      orc_gemm_nt(Cout, P, K, w, K, cols, K, out + n * Cout * HW + p0, HW, NULL, bias != NULL);
    }
  }
  free(cols);
}

/* ---- flow-matching sampler (scheduler.cpp:117-135, pipeline.cpp:237-243) ------------ */
/* sigma_i = shift s / (1 + (shift - 1) s), s from 1 down to 1/steps, sigma_steps = 0. The
 * reference is compiled for x86-64-v3, where its compiler fuses the denominator into one
 * multiply-add; fmaf reproduces that rounding. */
void orc_flow_sigmas(int steps, float shift, float* sig) {
  for (int i = 0; i < steps; ++i) {
    const float s = steps == 1 ? 1.0f : 1.0f - (float)i * (1.0f - 1.0f / (float)steps) / (float)(steps - 1);
    sig[i] = shift * s / fmaf(shift - 1.0f, s, 1.0f);
  }
  sig[steps] = 0.0f;
}

/* x += dt * (out + cfg (out - neg)) (neg NULL: x += dt * out). Built as the reference's
 * loops compile for x86-64-v3: the guidance mix as a separate multiply and add, the
 * Euler update as one fused multiply-add (pinned against the reference library). */
__attribute__((optimize("fp-contract=off"))) void orc_flow_step(float* x, const float* out, const float* neg,
                                                                float cfg, float dt, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float o = out[i];
    if (neg) {
      const float t = cfg * (o - neg[i]);
      o = o + t;
    }
    x[i] = fmaf(dt, o, x[i]);
  }
}
