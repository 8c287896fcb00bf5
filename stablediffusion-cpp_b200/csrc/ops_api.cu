// ops_api.cu - the compute half of the C ABI (sdb200.h): argument validation, operand
// preparation for the tensor-core GEMM, path selection, and the layer ops.
//
// GEMM path selection (gemm_nt_bf16 / gemm_nt_f32, backend_cuda.cu:453-477):
//   K == 0         C = bias (or C += bias)          - no contraction
//   M <= 16        memory-bound SIMT kernel, exact fp32 A (weights streamed once)
//   otherwise      tcgen05 GEMM (gemm_tc.cu). A fp32 is packed to bf16 (bf16 path,
//                  the reference's rounding) or rounded to tf32 (fp32 path) in the
//                  workspace with 16-byte-aligned rows; B is used in place when its
//                  base and row pitch meet TMA's 16-byte rule, else packed too.
#include <algorithm>
#include <cmath>
#include <string>

#include "internal.h"
#include "sdb200.h"

namespace sdb {

namespace {

constexpr int64_t kMaxDim = (int64_t)1 << 31;

void require(bool ok, const char* op, const std::string& what) {
  if (!ok) fail(kErrInvalidArg, std::string(op) + ": " + what);
}
void require_ptr(const void* p, const char* op, const char* name) {
  if (!p) fail(kErrInvalidArg, std::string(op) + ": null pointer " + name);
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

void check_gemm_args(const char* op, int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                     int64_t ldb, const void* C, int64_t ldc) {
  require(M < kMaxDim && N < kMaxDim && K < kMaxDim, op, "dimension >= 2^31");
  require(K >= 0, op, "K < 0");
  require_ptr(C, op, "C");
  require(ldc >= N, op, "ldc < N");
  if (K > 0) {
    require_ptr(A, op, "A");
    require_ptr(B, op, "B");
    require(lda >= K, op, "lda < K");
    require(ldb >= K, op, "ldb < K");
  }
  require((reinterpret_cast<uintptr_t>(C) & 3) == 0, op, "C not 4-byte aligned");
}

// bf16 x bf16 GEMM with A either fp32 (packed here) or bf16.
void gemm_bf16_core(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, bool a_bf16, const uint16_t* B,
                    int64_t ldb, void* C, int64_t ldc, bool c_bf16, const float* bias, bool acc, Epi epi,
                    const QkvRope* rope = nullptr, const ScatterOut* scatter = nullptr) {
  const int64_t Kp = round_up(K, 8);  // 16-byte rows of bf16
  const bool a_direct = a_bf16 && aligned16(A) && (lda % 8 == 0);
  const bool b_direct = aligned16(B) && (ldb % 8 == 0);
  const size_t a_bytes = a_direct ? 0 : align256((size_t)(M * Kp) * 2);
  const size_t b_bytes = b_direct ? 0 : align256((size_t)(N * Kp) * 2);
  uint8_t* ws = (a_bytes + b_bytes) ? static_cast<uint8_t*>(workspace(a_bytes + b_bytes)) : nullptr;
  const void* Ause = A;
  int64_t lda_use = lda;
  if (!a_direct) {
    uint16_t* pa = reinterpret_cast<uint16_t*>(ws);
    if (a_bf16)
      launch_copy2d(A, lda, pa, Kp, M, K, 2);
    else
      launch_pack_bf16(static_cast<const float*>(A), lda, pa, Kp, M, K);
    Ause = pa;
    lda_use = Kp;
  }
  const uint16_t* Buse = B;
  int64_t ldb_use = ldb;
  if (!b_direct) {
    uint16_t* pb = reinterpret_cast<uint16_t*>(ws + a_bytes);
    launch_copy2d(B, ldb, pb, Kp, N, K, 2);
    Buse = pb;
    ldb_use = Kp;
  }
  GemmCall g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = Ause;
  g.lda = lda_use;
  g.B = Buse;
  g.ldb = ldb_use;
  g.C = C;
  g.ldc = ldc;
  g.bias = bias;
  g.accumulate = acc;
  g.tf32 = false;
  g.epi = epi;
  g.out_bf16 = c_bf16;
  g.bn = 0;
  g.rope = rope;
  g.scatter = scatter;
  launch_gemm_tc(g);
}

// b_constant: B is a caller's weight buffer (the C-ABI entry), eligible for the opt-in
// packed-operand cache; internal callers pass activations or scratch as B.
void gemm_f32_core(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                   int64_t ldc, const float* bias, bool acc, bool b_constant) {
  const int64_t Kp = round_up(K, 4);  // 16-byte rows of fp32
  const bool cache_b = b_constant && operand_cache_on();
  const size_t a_bytes = align256((size_t)(M * Kp) * 4);
  const size_t b_bytes = cache_b ? 0 : align256((size_t)(N * Kp) * 4);
  uint8_t* ws = static_cast<uint8_t*>(workspace(a_bytes + b_bytes));
  float* pa = reinterpret_cast<float*>(ws);
  const float* pb;
  if (cache_b) {
    pb = cached_tf32_rows(B, N, K, ldb, Kp);  // the weights, packed once
    launch_pack_tf32(A, lda, pa, Kp, M, K);
  } else {
    float* pbw = reinterpret_cast<float*>(ws + a_bytes);
    launch_pack_tf32_pair(A, lda, pa, Kp, M, B, ldb, pbw, Kp, N, K);
    pb = pbw;
  }
  GemmCall g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = pa;
  g.lda = Kp;
  g.B = pb;
  g.ldb = Kp;
  g.C = C;
  g.ldc = ldc;
  g.bias = bias;
  g.accumulate = acc;
  g.tf32 = true;
  g.epi = Epi::kStore;
  g.out_bf16 = false;
  g.bn = 0;
  launch_gemm_tc(g);
}

bool skinny_ok(int64_t M, int64_t K) { return skinny_shape(M, K); }

}  // namespace

// Shared by the C ABI and by the DiT runner.
void gemm_nt_bf16_impl(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                       float* C, int64_t ldc, const float* bias, bool acc) {
  if (M <= 0 || N <= 0) return;  // no-op before any check, as backend_cuda.cu:455/:464
  check_gemm_args("gemm_nt_bf16", M, N, K, A, lda, B, ldb, C, ldc);
  if (K == 0) return launch_bias_fill(C, ldc, M, N, bias, acc);
  if (skinny_ok(M, K)) return launch_gemm_skinny(M, N, K, A, lda, B, ldb, true, C, ldc, bias, acc);
  gemm_bf16_core(M, N, K, A, lda, false, B, ldb, C, ldc, false, bias, acc, Epi::kStore);
}
void gemm_nt_bf16a_impl(int64_t M, int64_t N, int64_t K, const uint16_t* A, int64_t lda, const uint16_t* B,
                        int64_t ldb, float* C, int64_t ldc, const float* bias, bool acc) {
  if (M <= 0 || N <= 0) return;  // no-op before any check, as backend_cuda.cu:455/:464
  check_gemm_args("gemm_nt_bf16a", M, N, K, A, lda, B, ldb, C, ldc);
  if (K == 0) return launch_bias_fill(C, ldc, M, N, bias, acc);
  gemm_bf16_core(M, N, K, A, lda, true, B, ldb, C, ldc, false, bias, acc, Epi::kStore);
}
void gemm_nt_f32_impl(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc, const float* bias, bool acc, bool b_constant) {
  if (M <= 0 || N <= 0) return;  // no-op before any check, as backend_cuda.cu:455/:464
  check_gemm_args("gemm_nt_f32", M, N, K, A, lda, B, ldb, C, ldc);
  if (K == 0) return launch_bias_fill(C, ldc, M, N, bias, acc);
  if (skinny_ok(M, K)) return launch_gemm_skinny(M, N, K, A, lda, B, ldb, false, C, ldc, bias, acc);
  gemm_f32_core(M, N, K, A, lda, B, ldb, C, ldc, bias, acc, b_constant);
}
void gemm_tf32_direct(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                      float* C, int64_t ldc, const float* bias, bool acc) {
  if (M <= 0 || N <= 0) return;
  const bool ok = K > 0 && lda % 4 == 0 && ldb % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(B) & 15) == 0;
  if (!ok) fail(kErrInvalidArg, "gemm_tf32_direct: operands must be 16-byte aligned rows");
  GemmCall g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.A = A;
  g.lda = lda;
  g.B = B;
  g.ldb = ldb;
  g.C = C;
  g.ldc = ldc;
  g.bias = bias;
  g.accumulate = acc;
  g.tf32 = true;
  g.epi = Epi::kStore;
  g.out_bf16 = false;
  g.bn = 0;
  launch_gemm_tc(g);
}
void gemm_bf16_epilogue_impl(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, bool a_bf16,
                             const uint16_t* B, int64_t ldb, void* Y, int64_t ldy, bool y_bf16, const float* bias,
                             int epi) {
  const char* op = "gemm_bf16_epilogue";
  require(epi >= 0 && epi <= 2, op, "epi must be 0, 1 or 2");
  const int64_t ncols = epi == 0 ? N : N / 2;
  if (epi != 0) require(N % 32 == 0, op, "gated epilogues need N % 32 == 0 (16 + 16 interleaved columns)");
  if (M <= 0 || N <= 0) return;
  check_gemm_args(op, M, ncols, K, A, lda, B, ldb, Y, ldy);
  require(K > 0, op, "K == 0");
  gemm_bf16_core(M, N, K, A, lda, a_bf16, B, ldb, Y, ldy, y_bf16, bias, false, (Epi)epi);
}

// Fused-QKV projection with the attention prologue in the GEMM epilogue: X[M, K] times
// Wqkv[3 Dq, K]^T (+bias), then per head the q / k RMS norm, rotary embedding and fp16
// packing of zimage.cpp:117-120 (Epi::kQkvRope). q16 / k16 / v16 are fp16 [M, Dq].
void gemm_bf16_qkv_rope_impl(int64_t M, int64_t K, const void* A, int64_t lda, bool a_bf16, const uint16_t* B,
                             int64_t ldb, const float* bias, const QkvRope& r) {
  const char* op = "gemm_bf16_qkv_rope";
  require(r.Dq > 0 && r.Dq % 128 == 0, op, "Dq must be a positive multiple of 128");
  require(r.S > 0, op, "S must be positive");
  require_ptr(r.cs, op, "cs");
  require_ptr(r.sn, op, "sn");
  require_ptr(r.q16, op, "q16");
  require_ptr(r.k16, op, "k16");
  require_ptr(r.v16, op, "v16");
  require((((uintptr_t)r.q16 | (uintptr_t)r.k16 | (uintptr_t)r.v16 | (uintptr_t)r.cs | (uintptr_t)r.sn) & 15) == 0, op,
          "outputs and tables must be 16-byte aligned");
  if (M <= 0) return;
  const int64_t N = 3 * (int64_t)r.Dq;
  require(K > 0, op, "K == 0");
  require_ptr(A, op, "A");
  require_ptr(B, op, "B");
  require(lda >= K && ldb >= K, op, "leading dimension < K");
  QkvRope rv = r;
  rv.gamma_vec = ((reinterpret_cast<uintptr_t>(r.gq) | reinterpret_cast<uintptr_t>(r.gk)) & 15) == 0;
  gemm_bf16_core(M, N, K, A, lda, a_bf16, B, ldb, nullptr, N, false, bias, false, Epi::kQkvRope, &rv);
}

// Row-parallel projection of tensor parallelism: X[M, K] times W[N, K]^T (+bias), every
// output row stored into its owner rank's slot (Epi::kScatter) instead of C.
void gemm_bf16_scatter_impl(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, bool a_bf16, const uint16_t* B,
                            int64_t ldb, const float* bias, const ScatterOut& so) {
  const char* op = "gemm_bf16_scatter";
  if (M <= 0 || N <= 0) return;
  require(K > 0, op, "K == 0");
  require_ptr(A, op, "A");
  require_ptr(B, op, "B");
  require(lda >= K && ldb >= K, op, "leading dimension < K");
  require(N % 4 == 0, op, "N % 4 != 0 (16-byte rows)");
  gemm_bf16_core(M, N, K, A, lda, a_bf16, B, ldb, nullptr, N, false, bias, false, Epi::kScatter, nullptr, &so);
}

// Implicit-GEMM convolution for stride 1 (default); off: im2col for every stride.
static bool g_conv_implicit = true;
void set_conv_implicit(bool on) { g_conv_implicit = on; }

// conv2d (backend_cuda.cu:479-510). Stride 1 runs as an implicit GEMM on tf32 tensor
// cores (launch_conv_tc); other strides as im2col + tf32 GEMM writing NCHW directly
// (ldc = HW), as the reference does with cuBLAS.
void conv2d_impl(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                 int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out, int64_t Ho, int64_t Wo) {
  const char* op = "conv2d";
  require(N >= 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0 && kh > 0 && kw > 0 && stride > 0 && pad >= 0, op,
          "bad shape");
  require_ptr(x, op, "x");
  require_ptr(w, op, "w");
  require_ptr(out, op, "out");
  const int64_t K = Cin * kh * kw, HW = Ho * Wo;
  if (N == 0 || HW <= 0) return;
  if (stride == 1 && g_conv_implicit) {
    // Implicit GEMM: the input repacked once to NHWC, no im2col matrix.
    const int64_t cp = round_up(Cin, 4), cq = round_up(Cin, 32), taps = kh * kw;
    const bool cache_w = operand_cache_on();  // conv2d_impl serves only the C-ABI conv2d: w is the caller's
    const size_t xb = align256((size_t)(N * H * W * cp) * 4);
    const size_t wb = cache_w ? 0 : align256((size_t)(Cout * taps * cq) * 4);
    uint8_t* ws = static_cast<uint8_t*>(workspace(xb + wb));
    float* xh = reinterpret_cast<float*>(ws);
    const float* wp;
    if (cache_w) {
      wp = cached_conv_weight(w, Cout, Cin, taps, cq);  // the weights, packed once
    } else {
      float* wpw = reinterpret_cast<float*>(ws + xb);
      launch_conv_pack_w(w, wpw, Cout, Cin, taps, cq);
      wp = wpw;
    }
    launch_conv_pack_x(x, xh, N, Cin, H * W, cp);
    launch_conv_tc(xh, N, Cin, cp, H, W, wp, cq, Cout, (int)kh, (int)kw, pad, bias, nullptr, out, Ho, Wo);
    return;
  }
  const int64_t Kp = round_up(K, 4);
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(HW, ((int64_t)1 << 26) / Kp));
  // cols live in pool memory so that the GEMM's own workspace stays free.
  float* cols = static_cast<float*>(pool_malloc((size_t)(chunk * Kp) * 4));
  try {
    for (int64_t n = 0; n < N; ++n) {
      const float* xin = x + n * Cin * H * W;
      float* o = out + n * Cout * HW;
      for (int64_t p0 = 0; p0 < HW; p0 += chunk) {
        const int64_t P = std::min(chunk, HW - p0);
        op_im2col(xin, cols, Cin, H, W, kh, kw, Wo, stride, pad, p0, P, K, Kp);
        // out[co, p0 + p] = sum_k w[co, k] * cols[p, k]
        gemm_nt_f32_impl(Cout, P, K, w, K, cols, Kp, o + p0, HW, nullptr, false);
      }
      if (bias) op_add_bias_rows(o, HW, Cout, HW, bias);
    }
  } catch (...) {
    pool_free(cols);
    throw;
  }
  // The GEMMs above are stream-ordered; freeing into the cache is safe because the
  // next user of this block is also issued on the same stream.
  pool_free(cols);
}

}  // namespace sdb

// ===================================================================================
using namespace sdb;

#define SDB_GUARD(body)                 \
  try {                                 \
    body;                               \
    return kOk;                         \
  } catch (const sdb::Error& e) {       \
    sdb::set_last_error(e.msg);         \
    return e.code;                      \
  } catch (const std::exception& e) {   \
    sdb::set_last_error(e.what());      \
    return kErrCuda;                    \
  }

extern "C" {

int sdb200_set_gemm_tile(int bn) {
  SDB_GUARD({
    require(bn == 0 || bn == 64 || bn == 128 || bn == 192 || bn == 256, "set_gemm_tile",
            "bn must be 0, 64, 128, 192 or 256");
    sdb::set_gemm_tile(bn);
  })
}

int sdb200_set_gemm_pair(int enable) {
  SDB_GUARD({
    require(enable >= 0 && enable <= 2, "set_gemm_pair", "mode must be 0, 1 or 2");
    sdb::set_gemm_pair(enable);
  })
}

int sdb200_set_conv_implicit(int enable) {
  SDB_GUARD(sdb::set_conv_implicit(enable != 0))
}

int sdb200_set_attention_path(int path) {
  SDB_GUARD({
    require(path == 0 || path == 1, "set_attention_path", "path must be 0 (tensor cores) or 1 (exact fp32)");
    sdb::set_attention_tc(path == 0);
  })
}

int sdb200_gemm_nt_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                       float* C, int64_t ldc, const float* bias, int accumulate) {
  SDB_GUARD(gemm_nt_f32_impl(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0, /*b_constant=*/true))
}
int sdb200_gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B,
                        int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate) {
  SDB_GUARD(gemm_nt_bf16_impl(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0))
}
int sdb200_gemm_nt_bf16a(int64_t M, int64_t N, int64_t K, const uint16_t* A, int64_t lda, const uint16_t* B,
                         int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate) {
  SDB_GUARD(gemm_nt_bf16a_impl(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0))
}
int sdb200_set_operand_cache(int enable) { SDB_GUARD(operand_cache_enable(enable != 0)) }

int64_t sdb200_operand_cache_entries(void) {
  try {
    return operand_cache_entries();
  } catch (...) {
    return -1;
  }
}

int sdb200_pack_bf16(const float* src, int64_t ld, uint16_t* dst, int64_t ldo, int64_t rows, int64_t cols) {
  SDB_GUARD({
    require(rows >= 0 && cols >= 0, "pack_bf16", "rows and cols must be >= 0");
    if (rows == 0 || cols == 0) return kOk;
    require(ld >= cols && ldo >= cols, "pack_bf16", "ld or ldo < cols");
    require_ptr(src, "pack_bf16", "src");
    require_ptr(dst, "pack_bf16", "dst");
    require((reinterpret_cast<uintptr_t>(src) & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 1) == 0, "pack_bf16",
            "misaligned src or dst");
    launch_pack_bf16(src, ld, dst, ldo, rows, cols);
  })
}
int sdb200_gemm_bf16_epilogue(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, int a_bf16,
                              const uint16_t* B, int64_t ldb, void* Y, int64_t ldy, int y_bf16, const float* bias,
                              int epi) {
  SDB_GUARD(gemm_bf16_epilogue_impl(M, N, K, A, lda, a_bf16 != 0, B, ldb, Y, ldy, y_bf16 != 0, bias, epi))
}

int sdb200_gemm_bf16_qkv_rope(int64_t M, int64_t K, const void* X, int64_t ldx, int x_bf16, const uint16_t* Wqkv,
                              int64_t ldw, const float* bias, int64_t Dq, int64_t S, const float* cos, const float* sin,
                              const float* gq, const float* gk, float eps, void* q16, void* k16, void* v16) {
  SDB_GUARD({
    const char* op = "gemm_bf16_qkv_rope";
    require(M >= 0 && K > 0 && Dq > 0 && S > 0, op, "bad shape");
    require(Dq % 128 == 0 && Dq <= ((int64_t)1 << 30), op, "Dq must be a multiple of 128 (heads of 128)");
    require(S <= ((int64_t)1 << 30), op, "S too large");
    require_ptr(cos, op, "cos");
    require_ptr(sin, op, "sin");
    if (M == 0) return kOk;
    // The epilogue reads the tables as cos at both columns of a rotary pair and
    // (-sin, +sin); they are rebuilt from rope()'s layout for this call.
    float* t = static_cast<float*>(pool_malloc((size_t)(2 * S * 128) * sizeof(float)));
    try {
      op_rope_pair_tables(cos, sin, t, t + S * 128, S);
      QkvRope r{};
      r.S = (int)S;
      r.Dq = (int)Dq;
      r.gq = gq;
      r.gk = gk;
      r.cs = t;
      r.sn = t + S * 128;
      r.eps = eps;
      r.q16 = q16;
      r.k16 = k16;
      r.v16 = v16;
      gemm_bf16_qkv_rope_impl(M, K, X, ldx, x_bf16 != 0, Wqkv, ldw, bias, r);
    } catch (...) {
      pool_free(t);
      throw;
    }
    // Stream-ordered: the next user of this block is issued on the same stream.
    pool_free(t);
  })
}

int sdb200_dit_post_norm(const float* partials, int64_t slot_rows, int world, int64_t row0, int64_t rows, float* x,
                         int64_t D, const float* gamma2, const float* gate, const float* gamma_next,
                         const float* scale_next, uint16_t* const* h_dst, int n_dst, float eps) {
  SDB_GUARD({
    const char* op = "dit_post_norm";
    require(rows >= 0 && row0 >= 0 && D > 0 && D <= 12288, op, "bad shape (0 < D <= 12288)");
    require(world >= 1 && world <= 8 && slot_rows >= rows, op, "world must be 1..8 and slot_rows >= rows");
    require(n_dst == 0 || n_dst == world, op, "n_dst must be 0 or world");
    if (rows == 0) return kOk;
    require_ptr(partials, op, "partials");
    require_ptr(x, op, "x");
    if (n_dst) require_ptr(h_dst, op, "h_dst");
    for (int i = 0; i < n_dst; ++i) require_ptr(h_dst[i], op, "h_dst[i]");
    dit_post_norm_mod_bcast(partials, slot_rows, world, row0, rows, x, (int)D, gamma2, gate, gamma_next, scale_next,
                            h_dst, n_dst, eps);
  })
}

int sdb200_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                     int heads, int kv_heads, int64_t d, int causal) {
  SDB_GUARD({
    const char* op = "attention";
    require(N >= 0 && Sq >= 0 && Skv >= 0 && d > 0, op, "bad shape");
    require(heads > 0 && kv_heads > 0 && heads % kv_heads == 0, op, "heads must be a multiple of kv_heads");
    if (N == 0 || Sq == 0) return kOk;
    require_ptr(out, op, "out");
    if (Skv == 0) {
      // No keys: the reference's score matrix is empty and its P V product a K = 0 GEMM
      // that leaves zeros (tensor.cpp:354-394, :776-810), so out is zero.
      check_cuda(cudaMemsetAsync(out, 0, (size_t)(N * Sq * heads * d) * sizeof(float), ctx().stream),
                 "cudaMemsetAsync(attention)");
      return kOk;
    }
    require_ptr(q, op, "q");
    require_ptr(k, op, "k");
    require_ptr(v, op, "v");
    launch_attention(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal != 0);
  })
}

int sdb200_attention_f16(const void* q, const void* k, const void* v, void* out, int out_bf16, int64_t N, int64_t Sq,
                         int64_t Skv, int heads, int kv_heads, int64_t d, int64_t dp, int causal) {
  SDB_GUARD({
    const char* op = "attention_f16";
    require(N >= 0 && Sq >= 0 && Skv >= 0 && d > 0, op, "bad shape");
    require(heads > 0 && kv_heads > 0 && heads % kv_heads == 0, op, "heads must be a multiple of kv_heads");
    require((dp == 64 && d <= 64) || (dp == 128 && d <= 128), op, "dp must be 64 (d <= 64) or 128 (d <= 128)");
    require_ptr(out, op, "out");
    if (N == 0 || Sq == 0) return kOk;
    if (Skv == 0) {  // no keys: zero output, as sdb200_attention
      const size_t esz = out_bf16 ? 2 : 4;
      check_cuda(cudaMemsetAsync(out, 0, (size_t)(N * Sq * heads * d) * esz, ctx().stream),
                 "cudaMemsetAsync(attention_f16)");
      return kOk;
    }
    require_ptr(q, op, "q");
    require_ptr(k, op, "k");
    require_ptr(v, op, "v");
    require(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0, op, "q/k/v must be 16-byte aligned");
    launch_attention_f16(q, k, v, out, (long long)heads * d, (long long)Sq * heads * d, out_bf16 != 0, N, Sq, Skv,
                         heads, kv_heads, d, dp, causal != 0);
  })
}

int sdb200_pack_heads_f16(const float* x, void* y, int64_t rows, int heads, int64_t d, int64_t dp) {
  SDB_GUARD({
    require(dp >= d && heads > 0 && rows >= 0, "pack_heads_f16", "bad shape");
    require_ptr(x, "pack_heads_f16", "x");
    require_ptr(y, "pack_heads_f16", "y");
    launch_pack_heads_f16(x, y, rows, heads, d, dp);
  })
}

int sdb200_conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                  int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out, int64_t Ho, int64_t Wo) {
  SDB_GUARD(conv2d_impl(x, N, Cin, H, W, w, Cout, kh, kw, bias, stride, pad, out, Ho, Wo))
}
int sdb200_conv_pack_input(const float* x, float* xh, int64_t N, int64_t C, int64_t HW, int64_t cp) {
  SDB_GUARD({
    const char* op = "conv_pack_input";
    require(N >= 0 && C > 0 && HW >= 0 && cp >= C && cp % 4 == 0, op, "bad shape (cp must be >= C and % 4 == 0)");
    require_ptr(x, op, "x");
    require_ptr(xh, op, "xh");
    launch_conv_pack_x(x, xh, N, C, HW, cp);
  })
}
int sdb200_conv_pack_weight(const float* w, float* wp, int64_t Cout, int64_t Cin, int64_t taps, int64_t cq) {
  SDB_GUARD({
    const char* op = "conv_pack_weight";
    require(Cout > 0 && Cin > 0 && taps > 0 && cq >= Cin && cq % 32 == 0, op,
            "bad shape (cq must be >= Cin and % 32 == 0)");
    require_ptr(w, op, "w");
    require_ptr(wp, op, "wp");
    launch_conv_pack_w(w, wp, Cout, Cin, taps, cq);
  })
}
int sdb200_conv2d_nhwc(const float* xh, int64_t N, int64_t Cin, int64_t cp, int64_t H, int64_t W, const float* wp,
                       int64_t cq, int64_t Cout, int64_t kh, int64_t kw, int pad, const float* bias, const float* res,
                       float* out, int64_t Ho, int64_t Wo) {
  SDB_GUARD({
    const char* op = "conv2d_nhwc";
    require(N >= 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0 && kh > 0 && kw > 0 && pad >= 0 && Ho >= 0 && Wo >= 0,
            op, "bad shape");
    require(cp >= Cin && cp % 4 == 0 && cq >= Cin && cq % 32 == 0, op, "bad packed channel pitch");
    require_ptr(xh, op, "xh");
    require_ptr(wp, op, "wp");
    require_ptr(out, op, "out");
    require((reinterpret_cast<uintptr_t>(xh) & 15) == 0 && (reinterpret_cast<uintptr_t>(wp) & 15) == 0, op,
            "xh and wp must be 16-byte aligned");
    if (N > 0 && Ho > 0 && Wo > 0)
      launch_conv_tc(xh, N, Cin, cp, H, W, wp, cq, Cout, (int)kh, (int)kw, pad, bias, res, out, Ho, Wo);
  })
}
int sdb200_group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                      const float* beta, float eps) {
  SDB_GUARD({
    require(groups > 0 && C % groups == 0, "group_norm", "channels not divisible by groups");
    require_ptr(gamma, "group_norm", "gamma");
    require_ptr(beta, "group_norm", "beta");
    op_group_norm(x, y, N, C, HW, groups, gamma, beta, eps);
  })
}
int sdb200_layer_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta,
                      float eps) {
  SDB_GUARD(op_row_norm(x, y, rows, C, gamma, beta, eps, false))
}
int sdb200_rms_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, float eps) {
  SDB_GUARD(op_row_norm(x, y, rows, C, gamma, nullptr, eps, true))
}
int sdb200_rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps) {
  SDB_GUARD(op_rms_norm_heads(x, groups, dim, gamma, eps))
}
int sdb200_rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cos, const float* sin,
                int interleaved) {
  SDB_GUARD({
    require(dim > 0 && dim % 2 == 0 && inner % dim == 0, "rope", "inner must be a multiple of an even dim");
    op_rope(x, N, S, inner, dim, cos, sin, interleaved != 0);
  })
}
int sdb200_softmax_rows(float* x, int64_t rows, int64_t cols, float scale, int causal) {
  SDB_GUARD(op_softmax_rows(x, rows, cols, scale, causal != 0, rows > 0 ? rows : 1))
}
int sdb200_geglu(const float* x, float* y, int64_t rows, int64_t D) { SDB_GUARD(op_geglu(x, y, rows, D)) }
int sdb200_swiglu(const float* gate, const float* up, float* y, int64_t n) { SDB_GUARD(op_swiglu(gate, up, y, n)) }
int sdb200_silu(float* x, int64_t n) { SDB_GUARD(op_unary(x, n, 0)) }
int sdb200_gelu(float* x, int64_t n) { SDB_GUARD(op_unary(x, n, 1)) }
int sdb200_quick_gelu(float* x, int64_t n) { SDB_GUARD(op_unary(x, n, 2)) }
int sdb200_tanh(float* x, int64_t n) { SDB_GUARD(op_unary(x, n, 3)) }
int sdb200_add(float* a, const float* b, int64_t n) { SDB_GUARD(op_add(a, b, n)) }
int sdb200_scale(float* x, float s, int64_t n) { SDB_GUARD(op_affine(x, s, 0.0f, n)) }
int sdb200_affine(float* x, float a, float b, int64_t n) { SDB_GUARD(op_affine(x, a, b, n)) }
int sdb200_mul_rows(float* x, const float* v, int64_t rows, int64_t dim) { SDB_GUARD(op_mul_rows(x, v, rows, dim)) }
int sdb200_add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim) {
  SDB_GUARD(op_add_rows_scaled(x, y, g, rows, dim))
}
int sdb200_add_channel_bias(float* x, const float* b, int64_t N, int64_t C, int64_t HW) {
  SDB_GUARD(op_add_channel_bias(x, b, N, C, HW))
}
int sdb200_upsample_nearest2x(const float* x, float* y, int64_t NC, int64_t H, int64_t W) {
  SDB_GUARD(op_upsample2x(x, y, NC, H, W))
}
int sdb200_concat_channels(const float* a, const float* b, float* y, int64_t N, int64_t Ca, int64_t Cb, int64_t HW) {
  SDB_GUARD(op_concat_channels(a, b, y, N, Ca, Cb, HW))
}
int sdb200_nchw_to_nlc(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  SDB_GUARD(op_nchw_to_nlc(x, y, N, C, HW))
}
int sdb200_nlc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  SDB_GUARD(op_nlc_to_nchw(x, y, N, C, HW))
}
int sdb200_patchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  SDB_GUARD({
    require(p > 0 && H % p == 0 && W % p == 0, "patchify", "H and W must be multiples of p");
    op_patchify(x, y, C, H, W, p);
  })
}
int sdb200_unpatchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  SDB_GUARD({
    require(p > 0 && H % p == 0 && W % p == 0, "unpatchify", "H and W must be multiples of p");
    op_unpatchify(x, y, C, H, W, p);
  })
}

}  // extern "C"
