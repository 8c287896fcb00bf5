// sd_cuda_api.cpp - the reference backend's C++ entry points (namespace sd::cuda,
// src/backend_cuda.h:20-83) defined on top of this library's C ABI, so that the
// reference's tensor.cpp / zimage.cpp / unet.cpp link against libsdb200.so unchanged
// in place of build/backend_cuda.o (Makefile:35-47).
//
// The signatures have to be exactly the reference's (C++ linkage, int64_t sizes,
// bool flags) for the link to resolve; the declarations are written out here rather
// than included from the reference. Errors become std::runtime_error carrying the
// library's message, as backend_cuda.cu:41-48 reports failures.
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sdb200.h"

namespace {
inline void ok(int status, const char* what) {
  if (status != SDB200_OK) throw std::runtime_error(std::string(what) + ": " + sdb200_last_error());
}
}  // namespace

namespace sd {
namespace cuda {

bool available() { return sdb200_available() != 0; }
const char* device_name() { return sdb200_device_name(); }
size_t device_memory() { return sdb200_device_memory(); }

void* malloc(size_t bytes) {
  if (bytes == 0) return nullptr;
  void* p = sdb200_malloc(bytes);
  if (!p) throw std::runtime_error(std::string("cuda::malloc: ") + sdb200_last_error());
  return p;
}
void free(void* p) { ok(sdb200_free(p), "cuda::free"); }
void upload(void* dst, const void* src, size_t bytes) { ok(sdb200_upload(dst, src, bytes), "cuda::upload"); }
void download(void* dst, const void* src, size_t bytes) { ok(sdb200_download(dst, src, bytes), "cuda::download"); }
void copy(void* dst, const void* src, size_t bytes) { ok(sdb200_copy(dst, src, bytes), "cuda::copy"); }
void zero(void* dst, size_t bytes) { ok(sdb200_zero(dst, bytes), "cuda::zero"); }
void synchronize() { ok(sdb200_synchronize(), "cuda::synchronize"); }

void gemm_nt_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                 int64_t ldc, const float* bias, bool accumulate) {
  ok(sdb200_gemm_nt_f32(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate), "cuda::gemm_nt_f32");
}
void gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                  float* C, int64_t ldc, const float* bias, bool accumulate) {
  ok(sdb200_gemm_nt_bf16(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate), "cuda::gemm_nt_bf16");
}

void conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout, int64_t kh,
            int64_t kw, const float* bias, int stride, int pad, float* out, int64_t Ho, int64_t Wo) {
  ok(sdb200_conv2d(x, N, Cin, H, W, w, Cout, kh, kw, bias, stride, pad, out, Ho, Wo), "cuda::conv2d");
}
void group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                const float* beta, float eps) {
  ok(sdb200_group_norm(x, y, N, C, HW, groups, gamma, beta, eps), "cuda::group_norm");
}
void layer_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta, float eps) {
  ok(sdb200_layer_norm(x, y, rows, C, gamma, beta, eps), "cuda::layer_norm");
}
void rms_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, float eps) {
  ok(sdb200_rms_norm(x, y, rows, C, gamma, eps), "cuda::rms_norm");
}
void rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps) {
  ok(sdb200_rms_norm_heads(x, groups, dim, gamma, eps), "cuda::rms_norm_heads");
}
void rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cos, const float* sin,
          bool interleaved) {
  ok(sdb200_rope(x, N, S, inner, dim, cos, sin, interleaved), "cuda::rope");
}
void softmax_rows(float* x, int64_t rows, int64_t cols, float scale, bool causal) {
  ok(sdb200_softmax_rows(x, rows, cols, scale, causal), "cuda::softmax_rows");
}
void attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
               int heads, int kv_heads, int64_t d, bool causal) {
  ok(sdb200_attention(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal), "cuda::attention");
}
void geglu(const float* x, float* y, int64_t rows, int64_t D) { ok(sdb200_geglu(x, y, rows, D), "cuda::geglu"); }
void swiglu(const float* gate, const float* up, float* y, int64_t n) {
  ok(sdb200_swiglu(gate, up, y, n), "cuda::swiglu");
}

void silu(float* x, int64_t n) { ok(sdb200_silu(x, n), "cuda::silu"); }
void tanh(float* x, int64_t n) { ok(sdb200_tanh(x, n), "cuda::tanh"); }
void gelu(float* x, int64_t n) { ok(sdb200_gelu(x, n), "cuda::gelu"); }
void quick_gelu(float* x, int64_t n) { ok(sdb200_quick_gelu(x, n), "cuda::quick_gelu"); }
void add(float* a, const float* b, int64_t n) { ok(sdb200_add(a, b, n), "cuda::add"); }
void scale(float* x, float s, int64_t n) { ok(sdb200_scale(x, s, n), "cuda::scale"); }
void affine(float* x, float a, float b, int64_t n) { ok(sdb200_affine(x, a, b, n), "cuda::affine"); }
void mul_rows(float* x, const float* v, int64_t rows, int64_t dim) {
  ok(sdb200_mul_rows(x, v, rows, dim), "cuda::mul_rows");
}
void add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim) {
  ok(sdb200_add_rows_scaled(x, y, g, rows, dim), "cuda::add_rows_scaled");
}
void add_channel_bias(float* x, const float* b, int64_t N, int64_t C, int64_t HW) {
  ok(sdb200_add_channel_bias(x, b, N, C, HW), "cuda::add_channel_bias");
}
void upsample_nearest2x(const float* x, float* y, int64_t NC, int64_t H, int64_t W) {
  ok(sdb200_upsample_nearest2x(x, y, NC, H, W), "cuda::upsample_nearest2x");
}
void concat_channels(const float* a, const float* b, float* y, int64_t N, int64_t Ca, int64_t Cb, int64_t HW) {
  ok(sdb200_concat_channels(a, b, y, N, Ca, Cb, HW), "cuda::concat_channels");
}
void nchw_to_nlc(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  ok(sdb200_nchw_to_nlc(x, y, N, C, HW), "cuda::nchw_to_nlc");
}
void nlc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  ok(sdb200_nlc_to_nchw(x, y, N, C, HW), "cuda::nlc_to_nchw");
}
void patchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  ok(sdb200_patchify(x, y, C, H, W, p), "cuda::patchify");
}
void unpatchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  ok(sdb200_unpatchify(x, y, C, H, W, p), "cuda::unpatchify");
}

}  // namespace cuda
}  // namespace sd
