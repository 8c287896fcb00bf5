// ref_shim.cpp - TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// Exposes the reference's own CPU implementation (StableDiffusion-cpp src/tensor.cpp,
// src/zimage.cpp, src/modules.cpp, compiled unmodified from their location in the
// reference tree by oracle/Makefile) through plain C entry points, so the parity tests
// and the CPU baseline can call it with numpy buffers. Every function copies its
// inputs into sd::Tensor objects, runs the reference op, and copies the result out.
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "backend_cuda.h"
#include "safetensors.h"
#include "scheduler.h"
#include "tensor.h"
#include "unet.h"
#include "vae.h"
#include "zimage.h"

using namespace sd;

namespace {
thread_local std::string g_err;

Tensor make(const float* p, std::vector<int64_t> shape) {
  Tensor t(shape);
  if (t.numel()) std::memcpy(t.ptr(), p, (size_t)t.numel() * sizeof(float));
  return t;
}
void put(const Tensor& t, float* out) { std::memcpy(out, t.ptr(), (size_t)t.numel() * sizeof(float)); }

template <class F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}
}  // namespace

extern "C" {

const char* sdref_last_error() { return g_err.c_str(); }
void sdref_set_num_threads(int n) { set_num_threads(n); }
int sdref_num_threads() { return num_threads(); }

uint16_t sdref_f32_to_bf16(float f) { return f32_to_bf16(f); }
void sdref_f32_to_bf16_array(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f32_to_bf16(x[i]);
}

// tensor.cpp:354 gemm_nt
void sdref_gemm_nt(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                   int64_t ldc, const float* bias, int acc) {
  gemm_nt(M, N, K, A, lda, B, ldb, C, ldc, bias, acc != 0);
}
// tensor.cpp:412 gemm_nt_bf16
void sdref_gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B, int64_t ldb,
                        float* C, int64_t ldc, const float* bias, int acc) {
  gemm_nt_bf16(M, N, K, A, lda, B, ldb, C, ldc, bias, acc != 0);
}

// tensor.cpp:776 attention; q [N,Sq,heads*d], k/v [N,Skv,kv_heads*d]
int sdref_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq, int64_t Skv,
                    int heads, int kv_heads, int64_t d, int causal) {
  return guard([&] {
    Tensor tq = make(q, {N, Sq, heads * d});
    Tensor tk = make(k, {N, Skv, kv_heads * d});
    Tensor tv = make(v, {N, Skv, kv_heads * d});
    put(attention(tq, tk, tv, heads, causal != 0, kv_heads), out);
  });
}

// tensor.cpp:752 softmax_rows_ (in place)
void sdref_softmax_rows(float* x, int64_t rows, int64_t cols, float scale, int causal) {
  softmax_rows_(x, rows, cols, scale, causal != 0);
}

int sdref_rms_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, float eps) {
  return guard([&] {
    Tensor tx = make(x, {rows, C});
    Tensor g = gamma ? make(gamma, {C}) : Tensor();
    put(rms_norm(tx, gamma ? &g : nullptr, eps), y);
  });
}
int sdref_layer_norm(const float* x, float* y, int64_t rows, int64_t C, const float* gamma, const float* beta,
                     float eps) {
  return guard([&] {
    Tensor tx = make(x, {rows, C});
    Tensor g = gamma ? make(gamma, {C}) : Tensor();
    Tensor b = beta ? make(beta, {C}) : Tensor();
    put(layer_norm(tx, gamma ? &g : nullptr, beta ? &b : nullptr, eps), y);
  });
}
int sdref_rms_norm_heads(float* x, int64_t groups, int64_t dim, const float* gamma, float eps) {
  return guard([&] {
    Tensor tx = make(x, {groups, dim});
    Tensor g = gamma ? make(gamma, {dim}) : Tensor();
    rms_norm_heads_(tx, dim, gamma ? &g : nullptr, eps);
    put(tx, x);
  });
}
int sdref_rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cs, const float* sn,
               int interleaved) {
  return guard([&] {
    Tensor tx = make(x, {N, S, inner});
    Tensor c = make(cs, {S, dim}), s = make(sn, {S, dim});
    rope_(tx, dim, c, s, interleaved != 0);
    put(tx, x);
  });
}
int sdref_swiglu(const float* g, const float* u, float* y, int64_t n) {
  return guard([&] { put(swiglu(make(g, {n}), make(u, {n})), y); });
}
int sdref_geglu(const float* x, float* y, int64_t rows, int64_t D) {
  return guard([&] { put(geglu(make(x, {rows, 2 * D})), y); });
}
int sdref_group_norm(const float* x, float* y, int64_t N, int64_t C, int64_t HW, int groups, const float* gamma,
                     const float* beta, float eps) {
  return guard([&] {
    put(group_norm(make(x, {N, C, HW, 1}), groups, make(gamma, {C}), make(beta, {C}), eps), y);
  });
}
int sdref_conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                 int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out) {
  return guard([&] {
    Tensor tw = make(w, {Cout, Cin, kh, kw});
    Tensor b = bias ? make(bias, {Cout}) : Tensor();
    put(conv2d(make(x, {N, Cin, H, W}), tw, bias ? &b : nullptr, stride, pad), out);
  });
}
int sdref_mul_rows(float* x, const float* v, int64_t rows, int64_t dim) {
  return guard([&] {
    Tensor tx = make(x, {rows, dim});
    mul_rows_(tx, make(v, {dim}));
    put(tx, x);
  });
}
int sdref_add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim) {
  return guard([&] {
    Tensor tx = make(x, {rows, dim});
    add_rows_scaled_(tx, make(y, {rows, dim}), make(g, {dim}));
    put(tx, x);
  });
}

// ---- Z-Image transformer (zimage.cpp) on an in-memory random-init Weights ----------
void* sdref_weights_new() { return new Weights(); }
void sdref_weights_free(void* w) { delete static_cast<Weights*>(w); }
// Adds tensor `name`; bf16 != 0 stores it as BF16 with the reference's rounding
// (Tensor::to_bf16, tensor.cpp:128-134), as the loader does for large weights.
int sdref_weights_add(void* w, const char* name, const int64_t* shape, int ndim, const float* data, int bf16) {
  return guard([&] {
    std::vector<int64_t> s(shape, shape + ndim);
    Tensor t = make(data, s);
    if (bf16) t.to_bf16();
    static_cast<Weights*>(w)->tensors[name] = std::move(t);
  });
}
void* sdref_zimage_new(void* w, int heads, int patch, float norm_eps, float rope_theta, float t_scale, int ax0,
                       int ax1, int ax2) {
  try {
    ZImageTransformer::Config c;
    c.heads = heads;
    c.patch = patch;
    c.norm_eps = norm_eps;
    c.rope_theta = rope_theta;
    c.t_scale = t_scale;
    c.axes_dims[0] = ax0;
    c.axes_dims[1] = ax1;
    c.axes_dims[2] = ax2;
    return new ZImageTransformer(*static_cast<Weights*>(w), c);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void sdref_zimage_free(void* m) { delete static_cast<ZImageTransformer*>(m); }
// x [1, C, H, W], cap [1, L, capdim] -> out [1, C, H, W]
int sdref_zimage_forward(void* m, const float* x, int64_t C, int64_t H, int64_t W, float t, const float* cap,
                         int64_t L, int64_t capdim, float* out) {
  return guard([&] {
    Tensor tx = make(x, {1, C, H, W});
    Tensor tc = make(cap, {1, L, capdim});
    put(static_cast<ZImageTransformer*>(m)->forward(tx, t, tc), out);
  });
}

// ---- the reference's GPU backend (backend_cuda.cu + cuBLAS), in the build that links it
// instead of the stub (oracle/Makefile `refgpu`): a comparison column on the same B200.
int sdref_cuda_available() { return cuda::available() ? 1 : 0; }
int sdref_cuda_synchronize() { return guard([&] { cuda::synchronize(); }); }
// Weights::to_device(Device::CUDA) (safetensors.cpp:195-200): models keep their pointers.
int sdref_weights_to_cuda(void* w) { return guard([&] { static_cast<Weights*>(w)->to_device(Device::CUDA); }); }
// The transformer forward with its input moved to the device first and the output back.
int sdref_zimage_forward_cuda(void* m, const float* x, int64_t C, int64_t H, int64_t W, float t, const float* cap,
                              int64_t L, int64_t capdim, float* out) {
  return guard([&] {
    Tensor tx = make(x, {1, C, H, W}).to(Device::CUDA);
    Tensor tc = make(cap, {1, L, capdim}).to(Device::CUDA);
    put(static_cast<ZImageTransformer*>(m)->forward(tx, t, tc).to(Device::CPU), out);
  });
}
// Adds tensor `name` on the device with the contents of the caller's device buffer
// `src` (F32, or BF16 bit patterns when bf16 != 0), copied device to device. The storage
// is the reference's own (Tensor::to(Device::CUDA) of a zero host tensor, then
// cuda::copy), so its ops see a tensor exactly as Weights::to_device leaves one.
int sdref_weights_add_device(void* w, const char* name, const int64_t* shape, int ndim, const void* src, int bf16) {
  return guard([&] {
    std::vector<int64_t> s(shape, shape + ndim);
    Tensor host;
    host.shape = s;
    if (bf16) {
      host.dtype = DType::BF16;
      host.data16.assign((size_t)Tensor::numel_of(s), 0);
    } else {
      host.data.assign((size_t)Tensor::numel_of(s), 0.0f);
    }
    Tensor t = host.to(Device::CUDA);
    const size_t bytes = (size_t)Tensor::numel_of(s) * (bf16 ? 2 : 4);
    if (bytes) cuda::copy(bf16 ? (void*)t.dptr16() : (void*)t.dptr(), src, bytes);
    static_cast<Weights*>(w)->tensors[name] = std::move(t);
  });
}
// backend_cuda.h entry points on caller-owned device buffers.
int sdref_cuda_gemm_nt_bf16(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const uint16_t* B,
                            int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate) {
  return guard([&] { cuda::gemm_nt_bf16(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0); });
}
int sdref_cuda_gemm_nt_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                           float* C, int64_t ldc, const float* bias, int accumulate) {
  return guard([&] { cuda::gemm_nt_f32(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate != 0); });
}
int sdref_cuda_geglu(const float* x, float* y, int64_t rows, int64_t D) {
  return guard([&] { cuda::geglu(x, y, rows, D); });
}
int sdref_cuda_attention(const float* q, const float* k, const float* v, float* out, int64_t N, int64_t Sq,
                         int64_t Skv, int heads, int kv_heads, int64_t d, int causal) {
  return guard([&] { cuda::attention(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal != 0); });
}
int sdref_cuda_conv2d(const float* x, int64_t N, int64_t Cin, int64_t H, int64_t W, const float* w, int64_t Cout,
                      int64_t kh, int64_t kw, const float* bias, int stride, int pad, float* out, int64_t Ho,
                      int64_t Wo) {
  return guard([&] { cuda::conv2d(x, N, Cin, H, W, w, Cout, kh, kw, bias, stride, pad, out, Ho, Wo); });
}

// ---- SD 1.x UNet (unet.cpp) on an in-memory Weights ----------------------------------
void* sdref_unet_new(void* w, int heads) {
  try {
    return new UNet(*static_cast<Weights*>(w), heads);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void sdref_unet_free(void* m) { delete static_cast<UNet*>(m); }
// x [N, C, H, W], context [N, L, D] -> out [N, C, H, W]; on_device moves the inputs to the
// device first (weights already moved with sdref_weights_to_cuda) and the output back.
int sdref_unet_forward(void* m, const float* x, int64_t N, int64_t C, int64_t H, int64_t W, float t, const float* ctx,
                       int64_t L, int64_t D, float* out, int on_device) {
  return guard([&] {
    Tensor tx = make(x, {N, C, H, W}), tc = make(ctx, {N, L, D});
    if (on_device) {
      tx = tx.to(Device::CUDA);
      tc = tc.to(Device::CUDA);
    }
    Tensor y = static_cast<UNet*>(m)->forward(tx, t, tc);
    put(on_device ? y.to(Device::CPU) : y, out);
  });
}

// ---- VAE decoder (vae.cpp) on an in-memory Weights (sdref_weights_new / _add, fp32) --
void* sdref_vae_new(void* w, float scaling_factor, float shift_factor) {
  try {
    return new VAEDecoder(*static_cast<Weights*>(w), scaling_factor, shift_factor);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}
void sdref_vae_free(void* m) { delete static_cast<VAEDecoder*>(m); }
// The decode with the latent moved to the device and the image back (GPU backend build;
// the weights must have been moved with sdref_weights_to_cuda before sdref_vae_new).
int sdref_vae_decode_cuda(void* m, const float* z, int64_t N, int64_t C, int64_t h, int64_t w, float* out,
                          int64_t out_cap, int64_t* shape4) {
  return guard([&] {
    Tensor y = static_cast<VAEDecoder*>(m)->decode(make(z, {N, C, h, w}).to(Device::CUDA)).to(Device::CPU);
    if (y.ndim() != 4 || y.numel() > out_cap) throw std::runtime_error("sdref_vae_decode_cuda: output buffer too small");
    for (int i = 0; i < 4; ++i) shape4[i] = y.dim(i);
    put(y, out);
  });
}
// latents [N, C, h, w] -> out (capacity out_cap floats); shape4 receives the output shape.
int sdref_vae_decode(void* m, const float* z, int64_t N, int64_t C, int64_t h, int64_t w, float* out, int64_t out_cap,
                     int64_t* shape4) {
  return guard([&] {
    Tensor y = static_cast<VAEDecoder*>(m)->decode(make(z, {N, C, h, w}));
    if (y.ndim() != 4 || y.numel() > out_cap) throw std::runtime_error("sdref_vae_decode: output buffer too small");
    for (int i = 0; i < 4; ++i) shape4[i] = y.dim(i);
    put(y, out);
  });
}

// Weights::load_safetensors (safetensors.cpp:80-168) on one file; copies tensor `name`
// out as the reference stores it: BF16 bit patterns into out16 when it kept BF16, else
// F32 into out32. Returns 1 if BF16, 0 if F32, -1 on error (message in last_error), -2
// if the reference did not read that tensor.
int sdref_safetensors_tensor(const char* path, const char* name, int keep_bf16, int64_t min_numel, float* out32,
                             uint16_t* out16) {
  int res = -1;
  guard([&] {
    Weights w;
    w.load_safetensors(path, keep_bf16 != 0, min_numel);
    const Tensor* t = w.try_get(name);
    if (!t) {
      res = -2;
      return;
    }
    if (t->is_bf16()) {
      std::memcpy(out16, t->data16.data(), t->data16.size() * 2);
      res = 1;
    } else {
      std::memcpy(out32, t->data.data(), t->data.size() * 4);
      res = 0;
    }
  });
  return res;
}

// A ZImageTransformer over the checkpoint <dir>/<base> as the pipeline loads it
// (Weights::load_model with keep_bf16, pipeline.cpp:113); free with sdref_zimage_free and
// sdref_weights_free(*weights_out).
void* sdref_zimage_load(const char* dir, const char* base, int heads, int patch, float norm_eps, float rope_theta,
                        float t_scale, int ax0, int ax1, int ax2, void** weights_out) {
  void* model = nullptr;
  guard([&] {
    Weights* w = new Weights();
    try {
      w->load_model(dir, base, true);
      model = sdref_zimage_new(w, heads, patch, norm_eps, rope_theta, t_scale, ax0, ax1, ax2);
    } catch (...) {
      delete w;
      throw;
    }
    if (!model) {
      delete w;
      throw std::runtime_error(g_err);
    }
    *weights_out = w;
  });
  return model;
}

// FlowMatchScheduler (scheduler.cpp:117-135): sigmas[0..steps] and the model-facing times
// 1 - sigma_i of a `steps`-step schedule with the given shift.
int sdref_flow_sigmas(int steps, float shift, float* sigmas, float* model_times) {
  return guard([&] {
    FlowMatchScheduler s(shift);
    s.set_timesteps(steps);
    for (int i = 0; i <= steps; ++i) sigmas[i] = s.sigma(i);
    for (int i = 0; i < steps; ++i) model_times[i] = s.model_time(i);
  });
}

// One sampler step as the Z-Image pipeline takes it (pipeline.cpp:237-243): with cfg > 0,
// out += cfg * (out - neg) first, then FlowMatchScheduler::step(out, step, x).
int sdref_flow_step(float* x, const float* out, const float* neg, float cfg, int64_t n, int step, int steps,
                    float shift) {
  return guard([&] {
    FlowMatchScheduler s(shift);
    s.set_timesteps(steps);
    Tensor tx = make(x, {n});
    Tensor to = make(out, {n});
    if (neg && cfg > 0.0f)
      for (int64_t j = 0; j < n; ++j) to.ptr()[j] += cfg * (to.ptr()[j] - neg[j]);
    s.step(to, step, tx);
    put(tx, x);
  });
}

}  // extern "C"
