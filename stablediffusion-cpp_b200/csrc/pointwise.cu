// pointwise.cu - the value-wise and layout ops of the backend API that are not
// contractions (backend_cuda.h:60-80): activations, gated units, row and channel
// broadcasts, RoPE, and the NCHW / token layout changes. None of them is on the DiT's
// hot path - the device programs fold this work into GEMM epilogues and norm kernels -
// they are here so that the library replaces the whole backend interface.
//
// Design. Every value-wise op is a functor with a scalar form one(i) (one unit) and a
// vector form four(j) (units 4j .. 4j+3 through 16-byte loads and stores). One kernel
// template, k_pointwise, runs four() over the whole groups of four and one() over the
// tail; the launcher takes the vector form only when every pointer is 16-byte aligned
// and every width the op broadcasts over is a multiple of 4 (so a group of four never
// straddles a row, plane or head). Layout changes go through shared-memory tiles so that
// both the global reads and the global writes are contiguous.
//
// The value of each element is the reference CPU expression (tensor.cpp, cited per op)
// evaluated in the same order; the GPU tests hold the results to the reference's golden
// outputs.
#include <algorithm>
#include <cmath>

#include "internal.h"

namespace sdb {
namespace {

constexpr int kThreads = 256;

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float4 ld4(const float* p, int64_t j) { return reinterpret_cast<const float4*>(p)[j]; }
__device__ __forceinline__ void st4(float* p, int64_t j, float4 v) { reinterpret_cast<float4*>(p)[j] = v; }

template <class Op>
__global__ void __launch_bounds__(kThreads) k_pointwise(Op op, int64_t units, int vec) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  int64_t tail = 0;
  if (vec) {
    const int64_t groups = units >> 2;
    for (int64_t j = t; j < groups; j += step) op.four(j);
    tail = groups << 2;
  }
  for (int64_t i = tail + t; i < units; i += step) op.one(i);
}

// Grid of at most 16 CTAs per SM over `units` (four per thread in the vector form).
template <class Op>
void run_pointwise(const Op& op, int64_t units, bool vec, const char* what) {
  if (units <= 0) return;
  DeviceContext& c = ctx();
  const int64_t work = vec ? (units + 3) / 4 : units;
  const int64_t blocks = std::min<int64_t>((work + kThreads - 1) / kThreads, (int64_t)std::max(1, c.num_sms) * 16);
  k_pointwise<Op><<<(unsigned)std::max<int64_t>(1, blocks), kThreads, 0, c.stream>>>(op, units, vec ? 1 : 0);
  check_launch(what);
}

// ---- activations (tensor.cpp:843-867; backend_cuda.h:64-67) ---------------------------
__device__ __forceinline__ float activate(float v, int kind) {
  switch (kind) {
    case 0: return v / (1.0f + expf(-v));                               // silu
    case 1: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));  // gelu, erf form
    case 2: return v / (1.0f + expf(-1.702f * v));                      // quick_gelu
    default: return tanhf(v);                                           // tanh
  }
}
struct OpActivate {
  float* x;
  int kind;
  __device__ void one(int64_t i) const { x[i] = activate(x[i], kind); }
  __device__ void four(int64_t j) const {
    float4 v = ld4(x, j);
    v.x = activate(v.x, kind);
    v.y = activate(v.y, kind);
    v.z = activate(v.z, kind);
    v.w = activate(v.w, kind);
    st4(x, j, v);
  }
};

// x = x * a + b (tensor.cpp affine_)
struct OpAffine {
  float* x;
  float a, b;
  __device__ void one(int64_t i) const { x[i] = x[i] * a + b; }
  __device__ void four(int64_t j) const {
    float4 v = ld4(x, j);
    v.x = v.x * a + b;
    v.y = v.y * a + b;
    v.z = v.z * a + b;
    v.w = v.w * a + b;
    st4(x, j, v);
  }
};

// a += b (tensor.cpp add_)
struct OpAccumulate {
  float* a;
  const float* b;
  __device__ void one(int64_t i) const { a[i] += b[i]; }
  __device__ void four(int64_t j) const {
    float4 u = ld4(a, j);
    const float4 v = ld4(b, j);
    u.x += v.x;
    u.y += v.y;
    u.z += v.z;
    u.w += v.w;
    st4(a, j, u);
  }
};

// y = silu(g) * u (tensor.cpp:732-748)
__device__ __forceinline__ float swish_gate(float g, float u) { return g / (1.0f + expf(-g)) * u; }
struct OpSwiglu {
  const float* g;
  const float* u;
  float* y;
  __device__ void one(int64_t i) const { y[i] = swish_gate(g[i], u[i]); }
  __device__ void four(int64_t j) const {
    const float4 a = ld4(g, j), b = ld4(u, j);
    st4(y, j, make_float4(swish_gate(a.x, b.x), swish_gate(a.y, b.y), swish_gate(a.z, b.z), swish_gate(a.w, b.w)));
  }
};

// y[r, c] = x[r, c] * gelu_erf(x[r, D + c]) over [rows, 2D] -> [rows, D] (tensor.cpp:813-835)
__device__ __forceinline__ float erf_gate(float a, float g) {
  return a * 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
}
struct OpGeglu {
  const float* x;
  float* y;
  int64_t D;
  __device__ void one(int64_t i) const {
    const int64_t r = i / D, c = i - r * D;
    const float* row = x + 2 * D * r;
    y[i] = erf_gate(row[c], row[D + c]);
  }
  __device__ void four(int64_t j) const {  // D % 4 == 0: the four outputs share a row
    const int64_t i = 4 * j, r = i / D, c = i - r * D;
    const float* row = x + 2 * D * r;
    const float4 a = *reinterpret_cast<const float4*>(row + c), g = *reinterpret_cast<const float4*>(row + D + c);
    st4(y, j, make_float4(erf_gate(a.x, g.x), erf_gate(a.y, g.y), erf_gate(a.z, g.z), erf_gate(a.w, g.w)));
  }
};

// x[r, c] *= v[c] (tensor.cpp:889-901)
struct OpScaleColumns {
  float* x;
  const float* v;
  int64_t dim;
  __device__ void one(int64_t i) const { x[i] *= v[i % dim]; }
  __device__ void four(int64_t j) const {  // dim % 4 == 0
    float4 a = ld4(x, j);
    const float4 s = *reinterpret_cast<const float4*>(v + (4 * j) % dim);
    a.x *= s.x;
    a.y *= s.y;
    a.z *= s.z;
    a.w *= s.w;
    st4(x, j, a);
  }
};

// x[r, c] += g[c] * y[r, c] (tensor.cpp:903-917)
struct OpGatedAccumulate {
  float* x;
  const float* y;
  const float* g;
  int64_t dim;
  __device__ void one(int64_t i) const { x[i] += g[i % dim] * y[i]; }
  __device__ void four(int64_t j) const {  // dim % 4 == 0
    float4 a = ld4(x, j);
    const float4 b = ld4(y, j);
    const float4 s = *reinterpret_cast<const float4*>(g + (4 * j) % dim);
    a.x += s.x * b.x;
    a.y += s.y * b.y;
    a.z += s.z * b.z;
    a.w += s.w * b.w;
    st4(x, j, a);
  }
};

// x[plane, s] += b[plane] for planes of HW values (b is [N, C]; tensor.cpp:919-930)
struct OpPlaneBias {
  float* x;
  const float* b;
  int64_t HW;
  __device__ void one(int64_t i) const { x[i] += b[i / HW]; }
  __device__ void four(int64_t j) const {  // HW % 4 == 0: one plane per group
    float4 a = ld4(x, j);
    const float s = b[(4 * j) / HW];
    a.x += s;
    a.y += s;
    a.z += s;
    a.w += s;
    st4(x, j, a);
  }
};

// C[r, c] += b[r] over M x N with row pitch ldc (the bias of a conv GEMM lowered as
// out = W * cols, tensor.cpp:576-585)
struct OpRowBias {
  float* C;
  const float* b;
  int64_t N, ldc;
  __device__ void one(int64_t i) const {
    const int64_t r = i / N;
    C[r * ldc + (i - r * N)] += b[r];
  }
  __device__ void four(int64_t j) const {  // N % 4 == 0 and ldc % 4 == 0
    const int64_t i = 4 * j, r = i / N;
    float* p = C + r * ldc + (i - r * N);
    float4 a = *reinterpret_cast<float4*>(p);
    const float s = b[r];
    a.x += s;
    a.y += s;
    a.z += s;
    a.w += s;
    *reinterpret_cast<float4*>(p) = a;
  }
};

// Rotary embedding in place on x [N*S, inner], heads of `dim` values, tables [S, dim]
// (tensor.cpp:701-730). One unit is one rotated pair: (2k, 2k+1) with the angle at 2k when
// interleaved, else (k, k + dim/2) with the angles at k and k + dim/2.
__device__ __forceinline__ void rotate(float& u, float& w, float ca, float sa, float cb, float sb) {
  const float nu = u * ca - w * sa;
  const float nw = w * cb + u * sb;
  u = nu;
  w = nw;
}
// Rotary tables of rope() (cos / sin [S, 128], interleaved: pair i of row s uses column
// 2i) -> the operand layout of the fused QKV epilogue (Epi::kQkvRope): cs holds cos at
// 2i and 2i + 1, sn holds (-sin, +sin). One unit is one pair.
struct OpRopePairTables {
  const float* cos;
  const float* sin;
  float* cs;
  float* sn;
  __device__ void one(int64_t u) const {
    const int64_t o = 2 * u;  // row s * 128 + column 2i
    const float c = cos[o], sv = sin[o];
    cs[o] = c;
    cs[o + 1] = c;
    sn[o] = -sv;
    sn[o + 1] = sv;
  }
  __device__ void four(int64_t j) const {
#pragma unroll
    for (int q = 0; q < 4; ++q) one(4 * j + q);
  }
};
struct OpRope {
  float* x;
  const float* cs;
  const float* sn;
  int64_t S, inner, dim;
  int interleaved;
  __device__ void locate(int64_t pair, float*& head, const float*& c, const float*& s, int64_t& k) const {
    const int64_t half = dim / 2, per_token = (inner / dim) * half;
    const int64_t tok = pair / per_token, r = pair - tok * per_token, h = r / half;
    k = r - h * half;
    head = x + tok * inner + h * dim;
    c = cs + (tok % S) * dim;
    s = sn + (tok % S) * dim;
  }
  __device__ void one(int64_t pair) const {
    float* p;
    const float *c, *s;
    int64_t k;
    locate(pair, p, c, s, k);
    if (interleaved) {
      rotate(p[2 * k], p[2 * k + 1], c[2 * k], s[2 * k], c[2 * k], s[2 * k]);
    } else {
      const int64_t h2 = dim / 2;
      rotate(p[k], p[k + h2], c[k], s[k], c[k + h2], s[k + h2]);
    }
  }
  __device__ void four(int64_t j) const {  // (dim / 2) % 4 == 0: four pairs of one head
    float* p;
    const float *c, *s;
    int64_t k;
    locate(4 * j, p, c, s, k);
    if (interleaved) {  // pairs k..k+3 = values 2k..2k+7
      float4 a = *reinterpret_cast<float4*>(p + 2 * k), b = *reinterpret_cast<float4*>(p + 2 * k + 4);
      const float4 c0 = *reinterpret_cast<const float4*>(c + 2 * k), c1 = *reinterpret_cast<const float4*>(c + 2 * k + 4);
      const float4 s0 = *reinterpret_cast<const float4*>(s + 2 * k), s1 = *reinterpret_cast<const float4*>(s + 2 * k + 4);
      rotate(a.x, a.y, c0.x, s0.x, c0.x, s0.x);
      rotate(a.z, a.w, c0.z, s0.z, c0.z, s0.z);
      rotate(b.x, b.y, c1.x, s1.x, c1.x, s1.x);
      rotate(b.z, b.w, c1.z, s1.z, c1.z, s1.z);
      *reinterpret_cast<float4*>(p + 2 * k) = a;
      *reinterpret_cast<float4*>(p + 2 * k + 4) = b;
    } else {
      const int64_t h2 = dim / 2;
      float4 a = *reinterpret_cast<float4*>(p + k), b = *reinterpret_cast<float4*>(p + k + h2);
      const float4 ca = *reinterpret_cast<const float4*>(c + k), cb = *reinterpret_cast<const float4*>(c + k + h2);
      const float4 sa = *reinterpret_cast<const float4*>(s + k), sb = *reinterpret_cast<const float4*>(s + k + h2);
      rotate(a.x, b.x, ca.x, sa.x, cb.x, sb.x);
      rotate(a.y, b.y, ca.y, sa.y, cb.y, sb.y);
      rotate(a.z, b.z, ca.z, sa.z, cb.z, sb.z);
      rotate(a.w, b.w, ca.w, sa.w, cb.w, sb.w);
      *reinterpret_cast<float4*>(p + k) = a;
      *reinterpret_cast<float4*>(p + k + h2) = b;
    }
  }
};

// Nearest 2x upsampling of NC planes [H, W] -> [2H, 2W]; one unit is one input value,
// written to a 2 x 2 block (tensor.cpp upsample_nearest2x).
struct OpUpsample2x {
  const float* x;
  float* y;
  int64_t W;
  __device__ void one(int64_t i) const {
    const int64_t row = i / W, c = i - row * W;  // row indexes (plane, h) pairs
    float* o = y + 4 * W * row + 2 * c;
    const float v = x[i];
    o[0] = v;
    o[1] = v;
    o[2 * W] = v;
    o[2 * W + 1] = v;
  }
  __device__ void four(int64_t j) const {  // W % 4 == 0: four values of one input row
    const int64_t i = 4 * j, row = i / W, c = i - row * W;
    const float4 v = ld4(x, j);
    float* o = y + 4 * W * row + 2 * c;
    const float4 lo = make_float4(v.x, v.x, v.y, v.y), hi = make_float4(v.z, v.z, v.w, v.w);
    *reinterpret_cast<float4*>(o) = lo;
    *reinterpret_cast<float4*>(o + 4) = hi;
    *reinterpret_cast<float4*>(o + 2 * W) = lo;
    *reinterpret_cast<float4*>(o + 2 * W + 4) = hi;
  }
};

// y[n] = a[n] followed by b[n]: per sample, A = Ca*HW then B = Cb*HW contiguous values.
struct OpJoinSamples {
  const float* a;
  const float* b;
  float* y;
  int64_t A, B;
  __device__ float at(int64_t i) const {
    const int64_t n = i / (A + B), r = i - n * (A + B);
    return r < A ? a[n * A + r] : b[n * B + (r - A)];
  }
  __device__ void one(int64_t i) const { y[i] = at(i); }
  __device__ void four(int64_t j) const {  // A % 4 == 0 and B % 4 == 0: one source per group
    const int64_t i = 4 * j, n = i / (A + B), r = i - n * (A + B);
    const float4 v = r < A ? *reinterpret_cast<const float4*>(a + n * A + r)
                           : *reinterpret_cast<const float4*>(b + n * B + (r - A));
    st4(y, j, v);
  }
};

// ---- layout changes through shared memory ---------------------------------------------
// dst[z][c][r] = src[z][r][c] for `batch` matrices [rows, cols]: 32 x 32 tiles with a
// padded row (no bank conflicts), coalesced on both sides. NCHW <-> NLC per sample.
__global__ void __launch_bounds__(256) k_transpose_planes(const float* __restrict__ src, float* __restrict__ dst,
                                                          int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t z = blockIdx.z;
  const float* s = src + z * rows * cols;
  float* d = dst + z * rows * cols;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    const int64_t r = r0 + ty + k, c = c0 + tx;
    if (r < rows && c < cols) tile[ty + k][tx] = s[r * cols + c];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    const int64_t c = c0 + ty + k, r = r0 + tx;
    if (c < cols && r < rows) d[c * rows + r] = tile[tx][ty + k];
  }
}

void transpose_planes(const float* src, float* dst, int64_t batch, int64_t rows, int64_t cols, const char* what) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return;
  if (batch > 65535 || (rows + 31) / 32 > 65535) fail(kErrInvalidArg, std::string(what) + ": too many rows or samples");
  const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
  k_transpose_planes<<<grid, 256, 0, ctx().stream>>>(src, dst, rows, cols);
  check_launch(what);
}

// Image [C, H, W] <-> patch tokens [(H/p)(W/p), p*p*C] with token feature (ph*p + pw)*C + c
// (tensor.cpp patchify / unpatchify). One CTA moves `wt` tokens of one token row: the C*p
// image row segments they cover (wt*p contiguous values each) and their wt*p*p*C
// contiguous token values, both staged in shared memory as [c][ph][x].
template <bool kToTokens>
__global__ void __launch_bounds__(256) k_patch_rows(const float* __restrict__ src, float* __restrict__ dst, int C,
                                                    int H, int W, int p, int wt) {
  extern __shared__ float seg[];  // [C][p][wt * p]
  const int Wt = W / p, F = p * p * C, span = wt * p;
  const int h = blockIdx.y, w0 = blockIdx.x * wt;
  const int nw = min(wt, Wt - w0), nspan = nw * p;
  const int64_t tok0 = (int64_t)h * Wt + w0;
  if (kToTokens) {
    for (int e = threadIdx.x; e < C * p * nspan; e += blockDim.x) {
      const int line = e / nspan, x = e - line * nspan, c = line / p, ph = line - c * p;
      seg[line * span + x] = src[((int64_t)c * H + h * p + ph) * W + (int64_t)w0 * p + x];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nw * F; e += blockDim.x) {
      const int t = e / F, f = e - t * F, q = f / C, c = f - q * C, ph = q / p, pw = q - ph * p;
      dst[tok0 * F + e] = seg[(c * p + ph) * span + t * p + pw];
    }
  } else {
    for (int e = threadIdx.x; e < nw * F; e += blockDim.x) {
      const int t = e / F, f = e - t * F, q = f / C, c = f - q * C, ph = q / p, pw = q - ph * p;
      seg[(c * p + ph) * span + t * p + pw] = src[tok0 * F + e];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < C * p * nspan; e += blockDim.x) {
      const int line = e / nspan, x = e - line * nspan, c = line / p, ph = line - c * p;
      dst[((int64_t)c * H + h * p + ph) * W + (int64_t)w0 * p + x] = seg[line * span + x];
    }
  }
}

void patch_rows(const float* src, float* dst, int64_t C, int64_t H, int64_t W, int p, bool to_tokens) {
  if (C * H * W <= 0) return;
  const char* what = to_tokens ? "patchify" : "unpatchify";
  if (p < 1 || H % p || W % p) fail(kErrInvalidArg, std::string(what) + ": H and W must be multiples of p");
  if (C > (1 << 20) || H > (1 << 24) || W > (1 << 24)) fail(kErrInvalidArg, std::string(what) + ": size too large");
  const int64_t Wt = W / p, per_tok = (int64_t)p * p * C;  // values one token moves
  const int64_t wt = std::max<int64_t>(1, std::min<int64_t>(Wt, 8192 / per_tok));
  const size_t smem = (size_t)(C * p * wt * p) * sizeof(float);
  if (smem > 96 * 1024) fail(kErrInvalidArg, std::string(what) + ": p * p * C too large for one staging tile");
  const dim3 grid((unsigned)((Wt + wt - 1) / wt), (unsigned)(H / p));
  if (grid.y > 65535) fail(kErrInvalidArg, std::string(what) + ": too many token rows");
  if (to_tokens) {
    if (smem > 48 * 1024)
      check_cuda(cudaFuncSetAttribute(k_patch_rows<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024),
                 "patchify attr");
    k_patch_rows<true><<<grid, 256, smem, ctx().stream>>>(src, dst, (int)C, (int)H, (int)W, p, (int)wt);
  } else {
    if (smem > 48 * 1024)
      check_cuda(cudaFuncSetAttribute(k_patch_rows<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024),
                 "unpatchify attr");
    k_patch_rows<false><<<grid, 256, smem, ctx().stream>>>(src, dst, (int)C, (int)H, (int)W, p, (int)wt);
  }
  check_launch(what);
}

}  // namespace

// ---- launchers (declared in internal.h; arguments validated by the C ABI) -------------
void op_unary(float* x, int64_t n, int op) {
  run_pointwise(OpActivate{x, op}, n, al16(x), "unary");
}
void op_affine(float* x, float a, float b, int64_t n) { run_pointwise(OpAffine{x, a, b}, n, al16(x), "affine"); }
void op_add(float* a, const float* b, int64_t n) {
  run_pointwise(OpAccumulate{a, b}, n, al16(a) && al16(b), "add");
}
void op_swiglu(const float* g, const float* u, float* y, int64_t n) {
  run_pointwise(OpSwiglu{g, u, y}, n, al16(g) && al16(u) && al16(y), "swiglu");
}
void op_geglu(const float* x, float* y, int64_t rows, int64_t D) {
  run_pointwise(OpGeglu{x, y, D}, rows * D, D % 4 == 0 && al16(x) && al16(y), "geglu");
}
void op_mul_rows(float* x, const float* v, int64_t rows, int64_t dim) {
  run_pointwise(OpScaleColumns{x, v, dim}, rows * dim, dim % 4 == 0 && al16(x) && al16(v), "mul_rows");
}
void op_add_rows_scaled(float* x, const float* y, const float* g, int64_t rows, int64_t dim) {
  run_pointwise(OpGatedAccumulate{x, y, g, dim}, rows * dim, dim % 4 == 0 && al16(x) && al16(y) && al16(g),
                "add_rows_scaled");
}
void op_add_channel_bias(float* x, const float* b, int64_t N, int64_t C, int64_t HW) {
  run_pointwise(OpPlaneBias{x, b, HW}, N * C * HW, HW % 4 == 0 && al16(x), "add_channel_bias");
}
void op_add_bias_rows(float* C, int64_t ldc, int64_t M, int64_t N, const float* b) {
  run_pointwise(OpRowBias{C, b, N, ldc}, M * N, N % 4 == 0 && ldc % 4 == 0 && al16(C), "add_bias_rows");
}
void op_rope(float* x, int64_t N, int64_t S, int64_t inner, int64_t dim, const float* cs, const float* sn,
             bool interleaved) {
  const int64_t pairs = N * S * (inner / dim) * (dim / 2);
  const bool vec = (dim / 2) % 4 == 0 && inner % 4 == 0 && al16(x) && al16(cs) && al16(sn);
  run_pointwise(OpRope{x, cs, sn, S, inner, dim, interleaved ? 1 : 0}, pairs, vec, "rope");
}
void op_rope_pair_tables(const float* cos, const float* sin, float* cs, float* sn, int64_t S) {
  run_pointwise(OpRopePairTables{cos, sin, cs, sn}, S * 64, 1, "rope_pair_tables");
}
void op_upsample2x(const float* x, float* y, int64_t NC, int64_t H, int64_t W) {
  run_pointwise(OpUpsample2x{x, y, W}, NC * H * W, W % 4 == 0 && al16(x) && al16(y), "upsample_nearest2x");
}
void op_concat_channels(const float* a, const float* b, float* y, int64_t N, int64_t Ca, int64_t Cb, int64_t HW) {
  const int64_t A = Ca * HW, B = Cb * HW;
  run_pointwise(OpJoinSamples{a, b, y, A, B}, N * (A + B), A % 4 == 0 && B % 4 == 0 && al16(a) && al16(b) && al16(y),
                "concat_channels");
}
void op_nchw_to_nlc(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  transpose_planes(x, y, N, C, HW, "nchw_to_nlc");
}
void op_nlc_to_nchw(const float* x, float* y, int64_t N, int64_t C, int64_t HW) {
  transpose_planes(x, y, N, HW, C, "nlc_to_nchw");
}
void op_patchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  patch_rows(x, y, C, H, W, p, true);
}
void op_unpatchify(const float* x, float* y, int64_t C, int64_t H, int64_t W, int p) {
  patch_rows(x, y, C, H, W, p, false);
}

}  // namespace sdb
