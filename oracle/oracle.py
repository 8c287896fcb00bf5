"""TEST INFRASTRUCTURE ONLY: numpy front-end of the two CPU checkers.

* ``Oracle``  - the C restatement of the reference CPU path (``oracle/oracle.c`` ->
  ``oracle/liboracle.so``).
* ``RefCPU``  - the reference's own CPU path (StableDiffusion-cpp ``src/tensor.cpp``,
  ``src/zimage.cpp`` ...) compiled from its sources by ``oracle/Makefile`` into
  ``oracle/_ref/libsdref.so``; available where that library was built.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this module, and only as the checker / the timed CPU baseline. The product
(``libsdb200.so``) neither links nor calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsdref.so")
REF_CUDA_SO = os.path.join(HERE, "_ref", "libsdref_cuda.so")
REF_B200_SO = os.path.join(HERE, "_ref", "libsdref_b200.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def _ptr(a):
    """Pointer of a numpy array or NULL for None."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def build_oracle() -> None:
    """Compiles liboracle.so (gcc) if it is missing or older than oracle.c."""
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, capture_output=True)


class _Base:
    prefix = ""

    def __init__(self, path):
        self.lib = C.CDLL(path)

    def fn(self, name, argtypes, restype=None):
        f = getattr(self.lib, self.prefix + name)
        f.argtypes = argtypes
        f.restype = restype
        return f


class Oracle(_Base):
    """C restatement (oracle.c). Every method takes/returns float32 numpy arrays."""

    prefix = "orc_"

    def __init__(self, path: str = ORACLE_SO):
        build_oracle()
        super().__init__(path)
        v = C.c_void_p
        self._gemm = self.fn("gemm_nt", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int])
        self._gemm16 = self.fn("gemm_nt_bf16", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int])
        self._attn = self.fn("attention", [v, v, v, v, _i64, _i64, _i64, C.c_int, C.c_int, _i64, C.c_int])
        self._bf16 = self.fn("f32_to_bf16_array", [v, v, _i64])
        self._softmax = self.fn("softmax_rows", [v, _i64, _i64, C.c_float, C.c_int])
        self._rms = self.fn("rms_norm", [v, v, _i64, _i64, v, C.c_float])
        self._ln = self.fn("layer_norm", [v, v, _i64, _i64, v, v, C.c_float])
        self._rmsh = self.fn("rms_norm_heads", [v, _i64, _i64, v, C.c_float])
        self._rope = self.fn("rope", [v, _i64, _i64, _i64, _i64, v, v, C.c_int])
        self._swiglu = self.fn("swiglu", [v, v, v, _i64])
        self._geglu = self.fn("geglu", [v, v, _i64, _i64])
        self._mulrows = self.fn("mul_rows", [v, v, _i64, _i64])
        self._addrs = self.fn("add_rows_scaled", [v, v, v, _i64, _i64])
        self._gn = self.fn("group_norm", [v, v, _i64, _i64, _i64, C.c_int, v, v, C.c_float])
        self._conv = self.fn("conv2d", [v, _i64, _i64, _i64, _i64, v, _i64, _i64, _i64, v, C.c_int, C.c_int, v])
        self.set_num_threads = self.fn("set_num_threads", [C.c_int])
        self.num_threads = self.fn("num_threads", [], C.c_int)

    # bf16 rounding of the reference (tensor.cpp:114-121)
    def flow_sigmas(self, steps: int, shift: float = 3.0) -> np.ndarray:
        """FlowMatchScheduler::set_timesteps (scheduler.cpp:117-127): sigma_0..sigma_steps."""
        out = np.zeros(steps + 1, np.float32)
        self.fn("flow_sigmas", [C.c_int, C.c_float, C.c_void_p])(steps, shift, _ptr(out))
        return out

    def flow_step(self, x, out, neg, cfg, dt):
        """One sampler update (pipeline.cpp:237-243 + scheduler.cpp:129-134); returns new x."""
        x = np.ascontiguousarray(x, np.float32).copy()
        out = np.ascontiguousarray(out, np.float32)
        negp = _ptr(np.ascontiguousarray(neg, np.float32)) if neg is not None else None
        self.fn("flow_step", [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_float, _i64])(
            _ptr(x), _ptr(out), negp, cfg, dt, x.size)
        return x

    def to_bf16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.uint16)
        self._bf16(_ptr(x), _ptr(y), x.size)
        return y

    def gemm_nt(self, A, B, bias=None, C0=None, M=None, N=None, K=None, lda=None, ldb=None, ldc=None):
        """C[M,N] = A[M,K] B[N,K]^T (+bias) (+C0). A, B may have padded rows."""
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        M = A.shape[0] if M is None else M
        N = B.shape[0] if N is None else N
        K = A.shape[1] if K is None else K
        lda = A.shape[1] if lda is None else lda
        ldb = B.shape[1] if ldb is None else ldb
        if C0 is None:
            ldc = N if ldc is None else ldc
            Cm = np.zeros((M, ldc), np.float32)
            acc = 0
        else:
            Cm = np.array(C0, np.float32, copy=True, order="C")
            ldc = Cm.shape[1]
            acc = 1
        bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._gemm(M, N, K, _ptr(A), lda, _ptr(B), ldb, _ptr(Cm), ldc, _ptr(bias), acc)
        return Cm

    def gemm_nt_bf16(self, A, Bh, bias=None, C0=None, M=None, N=None, K=None, lda=None, ldb=None, ldc=None):
        """Same with B given as bf16 bit patterns (uint16)."""
        A = np.ascontiguousarray(A, np.float32)
        Bh = np.ascontiguousarray(Bh, np.uint16)
        M = A.shape[0] if M is None else M
        N = Bh.shape[0] if N is None else N
        K = A.shape[1] if K is None else K
        lda = A.shape[1] if lda is None else lda
        ldb = Bh.shape[1] if ldb is None else ldb
        if C0 is None:
            ldc = N if ldc is None else ldc
            Cm = np.zeros((M, ldc), np.float32)
            acc = 0
        else:
            Cm = np.array(C0, np.float32, copy=True, order="C")
            ldc = Cm.shape[1]
            acc = 1
        bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._gemm16(M, N, K, _ptr(A), lda, _ptr(Bh), ldb, _ptr(Cm), ldc, _ptr(bias), acc)
        return Cm

    def attention(self, q, k, v, heads, kv_heads=None, causal=False):
        """q [N,Sq,heads*d]; k, v [N,Skv,kv_heads*d] -> [N,Sq,heads*d]."""
        kv_heads = heads if kv_heads is None else kv_heads
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        N, Sq, inner = q.shape
        Skv = k.shape[1]
        d = inner // heads
        out = np.zeros_like(q)
        self._attn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), N, Sq, Skv, heads, kv_heads, d, int(causal))
        return out

    def softmax_rows(self, x, scale, causal=False):
        x = np.array(x, np.float32, copy=True, order="C")
        self._softmax(_ptr(x), x.shape[0], x.shape[1], scale, int(causal))
        return x

    def rms_norm(self, x, gamma=None, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        C_ = x.shape[-1]
        y = np.empty_like(x)
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        self._rms(_ptr(x), _ptr(y), x.size // C_, C_, _ptr(g), eps)
        return y

    def layer_norm(self, x, gamma=None, beta=None, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        C_ = x.shape[-1]
        y = np.empty_like(x)
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        b = None if beta is None else np.ascontiguousarray(beta, np.float32)
        self._ln(_ptr(x), _ptr(y), x.size // C_, C_, _ptr(g), _ptr(b), eps)
        return y

    def rms_norm_heads(self, x, dim, gamma=None, eps=1e-5):
        x = np.array(x, np.float32, copy=True, order="C")
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        self._rmsh(_ptr(x), x.size // dim, dim, _ptr(g), eps)
        return x

    def rope(self, x, dim, cos, sin, interleaved):
        x = np.array(x, np.float32, copy=True, order="C")
        N, S, inner = x.shape
        cos = np.ascontiguousarray(cos, np.float32)
        sin = np.ascontiguousarray(sin, np.float32)
        self._rope(_ptr(x), N, S, inner, dim, _ptr(cos), _ptr(sin), int(interleaved))
        return x

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        y = np.empty_like(g)
        self._swiglu(_ptr(g), _ptr(u), _ptr(y), g.size)
        return y

    def geglu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        D2 = x.shape[-1]
        y = np.empty(x.shape[:-1] + (D2 // 2,), np.float32)
        self._geglu(_ptr(x), _ptr(y), x.size // D2, D2 // 2)
        return y

    def mul_rows(self, x, v):
        x = np.array(x, np.float32, copy=True, order="C")
        v = np.ascontiguousarray(v, np.float32)
        self._mulrows(_ptr(x), _ptr(v), x.size // v.size, v.size)
        return x

    def add_rows_scaled(self, x, y, g):
        x = np.array(x, np.float32, copy=True, order="C")
        y = np.ascontiguousarray(y, np.float32)
        g = np.ascontiguousarray(g, np.float32)
        self._addrs(_ptr(x), _ptr(y), _ptr(g), x.size // g.size, g.size)
        return x

    def group_norm(self, x, groups, gamma, beta, eps):
        x = np.ascontiguousarray(x, np.float32)
        N, C_ = x.shape[:2]
        HW = x.size // (N * C_)
        y = np.empty_like(x)
        self._gn(_ptr(x), _ptr(y), N, C_, HW, groups, _ptr(np.ascontiguousarray(gamma, np.float32)),
                 _ptr(np.ascontiguousarray(beta, np.float32)), eps)
        return y

    def conv2d(self, x, w, bias, stride, pad):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        N, Cin, H, W = x.shape
        Cout, _, kh, kw = w.shape
        Ho = (H + 2 * pad - kh) // stride + 1
        Wo = (W + 2 * pad - kw) // stride + 1
        out = np.zeros((N, Cout, Ho, Wo), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._conv(_ptr(x), N, Cin, H, W, _ptr(w), Cout, kh, kw, _ptr(b), stride, pad, _ptr(out))
        return out


class RefCPU(_Base):
    """The reference's own CPU path (oracle/_ref/libsdref.so)."""

    prefix = "sdref_"

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        v = C.c_void_p
        self._gemm = self.fn("gemm_nt", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int])
        self._gemm16 = self.fn("gemm_nt_bf16", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int])
        self._attn = self.fn("attention", [v, v, v, v, _i64, _i64, _i64, C.c_int, C.c_int, _i64, C.c_int], C.c_int)
        self._bf16 = self.fn("f32_to_bf16_array", [v, v, _i64])
        self._softmax = self.fn("softmax_rows", [v, _i64, _i64, C.c_float, C.c_int])
        self._rms = self.fn("rms_norm", [v, v, _i64, _i64, v, C.c_float], C.c_int)
        self._ln = self.fn("layer_norm", [v, v, _i64, _i64, v, v, C.c_float], C.c_int)
        self._rmsh = self.fn("rms_norm_heads", [v, _i64, _i64, v, C.c_float], C.c_int)
        self._rope = self.fn("rope", [v, _i64, _i64, _i64, _i64, v, v, C.c_int], C.c_int)
        self._swiglu = self.fn("swiglu", [v, v, v, _i64], C.c_int)
        self._geglu = self.fn("geglu", [v, v, _i64, _i64], C.c_int)
        self._gn = self.fn("group_norm", [v, v, _i64, _i64, _i64, C.c_int, v, v, C.c_float], C.c_int)
        self._conv = self.fn("conv2d", [v, _i64, _i64, _i64, _i64, v, _i64, _i64, _i64, v, C.c_int, C.c_int, v],
                             C.c_int)
        self._mulrows = self.fn("mul_rows", [v, v, _i64, _i64], C.c_int)
        self._addrs = self.fn("add_rows_scaled", [v, v, v, _i64, _i64], C.c_int)
        self.set_num_threads = self.fn("set_num_threads", [C.c_int])
        self.num_threads = self.fn("num_threads", [], C.c_int)
        self.last_error = self.fn("last_error", [], C.c_char_p)
        self.w_new = self.fn("weights_new", [], v)
        self.w_free = self.fn("weights_free", [v])
        self.w_add = self.fn("weights_add", [v, C.c_char_p, v, C.c_int, v, C.c_int], C.c_int)
        self.z_new = self.fn("zimage_new", [v, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_int, C.c_int,
                                            C.c_int], v)
        self.z_free = self.fn("zimage_free", [v])
        self.z_fwd = self.fn("zimage_forward", [v, v, _i64, _i64, _i64, C.c_float, v, _i64, _i64, v], C.c_int)
        self.u_new = self.fn("unet_new", [v, C.c_int], v)
        self.u_free = self.fn("unet_free", [v])
        self.u_fwd = self.fn("unet_forward", [v, v, _i64, _i64, _i64, _i64, C.c_float, v, _i64, _i64, v, C.c_int],
                             C.c_int)
        self.v_new = self.fn("vae_new", [v, C.c_float, C.c_float], v)
        self.v_free = self.fn("vae_free", [v])
        self.v_dec = self.fn("vae_decode", [v, v, _i64, _i64, _i64, _i64, v, _i64, v], C.c_int)

    def _chk(self, rc):
        if rc:
            raise RuntimeError(self.last_error().decode())

    # The methods mirror Oracle's so tests can run both on the same inputs.
    to_bf16 = Oracle.to_bf16
    gemm_nt = Oracle.gemm_nt
    gemm_nt_bf16 = Oracle.gemm_nt_bf16
    softmax_rows = Oracle.softmax_rows
    mul_rows = Oracle.mul_rows
    add_rows_scaled = Oracle.add_rows_scaled

    def attention(self, q, k, v, heads, kv_heads=None, causal=False):
        kv_heads = heads if kv_heads is None else kv_heads
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        N, Sq, inner = q.shape
        out = np.zeros_like(q)
        self._chk(self._attn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), N, Sq, k.shape[1], heads, kv_heads,
                             inner // heads, int(causal)))
        return out

    def rms_norm(self, x, gamma=None, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        self._chk(self._rms(_ptr(x), _ptr(y), x.size // x.shape[-1], x.shape[-1], _ptr(g), eps))
        return y

    def layer_norm(self, x, gamma=None, beta=None, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        b = None if beta is None else np.ascontiguousarray(beta, np.float32)
        self._chk(self._ln(_ptr(x), _ptr(y), x.size // x.shape[-1], x.shape[-1], _ptr(g), _ptr(b), eps))
        return y

    def rms_norm_heads(self, x, dim, gamma=None, eps=1e-5):
        x = np.array(x, np.float32, copy=True, order="C")
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        self._chk(self._rmsh(_ptr(x), x.size // dim, dim, _ptr(g), eps))
        return x

    def rope(self, x, dim, cos, sin, interleaved):
        x = np.array(x, np.float32, copy=True, order="C")
        N, S, inner = x.shape
        self._chk(self._rope(_ptr(x), N, S, inner, dim, _ptr(np.ascontiguousarray(cos, np.float32)),
                             _ptr(np.ascontiguousarray(sin, np.float32)), int(interleaved)))
        return x

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        y = np.empty_like(g)
        self._chk(self._swiglu(_ptr(g), _ptr(u), _ptr(y), g.size))
        return y

    def geglu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        D2 = x.shape[-1]
        y = np.empty(x.shape[:-1] + (D2 // 2,), np.float32)
        self._chk(self._geglu(_ptr(x), _ptr(y), x.size // D2, D2 // 2))
        return y

    def group_norm(self, x, groups, gamma, beta, eps):
        x = np.ascontiguousarray(x, np.float32)
        N, C_ = x.shape[:2]
        y = np.empty_like(x)
        self._chk(self._gn(_ptr(x), _ptr(y), N, C_, x.size // (N * C_), groups,
                           _ptr(np.ascontiguousarray(gamma, np.float32)),
                           _ptr(np.ascontiguousarray(beta, np.float32)), eps))
        return y

    def conv2d(self, x, w, bias, stride, pad):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        N, Cin, H, W = x.shape
        Cout, _, kh, kw = w.shape
        Ho = (H + 2 * pad - kh) // stride + 1
        Wo = (W + 2 * pad - kw) // stride + 1
        out = np.zeros((N, Cout, Ho, Wo), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self._chk(self._conv(_ptr(x), N, Cin, H, W, _ptr(w), Cout, kh, kw, _ptr(b), stride, pad, _ptr(out)))
        return out

    # ---- flow-matching sampler (the reference's FlowMatchScheduler) ---------------
    def flow_sigmas(self, steps: int, shift: float = 3.0) -> np.ndarray:
        sig = np.zeros(steps + 1, np.float32)
        times = np.zeros(steps, np.float32)
        self._chk(self.fn("flow_sigmas", [C.c_int, C.c_float, C.c_void_p, C.c_void_p], C.c_int)(
            steps, shift, _ptr(sig), _ptr(times)))
        return sig

    def flow_step(self, x, out, neg, cfg, step, steps, shift=3.0):
        """FlowMatchScheduler::step after the pipeline's guidance mix; returns new x."""
        x = np.ascontiguousarray(x, np.float32).copy()
        out = np.ascontiguousarray(out, np.float32)
        negp = _ptr(np.ascontiguousarray(neg, np.float32)) if neg is not None else None
        self._chk(self.fn("flow_step", [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, _i64, C.c_int, C.c_int,
                                        C.c_float], C.c_int)(_ptr(x), _ptr(out), negp, cfg, x.size, step, steps, shift))
        return x

    # ---- checkpoints (the reference's safetensors reader) --------------------------
    def safetensors_tensor(self, path, name, keep_bf16, min_numel, numel):
        """Tensor `name` of `path` as Weights::load_safetensors stores it: (uint16 BF16 bits
        or float32 array of numel values, is_bf16), or None if the reference skipped it."""
        o32 = np.zeros(numel, np.float32)
        o16 = np.zeros(numel, np.uint16)
        rc = self.fn("safetensors_tensor", [C.c_char_p, C.c_char_p, C.c_int, _i64, C.c_void_p, C.c_void_p], C.c_int)(
            path.encode(), name.encode(), int(keep_bf16), int(min_numel), _ptr(o32), _ptr(o16))
        if rc == -1:
            raise RuntimeError(self.last_error().decode())
        if rc == -2:
            return None
        return (o16, True) if rc == 1 else (o32, False)

    def zimage_load(self, dir_, base, heads=30, patch=2, norm_eps=1e-5, rope_theta=256.0, t_scale=1000.0,
                    axes=(32, 48, 48)):
        """The reference ZImageTransformer over a checkpoint directory, loaded as the
        pipeline loads it; returns a callable like zimage()."""
        wout = C.c_void_p()
        load = self.fn("zimage_load", [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float,
                                       C.c_int, C.c_int, C.c_int, C.c_void_p], C.c_void_p)
        m = load(dir_.encode(), base.encode(), heads, patch, norm_eps, rope_theta, t_scale, *axes, C.byref(wout))
        if not m:
            raise RuntimeError(self.last_error().decode())
        return self._wrap_model(m, wout.value)

    # ---- Z-Image transformer on random-init weights ------------------------------
    def zimage(self, weights: dict, bf16_names: set, heads=30, patch=2, norm_eps=1e-5, rope_theta=256.0,
               t_scale=1000.0, axes=(32, 48, 48)):
        """Builds the reference ZImageTransformer over `weights` (name -> fp32 array);
        names in `bf16_names` are stored as BF16. Returns a callable
        f(x [1,C,H,W], t, cap [1,L,D]) -> out [1,C,H,W]."""
        w = self.w_new()
        for name, arr in weights.items():
            arr = np.ascontiguousarray(arr, np.float32)
            shape = (C.c_int64 * arr.ndim)(*arr.shape)
            self._chk(self.w_add(w, name.encode(), C.cast(shape, C.c_void_p), arr.ndim, _ptr(arr),
                                 int(name in bf16_names)))
        m = self.z_new(w, heads, patch, norm_eps, rope_theta, t_scale, *axes)
        if not m:
            self.w_free(w)
            raise RuntimeError(self.last_error().decode())
        return self._wrap_model(m, w)

    def unet(self, weights: dict, heads: int = 8, on_device: bool = False):
        """Builds the reference UNet (unet.cpp:18-56) over `weights` (name -> fp32 array);
        returns f(x [N,C,H,W], t, ctx [N,L,D]) -> out [N,C,H,W] running UNet::forward. With
        on_device the weights are moved with Weights::to_device and the inputs with
        Tensor::to (a library with a GPU backend)."""
        w = self.w_new()
        for name, arr in weights.items():
            arr = np.ascontiguousarray(arr, np.float32)
            shape = (C.c_int64 * arr.ndim)(*arr.shape)
            self._chk(self.w_add(w, name.encode(), C.cast(shape, C.c_void_p), arr.ndim, _ptr(arr), 0))
        if on_device:
            self._chk(self.fn("weights_to_cuda", [C.c_void_p], C.c_int)(w))
        m = self.u_new(w, heads)
        if not m:
            self.w_free(w)
            raise RuntimeError(self.last_error().decode())
        ref = self

        class _UNet:
            def __call__(self, x, t, ctx):
                x = np.ascontiguousarray(x, np.float32)
                ctx = np.ascontiguousarray(ctx, np.float32)
                out = np.empty_like(x)
                ref._chk(ref.u_fwd(m, _ptr(x), *x.shape, float(t), _ptr(ctx), ctx.shape[1], ctx.shape[2], _ptr(out),
                                   int(on_device)))
                return out

            def __del__(self):
                try:
                    ref.u_free(m)
                    ref.w_free(w)
                except Exception:
                    pass

        return _UNet()

    def vae(self, weights: dict, scaling_factor: float, shift_factor: float):
        """Builds the reference VAEDecoder (vae.cpp:15-32) over `weights` (name -> fp32
        array). Returns a callable f(z [N,C,h,w]) -> image [N,3,H,W] running
        VAEDecoder::decode (vae.cpp:35-51) on the CPU."""
        w = self.w_new()
        for name, arr in weights.items():
            arr = np.ascontiguousarray(arr, np.float32)
            shape = (C.c_int64 * arr.ndim)(*arr.shape)
            self._chk(self.w_add(w, name.encode(), C.cast(shape, C.c_void_p), arr.ndim, _ptr(arr), 0))
        m = self.v_new(w, scaling_factor, shift_factor)
        if not m:
            self.w_free(w)
            raise RuntimeError(self.last_error().decode())
        ref = self

        class _Vae:
            def __call__(self, z):
                z = np.ascontiguousarray(z, np.float32)
                cap = z.size * 64 * 4  # room for up to 8x upscaling to 4 channels
                out = np.empty(cap, np.float32)
                shp = (C.c_int64 * 4)()
                ref._chk(ref.v_dec(m, _ptr(z), *z.shape, _ptr(out), cap, C.cast(shp, C.c_void_p)))
                n = int(np.prod(list(shp)))
                return out[:n].reshape(tuple(shp)).copy()

            def __del__(self):
                try:
                    ref.v_free(m)
                    ref.w_free(w)
                except Exception:
                    pass

        return _Vae()

    def _wrap_model(self, m, w):
        ref = self

        class _Model:
            def __call__(self, x, t, cap):
                x = np.ascontiguousarray(x, np.float32)
                cap = np.ascontiguousarray(cap, np.float32)
                out = np.empty_like(x)
                _, Cc, H, W = x.shape
                ref._chk(ref.z_fwd(m, _ptr(x), Cc, H, W, float(t), _ptr(cap), cap.shape[1], cap.shape[2], _ptr(out)))
                return out

            def __del__(self):
                try:
                    ref.z_free(m)
                    ref.w_free(w)
                except Exception:
                    pass

        return _Model()


class RefCUDA(RefCPU):
    """The reference's GPU backend (src/backend_cuda.cu + cuBLAS) linked in place of the
    stub (oracle/_ref/libsdref_cuda.so): a comparison column timed on the same B200, never
    the product. Every RefCPU entry point is present; the extra ones take device pointers
    or move tensors to the device as the reference pipeline does."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_CUDA_SO)

    def __init__(self, path: str = REF_CUDA_SO):
        super().__init__(path)
        v = C.c_void_p
        self.cuda_available = self.fn("cuda_available", [], C.c_int)
        self.cuda_sync = self.fn("cuda_synchronize", [], C.c_int)
        self._w_cuda = self.fn("weights_to_cuda", [v], C.c_int)
        self._z_fwd_cuda = self.fn("zimage_forward_cuda", [v, v, _i64, _i64, _i64, C.c_float, v, _i64, _i64, v],
                                   C.c_int)
        self._gemm_cuda = self.fn("cuda_gemm_nt_bf16", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int],
                                  C.c_int)
        self._gemm32_cuda = self.fn("cuda_gemm_nt_f32", [_i64, _i64, _i64, v, _i64, v, _i64, v, _i64, v, C.c_int],
                                    C.c_int)
        self._geglu_cuda = self.fn("cuda_geglu", [v, v, _i64, _i64], C.c_int)
        self._attn_cuda = self.fn("cuda_attention", [v, v, v, v, _i64, _i64, _i64, C.c_int, C.c_int, _i64, C.c_int],
                                  C.c_int)
        self._conv_cuda = self.fn("cuda_conv2d", [v, _i64, _i64, _i64, _i64, v, _i64, _i64, _i64, v, C.c_int, C.c_int,
                                                  v, _i64, _i64], C.c_int)
        self._w_add_dev = self.fn("weights_add_device", [v, C.c_char_p, v, C.c_int, v, C.c_int], C.c_int)
        self._v_dec_cuda = self.fn("vae_decode_cuda", [v, v, _i64, _i64, _i64, _i64, v, _i64, v], C.c_int)

    def gemm_nt_bf16_dev(self, M, N, K, A, lda, B, ldb, Cp, ldc, bias, acc=False):
        self._chk(self._gemm_cuda(M, N, K, A, lda, B, ldb, Cp, ldc, bias, int(acc)))

    def gemm_nt_f32_dev(self, M, N, K, A, lda, B, ldb, Cp, ldc, bias, acc=False):
        self._chk(self._gemm32_cuda(M, N, K, A, lda, B, ldb, Cp, ldc, bias, int(acc)))

    def geglu_dev(self, x, y, rows, D):
        self._chk(self._geglu_cuda(x, y, rows, D))

    def attention_dev(self, q, k, v, out, N, Sq, Skv, heads, kv_heads, d, causal=False):
        self._chk(self._attn_cuda(q, k, v, out, N, Sq, Skv, heads, kv_heads, d, int(causal)))

    def conv2d_dev(self, x, N, Cin, H, W, w, Cout, kh, kw, bias, stride, pad, out, Ho, Wo):
        self._chk(self._conv_cuda(x, N, Cin, H, W, w, Cout, kh, kw, bias, stride, pad, out, Ho, Wo))

    def synchronize(self):
        self._chk(self.cuda_sync())

    def zimage_cuda(self, weights: dict, heads=30, patch=2, norm_eps=1e-5, rope_theta=256.0, t_scale=1000.0,
                    axes=(32, 48, 48)):
        """ZImageTransformer over `weights` (name -> torch CUDA tensor, float32 or bfloat16),
        copied device to device into the reference's own storage; f(x, t, cap) runs its
        forward on the GPU backend and returns the host output."""
        import torch

        w = self.w_new()
        for name, t in weights.items():
            t = t.contiguous()
            shape = (C.c_int64 * t.dim())(*t.shape)
            self._chk(self._w_add_dev(w, name.encode(), C.cast(shape, C.c_void_p), t.dim(), t.data_ptr(),
                                      int(t.dtype == torch.bfloat16)))
        self.synchronize()
        m = self.z_new(w, heads, patch, norm_eps, rope_theta, t_scale, *axes)
        if not m:
            self.w_free(w)
            raise RuntimeError(self.last_error().decode())
        ref = self

        class _Model:
            def __call__(self, x, t, cap):
                x = np.ascontiguousarray(x, np.float32)
                cap = np.ascontiguousarray(cap, np.float32)
                out = np.empty_like(x)
                _, Cc, H, W = x.shape
                ref._chk(ref._z_fwd_cuda(m, _ptr(x), Cc, H, W, float(t), _ptr(cap), cap.shape[1], cap.shape[2],
                                         _ptr(out)))
                return out

            def __del__(self):
                try:
                    ref.z_free(m)
                    ref.w_free(w)
                except Exception:
                    pass

        return _Model()

    def vae_cuda(self, weights: dict, scaling_factor: float, shift_factor: float):
        """VAEDecoder over `weights` (name -> fp32 numpy) moved to the device; f(z) decodes on
        the GPU backend and returns the host image."""
        w = self.w_new()
        for name, arr in weights.items():
            arr = np.ascontiguousarray(arr, np.float32)
            shape = (C.c_int64 * arr.ndim)(*arr.shape)
            self._chk(self.w_add(w, name.encode(), C.cast(shape, C.c_void_p), arr.ndim, _ptr(arr), 0))
        self._chk(self._w_cuda(w))
        m = self.v_new(w, scaling_factor, shift_factor)
        if not m:
            self.w_free(w)
            raise RuntimeError(self.last_error().decode())
        ref = self

        class _Vae:
            def __call__(self, z):
                z = np.ascontiguousarray(z, np.float32)
                cap = z.size * 64 * 4
                out = np.empty(cap, np.float32)
                shp = (C.c_int64 * 4)()
                ref._chk(ref._v_dec_cuda(m, _ptr(z), *z.shape, _ptr(out), cap, C.cast(shp, C.c_void_p)))
                n = int(np.prod(list(shp)))
                return out[:n].reshape(tuple(shp)).copy()

            def __del__(self):
                try:
                    ref.v_free(m)
                    ref.w_free(w)
                except Exception:
                    pass

        return _Vae()


class RefOnB200(RefCUDA):
    """The reference's own model code (tensor.cpp, modules.cpp, unet.cpp, zimage.cpp, vae.cpp)
    linked against libsdb200.so in place of its backend (oracle/_ref/libsdref_b200.so): the
    maintainer's drop-in link. Its Device::CUDA paths call this library's sd::cuda
    functions. Test infrastructure: it checks the boundary, it is not the product."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_B200_SO)

    def __init__(self, path: str = REF_B200_SO):
        super().__init__(path)
