"""sdb200 - Python binding of libsdb200.so, the B200 (sm_100a) backend for
StableDiffusion-cpp's dense-contraction path.

The library's public surface is the C ABI in ``include/sdb200.h`` (and the reference's
``sd::cuda::*`` C++ symbols built on it). This module binds that ABI with ctypes so
tests and benchmarks can drive it with device buffers owned by PyTorch; PyTorch is
used only for device memory and streams, never for the computation.

The shared library is built in-tree (``make -C stablediffusion-cpp_b200``) and loaded
from this directory. There is no fallback: if it is missing, importing the
functions raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsdb200.so")

OK = 0
ERR_INVALID_ARG = 1
ERR_NO_DEVICE = 2
ERR_CUDA = 3
ERR_DEVICE_WAIT = 4
ERR_OUT_OF_MEMORY = 5
ERR_UNSUPPORTED = 6


class SdbError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"sdb200 error {code}: {msg}")
        self.code = code


_lib = None

_i64 = C.c_int64
_v = C.c_void_p
_f = C.c_float
_i = C.c_int

# name -> (argtypes, restype)
_SIGS = {
    "sdb200_version": ([], _i),
    "sdb200_launch_count": ([], C.c_ulonglong),
    "sdb200_last_error": ([], C.c_char_p),
    "sdb200_available": ([], _i),
    "sdb200_device_count": ([], _i),
    "sdb200_device_name": ([], C.c_char_p),
    "sdb200_device_memory": ([], C.c_size_t),
    "sdb200_set_device": ([_i], _i),
    "sdb200_set_stream": ([_v], _i),
    "sdb200_get_stream": ([], _v),
    "sdb200_device_error_word": ([C.POINTER(_i)], _i),
    "sdb200_malloc": ([C.c_size_t], _v),
    "sdb200_free": ([_v], _i),
    "sdb200_upload": ([_v, _v, C.c_size_t], _i),
    "sdb200_download": ([_v, _v, C.c_size_t], _i),
    "sdb200_copy": ([_v, _v, C.c_size_t], _i),
    "sdb200_zero": ([_v, C.c_size_t], _i),
    "sdb200_synchronize": ([], _i),
    "sdb200_set_gemm_tile": ([_i], _i),
    "sdb200_set_gemm_pair": ([_i], _i),
    "sdb200_dit_post_norm": ([_v, _i64, _i, _i64, _i64, _v, _i64, _v, _v, _v, _v, _v, _i, _f], _i),
    "sdb200_set_conv_implicit": ([_i], _i),
    "sdb200_gemm_nt_f32": ([_i64, _i64, _i64, _v, _i64, _v, _i64, _v, _i64, _v, _i], _i),
    "sdb200_gemm_nt_bf16": ([_i64, _i64, _i64, _v, _i64, _v, _i64, _v, _i64, _v, _i], _i),
    "sdb200_gemm_nt_bf16_noalloc": ([_i64, _i64, _i64, _v, _i64, _v, _i64, _v, _i64, _v, _i], _i),
    "sdb200_gemm_nt_bf16a": ([_i64, _i64, _i64, _v, _i64, _v, _i64, _v, _i64, _v, _i], _i),
    "sdb200_pack_bf16": ([_v, _i64, _v, _i64, _i64, _i64], _i),
    "sdb200_set_operand_cache": ([_i], _i),
    "sdb200_operand_cache_entries": ([], _i64),
    "sdb200_gemm_bf16_epilogue": ([_i64, _i64, _i64, _v, _i64, _i, _v, _i64, _v, _i64, _i, _v, _i], _i),
    "sdb200_gemm_bf16_qkv_rope": ([_i64, _i64, _v, _i64, _i, _v, _i64, _v, _i64, _i64, _v, _v, _v, _v, _f, _v, _v, _v],
                                  _i),
    "sdb200_set_attention_path": ([_i], _i),
    "sdb200_attention_f16": ([_v, _v, _v, _v, _i, _i64, _i64, _i64, _i, _i, _i64, _i64, _i], _i),
    "sdb200_pack_heads_f16": ([_v, _v, _i64, _i, _i64, _i64], _i),
    "sdb200_attention": ([_v, _v, _v, _v, _i64, _i64, _i64, _i, _i, _i64, _i], _i),
    "sdb200_zimage_create": ([_i, _i, _f, _f, _f, _i, _i, _i], _v),
    "sdb200_zimage_set_weight": ([_v, C.c_char_p, _v, _i, C.POINTER(_i64), _i], _i),
    "sdb200_zimage_finalize": ([_v], _i),
    "sdb200_zimage_forward": ([_v, _v, _i64, _i64, _i64, _i64, _f, _v, _i64, _i64, _v], _i),
    "sdb200_zimage_destroy": ([_v], None),
    "sdb200_zimage_profile": ([_v, _i], _i),
    "sdb200_zimage_profile_read": ([_v, C.POINTER(C.c_double)], _i),
    "sdb200_zimage_profile_read_ex": ([_v, C.POINTER(C.c_double), _i], _i),
    "sdb200_zimage_set_tp": ([_v, _v], _i),
    "sdb200_zimage_set_tp_mode": ([_v, _i], _i),
    "sdb200_zimage_sample": ([_v, _v, _i64, _i64, _i64, _i64, _v, _v, _i64, _i64, _f, _i, _f], _i),
    "sdb200_flow_sigmas": ([_i, _f, _v], _i),
    "sdb200_zimage_load": ([_v, C.c_char_p, C.c_char_p, _i, _i, _i64], _i),
    "sdb200_vae_create": ([_f, _f], _v),
    "sdb200_vae_set_weight": ([_v, C.c_char_p, _v, C.POINTER(_i64), _i], _i),
    "sdb200_vae_load": ([_v, C.c_char_p, C.c_char_p], _i),
    "sdb200_vae_finalize": ([_v], _i),
    "sdb200_vae_info": ([_v, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)], _i),
    "sdb200_vae_decode": ([_v, _v, _i64, _i64, _i64, _i64, _v], _i),
    "sdb200_vae_destroy": ([_v], None),
    "sdb200_vae_profile": ([_v, _i], _i),
    "sdb200_vae_profile_read": ([_v, C.POINTER(C.c_double)], _i),
    "sdb200_safetensors_read": ([C.c_char_p, C.c_char_p, _i, _i64, _v, _i64, _v, _v, _v], _i),
    "sdb200_checkpoint_read_shard": ([C.c_char_p, C.c_char_p, C.c_char_p, _i, _i, _i, _i64, _v, _i64, _v, _v, _v],
                                     _i),
    "sdb200_zimage_get_weight": ([_v, C.c_char_p, _v, _i64, _v, _v, _v], _i),
    "sdb200_comm_unique_id": ([_v], _i),
    "sdb200_comm_create": ([_v, _i, _i], _v),
    "sdb200_comm_allreduce_sum_f32": ([_v, _v, C.c_size_t], _i),
    "sdb200_comm_set_barrier": ([_v, _i], _i),
    "sdb200_comm_barrier_selftest": ([_v, _i, _i, C.c_uint32], _i),
    "sdb200_comm_destroy": ([_v], None),
    "sdb200_conv2d": ([_v, _i64, _i64, _i64, _i64, _v, _i64, _i64, _i64, _v, _i, _i, _v, _i64, _i64], _i),
    "sdb200_conv_pack_input": ([_v, _v, _i64, _i64, _i64, _i64], _i),
    "sdb200_conv_pack_weight": ([_v, _v, _i64, _i64, _i64, _i64], _i),
    "sdb200_conv2d_nhwc": ([_v, _i64, _i64, _i64, _i64, _i64, _v, _i64, _i64, _i64, _i64, _i, _v, _v, _v, _i64,
                            _i64], _i),
    "sdb200_group_norm": ([_v, _v, _i64, _i64, _i64, _i, _v, _v, _f], _i),
    "sdb200_layer_norm": ([_v, _v, _i64, _i64, _v, _v, _f], _i),
    "sdb200_rms_norm": ([_v, _v, _i64, _i64, _v, _f], _i),
    "sdb200_rms_norm_heads": ([_v, _i64, _i64, _v, _f], _i),
    "sdb200_rope": ([_v, _i64, _i64, _i64, _i64, _v, _v, _i], _i),
    "sdb200_softmax_rows": ([_v, _i64, _i64, _f, _i], _i),
    "sdb200_geglu": ([_v, _v, _i64, _i64], _i),
    "sdb200_swiglu": ([_v, _v, _v, _i64], _i),
    "sdb200_silu": ([_v, _i64], _i),
    "sdb200_tanh": ([_v, _i64], _i),
    "sdb200_gelu": ([_v, _i64], _i),
    "sdb200_quick_gelu": ([_v, _i64], _i),
    "sdb200_add": ([_v, _v, _i64], _i),
    "sdb200_scale": ([_v, _f, _i64], _i),
    "sdb200_affine": ([_v, _f, _f, _i64], _i),
    "sdb200_mul_rows": ([_v, _v, _i64, _i64], _i),
    "sdb200_add_rows_scaled": ([_v, _v, _v, _i64, _i64], _i),
    "sdb200_add_channel_bias": ([_v, _v, _i64, _i64, _i64], _i),
    "sdb200_upsample_nearest2x": ([_v, _v, _i64, _i64, _i64], _i),
    "sdb200_concat_channels": ([_v, _v, _v, _i64, _i64, _i64, _i64], _i),
    "sdb200_nchw_to_nlc": ([_v, _v, _i64, _i64, _i64], _i),
    "sdb200_nlc_to_nchw": ([_v, _v, _i64, _i64, _i64], _i),
    "sdb200_patchify": ([_v, _v, _i64, _i64, _i64, _i], _i),
    "sdb200_unpatchify": ([_v, _v, _i64, _i64, _i64, _i], _i),
}


def lib():
    """Loads libsdb200.so (once) and declares every C-ABI signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libsdb200.so not built at {LIB_PATH}; run `make -C stablediffusion-cpp_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise SdbError(rc, lib().sdb200_last_error().decode(errors="replace"))


def available() -> bool:
    return bool(lib().sdb200_available())


from . import backend  # noqa: E402,F401  (torch-facing wrappers)


def flow_sigmas(steps: int, shift: float = 3.0):
    """The flow-matching schedule sigma_0..sigma_steps (scheduler.cpp:117-127), host-side."""
    import numpy as np

    out = np.zeros(steps + 1, dtype=np.float32)
    check(lib().sdb200_flow_sigmas(int(steps), float(shift), out.ctypes.data_as(C.c_void_p)))
    return out


def safetensors_read(path: str, name: str, keep_bf16: bool = True, bf16_min_numel: int = 1 << 20):
    """One tensor of a .safetensors file, converted as the reference converts it: a numpy
    uint16 array of BF16 bit patterns, or float32."""
    import numpy as np

    shape = (C.c_int64 * 8)()
    ndim, isb = C.c_int(0), C.c_int(0)
    check(lib().sdb200_safetensors_read(path.encode(), name.encode(), int(keep_bf16), int(bf16_min_numel), None, 0,
                                        shape, C.byref(ndim), C.byref(isb)))
    dims = [shape[i] for i in range(ndim.value)]
    out = np.empty(dims, dtype=np.uint16 if isb.value else np.float32)
    check(lib().sdb200_safetensors_read(path.encode(), name.encode(), int(keep_bf16), int(bf16_min_numel),
                                        out.ctypes.data_as(C.c_void_p), out.nbytes, shape, C.byref(ndim),
                                        C.byref(isb)))
    return out


def _read_tensor(call):
    """Runs a (dst, dst_bytes, shape, ndim, is_bf16) reader twice: shape query, then data.
    Returns a numpy uint16 (BF16 bits) or float32 array, or None when ndim < 0."""
    import numpy as np

    shape = (C.c_int64 * 8)()
    ndim, isb = C.c_int(0), C.c_int(0)
    check(call(None, 0, shape, C.byref(ndim), C.byref(isb)))
    if ndim.value < 0:
        return None
    out = np.empty([shape[i] for i in range(ndim.value)], dtype=np.uint16 if isb.value else np.float32)
    check(call(out.ctypes.data_as(C.c_void_p), out.nbytes, shape, C.byref(ndim), C.byref(isb)))
    return out


def checkpoint_read_shard(dir_: str, base: str, name: str, rank: int, world: int, heads: int,
                          bf16_min_numel: int = 1 << 20):
    """One tensor of a checkpoint as sdb200_zimage_load uploads it for rank of world
    (host only); None when this rank holds no part of it."""
    return _read_tensor(lambda d, nb, s, n, b: lib().sdb200_checkpoint_read_shard(
        dir_.encode(), base.encode(), name.encode(), int(rank), int(world), int(heads), int(bf16_min_numel), d, nb,
        s, n, b))
