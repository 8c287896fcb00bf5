"""GPU: the device bf16 rounding of the GEMM's activation operand, bit for bit.

sdb200_gemm_nt_bf16 rounds A to bf16 on the device before the tensor-core GEMM, with the
reference's rule (tensor.cpp:114-121 on the CPU, f32_to_bf16_d in backend_cuda.cu:183-188
on its GPU): round to nearest even on the raw bits; inf and NaN truncated, so a NaN keeps
its sign and the top 7 bits of its payload. sdb200_pack_bf16 runs that same pack kernel
on its own. Rounding is byte work, so the bar is bit equality with the reference's own
rounding (the golden vectors it wrote) and with the oracle, on ties, +-inf, NaN
payloads, subnormals, +-0, the overflow to inf, and random bit patterns, through both
the 16-byte vector kernel and the scalar kernel. The GEMM itself is then checked to use
exactly those rounded values: gemm_nt_bf16 on fp32 A equals gemm_nt_bf16a on the packed A.
"""
import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _special_bits():
    v = [
        0x00000000, 0x80000000,                          # +-0
        0x7F800000, 0xFF800000,                          # +-inf
        0x7FC00000, 0xFFC00000, 0x7F800001, 0xFF800001,  # quiet / signalling NaN
        0x7FFFFFFF, 0xFFFFFFFF, 0x7F80FFFF, 0x7FBF8000,  # NaN payloads (low bits dropped)
        0x3F808000, 0x3F818000, 0xBF808000, 0xBF818000,  # exact ties: even down, odd up
        0x3F807FFF, 0x3F808001, 0x3F80FFFF, 0x3F81FFFF,  # just below / above a tie
        0x00000001, 0x00008000, 0x00018000, 0x00007FFF,  # subnormals and their ties
        0x007FFFFF, 0x807FFFFF, 0x80008000, 0x80018000,
        0x007F8000, 0x007FC000,                          # largest subnormals -> min normal
        0x00800000, 0x80800000,                          # min normal
        0x7F7FFFFF, 0xFF7FFFFF, 0x7F7F8000, 0x7F7F7FFF,  # overflow to inf / stays finite
        0x7F7EFFFF, 0x3F800000, 0x40490FDB, 0xC0490FDB,  # ordinary values
    ]
    return np.array(v, dtype=np.uint32)


def _cases():
    rng = np.random.default_rng(13)
    rand = rng.integers(0, 2 ** 32, size=1 << 20, dtype=np.uint64).astype(np.uint32)
    # every exponent, with low halves on and around the tie
    e = (np.arange(256, dtype=np.uint32) << 23)
    lows = np.array([0x0000, 0x7FFF, 0x8000, 0x8001, 0xFFFF, 0x18000, 0x10000], np.uint32)
    grid = (e[:, None] | lows[None, :]).ravel()
    grid = np.concatenate([grid, grid | 0x80000000])
    return np.concatenate([_special_bits(), grid, rand]).view(np.float32)


def _pack(sdb, x2d, ld_pad=0, out_pad=0):
    """x2d fp32 [rows, cols] -> device pack with leading dims cols + pad."""
    import torch

    rows, cols = x2d.shape
    ld, ldo = cols + ld_pad, cols + out_pad
    src = torch.zeros((rows, ld), dtype=torch.float32)
    src[:, :cols] = torch.from_numpy(x2d)
    src = src.cuda()
    dst = torch.zeros((rows, ldo), dtype=torch.int16, device="cuda")
    sdb.check(sdb.lib().sdb200_pack_bf16(src.data_ptr(), ld, dst.data_ptr(), ldo, rows, cols))
    torch.cuda.synchronize()
    return dst.cpu().numpy().view(np.uint16)[:, :cols]


@pytest.mark.parametrize("layout", ["vector", "scalar_cols", "scalar_ld"])
def test_device_bf16_rounding_bit_exact(sdb, orc, layout):
    x = _cases()
    want = orc.to_bf16(x)
    if layout == "vector":       # cols % 8 == 0, 16-byte rows: the uint4 kernel
        cols, ld_pad, out_pad = 1024, 0, 8
    elif layout == "scalar_cols":  # odd width: the per-element kernel
        cols, ld_pad, out_pad = 1001, 0, 0
    else:                        # ld breaks 16-byte rows: the per-element kernel
        cols, ld_pad, out_pad = 1024, 1, 0
    n = x.size // cols * cols
    got = _pack(sdb, x[:n].reshape(-1, cols), ld_pad, out_pad).ravel()
    bad = np.nonzero(got != want[:n])[0]
    assert bad.size == 0, [(hex(int(x[:n].view(np.uint32)[i])), hex(int(got[i])), hex(int(want[i]))) for i in bad[:8]]


def test_device_bf16_rounding_vs_reference_golden(sdb):
    """The reference library's own rounding of its fixture inputs (tests/golden)."""
    g = load_golden("layers")
    x = np.ascontiguousarray(g["bf16_in"], np.float32)
    n = x.size // 8 * 8
    assert np.array_equal(_pack(sdb, x[:n].reshape(1, -1)).ravel(), g["bf16_out"][:n])
    assert np.array_equal(_pack(sdb, x.reshape(1, -1), ld_pad=1).ravel(), g["bf16_out"])


def test_gemm_uses_the_rounded_operand(sdb):
    """gemm_nt_bf16 (fp32 A, rounded inside) == gemm_nt_bf16a on the packed A, bit for bit."""
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    rng = np.random.default_rng(3)
    M, N, K = 300, 256, 520
    A = rng.standard_normal((M, K)).astype(np.float32)
    A.view(np.uint32)[:, ::7] = (A.view(np.uint32)[:, ::7] & 0xFFFF0000) | 0x8000  # exact ties
    Wb = torch.from_numpy(f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32)).view(np.int16))
    Wb = Wb.cuda()
    Ad = torch.from_numpy(A).cuda()
    Ah = torch.empty((M, K), dtype=torch.int16, device="cuda")
    L = sdb.lib()
    sdb.check(L.sdb200_pack_bf16(Ad.data_ptr(), K, Ah.data_ptr(), K, M, K))
    c1 = torch.empty((M, N), device="cuda")
    c2 = torch.empty((M, N), device="cuda")
    sdb.check(L.sdb200_gemm_nt_bf16(M, N, K, Ad.data_ptr(), K, Wb.data_ptr(), K, c1.data_ptr(), N, None, 0))
    sdb.check(L.sdb200_gemm_nt_bf16a(M, N, K, Ah.data_ptr(), K, Wb.data_ptr(), K, c2.data_ptr(), N, None, 0))
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
