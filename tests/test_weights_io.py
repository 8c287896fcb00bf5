"""Checkpoint reading on the host (sdb200_safetensors_read, the reader behind
sdb200_zimage_load): dtype conversion against the reference's own reader
(Weights::load_safetensors, safetensors.cpp:80-168, compiled into oracle/_ref) and
against numpy - every F16 bit pattern, F32 -> BF16 rounding, BF16 kept bit for bit, the
size threshold, skipped dtypes, malformed files."""
import os

import numpy as np
import pytest

from safetensors_writer import write_safetensors


@pytest.fixture(scope="module")
def host():
    import sdb200

    sdb200.lib()
    return sdb200


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    rng = np.random.default_rng(3)
    all_f16 = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    big = rng.standard_normal((300, 70)).astype(np.float32) * 3
    big[0, :6] = [np.inf, -np.inf, np.nan, 3.0e38, -1e-40, 1e-45]
    bf = (rng.standard_normal((40, 33)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    t = {
        "all_f16": ("F16", all_f16),
        "big_f32": ("F32", big),
        "small_f32": ("F32", rng.standard_normal((5, 7)).astype(np.float32)),
        "bf16": ("BF16", bf),
        "positions": ("I64", np.arange(12, dtype=np.int64)),
    }
    path = str(tmp_path_factory.mktemp("st") / "w.safetensors")
    write_safetensors(path, t, metadata={"format": "pt"})
    return path, t


def test_f16_every_bit_pattern(host, ckpt):
    path, t = ckpt
    got = host.safetensors_read(path, "all_f16", keep_bf16=False)
    want = t["all_f16"][1].astype(np.float32)
    assert got.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_conversions_match_reference_reader(host, ref, ckpt):
    path, t = ckpt
    for name in ("all_f16", "big_f32", "small_f32", "bf16"):
        n = int(np.prod(t[name][1].shape))
        for keep, min_numel in ((False, 1 << 20), (True, 1000), (True, 1 << 20)):
            want = ref.safetensors_tensor(path, name, keep, min_numel, n)
            got = host.safetensors_read(path, name, keep_bf16=keep, bf16_min_numel=min_numel)
            assert got.shape == t[name][1].shape
            assert (got.dtype == np.uint16) == want[1], (name, keep, min_numel)
            g = got.reshape(-1)
            w = want[0]
            assert np.array_equal(g.view(np.uint16 if want[1] else np.uint32), w.view(np.uint16 if want[1] else np.uint32))


def test_bf16_rounding_matches_oracle(host, orc, ckpt):
    path, t = ckpt
    got = host.safetensors_read(path, "big_f32", keep_bf16=True, bf16_min_numel=1000)
    assert got.dtype == np.uint16
    assert np.array_equal(got.reshape(-1), orc.to_bf16(t["big_f32"][1].reshape(-1)))
    kept = host.safetensors_read(path, "bf16", keep_bf16=True, bf16_min_numel=1)
    assert np.array_equal(kept, t["bf16"][1])


def test_skipped_dtype_and_errors(host, ckpt, tmp_path):
    path, _ = ckpt
    with pytest.raises(host.SdbError):
        host.safetensors_read(path, "positions")
    with pytest.raises(host.SdbError):
        host.safetensors_read(path, "missing")
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(np.uint64(1 << 40).tobytes() + b"{}")
    with pytest.raises(host.SdbError):
        host.safetensors_read(str(bad), "x")
    with pytest.raises(host.SdbError):
        host.safetensors_read(str(tmp_path / "absent.safetensors"), "x")
