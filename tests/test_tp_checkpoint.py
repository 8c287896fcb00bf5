"""The tensor-parallel cut of a Z-Image checkpoint (the reader behind sdb200_zimage_load
with world > 1) against the in-memory sharding sdb200.tp.shard_weights.

The reference reads the whole checkpoint on every process (Weights::load_model,
safetensors.cpp:80-194, pipeline.cpp:113-115) and has no tensor parallelism. Here each
rank reads only its Megatron shard: the q/k/v rows and to_out columns of its heads
(uneven when heads % world != 0), the w1/w3 rows and w2 columns of its 16-row FFN blocks,
the row-parallel biases on rank 0 only, everything else whole. Every tensor a rank
receives must equal, bit for bit, the same cut of the tensor as the reference's reader
converts it (BF16 kept, F16 / F32 widened, BF16 from bf16_min_numel elements up).

* host (no GPU): sdb200_checkpoint_read_shard for every rank of world 2, 4 and 8;
* GPU: sdb200_zimage_load for every rank of world 2 and 4 on one device, read back with
  sdb200_zimage_get_weight.
"""
import os

import numpy as np
import pytest

from safetensors_writer import write_checkpoint

MIN_NUMEL = 32768  # every block matrix of the test model is at least this large


def _cfg():
    from sdb200.zimage import ZConfig

    # 6 heads of 128 and 34 FFN blocks of 16: both split unevenly over 4 and 8 ranks
    return ZConfig(dim=768, heads=6, ffn=544, t_dim=256, t_hidden=256, cap_dim=128, layers=2, noise_refiners=1,
                   context_refiners=1)


def _bits(a):
    return a.view(np.uint16) if a.dtype == np.uint16 else a.view(np.uint32)


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    """A two-file checkpoint holding BF16, F16 and F32 block tensors, and each tensor as the
    reference's reader returns it (uint16 BF16 bits or float32)."""
    from sdb200.workloads import f32_to_bf16_bits
    from sdb200.zimage import random_weights_numpy

    w, bf = random_weights_numpy(_cfg(), 11)
    stored, as_read = {}, {}
    for i, (n, a) in enumerate(sorted(w.items())):
        if n in bf and i % 3 == 0:      # F32 on disk, rounded to BF16 by the reader
            stored[n] = ("F32", a)
        elif n in bf and i % 3 == 1:    # F16 on disk, widened then rounded
            stored[n] = ("F16", a.astype(np.float16))
            a = a.astype(np.float16).astype(np.float32)
        elif n in bf:
            stored[n] = ("BF16", f32_to_bf16_bits(a))
        else:
            stored[n] = ("F32", a)
        as_read[n] = f32_to_bf16_bits(a) if a.size >= MIN_NUMEL else a
    d = str(tmp_path_factory.mktemp("tpck"))
    write_checkpoint(d, "model", stored, shards=2)
    return d, as_read


def _expected(as_read, rank, world):
    from sdb200.tp import shard_weights

    return shard_weights(as_read, _cfg().heads, 128, rank, world)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_checkpoint_shard_cut_on_host(checkpoint, world):
    import sdb200

    d, as_read = checkpoint
    cfg = _cfg()
    for rank in range(world):
        want = _expected(as_read, rank, world)
        for name in as_read:
            got = sdb200.checkpoint_read_shard(d, "model", name, rank, world, cfg.heads, MIN_NUMEL)
            if name not in want:
                assert got is None, (name, rank, world)
                continue
            assert got is not None, (name, rank, world)
            assert got.dtype == want[name].dtype and got.shape == want[name].shape, (name, rank, world)
            assert np.array_equal(_bits(got), _bits(want[name])), (name, rank, world)
    # world 1 is the reader of sdb200_zimage_load without a cut
    name = "layers.0.feed_forward.w2.weight"
    assert np.array_equal(sdb200.checkpoint_read_shard(d, "model", name, 0, 1, cfg.heads, MIN_NUMEL), as_read[name])


def test_checkpoint_shard_rejects_bad_arguments(checkpoint):
    import sdb200

    d, _ = checkpoint
    with pytest.raises(sdb200.SdbError):
        sdb200.checkpoint_read_shard(d, "model", "layers.0.attention.to_q.weight", 2, 2, 6)
    with pytest.raises(sdb200.SdbError):
        sdb200.checkpoint_read_shard(os.path.join(d, "missing"), "model", "x_pad_token", 0, 2, 6)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_zimage_load_shard_on_one_gpu(sdb, checkpoint, world):
    """sdb200_zimage_load for each rank of `world` (one device, no communicator needed to
    load): the device copy of every tensor equals the in-memory shard."""
    from sdb200.zimage import ZImageB200

    d, as_read = checkpoint
    for rank in range(world):
        m = ZImageB200.from_checkpoint(d, "model", _cfg(), rank=rank, world=world, bf16_min_numel=MIN_NUMEL)
        want = _expected(as_read, rank, world)
        for name, arr in want.items():
            got = m.get_weight(name)
            assert got.dtype == arr.dtype and got.shape == arr.shape, (name, rank, world)
            assert np.array_equal(_bits(got), _bits(arr)), (name, rank, world)
        for name in set(as_read) - set(want):  # row-parallel biases live on rank 0 only
            with pytest.raises(sdb.SdbError):
                m.get_weight(name)
        del m
