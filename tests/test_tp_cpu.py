"""CPU, world size 2 over gloo: the tensor-parallel sharding of the DiT block weights
(sdb200.tp.shard_weights) reproduces the unsharded block projections once the
row-parallel partial outputs are summed across ranks, as the device runner does with its
NCCL all-reduce after to_out and w2. Uneven head and FFN splits and the rank-0-only
row-parallel biases are covered."""
import os
import socket

import numpy as np
import pytest

from sdb200.tp import ffn_split, head_split, shard_weights


def test_splits():
    assert head_split(30, 4) == [(0, 8), (8, 16), (16, 23), (23, 30)]
    assert head_split(30, 8)[-1] == (27, 30) and sum(b - a for a, b in head_split(30, 8)) == 30
    assert ffn_split(10240, 8) == [(i * 1280, (i + 1) * 1280) for i in range(8)]
    assert sum(b - a for a, b in ffn_split(528, 2)) == 528
    with pytest.raises(ValueError):
        ffn_split(100, 2)


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _block_weights(seed, D, heads, F):
    rng = np.random.default_rng(seed)
    p = "layers.0."
    w = {}
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        w[p + "attention." + n + ".weight"] = rng.standard_normal((D, D)) * 0.05
    w[p + "attention.to_out.0.bias"] = rng.standard_normal(D)
    w[p + "attention.to_q.bias"] = rng.standard_normal(D)
    w[p + "feed_forward.w1.weight"] = rng.standard_normal((F, D)) * 0.05
    w[p + "feed_forward.w3.weight"] = rng.standard_normal((F, D)) * 0.05
    w[p + "feed_forward.w2.weight"] = rng.standard_normal((D, F)) * 0.05
    w[p + "feed_forward.w2.bias"] = rng.standard_normal(D)
    w[p + "attention_norm1.weight"] = np.ones(D)
    w["x_pad_token"] = rng.standard_normal((1, D))
    return w


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        heads, hd, F = 3, 64, 528  # uneven: heads 2 + 1, FFN blocks 17 + 16
        D = heads * hd
        w = _block_weights(0, D, heads, F)
        sh = shard_weights(w, heads, hd, rank, world)
        p = "layers.0."
        rng = np.random.default_rng(1)
        h = rng.standard_normal((7, D))
        ao = rng.standard_normal((7, D))
        h0, h1 = head_split(heads, world)[rank]
        # column-parallel q: this rank's columns of the full projection
        q_r = h @ sh[p + "attention.to_q.weight"].T + sh[p + "attention.to_q.bias"]
        q_full = h @ w[p + "attention.to_q.weight"].T + w[p + "attention.to_q.bias"]
        ok_q = np.allclose(q_r, q_full[:, h0 * hd:h1 * hd])
        # row-parallel to_out: partial sums + bias on rank 0 only
        a_r = ao[:, h0 * hd:h1 * hd] @ sh[p + "attention.to_out.0.weight"].T
        if p + "attention.to_out.0.bias" in sh:
            a_r = a_r + sh[p + "attention.to_out.0.bias"]
        t = torch.from_numpy(a_r.copy())
        dist.all_reduce(t)
        a_full = ao @ w[p + "attention.to_out.0.weight"].T + w[p + "attention.to_out.0.bias"]
        ok_out = np.allclose(t.numpy(), a_full)
        # SwiGLU FFN: column-parallel w1/w3, row-parallel w2
        g_r = _silu(h @ sh[p + "feed_forward.w1.weight"].T) * (h @ sh[p + "feed_forward.w3.weight"].T)
        f_r = g_r @ sh[p + "feed_forward.w2.weight"].T
        if p + "feed_forward.w2.bias" in sh:
            f_r = f_r + sh[p + "feed_forward.w2.bias"]
        t = torch.from_numpy(f_r.copy())
        dist.all_reduce(t)
        g = _silu(h @ w[p + "feed_forward.w1.weight"].T) * (h @ w[p + "feed_forward.w3.weight"].T)
        f_full = g @ w[p + "feed_forward.w2.weight"].T + w[p + "feed_forward.w2.bias"]
        ok_ffn = np.allclose(t.numpy(), f_full)
        ok_rep = np.array_equal(sh["x_pad_token"], w["x_pad_token"]) and np.array_equal(
            sh[p + "attention_norm1.weight"], w[p + "attention_norm1.weight"])
        q.put((rank, bool(ok_q and ok_out and ok_ffn and ok_rep), ""))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


def test_tensor_parallel_shards_sum_to_full_projection():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res


def test_shard_identity_for_one_rank():
    w = _block_weights(3, 128, 2, 64)
    sh = shard_weights(w, 2, 64, 0, 1)
    assert all(np.array_equal(sh[k], w[k]) for k in w)
