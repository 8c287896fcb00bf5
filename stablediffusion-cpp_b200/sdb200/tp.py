"""Megatron-style tensor parallelism of the Z-Image DiT: sharding of
the block weights and the NCCL communicator the device runner reduces with.

Per block (reference names, zimage.cpp:38-46):
  column-parallel  attention.to_q / to_k / to_v  rows of this rank's heads (+ their biases)
                   feed_forward.w1 / w3          rows [F_r0, F_r1) (+ biases)
  row-parallel     attention.to_out.0            columns of this rank's heads; bias on rank 0
                   feed_forward.w2               columns [F_r0, F_r1); bias on rank 0
  replicated       norms, QK-norm gammas, adaLN, embeddings, final layer
Heads that do not divide evenly (30 over 4 or 8 GPUs) are split unevenly, the first
`heads % world` ranks taking one more. The sum of the row-parallel partial outputs over
the group equals the unsharded projection; the runner all-reduces it before each
post-norm (zimage.cpp:122, :131), which needs the full row.
"""
from __future__ import annotations

import ctypes as C


def head_split(heads: int, world: int):
    """[(h0, h1)] per rank, contiguous, sizes differing by at most one."""
    base, extra = divmod(heads, world)
    out, h = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((h, h + n))
        h += n
    return out


def ffn_split(F: int, world: int, block: int = 16):
    """[(f0, f1)] per rank in whole 16-row blocks (the SwiGLU interleave unit)."""
    nb = F // block
    if nb * block != F:
        raise ValueError("FFN width must be a multiple of 16")
    return [(a * block, b * block) for a, b in head_split(nb, world)]


def _is_block_param(name):
    return name.startswith(("layers.", "noise_refiner.", "context_refiner."))


def shard_weights(weights: dict, heads: int, head_dim: int, rank: int, world: int) -> dict:
    """This rank's view of a Z-Image weight dict (numpy arrays or torch tensors, the
    same names and dtypes). world == 1 returns the input unchanged."""
    if world == 1:
        return dict(weights)
    h0, h1 = head_split(heads, world)[rank]
    q0, q1 = h0 * head_dim, h1 * head_dim
    out = {}
    for name, w in weights.items():
        if not _is_block_param(name):
            out[name] = w
            continue
        leaf = name.split(".", 2)[2]  # e.g. "attention.to_q.weight"
        if leaf in ("attention.to_q.weight", "attention.to_k.weight", "attention.to_v.weight",
                    "attention.to_q.bias", "attention.to_k.bias", "attention.to_v.bias"):
            out[name] = w[q0:q1]
        elif leaf == "attention.to_out.0.weight":
            out[name] = w[:, q0:q1]
        elif leaf in ("attention.to_out.0.bias", "feed_forward.w2.bias"):
            if rank == 0:
                out[name] = w
        elif leaf in ("feed_forward.w1.weight", "feed_forward.w3.weight", "feed_forward.w1.bias",
                      "feed_forward.w3.bias"):
            F = weights[name.rsplit(".", 2)[0] + ".w1.weight"].shape[0]
            f0, f1 = ffn_split(F, world)[rank]
            out[name] = w[f0:f1]
        elif leaf == "feed_forward.w2.weight":
            f0, f1 = ffn_split(w.shape[1], world)[rank]
            out[name] = w[:, f0:f1]
        else:
            out[name] = w
    for name in list(out):
        t = out[name]
        if hasattr(t, "contiguous"):
            out[name] = t.contiguous()
        else:
            import numpy as np

            out[name] = np.ascontiguousarray(t)
    return out


class Comm:
    """A tensor-parallel NCCL communicator of libsdb200 on the current device. The
    128-byte unique id is created on rank 0 and shared over torch.distributed."""

    def __init__(self, rank: int, world: int, pg=None):
        from . import check, lib

        L = lib()
        uid = (C.c_char * 128)()
        if rank == 0:
            check(L.sdb200_comm_unique_id(uid))
        if world > 1:
            import torch.distributed as dist

            box = [bytes(uid.raw)]
            dist.broadcast_object_list(box, src=0, group=pg)
            C.memmove(uid, box[0], 128)
        self.handle = L.sdb200_comm_create(uid, rank, world)
        if not self.handle:
            raise RuntimeError(L.sdb200_last_error().decode())
        self.rank, self.world = rank, world

    def set_barrier(self, flags: bool):
        """Barrier between the fused tensor-parallel kernels: a flag exchange over NVLink
        (True, the default) or a 4-byte NCCL all-reduce (False). Same on every rank."""
        from . import check, lib

        check(lib().sdb200_comm_set_barrier(self.handle, 1 if flags else 0))

    def allreduce_sum_(self, t):
        """In-place sum over the group of a CUDA float32 tensor."""
        from . import backend, check, lib

        backend.bind_stream()
        check(lib().sdb200_comm_allreduce_sum_f32(self.handle, t.data_ptr(), t.numel()))
        return t

    def close(self):
        from . import lib

        if self.handle:
            lib().sdb200_comm_destroy(self.handle)
            self.handle = None
