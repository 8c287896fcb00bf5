"""Worker run under torchrun by tests/test_tp_gpu.py: the Z-Image forward with tensor
parallelism over the launched GPUs (heads 3 and FFN 528 split unevenly over 2 ranks), in
both exchange modes (fused into the kernels over NVLink - ordered by the flag barrier and
by the NCCL barrier - and NCCL all-reduce), against
the single-GPU forward and the CPU oracle, and the same model loaded per rank from a
checkpoint file. Rank 0 prints one JSON line."""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "stablediffusion-cpp_b200"), os.path.join(ROOT, "oracle")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    import sdb200
    from sdb200.tp import Comm, shard_weights
    from sdb200.zimage import ZConfig, ZImageB200, random_weights_numpy

    cfg = ZConfig(dim=384, heads=3, ffn=528, t_dim=256, t_hidden=256, cap_dim=128, layers=2, noise_refiners=1,
                  context_refiners=1)
    w, bf = random_weights_numpy(cfg, 0)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 16, 16, 24)).astype(np.float32)
    cap = rng.standard_normal((1, 20, 128)).astype(np.float32)
    xt, capt = torch.from_numpy(x).to(dev), torch.from_numpy(cap).to(dev)
    comm = Comm(rank, world)
    m = ZImageB200(shard_weights(w, cfg.heads, 128, rank, world), cfg, bf16_names=bf)
    ys = {}
    diffs = []
    # 1: exchange fused into the GEMM epilogue / post-norm, ordered by the flag barrier over
    # NVLink; "1n": the same with the NCCL all-reduce barrier; 0: NCCL all-reduce of the outputs
    for mode in (1, "1n", 0):
        comm.set_barrier(mode != "1n")
        m.set_tp(comm, mode=1 if mode == "1n" else mode)
        y = m.forward(xt, 0.6, capt)
        y = m.forward(xt, 0.6, capt)  # second call reuses the peer mappings
        torch.cuda.synchronize()
        y0 = y.clone()
        dist.broadcast(y0, src=0)
        diffs.append(float((y - y0).abs().max().item()))
        ys[mode] = y
    t = torch.tensor([max(diffs)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    m.set_tp(None)
    # The same model read from a checkpoint file, each rank reading only its shard
    # (sdb200_zimage_load): identical to the shards registered from memory.
    import tempfile

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from safetensors_writer import write_checkpoint
    from sdb200.workloads import f32_to_bf16_bits

    mn = 32768
    box = [tempfile.mkdtemp(prefix="tpck_") if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    if rank == 0:
        write_checkpoint(box[0], "model", {n: ("BF16", f32_to_bf16_bits(a)) if n in bf else ("F32", a)
                                           for n, a in w.items()}, shards=2)
    dist.barrier()
    w_read = {n: (f32_to_bf16_bits(a).astype(np.uint32) << 16).view(np.float32) if a.size >= mn else a
              for n, a in w.items()}
    bf_read = {n for n, a in w.items() if a.size >= mn}
    mf = ZImageB200.from_checkpoint(box[0], "model", cfg, rank=rank, world=world, bf16_min_numel=mn)
    mf.set_tp(comm)
    y_file = mf.forward(xt, 0.6, capt)
    mm = ZImageB200(shard_weights(w_read, cfg.heads, 128, rank, world), cfg, bf16_names=bf_read)
    mm.set_tp(comm)
    y_mem = mm.forward(xt, 0.6, capt)
    torch.cuda.synchronize()
    file_diff = torch.tensor([float((y_file - y_mem).abs().max().item())], device=dev)
    dist.all_reduce(file_diff, op=dist.ReduceOp.MAX)
    mf.set_tp(None)
    mm.set_tp(None)
    if rank == 0:
        from oracle import Oracle
        from zimage_oracle import ZImageOracle

        single = ZImageB200(w, cfg, bf16_names=bf).forward(xt, 0.6, capt).cpu().numpy()
        want = ZImageOracle(Oracle(), w, bf, heads=cfg.heads).forward(x, 0.6, cap)
        rel = lambda a, b: float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))  # noqa: E731
        fused, allred = ys[1].cpu().numpy(), ys[0].cpu().numpy()
        print(json.dumps({"world": world, "rel_vs_single_gpu": rel(fused, single), "rel_vs_oracle": rel(fused, want),
                          "allreduce_rel_vs_single_gpu": rel(allred, single),
                          "allreduce_rel_vs_oracle": rel(allred, want), "max_rank_diff": float(t.item()),
                          "checkpoint_vs_memory_max_diff": float(file_diff.item()),
                          "barrier_flags_vs_nccl_max_diff": float(np.abs(fused - ys["1n"].cpu().numpy()).max()),
                          "finite": bool(np.isfinite(fused).all() and np.isfinite(allred).all()),
                          "err_word": sdb200.backend.device_error_word()}), flush=True)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
