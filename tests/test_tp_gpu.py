"""GPU, 2 devices: the tensor-parallel Z-Image forward against the single-GPU forward
(relative Frobenius <= 1e-3, only the order of the fp32 partial sums differs) and the CPU
oracle (<= 1e-2), with all ranks holding identical outputs. Both exchange modes: the
row-parallel partial outputs scattered to their owner rank from the GEMM epilogue and
reduced in the sequence-sharded post-norm (default; ordered by a flag barrier over NVLink,
bit-identical to the same with an NCCL all-reduce as the barrier), and an NCCL all-reduce. Also each
rank reading only its shard from a checkpoint file (sdb200_zimage_load) against the
same shards registered from memory (identical outputs). Skipped where fewer than 2 GPUs
are visible."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_tensor_parallel_forward_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "tp_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1]
    r = json.loads(line)
    assert r["finite"] and r["err_word"] == 0
    assert r["max_rank_diff"] == 0.0
    assert r["rel_vs_single_gpu"] <= 1e-3, r
    assert r["rel_vs_oracle"] <= 1e-2, r
    assert r["allreduce_rel_vs_single_gpu"] <= 1e-3, r
    assert r["allreduce_rel_vs_oracle"] <= 1e-2, r
    assert r["checkpoint_vs_memory_max_diff"] == 0.0, r
    assert r["barrier_flags_vs_nccl_max_diff"] == 0.0, r


def test_flag_barrier_arrival_and_bounded_wait(sdb):
    """The tensor-parallel flag barrier on one GPU, every rank's flag words mapped to one
    local array (sdb200_comm_barrier_selftest). All peers arrived: it passes and leaves this
    rank's epoch in its word. One peer missing (a word nothing sets): the wait runs out after
    its 2 s bound, the device error word holds bit 64, sdb200_synchronize reports
    SDB200_ERR_DEVICE_WAIT and clears it, and the context still computes."""
    import time

    import torch

    L = sdb.lib()
    flags = torch.zeros(4, dtype=torch.int32, device="cuda")
    flags[1:] = 5
    torch.cuda.synchronize()  # the flags are written on torch's stream
    sdb.check(L.sdb200_comm_barrier_selftest(flags.data_ptr(), 4, 0, 5))
    assert L.sdb200_synchronize() == 0
    assert flags.tolist() == [5, 5, 5, 5]
    flags.zero_()
    flags[1] = 6
    flags[3] = 6  # rank 2 never arrives
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    sdb.check(L.sdb200_comm_barrier_selftest(flags.data_ptr(), 4, 0, 6))
    assert sdb.backend.device_error_word() == 64
    waited = time.perf_counter() - t0
    assert 1.5 <= waited <= 30.0, waited
    assert L.sdb200_synchronize() == 4  # SDB200_ERR_DEVICE_WAIT, word cleared
    assert sdb.backend.device_error_word() == 0
    a = torch.randn(64, 96, device="cuda")
    b = torch.randn(80, 96, device="cuda")
    got = sdb.backend.gemm_nt_f32(a, b)
    assert torch.allclose(got, a @ b.T, rtol=2e-2, atol=2e-2)
    assert L.sdb200_comm_barrier_selftest(flags.data_ptr(), 9, 0, 1) != 0  # world above 8: refused
