"""Benchmark of StableDiffusion-cpp's dense-contraction hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload gemm]

Workload `gemm`: the Z-Image fused-QKV projection
Y[4096, 11520] = X[4096, 3840] (fp32) * W[11520, 3840]^T (bf16) + b, fp32 accumulate,
through sdb200_gemm_nt_bf16 (the drop-in for the reference's gemm_nt_bf16). One step =
one such GEMM on each GPU. The GPUs run independent replicas (no collective: one GEMM
does not shard across devices), so the value is the sum over GPUs ("scaling": "weak").

Printed on rank 0 as one JSON line:
  value      TFLOP/s of the whole job, inputs resident in HBM (2*M*N*K per step)
  e2e        the same metric through the C ABI with pinned HOST buffers: H2D of X and
             D2H of Y inside the timed region (W is resident, as the reference keeps
             weights on the device after Weights::to_device)
  roofline   the tensor-core GEMM kernel alone (A pre-packed to bf16), timed with CUDA
             events on the library's stream, against MEASURED_PEAKS.json bf16 burst peak
  cpu_baseline  the reference's own CPU gemm_nt_bf16 (oracle/_ref, compiled from its
             sources) on this host's cores, rank 0 at N=1 only
The inputs (340 MB per step: X 63 MB, W 88 MB, Y 189 MB) exceed the 126 MB L2, so no
explicit flush is needed between timed iterations.

--impl reference runs the reference's CPU implementation of the same GEMM (rank 0
only) and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "stablediffusion-cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "bf16 GEMM TFLOP/s (% tcgen05 peak); Z-Image DiT ms/step @1024² at 1/2/4/8 GPUs"
M_, N_, K_ = 4096, 11520, 3840
FLOP = 2.0 * M_ * N_ * K_

THROTTLE_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def traffic_from_profile():
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemm_tc_cfg1.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons through NVML every
    2 ms from a background thread while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._ok = False
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            time.sleep(0.002)

    def __exit__(self, *a):
        self._stop.set()
        if self._ok:
            self._t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, bits in self.samples:
            for b, name in THROTTLE_BITS.items():
                if bits & b and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """The reference's own CPU GEMM (oracle/_ref) on this host's cores: bounded sample
    of the same workload per step (512 rows of X, i.e. 1/8 of the GEMM)."""
    if rank != 0:
        return
    import numpy as np

    from oracle import RefCPU

    ref = RefCPU()
    ref.set_num_threads(0)
    cores = ref.num_threads()
    rows = 512
    rng = np.random.default_rng(0)
    X = rng.standard_normal((rows, K_), dtype=np.float32)
    Wh = ref.to_bf16((0.02 * rng.standard_normal((N_, K_), dtype=np.float32)).astype(np.float32))
    b = (0.01 * rng.standard_normal(N_, dtype=np.float32)).astype(np.float32)
    for _ in range(args.warmup):
        ref.gemm_nt_bf16(X, Wh, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.gemm_nt_bf16(X, Wh, b)
    dt = (time.perf_counter() - t0) / args.steps
    tflops = 2.0 * rows * N_ * K_ / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 * (M_ / rows),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 x bf16 -> f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights)",
        "config": {"workload": "cfg1 fused-QKV GEMM 4096x11520x3840 bf16 weights (+bias)",
                   "parallelism": "reference CPU thread pool", "sample_rows": rows},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                         "sample": f"{rows} of 4096 rows of X per step (1/8 of the GEMM), all {N_} columns"},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """Reference CPU gemm_nt_bf16 timed on 512 rows (about 2-3 s of CPU work)."""
    try:
        import numpy as np

        from oracle import RefCPU

        if not RefCPU.available():
            return None
        ref = RefCPU()
        ref.set_num_threads(0)
        rows = 512
        rng = np.random.default_rng(0)
        X = rng.standard_normal((rows, K_), dtype=np.float32)
        Wh = ref.to_bf16((0.02 * rng.standard_normal((N_, K_), dtype=np.float32)).astype(np.float32))
        b = (0.01 * rng.standard_normal(N_, dtype=np.float32)).astype(np.float32)
        ref.gemm_nt_bf16(X, Wh, b)
        reps = 3
        t0 = time.perf_counter()
        for _ in range(reps):
            ref.gemm_nt_bf16(X, Wh, b)
        dt = (time.perf_counter() - t0) / reps
        return {"value": 2.0 * rows * N_ * K_ / dt / 1e12, "unit": "TFLOP/s", "cores": ref.num_threads(),
                "kind": "reference",
                "sample": f"{rows} of 4096 rows of the cfg1 GEMM, {reps} reps after 1 warm-up, reference "
                          "gemm_nt_bf16 (tensor.cpp:412) built from its sources"}
    except Exception as e:  # the baseline is reported, never required
        return {"value": None, "unit": "TFLOP/s", "cores": None, "kind": "reference", "sample": f"failed: {e}"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemm", choices=["gemm"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()

    if args.impl == "reference":
        return run_reference(args, world, rank)

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist

    import sdb200
    from sdb200 import backend as be

    if not sdb200.available():
        raise SystemExit("libsdb200: no usable sm_100 device: " + sdb200.lib().sdb200_last_error().decode())
    be.bind_stream()
    L = sdb200.lib()

    from sdb200.workloads import cfg1_inputs, f32_to_bf16_bits

    X, W, b = cfg1_inputs()
    Wbits = f32_to_bf16_bits(W)  # bf16 rounding of the weights, as Tensor::to_bf16 does at load time
    dev = torch.device("cuda", local)
    Xd = torch.from_numpy(X).to(dev)
    Wd = torch.from_numpy(Wbits.view(np.int16)).to(dev).view(torch.bfloat16)
    bd = torch.from_numpy(b).to(dev)
    Yd = torch.empty((M_, N_), device=dev)
    stream = torch.cuda.current_stream()

    def step():
        sdb200.check(L.sdb200_gemm_nt_bf16(M_, N_, K_, Xd.data_ptr(), K_, Wd.data_ptr(), K_, Yd.data_ptr(), N_,
                                           bd.data_ptr(), 0))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    t = torch.tensor([ms], device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_max = float(t.item())
    value = FLOP * args.steps * world / (ms_max * 1e-3) / 1e12

    # ---- dominant kernel alone: tcgen05 GEMM with A pre-packed to bf16 ----------
    Xbf = Xd.to(torch.bfloat16)  # A operand as the pack kernel produces it (RNE)
    for _ in range(3):
        sdb200.check(L.sdb200_gemm_nt_bf16a(M_, N_, K_, Xbf.data_ptr(), K_, Wd.data_ptr(), K_, Yd.data_ptr(), N_,
                                            bd.data_ptr(), 0))
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(args.steps, 10)
    k0.record(stream)
    for _ in range(reps):
        sdb200.check(L.sdb200_gemm_nt_bf16a(M_, N_, K_, Xbf.data_ptr(), K_, Wd.data_ptr(), K_, Yd.data_ptr(), N_,
                                            bd.data_ptr(), 0))
    k1.record(stream)
    torch.cuda.synchronize()
    kms = k0.elapsed_time(k1) / reps
    peak_tf, _, peak_kind = peaks()
    achieved = FLOP / (kms * 1e-3) / 1e12

    # ---- end to end through the C ABI with host buffers ---------------------------
    Xh = torch.from_numpy(X).pin_memory()
    Yh = torch.empty((M_, N_), dtype=torch.float32).pin_memory()
    Xs = torch.empty_like(Xd)

    def e2e_step():
        sdb200.check(L.sdb200_upload(Xs.data_ptr(), Xh.data_ptr(), Xh.numel() * 4))
        sdb200.check(L.sdb200_gemm_nt_bf16(M_, N_, K_, Xs.data_ptr(), K_, Wd.data_ptr(), K_, Yd.data_ptr(), N_,
                                           bd.data_ptr(), 0))
        sdb200.check(L.sdb200_download(Yh.data_ptr(), Yd.data_ptr(), Yh.numel() * 4))

    for _ in range(2):
        e2e_step()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a0.elapsed_time(a1)
    t = torch.tensor([e2e_ms], device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    e2e_value = FLOP * args.steps * world / (float(t.item()) * 1e-3) / 1e12
    ok_err = be.device_error_word()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 x bf16 -> f32 (A rounded from f32)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights, N(0,0.01) bias)",
            "config": {"workload": "cfg1 fused-QKV GEMM Y[4096,11520] = X[4096,3840] W[11520,3840]^T + b",
                       "global_batch": world, "parallelism": f"replicas x{world} (no collective)",
                       "l2": "inputs 340 MB/step > 126 MB L2, no flush"},
            "gpu_launches": 2 * args.steps,
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc<256,false> (tcgen05 kind::f16, 128x256 tiles)",
                         "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                         "peak_kind": f"{peak_kind} bf16 burst", "traffic": traffic_from_profile(),
                         "kernel_ms": kms},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": int(Xh.numel() * 4),
                    "d2h_bytes_per_step": int(Yh.numel() * 4)},
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "device_error_word": ok_err,
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
