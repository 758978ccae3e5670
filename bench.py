"""Decode-attention benchmark: µs/step and achieved HBM TB/s at 1/2/4/8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4]
    python bench.py --impl reference ...      # the reference's CPU kernel on this host

One JSON line on rank 0.  `value` is whole-job throughput in TB/s of
algorithmic bytes (KV read once + q + outputs, summed over ranks) divided by
the device-timed step (max over ranks), inputs resident in HBM.  `e2e` is the
same metric through the public API with the step's host buffers copied in
(H2D of q and of the new token's K/V, D2H of out + lse) inside the timed
region.  The KV cache itself is device-resident state, as the reference's
InplaceKVCache is host-resident state appended one token per step
(system/qwenoffload.py:100-122).

Workloads:
  cfg1  GQA Qwen3 layer, B=1, L=4096
  cfg2  GQA Mixtral layer, B=16, ragged L in [1024, 32768], two shares merged by LSE
  cfg4  GQA Qwen3, B=32, L=131072 sequence-sharded over N GPUs (default)
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn µs/step and achieved HBM TB/s (frac of peak) at 1/2/4/8 B200 vs CPU"


# ----------------------------------------------------------------- helpers
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(name):
    """dram read+write bytes per launch recorded from an ncu capture
    (profiles/<name>.txt holds a 'traffic_bytes_per_launch: N' line)."""
    path = os.path.join(ROOT, "profiles", name + ".txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"ws_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.idx)], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None:
            return None
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, x in enumerate(r) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def dist_info():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# --------------------------------------------------------------- workloads
class GqaLongCtx:
    """cfg4: Qwen3 shape, B=32, 32 q heads / 4 kv heads, D=128, L=131072 per
    sequence, KV sharded contiguously over the ranks: rank r holds tokens
    [r*L/N, (r+1)*L/N) of every (sequence, kv-head) row."""

    name = "cfg4"
    workload = "gqa_longctx_qwen3_b32_l131072_sharded"

    def __init__(self, world, rank, B=32, H=32, Hkv=4, D=128, L=131072):
        from scope_b200 import _lib
        self.world, self.rank = world, rank
        self.B, self.H, self.Hkv, self.D, self.L = B, H, Hkv, D, L
        self.G = H // Hkv
        assert L % world == 0
        self.Lloc = L // world
        self.scale = D ** -0.5
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(4000 + rank)
        rows = B * Hkv
        self.k = torch.randn(rows, self.Lloc, D, device=dev, dtype=torch.bfloat16, generator=g)
        self.v = torch.randn(rows, self.Lloc, D, device=dev, dtype=torch.bfloat16, generator=g)
        gq = torch.Generator(device=dev).manual_seed(4)
        self.q = torch.randn(B, H, D, device=dev, dtype=torch.bfloat16, generator=gq)
        self.qv = self.q.view(rows, self.G, D)
        self.lib = _lib.lib()
        self._lib = _lib
        if world == 1:
            self.out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
            self.lse = torch.empty(B, H, dtype=torch.float32, device=dev)
        else:
            self.part_o = torch.empty(B * H, D, dtype=torch.float32, device=dev)
            self.part_l = torch.empty(B * H, dtype=torch.float32, device=dev)
            self.all_o = torch.empty(world, B * H, D, dtype=torch.float32, device=dev)
            self.all_l = torch.empty(world, B * H, dtype=torch.float32, device=dev)
            self.out = torch.empty(B * H, D, dtype=torch.bfloat16, device=dev)
            self.lse = torch.empty(B * H, dtype=torch.float32, device=dev)
        nbytes = self.lib.ws_gqa_decode_workspace_size(rows, self.G, D, self.Lloc)
        self.ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)
        # host buffers for the end-to-end step
        self.q_host = torch.randn(B, H, D).bfloat16().pin_memory()
        self.knew_host = torch.randn(rows, D).bfloat16().pin_memory()
        self.vnew_host = torch.randn(rows, D).bfloat16().pin_memory()
        self.out_host = torch.empty(B * H * D, dtype=torch.bfloat16).pin_memory()
        self.lse_host = torch.empty(B * H, dtype=torch.float32).pin_memory()
        self.kernels_per_step = 1 if world == 1 else 2

    # algorithmic bytes of one local kernel launch, and of one step summed over ranks
    def kernel_bytes(self):
        rows = self.B * self.Hkv
        kv = 2 * rows * self.Lloc * self.D * 2
        q = self.B * self.H * self.D * 2
        out = self.B * self.H * (self.D * (2 if self.world == 1 else 4) + 4)
        return kv + q + out

    def step_bytes(self):
        kv = 2 * self.B * self.Hkv * self.L * self.D * 2
        return kv + self.B * self.H * self.D * 2 + self.B * self.H * (self.D * 2 + 4)

    def kernel(self):
        L_ = self.lib
        st = torch.cuda.current_stream().cuda_stream
        rows = self.B * self.Hkv
        if self.world == 1:
            rc = L_.ws_gqa_decode(self.qv.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.k.stride(0),
                                  self.k.stride(1), self.v.stride(0), self.v.stride(1), rows, self.G, self.D, self.D,
                                  self.Lloc, self.scale, self._lib.WS_DTYPE_BF16, self._lib.WS_OUT_NORM_BF16,
                                  self.out.data_ptr(), None, None, self.lse.data_ptr(), self.ws.data_ptr(),
                                  self.ws.numel(), st)
        else:
            rc = L_.ws_gqa_decode(self.qv.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.k.stride(0),
                                  self.k.stride(1), self.v.stride(0), self.v.stride(1), rows, self.G, self.D, self.D,
                                  self.Lloc, self.scale, self._lib.WS_DTYPE_BF16, self._lib.WS_OUT_NORM_F32,
                                  self.part_o.data_ptr(), None, None, self.part_l.data_ptr(), self.ws.data_ptr(),
                                  self.ws.numel(), st)
        if rc != 0:
            raise RuntimeError(L_.ws_last_error().decode())

    def step(self):
        self.kernel()
        if self.world > 1:
            import torch.distributed as dist
            from scope_b200 import lse_merge
            dist.all_gather_into_tensor(self.all_o.view(-1), self.part_o.view(-1))
            dist.all_gather_into_tensor(self.all_l.view(-1), self.part_l.view(-1))
            lse_merge(self.all_o, self.all_l, torch.bfloat16, out=self.out, out_lse=self.lse)

    def e2e_step(self):
        # H2D: this step's query, and the new token's K/V row appended to the last shard
        self.q.copy_(self.q_host, non_blocking=True)
        if self.rank == self.world - 1:
            self.k[:, self.Lloc - 1].copy_(self.knew_host, non_blocking=True)
            self.v[:, self.Lloc - 1].copy_(self.vnew_host, non_blocking=True)
        self.step()
        if self.rank == 0:
            self.out_host.copy_(self.out.view(-1), non_blocking=True)
            self.lse_host.copy_(self.lse.view(-1), non_blocking=True)

    def e2e_bytes(self):
        h2d = self.world * self.q.numel() * 2 + 2 * self.knew_host.numel() * 2
        d2h = self.out.numel() * 2 + self.lse.numel() * 4
        return h2d, d2h

    def config(self):
        return {"workload": self.workload, "batch": self.B, "q_heads": self.H, "kv_heads": self.Hkv,
                "head_dim": self.D, "kv_len": self.L, "kv_len_per_gpu": self.Lloc,
                "parallelism": f"seq-shard{self.world}", "l2": "inputs > L2 (KV 8.6 GB total)",
                "exchange": "nccl all_gather of (o fp32, lse) + lse_merge kernel" if self.world > 1 else "none"}

    # reference CPU sample: same op (fused_cpu_attn, B_kv = 128 rows), shorter KV
    def cpu_sample(self, L_s=4096):
        return dict(rows=self.B * self.Hkv, G=self.G, D=self.D, L=L_s)


def cpu_reference_time(sample, budget_s=10.0, max_calls=200, warm=1, kind_pref="reference"):
    """Time the reference's own CPU kernel (oracle/_ref) -- or the oracle port
    when the compiled reference cannot run here -- on a bounded sample.
    Returns (bytes_per_second, dict)."""
    import oracle
    rows, G, D, L = sample["rows"], sample["G"], sample["D"], sample["L"]
    torch.manual_seed(11)
    ncores = os.cpu_count() or 1
    q = torch.randn(rows, G, D).bfloat16()
    k = torch.randn(rows, L, D).bfloat16()
    v = torch.randn(rows, L, D).bfloat16()
    nbytes = 2 * rows * L * D * 2 + rows * G * D * 2 + rows * G * (D * 2 + 4)
    kind = "port"
    if kind_pref == "reference" and oracle.ref_available():
        try:
            ref = oracle.load_ref("cpu_attn_ext")
            ref.set_num_threads(ncores)
            torch.set_num_threads(ncores)
            fn = lambda: ref.fused_cpu_attn(q, k, v, D ** -0.5)  # noqa: E731
            kind = "reference"
        except Exception:
            kind = "port"
    if kind == "port":
        qb, kb, vb = oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v)
        fn = lambda: oracle.gqa_decode(qb, kb, vb, D ** -0.5)  # noqa: E731
    for _ in range(warm):
        fn()
    times = []
    t_start = time.perf_counter()
    while len(times) < max_calls and (time.perf_counter() - t_start) < budget_s:
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return nbytes / t, {"kind": kind, "cores": ncores, "calls": len(times), "sec_per_call": t,
                        "sample": f"fused_cpu_attn bf16, B_kv={rows}, G={G}, D={D}, L={L} "
                                  f"({nbytes / 1e6:.0f} MB algorithmic per call)"}


WORKLOADS = {"cfg4": GqaLongCtx}


# -------------------------------------------------------------------- main
def time_loop(fn, steps, warmup, world):
    for _ in range(warmup):
        fn()
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3 / steps, world)


def run_reference_arm(args):
    world, rank, _ = dist_info()
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    # one step = one reference call on a bounded sample of the workload (same rows, shorter KV)
    sample = {"rows": 128, "G": 8, "D": 128, "L": 2048}
    bps, info = cpu_reference_time(sample, budget_s=1e9, max_calls=args.steps, warm=args.warmup)
    value = bps / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": info["sec_per_call"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl.workload, "sample": info["sample"]},
            "cpu_baseline": {"value": value, "unit": "TB/s", "cores": info["cores"], "kind": info["kind"],
                             "sample": info["sample"]},
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference_arm(args)
        return

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import scope_b200
    scope_b200.build()
    wl = WORKLOADS[args.workload](world, rank)

    # 1) dominant kernel alone (roofline)
    t_kernel = time_loop(wl.kernel, args.steps, args.warmup, world)
    # 2) full step, device-resident inputs (value)
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local
    with ClockSampler(gpu_index) as clk:
        t_step = time_loop(wl.step, args.steps, args.warmup, world)
    clocks = clk.summary()
    # 3) end to end through the public path with host buffers
    t_e2e = time_loop(wl.e2e_step, args.steps, args.warmup, world)

    hbm, peak_src = peaks()
    kb = wl.kernel_bytes()
    achieved = kb / t_kernel / 1e9
    value = wl.step_bytes() / t_step / 1e12
    h2d, d2h = wl.e2e_bytes()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        bps, info = cpu_reference_time(wl.cpu_sample())
        cpu = {"value": bps / 1e12, "unit": "TB/s", "cores": info["cores"], "kind": info["kind"],
               "sample": info["sample"] + f"; median of {info['calls']} calls"}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_step * 1e3, "us_per_step": t_step * 1e6,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) q/k/v)", "config": wl.config(),
                "e2e": {"value": wl.step_bytes() / t_e2e / 1e12, "unit": "TB/s", "us_per_step": t_e2e * 1e6,
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "peak_source": peak_src,
                             "kernel": "gqa_decode_kernel<128,128,1,4>", "kernel_us": t_kernel * 1e6,
                             "algorithmic_bytes_per_launch": kb,
                             "traffic": profile_traffic(f"gqa_decode_{wl.name}")},
                "gpu_launches": wl.kernels_per_step * args.steps,
                "clocks": clocks, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
