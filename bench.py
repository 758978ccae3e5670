"""Decode-attention benchmark: µs/step and achieved HBM TB/s at 1/2/4/8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4]
    python bench.py --impl reference ...      # the reference's CPU kernel on this host

One JSON line on rank 0.  `value` is whole-job throughput in TB/s of
algorithmic bytes (KV read once + q + outputs, summed over ranks) divided by
the device-timed step (CUDA events, max over ranks), inputs resident in HBM
and larger than L2 (small workloads rotate over enough copies of their inputs
to exceed L2).  `e2e` is the same metric through the public API with the
step's host buffers copied in (H2D of q and of the new token's K/V) and the
result copied out (D2H of out + lse) inside the timed region.  The KV cache
itself is device-resident state, as the reference's InplaceKVCache is
host-resident state appended one token per step (system/qwenoffload.py:100-122).

Workloads (the default is the one the metric's
1/2/4/8-GPU scaling is quoted on):
  cfg1  GQA Qwen3 layer, B=1, L=4096
  cfg2  GQA Mixtral layer, B=16, ragged L in [1024, 32768], two shares merged by LSE
  cfg3  absorbed MLA, DeepSeek-V2-Lite: B=8, 16 heads, latent 512 + rope 64, S=16384
  cfg4  GQA Qwen3, B=32, L=131072 sequence-sharded over N GPUs (default)
  cfg5  CSA sparse decode, DeepSeek-V4 style: bs=16, 64 heads, 65536 int8
        entries, top-2048 gather, entry-sharded over N GPUs
  idx   the CSA indexer top-k that produces cfg5's ids (one GPU)
  mla_abs  cfg3 with the absorb and up-projection GEMMs either side (one GPU)
"""
from __future__ import annotations

import argparse
import json
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
L2_BYTES = 126 * 2 ** 20


# ----------------------------------------------------------------- helpers
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_roofline(wl, t_kernel):
    """For tensor-core workloads: the dominant kernel's FLOP rate against the
    measured dense bf16 peak (burst figure: the kernel is timed alone)."""
    if not hasattr(wl, "kernel_flops"):
        return None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        peak, src = 1590.0, "fallback"
    achieved = wl.kernel_flops() / t_kernel / 1e12
    return {"achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": src,
            "flops_per_launch": wl.kernel_flops()}


def profile_traffic(name, kernel_bytes):
    """dram read+write bytes per launch from an ncu capture of the N=1
    workload (profiles/<name>.txt: 'traffic_bytes_per_launch: T' and, when the
    capture's launch moved other algorithmic bytes than this one, e.g. one
    rank's 1/N shard, 'traffic_algorithmic_bytes: A'), scaled to this launch
    by its algorithmic bytes: T * kernel_bytes / A.  Returns (bytes, note)."""
    path = os.path.join(ROOT, "profiles", name + ".txt")
    t = a = None
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                t = float(line.split(":", 1)[1])
            elif line.startswith("traffic_algorithmic_bytes:"):
                a = float(line.split(":", 1)[1])
    except OSError:
        pass
    if t is None:
        return None, None
    if a is None or abs(a - kernel_bytes) <= 1e-6 * a:
        return t, f"profiles/{name}.txt"
    return t * kernel_bytes / a, (f"profiles/{name}.txt ({t:.0f} B for {a:.0f} algorithmic B), scaled to this "
                                  f"launch's {kernel_bytes} algorithmic B")


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
            time.sleep(0.3)
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
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


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


def bf16_randn(shape, gen, device):
    return torch.randn(*shape, device=device, dtype=torch.bfloat16, generator=gen)


def median_time(fn, budget_s, max_calls, warm=1):
    for _ in range(warm):
        fn()
    times = []
    t_start = time.perf_counter()
    while len(times) < max_calls and (time.perf_counter() - t_start) < budget_s:
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def load_cpu_ref(module="cpu_attn_ext"):
    """The reference's own extension from oracle/_ref on all host cores, or None."""
    import oracle
    if not oracle.ref_available():
        return None
    try:
        ref = oracle.load_ref(module)
    except Exception:
        return None
    n = os.cpu_count() or 1
    ref.set_num_threads(n)
    torch.set_num_threads(n)
    return ref


# --------------------------------------------------------------- workloads
class Workload:
    """Common harness: kernel(i) is the dominant launch on input copy i,
    step(i) the full decode step, e2e_step(i) the step through the public API
    with host buffers.  `copies` input sets rotate so that the bytes touched
    between two uses of one set exceed L2."""

    name = ""
    workload = ""
    copies = 1
    graph = False
    kernel_name = ""

    def kernel_bytes(self):
        raise NotImplementedError

    def step_bytes(self):
        return self.kernel_bytes()


class GqaDense(Workload):
    """Dense GQA decode through ws_gqa_decode over [B*Hkv, L, D] rows.

    cfg4 (default): Qwen3 shape, B=32, 32 q heads / 4 kv heads, D=128,
    L=131072, KV sharded contiguously over the ranks -- rank r holds tokens
    [r*L/N, (r+1)*L/N) of every (sequence, kv-head) row; partials are
    exchanged with NCCL all_gather and merged with ws_lse_merge.
    cfg1: the same layer shape at B=1, L=4096 on one GPU."""

    kernel_name = "gqa_decode_kernel<128,128,1,4>"

    def __init__(self, world, rank, name, B, H, Hkv, D, L, seed, exchange="peer"):
        from scope_b200 import _lib
        self.name = name
        self.exchange = exchange if world > 1 else "none"
        self.world, self.rank = world, rank
        self.B, self.H, self.Hkv, self.D, self.L = B, H, Hkv, D, L
        self.G = H // Hkv
        assert L % world == 0
        self.Lloc = L // world
        self.scale = D ** -0.5
        self.workload = (f"gqa_qwen3_b{B}_l{L}" + ("_sharded" if name == "cfg4" else ""))
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        rows = B * Hkv
        per_copy = 2 * rows * self.Lloc * D * 2
        self.copies = max(1, -(-3 * L2_BYTES // per_copy)) if per_copy < 3 * L2_BYTES else 1
        self.graph = per_copy < 64 * 2 ** 20
        g = torch.Generator(device=dev).manual_seed(seed + rank)
        self.k = [bf16_randn((rows, self.Lloc, D), g, dev) for _ in range(self.copies)]
        self.v = [bf16_randn((rows, self.Lloc, D), g, dev) for _ in range(self.copies)]
        gq = torch.Generator(device=dev).manual_seed(seed)
        # q, then the new token's K and V rows, in one device block that a public-API step fills from one
        # pinned host block with one copy; out, then lse, in one block read back with one copy
        self.nq, self.nkv = B * H * D, rows * D
        self.in_dev = torch.empty(self.nq + 2 * self.nkv, dtype=torch.bfloat16, device=dev)
        self.q = self.in_dev[:self.nq].view(B, H, D)
        self.q.copy_(bf16_randn((B, H, D), gq, dev))
        self.qv = self.q.view(rows, self.G, D)
        self.lib, self._lib = _lib.lib(), _lib
        ob, lb = B * H * D * 2, B * H * 4
        self.out_dev = torch.empty(ob + lb, dtype=torch.uint8, device=dev)
        out_v, lse_v = self.out_dev[:ob].view(torch.bfloat16), self.out_dev[ob:].view(torch.float32)
        if world == 1:
            self.out, self.lse = out_v.view(B, H, D), lse_v.view(B, H)
        else:
            from scope_b200.shard import PartialExchange, PeerExchange, ScatterExchange
            if self.exchange == "peer":
                self.ex = PeerExchange(B * H, D, world, rank, dev)
            elif self.exchange == "scatter":
                self.ex = ScatterExchange(B * H, D, world, rank, dev)
            else:
                self.ex = PartialExchange(B * H, D, world, dev)
                self.part_o, self.part_l = self.ex.part_o, self.ex.part_l
            self.out, self.lse = out_v.view(B * H, D), lse_v.view(B * H)
        nbytes = self.lib.ws_gqa_decode_workspace_size(rows, self.G, D, self.Lloc)
        self.ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)
        self.in_host = torch.randn(self.nq + 2 * self.nkv).bfloat16().pin_memory()
        self.out_host = torch.empty(ob + lb, dtype=torch.uint8).pin_memory()
        # the decode, its deferred merge when a row's tiles span more than eight CTAs (the rule in
        # gqa_decode.cu's host code), and with N > 1 the merge of the exchanged partials
        tpr = -(-self.Lloc // 64)
        total = rows * tpr
        nctas = min(torch.cuda.get_device_properties(dev).multi_processor_count, 156, max(total, 1))
        per_cta = -(-total // nctas)
        deferred = self.Lloc > 0 and -(-tpr // per_cta) + 1 > 8
        self.kernels_per_step = 1 + int(deferred) + int(world > 1)

    def kernel_bytes(self):
        rows = self.B * self.Hkv
        return (2 * rows * self.Lloc * self.D * 2 + self.B * self.H * self.D * 2
                + self.B * self.H * (self.D * (2 if self.world == 1 else 4) + 4))

    def step_bytes(self):
        return (2 * self.B * self.Hkv * self.L * self.D * 2 + self.B * self.H * self.D * 2
                + self.B * self.H * (self.D * 2 + 4))

    def kernel(self, i):
        L_, c = self.lib, i % self.copies
        k, v = self.k[c], self.v[c]
        st = self._lib.stream_ptr(self.dev)
        rows = self.B * self.Hkv
        if self.world == 1:
            out, lse, mode = self.out.data_ptr(), self.lse.data_ptr(), self._lib.WS_OUT_NORM_BF16
        elif self.exchange in ("peer", "scatter"):   # rank 0's own slot, or a local block the exchange copies
            (out, lse), mode = self.ex.slot(), self._lib.WS_OUT_NORM_F32
        else:
            out, lse, mode = self.part_o.data_ptr(), self.part_l.data_ptr(), self._lib.WS_OUT_NORM_F32
        rc = L_.ws_gqa_decode(self.qv.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                              v.stride(0), v.stride(1), rows, self.G, self.D, self.D, self.Lloc, self.scale,
                              self._lib.WS_DTYPE_BF16, mode, out, None, None, lse,
                              self.ws.data_ptr(), self.ws.numel(), st)
        if rc != 0:
            raise RuntimeError(L_.ws_last_error().decode())

    def exchange_step(self, i):
        """The exchange of one step alone (N > 1): the partials already sit in their blocks."""
        if self.exchange in ("peer", "scatter"):
            self.ex.step(out=self.out if self.rank == 0 else None, out_lse=self.lse if self.rank == 0 else None)
        elif self.world > 1:
            self.ex.step(torch.bfloat16, out=self.out, out_lse=self.lse)

    def step(self, i):
        self.kernel(i)
        self.exchange_step(i)

    def close(self):
        if self.exchange in ("peer", "scatter"):
            self.ex.close()

    def e2e_step(self, i):
        """Through the public API with host buffers: q (and, on the rank holding the last shard, the new
        token's K and V rows) arrive in one copy from pinned memory, the token is appended to the cache
        with ws_kv_append, the decode (and exchange) runs, and out + lse leave in one copy."""
        c = i % self.copies
        last = self.rank == self.world - 1   # the new token lands in the last shard
        n = self.nq + 2 * self.nkv if last else self.nq
        self.in_dev[:n].copy_(self.in_host[:n], non_blocking=True)
        if last:
            st = self._lib.stream_ptr(self.dev)
            rows = self.B * self.Hkv
            for cache, off in ((self.k[c], self.nq), (self.v[c], self.nq + self.nkv)):
                rc = self.lib.ws_kv_append(cache.data_ptr(), cache.stride(0), cache.stride(1), self.Lloc,
                                           self.in_dev[off:].data_ptr(), self.D, self.D, rows, 1, self.D,
                                           self._lib.WS_DTYPE_BF16, self.Lloc - 1, st)
                if rc != 0:
                    raise RuntimeError(self.lib.ws_last_error().decode())
        self.step(i)
        if self.rank == 0:
            self.out_host.copy_(self.out_dev, non_blocking=True)

    def e2e_bytes(self):
        return ((self.world * self.nq + 2 * self.nkv) * 2, self.out_dev.numel())

    def parity_check(self, seed):
        """N > 1, before timing: one step on input copy 0, then rank 0 rebuilds
        whole rows from every rank's shard (each shard is drawn from the
        generator seeded seed + rank, so rank 0 can draw any of them again)
        and compares the merged output of those rows with a single-GPU
        ws_gqa_decode over the whole row.  Every rank takes the same
        collective steps; only rank 0 computes the check."""
        if self.world == 1:
            return None
        self.step(0)
        torch.cuda.synchronize()
        res = None
        if self.rank == 0:
            dev = self.q.device
            rows = self.B * self.Hkv
            sel = torch.tensor([0, rows // 2 + 1, rows - 1], device=dev)
            ks, vs = [], []
            for r in range(self.world):
                g = torch.Generator(device=dev).manual_seed(seed + r)
                kr = [bf16_randn((rows, self.Lloc, self.D), g, dev) for _ in range(self.copies)][0][sel]
                vr = [bf16_randn((rows, self.Lloc, self.D), g, dev) for _ in range(self.copies)][0][sel]
                ks.append(kr)
                vs.append(vr)
            kf, vf = torch.cat(ks, dim=1).contiguous(), torch.cat(vs, dim=1).contiguous()
            del ks, vs
            n = sel.numel()
            q = self.qv[sel].contiguous()
            out = torch.empty(n, self.G, self.D, dtype=torch.bfloat16, device=dev)
            lse = torch.empty(n, self.G, dtype=torch.float32, device=dev)
            ws = torch.zeros(self.lib.ws_gqa_decode_workspace_size(n, self.G, self.D, self.L), dtype=torch.uint8,
                             device=dev)
            rc = self.lib.ws_gqa_decode(q.data_ptr(), kf.data_ptr(), vf.data_ptr(), kf.stride(0), kf.stride(1),
                                        vf.stride(0), vf.stride(1), n, self.G, self.D, self.D, self.L, self.scale,
                                        self._lib.WS_DTYPE_BF16, self._lib.WS_OUT_NORM_BF16, out.data_ptr(), None,
                                        None, lse.data_ptr(), ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream().cuda_stream)
            if rc != 0:
                raise RuntimeError(self.lib.ws_last_error().decode())
            heads = (sel[:, None] * self.G + torch.arange(self.G, device=dev)[None, :]).reshape(-1)
            got_o = self.out.view(-1, self.D)[heads].float()
            got_l = self.lse.view(-1)[heads]
            res = {"rows_checked": int(heads.numel()),
                   "max_abs_out": float((got_o - out.view(-1, self.D).float()).abs().max()),
                   "max_abs_lse": float((got_l - lse.view(-1)).abs().max()),
                   "against": "one-GPU ws_gqa_decode over the whole row, rebuilt from every rank's shard"}
            del kf, vf, ws
            torch.cuda.empty_cache()
        barrier(self.world)
        return res

    def config(self):
        return {"workload": self.workload, "batch": self.B, "q_heads": self.H, "kv_heads": self.Hkv,
                "head_dim": self.D, "kv_len": self.L, "kv_len_per_gpu": self.Lloc,
                "parallelism": f"seq-shard{self.world}",
                "l2": (f"inputs {2 * self.B * self.Hkv * self.Lloc * self.D * 2 / 1e9:.2f} GB per GPU > L2"
                       if self.copies == 1 else f"{self.copies} rotating input copies > 3x L2"),
                "timing": "cuda-graph replay" if self.graph else "stream launches",
                "exchange": {"peer": "partials pushed into rank 0's IPC-mapped slots over NVLink (one launch per rank), "
                                     "rank 0's merge kernel after a bounded acquire wait on the ranks' flags",
                             "scatter": "each rank merges its share of the rows from its peers' copies (IPC-mapped "
                                        "buffers over NVLink) and stores the merged share in rank 0's gather area",
                             "nccl": "nccl all_gather of (o fp32, lse) + lse_merge kernel on every rank",
                             "none": "none"}[self.exchange]}

    def cpu_reference(self, budget_s, max_calls, warm=1):
        return cpu_ref_dense(self.B, self.Hkv, self.G, self.D, self.L, budget_s, max_calls, warm)


class GqaShares(Workload):
    """cfg2: Mixtral layer shape, B=16, 32 q heads / 8 kv heads (G=4), D=128,
    ragged per-sequence KV lengths ~ U[1024, 32768] (seed 2), each sequence's
    KV split at r in {0.25, 0.5, 0.75} into two physical shares (share 0 =
    tokens [0, floor(r*L)), share 1 = the rest), one launch of
    ws_gqa_decode_shares decodes both and merges them by LSE."""

    name = "cfg2"
    kernel_name = "gqa_decode_kernel<128,128,1,4> (2 shares)"

    def __init__(self, world, rank, B=16, H=32, Hkv=8, D=128, seed=2):
        import scope_b200
        self.world, self.rank = world, rank
        self.B, self.H, self.Hkv, self.D = B, H, Hkv, D
        self.G = H // Hkv
        self.scale = D ** -0.5
        self.lens, self.ratio, self.L0, self.L1 = cfg2_geometry(B, seed)
        self.workload = f"gqa_mixtral_b{B}_ragged_1024_32768_two_shares"
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(seed)
        self.q = bf16_randn((B, H, D), g, dev)
        self.total_tokens = int(self.lens.sum())
        # each share is the reference's cache layout: [B*Hkv, capacity, D] rows per
        # (sequence, kv-head), valid tokens [0, len) (system/qwenoffload.py:59-141)
        cap0, cap1 = int(self.L0.max()), int(self.L1.max())
        self.k0, self.v0 = bf16_randn((B * Hkv, cap0, D), g, dev), bf16_randn((B * Hkv, cap0, D), g, dev)
        self.k1, self.v1 = bf16_randn((B * Hkv, cap1, D), g, dev), bf16_randn((B * Hkv, cap1, D), g, dev)
        n0 = torch.tensor(self.L0, dtype=torch.int32, device=dev)
        n1 = torch.tensor(self.L1, dtype=torch.int32, device=dev)
        self.shares = [scope_b200.Share(self.k0, self.v0, seqlens=n0), scope_b200.Share(self.k1, self.v1, seqlens=n1)]
        self.out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty(B, H, dtype=torch.float32, device=dev)
        self.q_host = torch.randn(B, H, D).bfloat16().pin_memory()
        self.out_host = torch.empty(B, H, D, dtype=torch.bfloat16).pin_memory()
        self.lse_host = torch.empty(B, H, dtype=torch.float32).pin_memory()
        self.copies = 1
        self.graph = True
        self.kernels_per_step = 2   # the decode and the deferred merge of the ragged groups' pieces
        self._decode = scope_b200.gqa_decode_shares

    def kernel_bytes(self):
        return 2 * self.total_tokens * self.Hkv * self.D * 2 + self.B * self.H * (self.D * 2 * 2 + 4)

    def kernel(self, i):
        self._decode(self.q, self.shares, self.scale, out=self.out, lse=self.lse)

    step = kernel

    def e2e_step(self, i):
        self.q.copy_(self.q_host, non_blocking=True)
        self._decode(self.q, self.shares, self.scale, out=self.out, lse=self.lse)
        self.out_host.copy_(self.out, non_blocking=True)
        self.lse_host.copy_(self.lse, non_blocking=True)

    def e2e_bytes(self):
        return self.q.numel() * 2, self.out.numel() * 2 + self.lse.numel() * 4

    def config(self):
        return {"workload": self.workload, "batch": self.B, "q_heads": self.H, "kv_heads": self.Hkv,
                "head_dim": self.D, "kv_len_sum": int(self.lens.sum()), "kv_len_min": int(self.lens.min()),
                "kv_len_max": int(self.lens.max()), "share_ratios": [float(r) for r in self.ratio],
                "layout": "two padded shares [B*Hkv, cap, D] per sequence split",
                "parallelism": "single-gpu", "l2": f"inputs {self.kernel_bytes() / 1e9:.2f} GB > L2",
                "timing": "cuda-graph replay"}

    def cpu_reference(self, budget_s, max_calls, warm=1):
        return cpu_ref_shares(self.B, self.H, self.Hkv, self.D, budget_s, max_calls, warm)


class Mla(Workload):
    """cfg3: absorbed MLA, DeepSeek-V2-Lite shape: B=8, 16 heads sharing one
    latent KV of 512 + 64 rope dims, S=16384, scale 1/sqrt(192); output
    [8*16, 512] bf16 normalised + fp32 LSE (ws_mla_decode: the tcgen05 split-KV
    kernel and its merge kernel)."""

    name = "cfg3"
    kernel_name = "mla_decode_kernel (tcgen05) + mla_merge_kernel"
    profile_name = "mla_decode_cfg3"

    def __init__(self, world, rank, B=8, nH=16, S=16384, seed=3):
        from scope_b200 import cpu_attn
        self.world, self.rank = world, rank
        self.B, self.nH, self.S = B, nH, S
        self.scale = 192 ** -0.5
        self.workload = f"mla_absorbed_ds2lite_b{B}_h{nH}_s{S}"
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed)
        per_copy = B * S * (512 + 64) * 2
        self.copies = max(1, -(-3 * L2_BYTES // per_copy))
        self.graph = True
        self.c = [bf16_randn((B, S, 512), g, dev) for _ in range(self.copies)]
        self.p = [bf16_randn((B, S, 64), g, dev) for _ in range(self.copies)]
        self.qp = bf16_randn((B * nH, 512), g, dev)
        self.qpe = bf16_randn((B * nH, 64), g, dev)
        self._decode = cpu_attn.mla_decode
        self.qp_host = torch.randn(B * nH, 512).bfloat16().pin_memory()
        self.qpe_host = torch.randn(B * nH, 64).bfloat16().pin_memory()
        self.cnew_host = torch.randn(B, 512).bfloat16().pin_memory()
        self.pnew_host = torch.randn(B, 64).bfloat16().pin_memory()
        self.out_host = torch.empty(B * nH, 512, dtype=torch.bfloat16).pin_memory()
        self.lse_host = torch.empty(B * nH, dtype=torch.float32).pin_memory()
        self.kernels_per_step = 2

    def kernel_bytes(self):
        return self.B * self.S * (512 + 64) * 2 + self.B * self.nH * (576 * 2 + 512 * 2 + 4)

    def kernel(self, i):
        c = i % self.copies
        self.out, self.lse = self._decode(self.qp, self.qpe, self.c[c], self.p[c], self.scale)

    step = kernel

    def e2e_step(self, i):
        c = i % self.copies
        self.qp.copy_(self.qp_host, non_blocking=True)
        self.qpe.copy_(self.qpe_host, non_blocking=True)
        self.c[c][:, self.S - 1].copy_(self.cnew_host, non_blocking=True)   # the new token's latent
        self.p[c][:, self.S - 1].copy_(self.pnew_host, non_blocking=True)
        out, lse = self._decode(self.qp, self.qpe, self.c[c], self.p[c], self.scale)
        self.out_host.copy_(out, non_blocking=True)
        self.lse_host.copy_(lse, non_blocking=True)

    def e2e_bytes(self):
        return ((self.qp_host.numel() + self.qpe_host.numel() + self.cnew_host.numel() + self.pnew_host.numel()) * 2,
                self.out_host.numel() * 2 + self.lse_host.numel() * 4)

    def config(self):
        return {"workload": self.workload, "batch": self.B, "heads": self.nH, "kv_lora_rank": 512, "rope_dims": 64,
                "kv_len": self.S, "parallelism": "single-gpu",
                "l2": f"{self.copies} rotating input copies > 3x L2", "timing": "cuda-graph replay"}

    def cpu_reference(self, budget_s, max_calls, warm=1):
        return cpu_ref_mla(self.B, self.nH, self.S, budget_s, max_calls, warm)


class MlaAbsorbed(Mla):
    """mla_abs: cfg3's absorbed-MLA step with the projections either side
    (ws_mla_decode_absorbed: q_nope . W_UK, the tcgen05 decode, and the merge
    fused with the up-projection o . W_UV^T), DeepSeek-V2-Lite shapes: nop = 128,
    vhd = 128, random-init kv_b_proj weight; output [8, 16, 128] bf16.  The
    reference runs this step as torch.bmm + fused_cpu_attn_mla_compressed + bmm
    (system/deepseek.py:257-265, :355-407)."""

    name = "mla_abs"
    kernel_name = "mla_absorb_kernel + mla_decode_kernel (tcgen05) + mla_merge_up_kernel"
    profile_name = "mla_decode_cfg3"

    def __init__(self, world, rank, B=8, nH=16, S=16384, seed=3):
        super().__init__(world, rank, B=B, nH=nH, S=S, seed=seed)
        from scope_b200 import cpu_attn
        self.workload = f"mla_absorbed_step_ds2lite_b{B}_h{nH}_s{S}_nop128_vhd128"
        dev = self.qp.device
        g = torch.Generator(device=dev).manual_seed(seed + 100)
        self.nop = self.vhd = 128
        self.q_nope = bf16_randn((B, nH, self.nop), g, dev)
        self.w = (torch.randn(nH * (self.nop + self.vhd), 512, generator=g, device=dev) * 0.05).bfloat16()
        self._absorbed = cpu_attn.mla_decode_absorbed
        self.qn_host = torch.randn(B, nH, self.nop).bfloat16().pin_memory()
        self.outv_host = torch.empty(B, nH, self.vhd, dtype=torch.bfloat16).pin_memory()
        self.kernels_per_step = 4   # absorb, decode, merge, up-projection

    def kernel_bytes(self):
        return (self.B * self.S * (512 + 64) * 2 + self.B * self.nH * (self.nop + 64 + self.vhd) * 2
                + 2 * self.nH * 128 * 512 * 2 + self.B * self.nH * 4)

    def kernel(self, i):
        c = i % self.copies
        self.out = self._absorbed(self.q_nope, self.qpe, self.c[c], self.p[c], self.w, self.scale)

    step = kernel

    def e2e_step(self, i):
        c = i % self.copies
        self.q_nope.copy_(self.qn_host, non_blocking=True)
        self.qpe.copy_(self.qpe_host, non_blocking=True)
        self.c[c][:, self.S - 1].copy_(self.cnew_host, non_blocking=True)
        self.p[c][:, self.S - 1].copy_(self.pnew_host, non_blocking=True)
        out = self._absorbed(self.q_nope, self.qpe, self.c[c], self.p[c], self.w, self.scale)
        self.outv_host.copy_(out, non_blocking=True)

    def e2e_bytes(self):
        return ((self.qn_host.numel() + self.qpe_host.numel() + self.cnew_host.numel() + self.pnew_host.numel()) * 2,
                self.outv_host.numel() * 2)

    def config(self):
        d = super().config()
        d.update({"workload": self.workload, "qk_nope_head_dim": self.nop, "v_head_dim": self.vhd,
                  "weights": "random-init kv_b_proj (N(0,1) x 0.05)"})
        return d


class Csa(Workload):
    """cfg5: CSA sparse decode (DeepSeek-V4 style), bs=16, 64 heads over a
    512-wide latent, nc=65536 int8 entries with one fp32 scale each, top-2048
    sorted unique ids per sequence, bf16 q, scale 1/sqrt(512); out bf16
    normalised + fp32 LSE (ws_csa_decode).  With N GPUs rank r holds entries
    [r*nc/N, (r+1)*nc/N) of every sequence, attends to the ids that fall in
    its shard (rebased locally), and the fp32 partials are exchanged with NCCL
    all_gather and merged with ws_lse_merge.

    Inputs larger than L2: steps rotate over 32 top-k id sets and 32 query
    copies, and over enough copies of this rank's KV shard to exceed 3x L2,
    so the rows one step reads were last read many steps (and > L2 bytes) ago."""

    name = "cfg5"
    kernel_name = "csa_decode_kernel<int8,bf16 q> (tcgen05, 9 CTAs per sequence) + lse_merge_vec_kernel"
    profile_name = "csa_decode_cfg5"
    graph = True

    def __init__(self, world, rank, bs=16, nH=64, nc=65536, k=2048, seed=5, exchange="peer"):
        from scope_b200 import _lib
        self.world, self.rank = world, rank
        self.exchange = exchange if world > 1 else "none"
        self.bs, self.nH, self.nc, self.k = bs, nH, nc, k
        self.scale = 512 ** -0.5
        self.workload = f"csa_ds4_b{bs}_h{nH}_nc{nc}_top{k}_int8"
        dev = torch.device("cuda", torch.cuda.current_device())
        from scope_b200.shard import shard_bounds
        self.lo, self.hi = shard_bounds(nc, world, rank)
        ncl = self.hi - self.lo
        shard_bytes = bs * ncl * (512 + 4)
        self.n_kv = max(1, -(-3 * L2_BYTES // shard_bytes))
        self.n_sets = 32
        self.copies = self.n_sets
        g = torch.Generator(device=dev).manual_seed(seed + 17 * rank)
        self.kv, self.kv_scales = [], []
        for _ in range(self.n_kv):
            kv = torch.empty(bs, ncl, 512, dtype=torch.int8, device=dev)
            for b in range(bs):   # round(N(0,1) * 32) clipped to +-127, per sequence to bound the temporary
                kv[b] = (torch.randn(ncl, 512, generator=g, device=dev) * 32).round_().clamp_(-127, 127)
            self.kv.append(kv)
            self.kv_scales.append(torch.rand(bs, ncl, generator=g, device=dev) * 0.04 + 0.01)
        gi = torch.Generator().manual_seed(seed)
        self.idx = [torch.stack([torch.randperm(nc, generator=gi)[:k].sort().values for _ in range(bs)]).int().to(dev)
                    for _ in range(self.n_sets)]
        self.n_local = [int(((t >= self.lo) & (t < self.hi)).sum()) for t in self.idx]
        # shard load balance: selected entries per rank (all ranks' shards, from the same id sets), as
        # max / mean over ranks, averaged over the sets; the per-sequence worst case alongside
        bounds = [shard_bounds(nc, world, r) for r in range(world)]
        whole, per_seq = [], []
        for t in self.idx:
            cnt = torch.stack([((t >= lo_r) & (t < hi_r)).sum(dim=1) for lo_r, hi_r in bounds]).float()  # [world, bs]
            tot = cnt.sum(dim=1)
            whole.append(float(tot.max() / tot.mean()))
            per_seq.append(float((cnt.max(dim=0).values / cnt.mean(dim=0).clamp(min=1e-9)).max()))
        self.shard_load = (sum(whole) / len(whole), max(per_seq))
        gq = torch.Generator(device=dev).manual_seed(seed + 1)
        self.q = [torch.randn(bs, nH, 512, generator=gq, device=dev).bfloat16() for _ in range(self.n_sets)]
        self.lib, self._lib = _lib.lib(), _lib
        if world == 1:
            self.out = torch.empty(bs, nH, 512, dtype=torch.bfloat16, device=dev)
            self.lse = torch.empty(bs, nH, dtype=torch.float32, device=dev)
        else:
            from scope_b200.shard import PartialExchange, PeerExchange, ScatterExchange
            if self.exchange == "peer":
                self.ex = PeerExchange(bs * nH, 512, world, rank, dev)
            elif self.exchange == "scatter":
                self.ex = ScatterExchange(bs * nH, 512, world, rank, dev)
            else:
                self.ex = PartialExchange(bs * nH, 512, world, dev)
                self.part_o, self.part_l = self.ex.part_o, self.ex.part_l
            self.out = torch.empty(bs * nH, 512, dtype=torch.bfloat16, device=dev)
            self.lse = torch.empty(bs * nH, dtype=torch.float32, device=dev)
        self.ws = torch.zeros(self.lib.ws_csa_decode_workspace_size(bs, nH, self._lib.WS_DTYPE_BF16),
                              dtype=torch.uint8, device=dev)
        self.q_host = torch.randn(bs, nH, 512).bfloat16().pin_memory()
        self.idx_host = self.idx[0].cpu().pin_memory()
        self.out_host = torch.empty(bs * nH * 512, dtype=torch.bfloat16).pin_memory()
        self.lse_host = torch.empty(bs * nH, dtype=torch.float32).pin_memory()
        # the decode and the merge of its split partials (9 CTAs per sequence here), and with N > 1 the
        # merge of the exchanged partials
        self.kernels_per_step = 2 + int(world > 1)

    def parity_check(self, seed):
        """N > 1, before timing: one step on id set 0 and KV copy 0, then rank 0
        rebuilds the whole entry buffer from every rank's shard (drawn again
        from the generator seeded seed + 17 * rank) and compares the merged
        output with a single-GPU ws_csa_decode over it.  Every rank takes the
        same collective steps; only rank 0 computes the check."""
        if self.world == 1:
            return None
        from scope_b200.shard import shard_bounds
        self.step(0)
        torch.cuda.synchronize()
        res = None
        if self.rank == 0:
            dev = self.q[0].device
            kvs, scs = [], []
            for r in range(self.world):
                lo, hi = shard_bounds(self.nc, self.world, r)
                g = torch.Generator(device=dev).manual_seed(seed + 17 * r)
                kv = torch.empty(self.bs, hi - lo, 512, dtype=torch.int8, device=dev)
                for b in range(self.bs):
                    kv[b] = (torch.randn(hi - lo, 512, generator=g, device=dev) * 32).round_().clamp_(-127, 127)
                kvs.append(kv)
                scs.append(torch.rand(self.bs, hi - lo, generator=g, device=dev) * 0.04 + 0.01)
            kvf, scf = torch.cat(kvs, dim=1).contiguous(), torch.cat(scs, dim=1).contiguous()
            del kvs, scs
            out = torch.empty(self.bs * self.nH, 512, dtype=torch.bfloat16, device=dev)
            lse = torch.empty(self.bs * self.nH, dtype=torch.float32, device=dev)
            ws = torch.zeros(self.lib.ws_csa_decode_workspace_size(self.bs, self.nH, self._lib.WS_DTYPE_BF16),
                             dtype=torch.uint8, device=dev)
            rc = self.lib.ws_csa_decode(self.q[0].data_ptr(), self._lib.WS_DTYPE_BF16, self.bs, self.nH, 512,
                                        kvf.data_ptr(), self._lib.WS_DTYPE_I8, scf.data_ptr(), self.nc, 0,
                                        self.idx[0].data_ptr(), self.k, self._lib.WS_CSA_IDX_ALL, 0, 0, self.scale,
                                        out.data_ptr(), self._lib.WS_DTYPE_BF16, lse.data_ptr(), ws.data_ptr(),
                                        ws.numel(), torch.cuda.current_stream().cuda_stream)
            if rc != 0:
                raise RuntimeError(self.lib.ws_last_error().decode())
            res = {"rows_checked": self.bs * self.nH,
                   "max_abs_out": float((self.out.float() - out.float()).abs().max()),
                   "max_abs_lse": float((self.lse - lse).abs().max()),
                   "against": "one-GPU ws_csa_decode over the whole entry buffer, rebuilt from every rank's shard"}
            del kvf, scf, ws
            torch.cuda.empty_cache()
        barrier(self.world)
        return res

    def kernel_bytes(self):
        """Per launch on this rank, averaged over the rotating id sets."""
        out_b = 2 * 512 if self.world == 1 else 4 * 512
        n_local = sum(self.n_local) / len(self.n_local)
        return n_local * (512 + 4 + 4) + self.bs * self.nH * (512 * 2 + out_b + 4)

    def step_bytes(self):
        return self.bs * self.k * (512 + 4 + 4) + self.bs * self.nH * (512 * 2 + 512 * 2 + 4)

    def kernel_flops(self):
        n_local = sum(self.n_local) / len(self.n_local)
        return 2 * 2 * n_local * self.nH * 512

    def kernel(self, i):
        L_ = self.lib
        st = torch.cuda.current_stream().cuda_stream
        c, kvc = i % self.n_sets, i % self.n_kv
        if self.world == 1:
            out, lse = self.out.data_ptr(), self.lse.data_ptr()
            odt, mode, lo = self._lib.WS_DTYPE_BF16, self._lib.WS_CSA_IDX_ALL, 0
        else:
            out, lse = (self.ex.slot() if self.exchange in ("peer", "scatter")
                        else (self.part_o.data_ptr(), self.part_l.data_ptr()))
            odt, mode, lo = self._lib.WS_DTYPE_F32, self._lib.WS_CSA_IDX_SORTED_SHARD, self.lo
        kv = self.kv[kvc]
        rc = L_.ws_csa_decode(self.q[c].data_ptr(), self._lib.WS_DTYPE_BF16, self.bs, self.nH, 512, kv.data_ptr(),
                              self._lib.WS_DTYPE_I8, self.kv_scales[kvc].data_ptr(), kv.shape[1], lo,
                              self.idx[c].data_ptr(), self.k, mode, 0, 0, self.scale, out, odt,
                              lse, self.ws.data_ptr(), self.ws.numel(), st)
        if rc != 0:
            raise RuntimeError(L_.ws_last_error().decode())

    def exchange_step(self, i):
        """The exchange of one step alone (N > 1): the partials already sit in their blocks."""
        if self.exchange in ("peer", "scatter"):
            self.ex.step(out=self.out if self.rank == 0 else None, out_lse=self.lse if self.rank == 0 else None)
        elif self.world > 1:
            self.ex.step(torch.bfloat16, out=self.out, out_lse=self.lse)

    def step(self, i):
        self.kernel(i)
        self.exchange_step(i)

    def close(self):
        if self.exchange in ("peer", "scatter"):
            self.ex.close()

    def e2e_step(self, i):
        """Through the public API: q and the step's top-k ids come from host
        memory, out and lse go back to it."""
        from scope_b200 import csa_attn
        c, kvc = i % self.n_sets, i % self.n_kv
        q, idx = self.q[c], self.idx[c]
        q.copy_(self.q_host, non_blocking=True)
        idx.copy_(self.idx_host, non_blocking=True)
        if self.world == 1:
            out, lse = csa_attn.csa_sparse_decode(q, self.kv[kvc], idx, self.scale, self.kv_scales[kvc])
        elif self.exchange in ("peer", "scatter"):   # the C-ABI decode into the exchange slot, then the exchange
            self.step(i)
            out, lse = self.out, self.lse
        else:
            po, pl = csa_attn.csa_sparse_decode(q, self.kv[kvc], idx, self.scale, self.kv_scales[kvc],
                                                shard_lo=self.lo, idx_mode="sorted_shard", out_dtype=torch.float32)
            self.ex.part_o.copy_(po.view(-1, 512))
            self.ex.part_l.copy_(pl.view(-1))
            out, lse = self.ex.step(torch.bfloat16)
        if self.rank == 0:
            self.out_host.copy_(out.view(-1), non_blocking=True)
            self.lse_host.copy_(lse.view(-1), non_blocking=True)

    def e2e_bytes(self):
        return (self.world * (self.q_host.numel() * 2 + self.idx_host.numel() * 4),
                self.out_host.numel() * 2 + self.lse_host.numel() * 4)

    def config(self):
        return {"workload": self.workload, "batch": self.bs, "heads": self.nH, "kv_lora_rank": 512,
                "n_compressed": self.nc, "topk": self.k, "kv_dtype": "int8 + fp32 scale per entry",
                "entries_per_gpu": self.hi - self.lo,
                "selected_entries_this_rank": sum(self.n_local) / len(self.n_local),
                "shard_load_max_over_mean": round(self.shard_load[0], 4),
                "shard_load_max_over_mean_worst_sequence": round(self.shard_load[1], 4),
                "parallelism": f"entry-shard{self.world}",
                "l2": (f"{self.n_sets} rotating top-k sets and q copies, {self.n_kv} KV shard copies "
                       f"({self.n_kv * self.kv[0].numel() / 2 ** 20:.0f} MiB) > 3x L2"),
                "timing": "cuda-graph replay",
                "exchange": {"peer": "partials pushed into rank 0's IPC-mapped slots over NVLink (one launch per rank), "
                                     "rank 0's merge kernel after a bounded acquire wait on the ranks' flags",
                             "scatter": "each rank merges its share of the rows from its peers' copies (IPC-mapped "
                                        "buffers over NVLink) and stores the merged share in rank 0's gather area",
                             "nccl": "nccl all_gather of (o fp32, lse) + lse_merge kernel",
                             "none": "none"}[self.exchange]}

    def cpu_reference(self, budget_s, max_calls, warm=1):
        return cpu_ref_csa(self.bs, self.nH, self.nc, self.k, budget_s, max_calls, warm)


class Indexer(Workload):
    """idx: the CSA indexer top-k that produces cfg5's ids (the step before the CSA decode):
    bs=16 sequences, 64 index heads x 128 dims over nc=65536 compressed entries,
    bf16 q/kv (the dtype the DeepSeek-V4 runtime passes, system/ds4offload.py:95-125),
    fp32 weights, top-2048 by descending score (ws_indexer_topk: scoring kernel +
    select kernel).  Inputs larger than L2 (256 MiB of kv)."""

    name = "idx"
    kernel_name = "indexer_score_tc_kernel<bf16> (tcgen05) + indexer_select_kernel"
    profile_name = "indexer_topk_idx"
    graph = True

    def __init__(self, world, rank, bs=16, nH=64, hd=128, nc=65536, k=2048, seed=6):
        from scope_b200 import _lib
        self.world, self.rank = world, rank
        self.bs, self.nH, self.hd, self.nc, self.k = bs, nH, hd, nc, k
        self.workload = f"indexer_ds4_b{bs}_h{nH}_d{hd}_nc{nc}_top{k}_bf16"
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed)
        self.copies = max(1, -(-3 * L2_BYTES // (bs * nc * hd * 2)))
        self.kv = [bf16_randn((bs, nc, hd), g, dev) for _ in range(self.copies)]
        self.q = bf16_randn((bs, nH, hd), g, dev)
        self.w = torch.rand(bs, nH, generator=g, device=dev)
        self.ids = torch.empty(bs, k, dtype=torch.int32, device=dev)
        self.lib, self._lib = _lib.lib(), _lib
        self.ws = torch.zeros(self.lib.ws_indexer_topk_workspace_size(bs, nc), dtype=torch.uint8, device=dev)
        self.q_host = torch.randn(bs, nH, hd).bfloat16().pin_memory()
        self.ids_host = torch.empty(bs, k, dtype=torch.int32).pin_memory()
        self.kernels_per_step = 2

    def kernel_bytes(self):
        return self.bs * self.nc * self.hd * 2 + self.bs * self.nH * (self.hd * 2 + 4) + self.bs * self.k * 4

    def kernel_flops(self):
        return 2 * self.bs * self.nc * self.nH * self.hd

    def kernel(self, i):
        kv = self.kv[i % self.copies]
        rc = self.lib.ws_indexer_topk(self.q.data_ptr(), kv.data_ptr(), self._lib.WS_DTYPE_BF16, self.w.data_ptr(),
                                      self.bs, self.nH, self.hd, self.nc, self.k, self._lib.WS_TOPK_BY_SCORE,
                                      self.ids.data_ptr(), None, self.ws.data_ptr(), self.ws.numel(),
                                      torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(self.lib.ws_last_error().decode())

    step = kernel

    def e2e_step(self, i):
        from scope_b200 import csa_attn
        self.q.copy_(self.q_host, non_blocking=True)
        ids = csa_attn.indexer_topk(self.q, self.kv[i % self.copies], self.w, self.k)
        self.ids_host.copy_(ids, non_blocking=True)

    def e2e_bytes(self):
        return self.q_host.numel() * 2, self.ids_host.numel() * 4

    def config(self):
        return {"workload": self.workload, "batch": self.bs, "index_heads": self.nH, "head_dim": self.hd,
                "n_compressed": self.nc, "topk": self.k, "dtype_in": "bf16 q/kv, fp32 weights, fp32 math",
                "parallelism": "single-gpu", "l2": f"{self.copies} rotating kv copies > 3x L2",
                "timing": "cuda-graph replay"}

    def cpu_reference(self, budget_s, max_calls, warm=1):
        return cpu_ref_indexer(self.bs, self.nH, self.hd, self.nc, self.k, budget_s, max_calls, warm)


# ------------------------------------------------- reference CPU measurements
def cfg2_geometry(B=16, seed=2):
    """Seeded ragged lengths ~ U[1024, 32768] and share ratios in {.25, .5, .75}."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(1024, 32768, size=B, endpoint=True)
    ratio = rng.choice([0.25, 0.5, 0.75], size=B)
    L0 = np.floor(ratio * lens).astype(np.int64)
    return lens, ratio, L0, lens - L0


def randn_bf16_host(shape, seed):
    """A host bf16 tensor of N(0,1) values, filled one leading-dim slice per
    task on all host cores (each slice from its own seeded generator), so the
    8.6 GB of cfg4's KV are drawn in seconds."""
    import concurrent.futures as cf
    x = torch.empty(*shape, dtype=torch.bfloat16)

    def fill(i):
        x[i].normal_(generator=torch.Generator().manual_seed(seed * 100003 + i))
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        list(ex.map(fill, range(shape[0])))
    return x


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_ref_dense(B, Hkv, G, D, L, budget_s, max_calls, warm=1):
    """The reference's fused_cpu_attn on all host cores over the whole
    workload: B*Hkv rows of L tokens (cfg4: 128 rows x 131072 tokens, 8.6 GB
    of host KV, one call per step).  Returns (bytes/s, info)."""
    import oracle
    rows = B * Hkv
    torch.manual_seed(11)
    q = torch.randn(rows, G, D).bfloat16()
    k = randn_bf16_host((rows, L, D), 12)
    v = randn_bf16_host((rows, L, D), 13)
    nbytes = 2 * rows * L * D * 2 + rows * G * D * 2 + rows * G * (D * 2 + 4)
    ref = load_cpu_ref()
    if ref is not None:
        kind, fn = "reference", (lambda: ref.fused_cpu_attn(q, k, v, D ** -0.5))
    else:
        qb, kb, vb = oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v)
        kind, fn = "port", (lambda: oracle.gqa_decode(qb, kb, vb, D ** -0.5))
    t, n = median_time(fn, budget_s, max_calls, warm)
    return nbytes / t, {"kind": kind, "cores": os.cpu_count() or 1, "calls": n, "sec_per_call": t,
                        "cpu_model": cpu_model(),
                        "sample": f"fused_cpu_attn bf16, B_kv={rows}, G={G}, D={D}, L={L}: the whole workload "
                                  f"per call ({nbytes / 1e6:.1f} MB)"}


def cpu_ref_shares(B, H, Hkv, D, budget_s, max_calls, warm=1):
    """cfg2 on the host: per sequence and share the reference's fused_cpu_attn
    (bf16), then the runtime's merge (system/mixoffload.py:1333-1334,
    :1456-1464) in torch.  Returns (bytes/s, info)."""
    import oracle
    G = H // Hkv
    lens, ratio, L0, L1 = cfg2_geometry(B)
    torch.manual_seed(12)
    q = torch.randn(B, H, D).bfloat16()
    ks0 = [torch.randn(Hkv, int(a), D).bfloat16() for a in L0]
    vs0 = [torch.randn(Hkv, int(a), D).bfloat16() for a in L0]
    ks1 = [torch.randn(Hkv, int(a), D).bfloat16() for a in L1]
    vs1 = [torch.randn(Hkv, int(a), D).bfloat16() for a in L1]
    nbytes = 2 * int(lens.sum()) * Hkv * D * 2 + B * H * (D * 2 * 2 + 4)
    ref = load_cpu_ref()

    def one(kb, vb, qb):
        if ref is not None:
            o, m, s = ref.fused_cpu_attn(qb, kb, vb, D ** -0.5)
            return o.float() * s.float(), m.float(), s.float()
        o, m, s = oracle.gqa_decode(oracle.bf16_bits(qb), oracle.bf16_bits(kb), oracle.bf16_bits(vb), D ** -0.5)
        return torch.from_numpy(o * s[..., None]), torch.from_numpy(m)[..., None], torch.from_numpy(s)[..., None]

    def run():
        for b in range(B):
            qb = q[b].view(Hkv, G, D)
            o0, m0, s0 = one(ks0[b], vs0[b], qb)
            o1, m1, s1 = one(ks1[b], vs1[b], qb)
            M = torch.maximum(m0, m1)
            w0, w1 = torch.exp(m0 - M), torch.exp(m1 - M)
            _ = (o0 * w0 + o1 * w1) / (w0 * s0 + w1 * s1).clamp(min=1e-3)

    t, n = median_time(run, budget_s, max_calls, warm)
    return nbytes / t, {"kind": "reference" if ref is not None else "port", "cores": os.cpu_count() or 1,
                        "calls": n, "sec_per_call": t,
                        "sample": f"full cfg2 step ({nbytes / 1e9:.2f} GB): per sequence and share "
                                  "fused_cpu_attn + torch LSE merge"}


def cpu_ref_mla(B, nH, S, budget_s, max_calls, warm=1):
    """The reference's fused_cpu_attn_mla_compressed on all host cores (full cfg3)."""
    import oracle
    torch.manual_seed(13)
    qp = torch.randn(B * nH, 512).bfloat16()
    qpe = torch.randn(B * nH, 64).bfloat16()
    c = torch.randn(B, S, 512).bfloat16()
    p = torch.randn(B, S, 64).bfloat16()
    nbytes = B * S * 576 * 2 + B * nH * (576 * 2 + 512 * 4 + 8)
    ref = load_cpu_ref()
    if ref is not None:
        kind, fn = "reference", (lambda: ref.fused_cpu_attn_mla_compressed(qp, qpe, c, p, 192 ** -0.5))
    else:
        bits = [oracle.bf16_bits(t) for t in (qp, qpe, c, p)]
        kind, fn = "port", (lambda: oracle.mla_compressed(*bits, 192 ** -0.5))
    t, n = median_time(fn, budget_s, max_calls, warm)
    return nbytes / t, {"kind": kind, "cores": os.cpu_count() or 1, "calls": n, "sec_per_call": t,
                        "sample": f"fused_cpu_attn_mla_compressed, B={B}, nH={nH}, S={S} (full cfg3, "
                                  f"{nbytes / 1e6:.1f} MB per call)"}


def cpu_ref_csa(bs, nH, nc, k, budget_s, max_calls, warm=1):
    """cfg5 on the host: the reference's indexer_attn_cpu (csa_attn.cpp:1819-1883)
    on all cores over a bf16 copy of the dequantised entries (int8 * scale,
    made outside the timing), fp32 q, the same sorted top-k ids.  Full cfg5
    step; bytes are the workload's algorithmic bytes."""
    import oracle
    torch.manual_seed(15)
    kv = torch.empty(bs, nc, 512, dtype=torch.bfloat16)
    sc = torch.rand(bs, nc) * 0.04 + 0.01
    for b in range(bs):
        kv[b] = ((torch.randn(nc, 512) * 32).round_().clamp_(-127, 127) * sc[b, :, None]).bfloat16()
    g = torch.Generator().manual_seed(5)
    idx = torch.stack([torch.randperm(nc, generator=g)[:k].sort().values for _ in range(bs)]).int()
    q = torch.randn(bs, nH, 512).bfloat16().float()
    o = torch.empty(bs, nH, 512)
    lse = torch.empty(bs, nH)
    nbytes = bs * k * (512 + 4 + 4) + bs * nH * (512 * 2 + 512 * 2 + 4)
    ref = load_cpu_ref("csa_attn_kernel")
    n = os.cpu_count() or 1
    if ref is not None:
        kind, fn = "reference", (lambda: ref.indexer_attn_cpu(q, kv, idx, 512 ** -0.5, o, lse, n))
    else:
        qn, kvn, idn = q.numpy(), oracle.bf16_bits(kv), idx.numpy()
        kind, fn = "port", (lambda: oracle.csa_attend(qn, kvn, 512 ** -0.5, idx=idn))
    t, calls = median_time(fn, budget_s, max_calls, warm)
    return nbytes / t, {"kind": kind, "cores": n, "calls": calls, "sec_per_call": t,
                        "sample": f"indexer_attn_cpu, bs={bs}, nH={nH}, nc={nc}, k={k} on bf16 dequantised "
                                  f"entries (full cfg5 step, {nbytes / 1e6:.1f} MB algorithmic)"}


def cpu_ref_indexer(bs, nH, hd, nc, k, budget_s, max_calls, warm=1):
    """The reference's indexer_topk_cpu (csa_attn.cpp:1658-1736) on all cores,
    fp32 copies of the same shapes (the reference op takes fp32)."""
    import oracle
    torch.manual_seed(16)
    q = torch.randn(bs, nH, hd)
    kv = torch.randn(bs, nc, hd)
    w = torch.rand(bs, nH)
    nbytes = bs * nc * hd * 2 + bs * nH * (hd * 2 + 4) + bs * k * 4
    ref = load_cpu_ref("csa_attn_kernel")
    n = os.cpu_count() or 1
    if ref is not None:
        kind, fn = "reference", (lambda: ref.indexer_topk_cpu(q, kv, w, k, n))
    else:
        qn, kvn, wn = q.numpy(), kv.numpy(), w.numpy()
        kind, fn = "port", (lambda: oracle.indexer_topk(qn, kvn, wn, k))
    t, calls = median_time(fn, budget_s, max_calls, warm)
    return nbytes / t, {"kind": kind, "cores": n, "calls": calls, "sec_per_call": t,
                        "sample": f"indexer_topk_cpu fp32, bs={bs}, nH={nH}, hd={hd}, nc={nc}, k={k} (full step; "
                                  f"bytes counted as the bf16 GPU workload's)"}


def cpu_reference_for(name, args, budget_s, max_calls, warm):
    if name == "cfg4":
        return cpu_ref_dense(32, 4, 8, 128, args.kv_len or 131072, budget_s, max_calls, warm), \
            "gqa_qwen3_b32_l131072_sharded"
    if name == "cfg1":
        return cpu_ref_dense(1, 4, 8, 128, args.kv_len or 4096, budget_s, max_calls, warm), "gqa_qwen3_b1_l4096"
    if name == "cfg2":
        return cpu_ref_shares(16, 32, 8, 128, budget_s, max_calls, warm), \
            "gqa_mixtral_b16_ragged_1024_32768_two_shares"
    if name in ("cfg3", "mla_abs"):   # the reference's CPU part of the step (its bmm's run on the GPU)
        return cpu_ref_mla(8, 16, 16384, budget_s, max_calls, warm), "mla_absorbed_ds2lite_b8_h16_s16384"
    if name == "cfg5":
        return cpu_ref_csa(16, 64, 65536, 2048, budget_s, max_calls, warm), "csa_ds4_b16_h64_nc65536_top2048_int8"
    if name == "idx":
        return cpu_ref_indexer(16, 64, 128, 65536, 2048, budget_s, max_calls, warm), \
            "indexer_ds4_b16_h64_d128_nc65536_top2048_bf16"
    raise ValueError(name)


def make_workload(name, world, rank, args):
    if name == "cfg4":
        return GqaDense(world, rank, "cfg4", 32, 32, 4, 128, args.kv_len or 131072, SEEDS["cfg4"],
                        exchange=args.exchange)
    if name == "cfg1":
        return GqaDense(world, rank, "cfg1", 1, 32, 4, 128, args.kv_len or 4096, SEEDS["cfg1"])
    if name == "cfg2":
        return GqaShares(world, rank)
    if name == "cfg3":
        return Mla(world, rank, S=args.kv_len or 16384)
    if name == "mla_abs":
        return MlaAbsorbed(world, rank, S=args.kv_len or 16384)
    if name == "cfg5":
        return Csa(world, rank, nc=args.kv_len or 65536, seed=SEEDS["cfg5"], exchange=args.exchange)
    if name == "idx":
        return Indexer(world, rank, nc=args.kv_len or 65536)
    raise ValueError(name)


WORKLOADS = ("cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "idx", "mla_abs", "aux")
SEEDS = {"cfg4": 4000, "cfg1": 1000, "cfg5": 5}


# -------------------------------------------------------------------- main
def make_runner(wl, fn, graph=None):
    """Returns run(n) that issues n steps.  Small workloads are captured once
    (one pass over all input copies) in a CUDA graph and replayed."""
    if not (wl.graph if graph is None else graph):
        state = {"i": 0}

        def run(n):
            for _ in range(n):
                fn(state["i"])
                state["i"] += 1
        return run, 1
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    per = max(wl.copies, 8)
    with torch.cuda.stream(s):
        for i in range(per):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(per):
            fn(i)

    def run(n):
        for _ in range(max(1, n // per)):
            g.replay()
    run.graph = g
    return run, per


def time_steps_flushed(wl, fn, steps, warmup, world):
    """One CUDA-event pair per step, with an L2 flush (untimed) before each."""
    for i in range(warmup):
        wl.flush(i)
        fn(i)
    barrier(world)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i, (a, b) in enumerate(evs):
        wl.flush(i)
        a.record()
        fn(i)
        b.record()
    torch.cuda.synchronize()
    barrier(world)
    total = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    return max_over_ranks(total / steps, world), steps


def time_steps(wl, fn, steps, warmup, world, graph=None):
    if getattr(wl, "flush_l2", False):
        return time_steps_flushed(wl, fn, steps, warmup, world)
    run, per = make_runner(wl, fn, graph)
    run(max(warmup, per))
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n = max(steps // per, 1) * per
    e0.record()
    run(n)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3 / n, world), n


def time_e2e(wl, steps, warmup, world):
    """Public-API steps with host buffers; no graph (a user calls the API)."""
    if getattr(wl, "flush_l2", False):
        return time_steps_flushed(wl, wl.e2e_step, steps, warmup, world)[0]
    for i in range(warmup):
        wl.e2e_step(i)
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        wl.e2e_step(i)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3 / steps, world)


def run_aux(args):
    """--workload aux: the auxiliary kernels of the path, each timed alone on
    inputs larger than L2 (CUDA events, mean over --steps launches after
    --warmup), with its algorithmic bytes per launch: the int8 / u8
    quantisers, the fp32 GQA decode, the two log-sum-exp merges (the strided
    one at a sharded-exchange shape) and the KV-cache append (one token; a
    latency-bound launch).  One JSON line; per-kernel results in "ops"."""
    from scope_b200 import _lib
    L_ = _lib.lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = lambda: torch.cuda.current_stream().cuda_stream   # noqa: E731
    g = torch.Generator(device=dev).manual_seed(77)
    hbm, peak_src = peaks()

    def chk(rc):
        if rc != 0:
            raise RuntimeError(L_.ws_last_error().decode())

    def timed(fn, nbytes):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        return {"us": us, "bytes": nbytes, "GB/s": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / hbm}

    ops = {}
    # kv_quantize_bf16_to_int8 over [8, 32768, 512] bf16 (two copies, alternating)
    rows, hd = 8 * 32768, 512
    kvs = [bf16_randn((rows, hd), g, dev) for _ in range(2)]
    k8 = torch.empty(rows, hd, dtype=torch.int8, device=dev)
    ksc = torch.empty(rows, dtype=torch.float32, device=dev)
    ksm = torch.empty(rows, dtype=torch.int32, device=dev)
    ops["csa_kv_quantize_s8"] = timed(lambda i: chk(L_.ws_csa_kv_quantize_s8(
        kvs[i % 2].data_ptr(), rows, hd, k8.data_ptr(), ksc.data_ptr(), ksm.data_ptr(), st())), rows * hd * 3 + rows * 8)
    del kvs, k8, ksc, ksm
    # q_quantize_fp32_to_u8 over [131072, 512] fp32
    rows = 131072
    qs = [torch.randn(rows, hd, generator=g, device=dev) for _ in range(2)]
    qu = torch.empty(rows, hd, dtype=torch.uint8, device=dev)
    qsc = torch.empty(rows, dtype=torch.float32, device=dev)
    ops["csa_q_quantize_u8"] = timed(lambda i: chk(L_.ws_csa_q_quantize_u8(
        qs[i % 2].data_ptr(), rows, hd, qu.data_ptr(), qsc.data_ptr(), st())), rows * hd * 5 + rows * 4)
    del qs, qu, qsc
    # fp32 GQA decode (gqa_f32_kernel): 32 kv rows x 16384 tokens x 128, G = 8
    B_kv, G, D, L = 32, 8, 128, 16384
    q = torch.randn(B_kv, G, D, generator=g, device=dev)
    k = torch.randn(B_kv, L, D, generator=g, device=dev)
    v = torch.randn(B_kv, L, D, generator=g, device=dev)
    out = torch.empty(B_kv, G, D, device=dev)
    lse = torch.empty(B_kv, G, device=dev)
    ws = torch.zeros(L_.ws_gqa_decode_workspace_size(B_kv, G, D, L), dtype=torch.uint8, device=dev)
    ops["gqa_f32_decode"] = timed(lambda i: chk(L_.ws_gqa_decode(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), v.stride(0), v.stride(1), B_kv, G, D, D,
        L, D ** -0.5, _lib.WS_DTYPE_F32, _lib.WS_OUT_NORM_F32, out.data_ptr(), None, None, lse.data_ptr(),
        ws.data_ptr(), ws.numel(), st())), 2 * B_kv * L * D * 4 + B_kv * G * (2 * D * 4 + 4))
    del q, k, v, out, lse, ws
    # strided merge of 8 gathered [o, lse] blocks (the NCCL exchange's merge), 131072 rows x 128
    P, R, D = 8, 131072, 128
    blk = R * D + R
    parts = torch.randn(P, blk, generator=g, device=dev)
    out = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(R, device=dev)
    ops["lse_merge_strided"] = timed(lambda i: chk(L_.ws_lse_merge_strided(
        parts.data_ptr(), blk, parts.data_ptr() + 4 * R * D, blk, P, R, D, out.data_ptr(), _lib.WS_DTYPE_BF16,
        lse.data_ptr(), st())), P * blk * 4 + R * (D * 2 + 4))
    del parts, out, lse
    # vectorised merge of 9 split partials (the CSA split merge shape), 16384 rows x 512
    P, R, D = 9, 16384, 512
    po = torch.randn(P, R, D, generator=g, device=dev)
    pl = torch.randn(P, R, generator=g, device=dev)
    out = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(R, device=dev)
    ops["lse_merge"] = timed(lambda i: chk(L_.ws_lse_merge(
        po.data_ptr(), pl.data_ptr(), P, R, D, out.data_ptr(), _lib.WS_DTYPE_BF16, lse.data_ptr(), st())),
        P * R * (D + 1) * 4 + R * (D * 2 + 4))
    del po, pl, out, lse
    # KV-cache append of one decode token into [128 rows, 8192, 128] (one launch per token)
    rows, cap, D = 128, 8192, 128
    cache = torch.zeros(rows, cap, D, dtype=torch.bfloat16, device=dev)
    new = bf16_randn((rows, 1, D), g, dev)
    # one launch per token is far shorter than a Python-side launch: the launches are captured in a CUDA
    # graph (args.steps appends at successive positions) and the graph is timed, so the events see device time
    gs = torch.cuda.Stream()
    gs.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for i in range(args.steps):
            chk(L_.ws_kv_append(cache.data_ptr(), cache.stride(0), cache.stride(1), cap, new.data_ptr(),
                                new.stride(0), new.stride(1), rows, 1, D, _lib.WS_DTYPE_BF16, i % cap,
                                torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    r = timed(lambda i: graph.replay(), 2 * rows * D * 2 * args.steps)
    ops["kv_append_1tok"] = {"us": r["us"] / args.steps, "bytes": 2 * rows * D * 2, "GB/s": r["GB/s"],
                             "frac": r["frac"], "note": "per launch, from a CUDA graph of back-to-back appends"}
    tot_b = sum(o["bytes"] for o in ops.values())
    tot_us = sum(o["us"] for o in ops.values())
    line = {"metric": METRIC, "value": tot_b / tot_us / 1e6, "unit": "TB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tot_us / 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16/fp32", "data": "synthetic (seeded normal)",
            "config": {"workload": "aux_kernels", "peak_GBps": hbm, "peak_source": peak_src,
                       "l2": "every input but the append's is larger than L2"},
            "ops": ops, "gpu_launches": len(ops) * args.steps}
    print(json.dumps(line), flush=True)


OTHER_WORKLOADS = ("cfg1", "cfg2", "cfg3", "cfg5", "idx", "mla_abs")


def run_others(args, hbm):
    """The other BASELINE configs (and the indexer / absorbed-MLA steps), one GPU each, measured in the
    same process after the headline: per workload the device-timed step and its dominant kernel (inputs
    rotated past L2 as in their own runs), the step through the public API with host buffers, and the
    reference's CPU kernel on a bounded number of calls.  Returns {name: summary}."""
    import argparse as _ap
    steps = min(max(args.steps, 200), 2000)
    warm = max(args.warmup, 10)
    res = {}
    gpu_index = int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[0]) if os.environ.get("CUDA_VISIBLE_DEVICES") \
        else torch.cuda.current_device()
    with ClockSampler(gpu_index) as clk:
        for name in OTHER_WORKLOADS:
            sub = _ap.Namespace(**vars(args))
            sub.kv_len, sub.workload = 0, name
            wl = None
            try:
                wl = make_workload(name, 1, 0, sub)
                t_kernel, _ = time_steps(wl, wl.kernel, steps, warm, 1)
                t_step, n_timed = time_steps(wl, wl.step, steps, warm, 1)
                t_e2e = time_e2e(wl, min(steps, 200), warm, 1)
                kb = wl.kernel_bytes()
                r = {"workload": wl.config()["workload"], "us_per_step": t_step * 1e6,
                     "value": wl.step_bytes() / t_step / 1e12, "unit": "TB/s", "timed_steps": n_timed,
                     "kernel": wl.kernel_name, "kernel_us": t_kernel * 1e6, "algorithmic_bytes_per_launch": kb,
                     "achieved_gbs": kb / t_kernel / 1e9, "frac": kb / t_kernel / 1e9 / hbm,
                     "e2e_us": t_e2e * 1e6, "e2e_value": wl.step_bytes() / t_e2e / 1e12,
                     "gpu_launches_per_step": wl.kernels_per_step}
                tr = tensor_roofline(wl, t_kernel)
                if tr is not None:
                    r["tensor_frac"] = tr["frac"]
                if not args.no_cpu_baseline:
                    bps, info = wl.cpu_reference(budget_s=2.0, max_calls=20)
                    r["cpu_reference"] = {"value": bps / 1e12, "unit": "TB/s", "us_per_call": info["sec_per_call"] * 1e6,
                                          "calls": info["calls"], "cores": info["cores"], "kind": info["kind"],
                                          "sample": info["sample"]}
                res[name] = r
            except Exception as e:   # one workload's failure leaves the headline line intact
                res[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
            if wl is not None and hasattr(wl, "close"):
                wl.close()
            del wl
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    res["clocks"] = clk.summary()
    return res


def run_reference_arm(args):
    """The reference's own CPU kernel on this host's cores, one bounded sample
    of the workload per step.  Touches no GPU and loads nothing of scope_b200."""
    world, rank, _ = dist_info()
    if rank != 0:
        return
    (bps, info), workload = cpu_reference_for(args.workload, args, budget_s=1e9, max_calls=args.steps,
                                              warm=args.warmup)
    value = bps / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus, "steps": info["calls"],
            "warmup": args.warmup, "ms_per_step": info["sec_per_call"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {"workload": workload, "sample": info["sample"]},
            "cpu_baseline": {"value": value, "unit": "TB/s", "cores": info["cores"], "kind": info["kind"],
                             "cpu_model": info.get("cpu_model", cpu_model()), "sample": info["sample"]},
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="cfg4", choices=WORKLOADS)
    ap.add_argument("--kv-len", type=int, default=0, help="override KV length (profiling on a small case)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-others", action="store_true",
                    help="N = 1, cfg4: skip the other workloads measured after the headline ('workloads' key)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "scatter", "nccl"],
                    help="cfg4 / cfg5 at N > 1: partials pushed over NVLink to rank 0 (peer), merged in shares "
                         "by every rank and gathered on rank 0 (scatter), or an NCCL all_gather (nccl)")
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
    if args.workload == "aux":
        if world > 1:
            raise SystemExit("--workload aux runs on one GPU")
        run_aux(args)
        return
    wl = make_workload(args.workload, world, rank, args)
    parity = wl.parity_check(SEEDS[args.workload]) if hasattr(wl, "parity_check") else None

    t_kernel, _ = time_steps(wl, wl.kernel, args.steps, args.warmup, world)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = int(vis.split(",")[local]) if vis else local
    with ClockSampler(gpu_index) as clk:
        t_step, n_timed = time_steps(wl, wl.step, args.steps, args.warmup, world)
    clocks = clk.summary()
    t_e2e = time_e2e(wl, min(args.steps, 500), args.warmup, world)
    # N > 1: the exchange alone, back to back (push + merge, or all_gather + merge), every rank in step; the
    # peer forms from a CUDA graph, so that host launch overhead is not what is timed
    t_ex = (time_steps(wl, wl.exchange_step, min(args.steps, 200), args.warmup, world,
                       graph=True if getattr(wl, "exchange", "") in ("peer", "scatter") else None)[0]
            if world > 1 and hasattr(wl, "exchange_step") else None)

    hbm, peak_src = peaks()
    kb = wl.kernel_bytes()
    traffic, traffic_src = profile_traffic(getattr(wl, "profile_name", f"gqa_decode_{wl.name}"), kb)
    achieved = kb / t_kernel / 1e9
    value = wl.step_bytes() / t_step / 1e12
    h2d, d2h = wl.e2e_bytes()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        bps, info = wl.cpu_reference(budget_s=10.0, max_calls=200)
        cpu = {"value": bps / 1e12, "unit": "TB/s", "cores": info["cores"], "kind": info["kind"],
               "cpu_model": info.get("cpu_model", cpu_model()),
               "sample": info["sample"] + f"; median of {info['calls']} calls",
               "us_per_call": info["sec_per_call"] * 1e6}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "timed_steps": n_timed, "ms_per_step": t_step * 1e3, "us_per_step": t_step * 1e6,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) q/k/v)", "config": wl.config(),
                "e2e": {"value": wl.step_bytes() / t_e2e / 1e12, "unit": "TB/s", "us_per_step": t_e2e * 1e6,
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "peak_source": peak_src, "kernel": wl.kernel_name,
                             "kernel_us": t_kernel * 1e6, "algorithmic_bytes_per_launch": kb,
                             "traffic": traffic, "traffic_source": traffic_src},
                "tensor": tensor_roofline(wl, t_kernel),
                "gpu_launches": wl.kernels_per_step * n_timed,
                "clocks": clocks, "cpu_baseline": cpu}
        if parity is not None:
            line["parity"] = parity
        if t_ex is not None:
            line["exchange_us"] = t_ex * 1e6
        if world == 1 and args.workload == "cfg4" and not args.kv_len and not args.no_others:
            # the headline's buffers go before the other workloads allocate theirs
            if hasattr(wl, "close"):
                wl.close()
            wl = None
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            line["workloads"] = run_others(args, hbm)
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
    status = scope_b200.status_take()
    if status != 0:
        raise RuntimeError(f"rank {rank}: a kernel reported a device-side failure (status {status})")
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
