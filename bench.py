"""Benchmark of the sm_100a paged-attention backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg4|cfg3|cfg5-t512|cfg5-t64|scatter|qkv-prefill|qkv-decode]

One step = one launch of the hot path over one batch of the workload, with
inputs resident in HBM (``value``), and the same step through the public
Python API with the step's inputs copied from pinned host memory and its
result copied back, plus a host synchronisation (``e2e``):

* cfg4 (default): configuration 4 -- fused KV write + paged decode, bf16 KV,
  64 requests per GPU, every context 32768 tokens, 32 heads x 128 dims, block
  size 16, randomly permuted block tables; 34.7 GB of KV per GPU (larger than
  the 126 MB L2, so no flush is needed between steps).  Requests are sharded
  across GPUs (weak scaling: each rank owns 64 requests of the global batch).
* cfg3: configuration 3 at batch 256 -- ragged contexts ~U[1, 4096].
* cfg5-t512 / cfg5-t64: configuration 5 -- one batched tcgen05 chunked
  prefill launch over 16 sequences, chunk 512 or 64 tokens, prefixes
  16*U{0..252}; the KV pool is ~2-4 GB (larger than L2).
* scatter: the slot-mapping KV scatter of 16 x 512 prefill tokens (bf16).
* qkv-prefill / qkv-decode: the attention's QKV projection with the KV write
  in its epilogue (tcgen05 GEMM), hidden 4096, over 8192 prefill tokens
  (TFLOP/s, tensor roofline) or 64 decode tokens (GB/s, HBM roofline: the
  100 MB weight read dominates); the line also carries the unfused sequence
  (cuBLAS matmul, then the scatter) timed in the same run.

Under torchrun (N>1) each rank runs its shard on its own GPU; the only
collective is the all-reduce(MAX) of the timings.  Rank 0 prints one JSON
line.  ``--impl reference`` times the reference algorithm's CPU restatement
(oracle/: paged_attention_batch_online_v1, the SDPA v2 prefill, the KV
write loop of minivllm) on the host cores instead; under torchrun only
rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path
from types import SimpleNamespace

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "mini-gpt-inference_b200"))

METRIC = "paged decode attn HBM GB/s (% of 8 TB/s); decode tokens/sec at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
H, D, S = 32, 128, 16


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peak(key: str) -> tuple[float, str]:
    try:
        return float(json.loads((REPO / "MEASURED_PEAKS.json").read_text())[key]), "measured"
    except Exception:
        return FALLBACK[key], "fallback"


def _tables(counts, perm):
    width = max(counts)
    t = torch.full((len(counts), width), -1, dtype=torch.int64)
    nxt = 0
    for b, c in enumerate(counts):
        t[b, :c] = perm[nxt:nxt + c]
        nxt += c
    return t


# ------------------------------------------------------------------ workloads
class DecodeWorkload:
    """Fused KV write + paged decode over one batch (configuration 4 or 3)."""

    bound, unit = "hbm", "GB/s"

    def __init__(self, name, rank, device, batch=None, ctx=None, kv_dtype="bf16"):
        self.name, self.device = name, device
        self.kv_name = kv_dtype
        self.dt = torch.float32 if kv_dtype == "f32" else torch.bfloat16
        self.es = 4 if kv_dtype == "f32" else 2
        if name == "cfg4":
            self.B = batch or 64
            lens = [ctx or 32768] * self.B
            self.desc = (f"config 4: long-context split-K decode, {kv_dtype} KV, {self.B} requests/GPU"
                         f" x {lens[0]} tokens, H=32, D=128, S=16, fused KV write")
        else:
            self.B = batch or 256
            g = torch.Generator().manual_seed(1000 + rank)
            lens = torch.randint(1, 4097, (self.B,), generator=g).tolist()
            lens[0] = 1
            if lens[-1] % S == 0:
                lens[-1] -= 1
            self.desc = (f"config 3: ragged decode, {kv_dtype} KV, batch {self.B}/GPU, contexts"
                         " ~U[1,4096], H=32, D=128, S=16, fused KV write")
        self.lens = lens
        counts = [math.ceil(n / S) for n in lens]
        P = sum(counts) + max(1, sum(counts) // 100)
        g = torch.Generator(device=device).manual_seed(20260000 + rank)
        self.k = torch.empty((1, P, S, H, D), dtype=self.dt, device=device).normal_(generator=g)
        self.v = torch.empty_like(self.k).normal_(generator=g)
        tables = _tables(counts, torch.randperm(P, generator=g, device=device).cpu())
        slots = [int(tables[b, (n - 1) // S]) * S + (n - 1) % S for b, n in enumerate(lens)]
        hg = torch.Generator().manual_seed(rank)
        self.host = {
            "q": torch.randn((self.B, H, D), generator=hg).to(self.dt).pin_memory(),
            "k_new": torch.randn((self.B, H, D), generator=hg).to(self.dt).pin_memory(),
            "v_new": torch.randn((self.B, H, D), generator=hg).to(self.dt).pin_memory(),
            "tables": tables.pin_memory(),
            "ctx": torch.tensor(lens, dtype=torch.int64).pin_memory(),
            "slots": torch.tensor(slots, dtype=torch.int64).pin_memory(),
        }
        self.dev = {k: v.to(device) for k, v in self.host.items()}
        self.out_h = torch.empty((self.B, H, D), dtype=self.dt).pin_memory()
        self.pool = SimpleNamespace(k=self.k, v=self.v, block_size=S)
        self.kv_gb = 2 * self.k.numel() * self.k.element_size() / 1e9

    def _call(self, t, prepare=False, out=None):
        from b200attn import paged_attention_batch_b200
        return paged_attention_batch_b200(t["q"], self.pool, t["tables"], t["ctx"], 0,
                                          k_new=t["k_new"], v_new=t["v_new"],
                                          slot_mapping=t["slots"], out=out, prepare=prepare)

    def prepare(self):
        self.call = self._call(self.dev, prepare=True,
                               out=torch.empty((self.B, H, D), dtype=self.dt,
                                               device=self.device))

    def step(self):
        self.call()

    def e2e_step(self):
        t = {k: v.to(self.device, non_blocking=True) for k, v in self.host.items()}
        self.out_h.copy_(self._call(t), non_blocking=True)

    def work(self) -> float:  # algorithmic bytes per step
        from b200attn import decode_bytes
        return decode_bytes(self.lens, H, D, S, kv_bytes=self.es, q_bytes=self.es,
                            out_bytes=self.es, idx_bytes=8, fused_in_bytes=self.es)

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.host.values())

    def d2h_bytes(self):
        return self.out_h.numel() * self.out_h.element_size()

    def config(self, world):
        return {"workload": self.desc, "batch_per_gpu": self.B, "global_batch": self.B * world,
                "context_lens": str(self.lens[0]) if self.name == "cfg4" else "U[1,4096]",
                "heads": H, "head_dim": D, "block_size": S, "kv_dtype": self.kv_name,
                "q_dtype": self.kv_name, "accumulate": "f32", "fused_kv_write": True,
                "l2": "inputs larger than L2 (KV pool %.1f GB per GPU), no flush" % self.kv_gb,
                "parallelism": f"request-sharded dp{world} (no data-path collective)"}

    def extra(self, ms_max, world, steps):
        value = self.work() * world * steps / (ms_max * 1e-3) / 1e9
        return {"pct_of_8tbs": 100.0 * value / world / NOMINAL_HBM_GBS,
                "decode_tokens_per_s": self.B * world * steps / (ms_max * 1e-3)}


class PrefillWorkload:
    """One batched tcgen05 chunked-prefill launch over 16 sequences (configuration 5)."""

    unit = "TFLOP/s"

    def __init__(self, T, rank, device, nseq=16):
        self.T, self.device, self.nseq = T, device, nseq
        self.bound = "tensor" if T >= 512 else "hbm"
        g = torch.Generator().manual_seed(rank)
        self.prefix = (torch.randint(0, 253, (nseq,), generator=g) * 16).tolist()
        counts = [math.ceil((p + T) / S) for p in self.prefix]
        P = sum(counts) + 16
        gd = torch.Generator(device=device).manual_seed(30260000 + rank)
        self.k = torch.empty((1, P, S, H, D), dtype=torch.bfloat16, device=device).normal_(generator=gd)
        self.v = torch.empty_like(self.k).normal_(generator=gd)
        perm = torch.randperm(P, generator=gd, device=device).cpu()
        self.tables_h, nxt = [], 0
        for c in counts:
            self.tables_h.append(perm[nxt:nxt + c].clone().pin_memory())
            nxt += c
        self.q_h = [torch.randn((T, H, D), generator=g).to(torch.bfloat16).pin_memory()
                    for _ in range(nseq)]
        self.tables = [t.to(device) for t in self.tables_h]
        self.q = [q.to(device) for q in self.q_h]
        self.out_h = [torch.empty((T, H, D), dtype=torch.bfloat16).pin_memory() for _ in range(nseq)]
        self.pool = SimpleNamespace(k=self.k, v=self.v, block_size=S)
        self.kv_gb = 2 * self.k.numel() * self.k.element_size() / 1e9
        self.desc = (f"config 5: prefix-aware chunked prefill (tcgen05), bf16, {nseq} sequences,"
                     f" chunk {T}, prefixes 16*U{{0..252}}, H=32, D=128, S=16")

    def prepare(self):
        from b200attn import chunked_prefill_batch_b200
        self.call = chunked_prefill_batch_b200(self.q, self.pool, self.tables, self.prefix, 0,
                                               prepare=True)

    def step(self):
        self.call()

    def e2e_step(self):
        from b200attn import chunked_prefill_batch_b200
        qs = [q.to(self.device, non_blocking=True) for q in self.q_h]
        ts = [t.to(self.device, non_blocking=True) for t in self.tables_h]
        outs = chunked_prefill_batch_b200(qs, self.pool, ts, self.prefix, 0)
        for o, oh in zip(outs, self.out_h):
            oh.copy_(o, non_blocking=True)

    def flops(self) -> float:
        T = self.T
        return sum(4.0 * H * D * (T * p + T * (T + 1) / 2) for p in self.prefix)

    def bytes(self) -> float:
        kv = sum((p + self.T) * H * D * 2 * 2 for p in self.prefix)
        return kv + 2 * self.nseq * self.T * H * D * 2

    def work(self) -> float:
        return self.flops()

    def h2d_bytes(self):
        return sum(q.numel() * 2 for q in self.q_h) + sum(t.numel() * 8 for t in self.tables_h)

    def d2h_bytes(self):
        return sum(o.numel() * 2 for o in self.out_h)

    def config(self, world):
        return {"workload": self.desc, "seqs_per_gpu": self.nseq, "chunk": self.T, "heads": H,
                "head_dim": D, "block_size": S, "kv_dtype": "bf16", "accumulate": "f32",
                "l2": "KV pool %.1f GB per GPU (larger than L2), no flush" % self.kv_gb,
                "parallelism": f"sequence-sharded dp{world}"}

    def extra(self, ms_max, world, steps):
        sec = ms_max * 1e-3 / steps
        return {"prefill_gbs": self.bytes() * world / sec / 1e9,
                "prefill_tokens_per_s": self.nseq * self.T * world / sec}


class ScatterWorkload:
    """Slot-mapping scatter of 16 x 512 prefill tokens into a bf16 pool."""

    bound, unit = "hbm", "GB/s"

    def __init__(self, rank, device, n=16 * 512):
        self.n, self.device = n, device
        P = n // S * 8
        self.k = torch.zeros((1, P, S, H, D), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        g = torch.Generator().manual_seed(rank)
        self.kn_h = torch.randn((n, H, D), generator=g).to(torch.bfloat16).pin_memory()
        self.vn_h = torch.randn((n, H, D), generator=g).to(torch.bfloat16).pin_memory()
        self.slots_h = torch.randperm(P * S, generator=g)[:n].pin_memory()
        self.kn, self.vn, self.slots = (t.to(device) for t in (self.kn_h, self.vn_h, self.slots_h))
        self.pool = SimpleNamespace(k=self.k, v=self.v, block_size=S)
        self.desc = f"slot-mapping KV scatter: {n} tokens x 32 heads x 128 dims, bf16"

    def prepare(self):
        from b200attn import kv_scatter_b200
        self.call = kv_scatter_b200(self.kn, self.vn, self.pool, self.slots, 0, prepare=True)

    def step(self):
        self.call()

    def e2e_step(self):
        from b200attn import kv_scatter_b200
        kv_scatter_b200(self.kn_h.to(self.device, non_blocking=True),
                        self.vn_h.to(self.device, non_blocking=True), self.pool,
                        self.slots_h.to(self.device, non_blocking=True), 0)

    def work(self) -> float:
        return self.n * H * D * 2 * (2 + 2) + self.n * 8

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.kn_h, self.vn_h, self.slots_h))

    def d2h_bytes(self):
        return 0

    def config(self, world):
        return {"workload": self.desc, "tokens_per_gpu": self.n, "heads": H, "head_dim": D,
                "block_size": S, "kv_dtype": "bf16",
                "l2": "each step moves %.0f MB; no flush between steps" % (self.work() / 1e6),
                "parallelism": f"token-sharded dp{world}"}

    def extra(self, ms_max, world, steps):
        return {}


class QkvWorkload:
    """The attention's QKV projection with the KV write in its epilogue
    (b200_qkv_kv_write), bf16, hidden 4096 (H=32, D=128): a prefill batch
    of 16 x 512 tokens (tensor-bound) or a decode batch of 64 tokens
    (bound by the 100 MB weight read)."""

    def __init__(self, name, rank, device):
        self.name, self.device = name, device
        self.T = 16 * 512 if name == "qkv-prefill" else 64
        self.C = H * D
        self.bound, self.unit = ("tensor", "TFLOP/s") if name == "qkv-prefill" else ("hbm", "GB/s")
        T, C = self.T, self.C
        g = torch.Generator().manual_seed(rank)
        gd = torch.Generator(device=device).manual_seed(40260000 + rank)
        P = T // S * 2
        self.k = torch.zeros((1, P, S, H, D), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.pool = SimpleNamespace(k=self.k, v=self.v, block_size=S)
        self.w = (torch.empty((3 * C, C), dtype=torch.bfloat16, device=device)
                  .normal_(0.0, 0.02, generator=gd))
        self.x_h = torch.randn((T, C), generator=g).to(torch.bfloat16).pin_memory()
        self.slots_h = torch.randperm(P * S, generator=g)[:T].pin_memory()
        self.x, self.slots = self.x_h.to(device), self.slots_h.to(device)
        self.q_h = torch.empty((T, C), dtype=torch.bfloat16).pin_memory()
        self.desc = (f"fused QKV projection + KV write (tcgen05), bf16, {T} tokens, hidden {C}"
                     f" (H=32, D=128), weight [3C, C], S=16")

    def prepare(self):
        from b200attn import qkv_kv_write_b200
        self.call = qkv_kv_write_b200(self.x, self.w, self.pool, self.slots, 0, prepare=True)

    def step(self):
        self.call()

    def e2e_step(self):
        from b200attn import qkv_kv_write_b200
        q = qkv_kv_write_b200(self.x_h.to(self.device, non_blocking=True), self.w, self.pool,
                              self.slots_h.to(self.device, non_blocking=True), 0)
        self.q_h.copy_(q.view(self.T, self.C), non_blocking=True)

    def flops(self) -> float:
        return 2.0 * self.T * self.C * 3 * self.C

    def bytes(self) -> float:
        T, C = self.T, self.C
        return 2.0 * (3 * C * C + T * C + T * 3 * C) + 8 * T

    def work(self) -> float:
        return self.flops() if self.bound == "tensor" else self.bytes()

    def h2d_bytes(self):
        return self.x_h.numel() * 2 + self.slots_h.numel() * 8

    def d2h_bytes(self):
        return self.q_h.numel() * 2

    def config(self, world):
        return {"workload": self.desc, "tokens_per_gpu": self.T, "hidden": self.C, "heads": H,
                "head_dim": D, "block_size": S, "accumulate": "f32",
                "l2": "weights %.0f MB, no flush between steps" % (3 * self.C * self.C * 2 / 1e6),
                "parallelism": f"token-sharded dp{world}"}

    def extra(self, ms_max, world, steps):
        """The unfused sequence the kernel replaces, timed the same way:
        torch's bf16 matmul (cuBLAS) into a [T, 3C] tensor, then the
        slot-mapping scatter of its k and v thirds."""
        from b200attn import kv_scatter_b200
        T, C = self.T, self.C
        y = torch.empty((T, 3 * C), dtype=torch.bfloat16, device=self.device)

        def unfused(scatter):
            torch.matmul(self.x, self.w.t(), out=y)
            if scatter:
                kv_scatter_b200(y[:, C:2 * C].view(T, H, D), y[:, 2 * C:].view(T, H, D),
                                self.pool, self.slots, 0)

        res = {}
        with torch.inference_mode():
            for scatter in (False, True):
                for _ in range(3):
                    unfused(scatter)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    unfused(scatter)
                e1.record()
                torch.cuda.synchronize(self.device)
                ms = e0.elapsed_time(e1) / steps
                key = "cublas_matmul_plus_scatter" if scatter else "cublas_matmul_alone"
                res[key] = {"ms_per_step": ms,
                            "value": self.work() / (ms * 1e-3) / (1e12 if self.bound == "tensor" else 1e9),
                            "unit": self.unit}
        res["fused_ms_per_step"] = ms_max / steps
        return {"unfused_comparison": res}


def make_workload(name, rank, device, args):
    if name in ("cfg4", "cfg3"):
        return DecodeWorkload(name, rank, device, args.batch, args.ctx, args.kv_dtype)
    if name == "cfg5-t512":
        return PrefillWorkload(512, rank, device)
    if name == "cfg5-t64":
        return PrefillWorkload(64, rank, device)
    if name == "scatter":
        return ScatterWorkload(rank, device)
    if name in ("qkv-prefill", "qkv-decode"):
        return QkvWorkload(name, rank, device)
    raise SystemExit(f"unknown workload {name}")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons of the GPUs in use
    every few milliseconds (NVML, read-only).  The sampler starts before the
    warm-up so that it is running when the timed region begins; summary()
    keeps the samples taken between mark_start() and mark_stop()."""

    def __init__(self, indices: list, period_s: float = 0.002):
        self.indices, self.period = indices, period_s
        self.samples: list[tuple[float, float, float, int]] = []  # (t, sm, max, reasons)
        self._stop = None
        self._thread = None
        self._t0, self._t1 = None, None

    def mark_start(self) -> None:
        self._t0 = time.perf_counter()

    def mark_stop(self) -> None:
        self._t1 = time.perf_counter()

    def _run(self):
        import pynvml
        try:
            handles = []
            for ident in self.indices:
                if isinstance(ident, int) or str(ident).isdigit():
                    handles.append(pynvml.nvmlDeviceGetHandleByIndex(int(ident)))
                else:
                    handles.append(pynvml.nvmlDeviceGetHandleByUUID(str(ident)))
            while not self._stop.is_set():
                for h in handles:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((time.perf_counter(), float(sm), float(mx), int(rs)))
                self._stop.wait(self.period)
        except Exception:
            pass

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
        except Exception:
            return self
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        return False

    def summary(self) -> dict:
        t0 = self._t0 if self._t0 is not None else float("-inf")
        t1 = self._t1 if self._t1 is not None else float("inf")
        window = [s[1:] for s in self.samples if t0 <= s[0] <= t1]
        widened = False
        if not window:
            # A timed region shorter than the sampling period: take the
            # samples within two periods of it instead, and say so.
            pad = 2 * self.period + 0.005
            window = [s[1:] for s in self.samples if t0 - pad <= s[0] <= t1 + pad]
            widened = True
        if not window:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        import pynvml
        names = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted(n for n, bit in names.items() if any(s[2] & bit for s in window))
        out = {"sm_mhz": statistics.median(s[0] for s in window),
               "sm_max_mhz": max(s[1] for s in window), "reasons": reasons,
               "samples": len(window), "source": "nvml"}
        if widened:
            out["window"] = "timed region shorter than the sampling period; samples within 2 periods"
        return out


def gpu_indices(world: int) -> list:
    """NVML identifiers (index or UUID) of the GPUs this job's ranks use."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        return ids[:world]
    return list(range(world))


# ------------------------------------------------------------------ CPU leg
def usable_cpus() -> int:
    """CPUs this process may run on: the affinity mask, capped by a cgroup
    v2 CPU quota when one is set (os.cpu_count() sees neither)."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        quota, period = Path("/sys/fs/cgroup/cpu.max").read_text().split()[:2]
        if quota != "max":
            n = min(n, max(1, math.ceil(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), or the platform's."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()


def cpu_reference_sample(workload: str, steps: int, warmup: int,
                         threads: int | None = None) -> dict:
    """Times the reference algorithm (its CPU restatement under oracle/) on
    the host cores, all threads, on a bounded sample of the workload."""
    sys.path.insert(0, str(REPO))
    import oracle
    from b200attn.ops import decode_bytes

    threads = threads or usable_cpus()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(5)
    if workload in ("cfg4", "cfg3"):
        # paged_attention_batch_online_v1 on 4 requests x 32768 tokens (cfg4)
        # or 8 ragged requests (cfg3); the reference cannot mix bf16 KV with
        # fp32 q, so the bf16 sample pool is upcast to fp32 first.
        # (one request for the single-thread figure, which runs ~4x slower)
        lens = [32768] * (1 if threads == 1 else 4) if workload == "cfg4" else \
            torch.randint(1, 4097, (8,), generator=g).tolist()
        counts = [math.ceil(n / S) for n in lens]
        P = sum(counts)
        kf = torch.randn((1, P, S, H, D), generator=g).to(torch.bfloat16).float()
        vf = torch.randn((1, P, S, H, D), generator=g).to(torch.bfloat16).float()
        tables = _tables(counts, torch.randperm(P, generator=g))
        ctx = torch.tensor(lens)
        q = torch.randn((len(lens), H, D), generator=g)
        fn = lambda: oracle.paged_decode_online(q, kf, vf, tables, ctx, 0)
        work = decode_bytes(lens, H, D, S, kv_bytes=2, q_bytes=2, out_bytes=2)
        unit = "GB/s"
        ctx_desc = f"{len(lens)} x {lens[0]}" if workload == "cfg4" else "U[1,4096]"
        sample = (f"{len(lens)} request(s), contexts {ctx_desc},"
                  " H=32, D=128, S=16, bf16 KV upcast to fp32, paged_attention_batch_online_v1"
                  " restatement (oracle/)")
    elif workload.startswith("cfg5"):
        T = 512 if workload.endswith("512") else 64
        prefix = [2016, 1024]
        k_pool = torch.randn((1, sum(math.ceil((p + T) / S) for p in prefix), S, H, D),
                             generator=g).to(torch.bfloat16).float()
        v_pool = torch.randn_like(k_pool)
        qs = [torch.randn((T, H, D), generator=g) for _ in prefix]
        tables, nxt = [], 0
        for p in prefix:
            c = math.ceil((p + T) / S)
            tables.append(list(range(nxt, nxt + c)))
            nxt += c

        def fn():
            for q, t, p in zip(qs, tables, prefix):
                oracle.prefix_prefill_from_pool(q, k_pool, v_pool, t, p, 0)
        work = sum(4.0 * H * D * (T * p + T * (T + 1) / 2) for p in prefix)
        unit = "TFLOP/s"
        sample = (f"2 sequences (prefix 2016 and 1024, chunk {T}), H=32, D=128, fp32, SDPA v2"
                  " prefill restatement (oracle/)")
    elif workload.startswith("qkv"):
        # The reference's own CPU path: the qkv Linear (torch, fp32) on a
        # 256-token sample, chunk(3), then the per-token write loop.
        n, C = 256, H * D
        x = torch.randn((n, C), generator=g)
        w = torch.randn((3 * C, C), generator=g) * 0.02
        k_pool = torch.zeros((1, n // S * 2, S, H, D))
        v_pool = torch.zeros_like(k_pool)
        slots = torch.randperm(k_pool.shape[1] * S, generator=g)[:n].tolist()

        def fn():
            q, k, v = torch.nn.functional.linear(x, w).chunk(3, dim=-1)
            oracle.kv_scatter(k_pool, v_pool, k.reshape(n, H, D), v.reshape(n, H, D), slots, 0)
        if workload == "qkv-prefill":
            work, unit = 2.0 * n * C * 3 * C, "TFLOP/s"
        else:
            work, unit = 4.0 * (3 * C * C + n * C + n * 3 * C), "GB/s"
        sample = (f"{n} tokens, hidden {C}, fp32 qkv Linear + per-token KVBlockPool.write_layer"
                  " loop restatement (oracle/)")
    else:
        n = 2048
        k_pool = torch.zeros((1, n // S * 8, S, H, D), dtype=torch.bfloat16)
        v_pool = torch.zeros_like(k_pool)
        kn = torch.randn((n, H, D), generator=g).to(torch.bfloat16)
        slots = torch.randperm(k_pool.shape[1] * S, generator=g)[:n].tolist()
        fn = lambda: oracle.kv_scatter(k_pool, v_pool, kn, kn, slots, 0)
        work = n * H * D * 2 * 4 + n * 8
        unit = "GB/s"
        sample = f"{n} tokens, per-token KVBlockPool.write_layer loop restatement (oracle/)"
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    return {"value": work / sec / scale, "unit": unit, "cores": threads, "kind": "port",
            "sample": sample, "seconds_per_step": sec}


def metric_name(workload: str, unit: str) -> str:
    """The metric string of a workload, shared by both arms."""
    if workload in ("cfg4", "cfg3"):
        return METRIC
    what = {"cfg5": "chunked prefill attention", "scatter": "KV scatter",
            "qkv": "fused QKV projection + KV write"}[workload.split("-")[0]]
    return f"{workload} {what} {unit}"


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    r = cpu_reference_sample(args.workload, args.steps, args.warmup)
    line = {"metric": metric_name(args.workload, r["unit"]),
            "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["seconds_per_step"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{args.workload} bounded sample on host CPU",
                       "sample": r["sample"]},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg
TRAFFIC_FILES = {"cfg4": "paged_decode_cfg4_traffic.json", "cfg3": "paged_decode_cfg3_traffic.json",
                 "qkv-prefill": "qkv_kv_write_prefill_traffic.json",
                 "qkv-decode": "qkv_kv_write_decode_traffic.json"}


def traffic_from_profile(workload: str) -> float | None:
    if workload not in TRAFFIC_FILES:
        return None
    p = REPO / "profiles" / TRAFFIC_FILES[workload]
    try:
        return float(json.loads(p.read_text())["dram_bytes_per_launch_full_size"])
    except Exception:
        return None


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = world > 1
    if pg:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    wl = make_workload(args.workload, rank, dev, args)
    stream = torch.cuda.current_stream(dev)
    with torch.inference_mode(), ClockSampler(gpu_indices(world)) as clocks:
        wl.prepare()
        for _ in range(args.warmup):
            wl.step()
        torch.cuda.synchronize(dev)
        if pg:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            wl.step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        clocks.mark_stop()
        ms = ev0.elapsed_time(ev1)
        if pg:
            dist.barrier()
        # End to end through the public API: H2D of the step's inputs from
        # pinned memory, the call, D2H of the result, host synchronisation.
        for _ in range(2):
            wl.e2e_step()
        stream.synchronize()
        if pg:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            wl.e2e_step()
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    times = torch.tensor([ms, e2e_s * 1e3], dtype=torch.float64, device=dev)
    if pg:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_max, e2e_ms_max = float(times[0]), float(times[1])
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = wl.work() * world * args.steps / (ms_max * 1e-3) / scale
    e2e_value = wl.work() * world * args.steps / (e2e_ms_max * 1e-3) / scale
    per_launch_s = ms * 1e-3 / args.steps  # this rank's own kernel time
    if wl.bound == "tensor":
        peak, src = measured_peak("bf16_tflops")
        achieved, r_unit = wl.flops() / per_launch_s / 1e12, "TFLOP/s"
    else:
        peak, src = measured_peak("hbm_gbs")
        nbytes = wl.bytes() if hasattr(wl, "bytes") else wl.work()
        achieved, r_unit = nbytes / per_launch_s / 1e9, "GB/s"
    cpu = None
    # The CPU baseline is an N=1 figure (under torchrun the other ranks would
    # wait for it in the closing barrier).
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_sample(args.workload, steps=3, warmup=0)
        cpu.pop("seconds_per_step")
        # The reference's own harnesses time one thread; record that too.
        one = cpu_reference_sample(args.workload, steps=1, warmup=0, threads=1)
        cpu["value_1_thread"] = one["value"]
        cpu["cpu_model"] = cpu_model()
    if rank == 0:
        metric = metric_name(args.workload, wl.unit)
        line = {
            "metric": metric, "value": value, "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": getattr(wl, "kv_name", "bf16"), "data": "synthetic", "config": wl.config(world),
            **wl.extra(ms_max, world, args.steps),
            "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": r_unit,
                         "frac": achieved / peak, "peak_source": src,
                         "traffic": traffic_from_profile(args.workload),
                         "algorithmic_per_launch": wl.work()},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes(),
                    "d2h_bytes_per_step": wl.d2h_bytes(), "ms_per_step": e2e_ms_max / args.steps},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps,
        }
        print(json.dumps(line), flush=True)
    if pg:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg4",
                    choices=("cfg4", "cfg3", "cfg5-t512", "cfg5-t64", "scatter", "qkv-prefill",
                             "qkv-decode"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="decode requests per GPU (default: the workload's; smaller for profiling)")
    ap.add_argument("--kv-dtype", choices=("bf16", "f32"), default="bf16",
                    help="KV pool dtype of the decode workloads (configuration 3 is specified for both)")
    ap.add_argument("--ctx", type=int, default=None,
                    help="context length of cfg4 requests (default 32768)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local_rank = env_rank()
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
