"""Benchmark of the sm_100a paged-attention backend.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg4|cfg3|cfg5-t512|cfg5-t64|scatter|qkv-prefill|qkv-decode]
                    [--only]

One step = one launch of the hot path over one batch of the workload, with
inputs resident in HBM (``value``), and the same step through the public
Python API with the step's inputs copied from pinned host memory and its
result copied back, plus a host synchronisation (``e2e``).  Workloads:

* cfg4 (the headline): configuration 4 -- fused KV write + paged decode, bf16
  KV, 64 requests per GPU, every context 32768 tokens, 32 heads x 128 dims,
  block size 16, randomly permuted block tables; 37.8 GB of KV per GPU
  (larger than the 126 MB L2, so no flush is needed between steps).
* cfg3 / cfg3-f32: configuration 3 at batch 256 -- ragged contexts
  ~U[1, 4096], bf16 or fp32 KV.
* cfg5-t512 / cfg5-t64: configuration 5 -- one batched tcgen05 chunked
  prefill launch over 16 sequences, chunk 512 or 64 tokens, prefixes
  16*U{0..252}; the KV pool is ~2-4 GB (larger than L2).
* scatter: the slot-mapping KV scatter of 16 x 512 prefill tokens (bf16).
* qkv-prefill / qkv-decode: the attention's QKV projection with the KV write
  in its epilogue (tcgen05 GEMM), hidden 4096, over 8192 prefill tokens
  (TFLOP/s, tensor roofline) or 64 decode tokens (GB/s, HBM roofline: the
  100 MB weight read dominates); the object also carries the unfused
  sequence (cuBLAS matmul, then the scatter) timed in the same run.

The JSON line's top level is the --workload (default cfg4; weak scaling:
every rank owns 64 requests).  Unless --only is given, the same line also
carries
* ``workloads``: every other workload above, one sub-object each with its
  own ms_per_step, roofline, e2e and clocks;
* ``strong_scaling`` (cfg4): configuration 4 as specified, 64 requests in
  all, rank r owning requests r, r + N, ...;
* ``runtime``: decode tokens/s of request-sharded serving through the runtime
  harness, the NCCL all-gather of finished token ids inside the timed region.

Every N runs under a process group (a single-rank one at N=1); times are
taken on the device and reduced MAX over ranks, work is summed.  Rank 0
prints one JSON line.  ``--impl reference`` times the reference algorithm's
CPU restatement (oracle/: paged_attention_batch_online_v1, the SDPA v2
prefill, the KV write loop of minivllm) on the host cores instead; under
torchrun only rank 0 runs it.
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
    """Fused KV write + paged decode over one batch (configuration 4 or 3).

    Weak scaling (default): every rank owns ``batch`` requests.  With
    ``strong=True`` the batch is the global one and rank r owns requests
    r, r + world, ... of it (configuration 4 as specified: 64 requests in
    all, sharded by request).
    """

    bound, unit = "hbm", "GB/s"

    def __init__(self, name, rank, device, batch=None, ctx=None, kv_dtype="bf16",
                 world=1, strong=False):
        self.name, self.device = name, device
        self.kv_name = kv_dtype
        self.dt = torch.float32 if kv_dtype == "f32" else torch.bfloat16
        self.es = 4 if kv_dtype == "f32" else 2
        self.strong, self.world = strong, world
        if name == "cfg4":
            self.global_B = batch or 64
            lens = [ctx or 32768] * self.global_B
            per = "in all" if strong else "per GPU"
            self.desc = (f"config 4: long-context split-K decode, {kv_dtype} KV, {self.global_B}"
                         f" requests {per} x {lens[0]} tokens, H=32, D=128, S=16, fused KV write")
        else:
            self.global_B = batch or 256
            # Configuration 3: contexts ~U[1, 4096] (seed 0 on every rank, so
            # each rank of the weak-scaling run has the same work), the first
            # one 1 and the last one forced to a non-multiple of the block size.
            g = torch.Generator().manual_seed(0)
            lens = torch.randint(1, 4097, (self.global_B,), generator=g).tolist()
            lens[0] = 1
            if lens[-1] % S == 0:
                lens[-1] -= 1
            per = "in all" if strong else "per GPU"
            self.desc = (f"config 3: ragged decode, {kv_dtype} KV, batch {self.global_B} {per},"
                         " contexts ~U[1,4096], H=32, D=128, S=16, fused KV write")
        if strong:
            lens = lens[rank::world]
        self.B = len(lens)
        self.lens = lens
        counts = [math.ceil(n / S) for n in lens]
        # The pool holds the needed blocks plus 10 % spare (configuration 3's
        # sizing; configuration 4 uses the same rule).
        P = math.ceil(1.1 * sum(counts))
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
        glob = self.global_B if self.strong else self.B * world
        return {"workload": self.desc, "batch_per_gpu": self.B, "global_batch": glob,
                "context_lens": str(self.lens[0]) if self.name == "cfg4" else "U[1,4096]",
                "heads": H, "head_dim": D, "block_size": S, "kv_dtype": self.kv_name,
                "q_dtype": self.kv_name, "accumulate": "f32", "fused_kv_write": True,
                "l2": "inputs larger than L2 (KV pool %.1f GB per GPU), no flush" % self.kv_gb,
                "parallelism": f"request-sharded dp{world} (no data-path collective)"}

    def extra(self, value, ms_max, world, steps):
        glob = self.global_B if self.strong else self.B * world
        # One decode-attention launch serves one layer of one decode step of
        # every request in the batch: this is a per-layer attention rate, not
        # the runtime's decode tokens/s (that is the "runtime" object).
        return {"pct_of_8tbs": 100.0 * value / world / NOMINAL_HBM_GBS,
                "attention_launch_rows_per_s": glob * steps / (ms_max * 1e-3)}


class PrefillWorkload:
    """One batched tcgen05 chunked-prefill launch over 16 sequences (configuration 5)."""

    unit = "TFLOP/s"

    def __init__(self, T, rank, device, nseq=16):
        self.T, self.device, self.nseq = T, device, nseq
        self.bound = "tensor" if T >= 512 else "hbm"
        # The prefixes come from seed 0 on every rank (each rank of the
        # weak-scaling run has the same work); the tensors' values from the rank.
        self.prefix = (torch.randint(0, 253, (nseq,), generator=torch.Generator().manual_seed(0))
                       * 16).tolist()
        g = torch.Generator().manual_seed(rank)
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

    def extra(self, value, ms_max, world, steps):
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

    def extra(self, value, ms_max, world, steps):
        """A plain device copy of the same bytes (k and v into fresh tensors,
        torch ``copy_``), timed like the steps: the bandwidth a copy of this
        size reaches, below the measured peak, which comes from a 4 GB copy."""
        kd, vd = torch.empty_like(self.kn), torch.empty_like(self.vn)

        def copy():
            kd.copy_(self.kn)
            vd.copy_(self.vn)

        for _ in range(3):
            copy()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            copy()
        e1.record()
        torch.cuda.synchronize(self.device)
        ms = e0.elapsed_time(e1) / steps
        moved = 2 * (kd.numel() + vd.numel()) * kd.element_size()
        return {"same_bytes_copy": {"ms_per_step": round(ms, 5), "GB/s": round(moved / ms / 1e6, 1),
                                    "bytes": moved}}


class QkvWorkload:
    """The attention's QKV projection with the KV write in its epilogue
    (b200_qkv_kv_write), bf16, hidden 4096 (H=32, D=128): a prefill batch
    of 16 x 512 tokens (tensor-bound) or a decode batch of 64 tokens
    (bound by the 100 MB weight read).  Step i projects with layer i % LAYERS
    of LAYERS weight matrices and writes that layer's pool rows, as a
    model's forward does: 403 MB of weights, so no step finds its weights
    in the 126 MB L2 (one 100 MB matrix reused every step would mostly
    stay there)."""

    LAYERS = 4

    def __init__(self, name, rank, device):
        self.name, self.device = name, device
        self.T = 16 * 512 if name == "qkv-prefill" else 64
        self.C = H * D
        self.bound, self.unit = ("tensor", "TFLOP/s") if name == "qkv-prefill" else ("hbm", "GB/s")
        T, C = self.T, self.C
        g = torch.Generator().manual_seed(rank)
        gd = torch.Generator(device=device).manual_seed(40260000 + rank)
        P = T // S * 2
        self.k = torch.zeros((self.LAYERS, P, S, H, D), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.pool = SimpleNamespace(k=self.k, v=self.v, block_size=S)
        self.ws = [torch.empty((3 * C, C), dtype=torch.bfloat16, device=device)
                   .normal_(0.0, 0.02, generator=gd) for _ in range(self.LAYERS)]
        self.i = self.j = 0
        self.x_h = torch.randn((T, C), generator=g).to(torch.bfloat16).pin_memory()
        self.slots_h = torch.randperm(P * S, generator=g)[:T].pin_memory()
        self.x, self.slots = self.x_h.to(device), self.slots_h.to(device)
        self.q_h = torch.empty((T, C), dtype=torch.bfloat16).pin_memory()
        self.desc = (f"fused QKV projection + KV write (tcgen05), bf16, {T} tokens, hidden {C}"
                     f" (H=32, D=128), weight [3C, C], S=16")

    def prepare(self):
        from b200attn import qkv_kv_write_b200
        self.calls = [qkv_kv_write_b200(self.x, w, self.pool, self.slots, layer, prepare=True)
                      for layer, w in enumerate(self.ws)]

    def step(self):
        self.calls[self.i % self.LAYERS]()
        self.i += 1

    def e2e_step(self):
        from b200attn import qkv_kv_write_b200
        layer = self.j % self.LAYERS
        self.j += 1
        q = qkv_kv_write_b200(self.x_h.to(self.device, non_blocking=True), self.ws[layer], self.pool,
                              self.slots_h.to(self.device, non_blocking=True), layer)
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
                "l2": "%d weight matrices of %.0f MB cycled step by step (%.0f MB, larger than L2);"
                      " no flush" % (self.LAYERS, 3 * self.C * self.C * 2 / 1e6,
                                     self.LAYERS * 3 * self.C * self.C * 2 / 1e6),
                "parallelism": f"token-sharded dp{world}"}

    def extra(self, value, ms_max, world, steps):
        """The unfused sequence the kernel replaces, timed the same way:
        torch's bf16 matmul (cuBLAS) into a [T, 3C] tensor, then the
        slot-mapping scatter of its k and v thirds (a prepared call), cycling
        over the layers like the steps.  The ``cuda_graph`` entry times the
        fused call and both unfused sequences as CUDA graphs of 12 calls
        (three passes over the layers), device time without host overhead,
        which at decode sizes is larger than the kernels themselves."""
        from b200attn import kv_scatter_b200
        T, C = self.T, self.C
        dev = self.device
        y = torch.empty((T, 3 * C), dtype=torch.bfloat16, device=dev)
        with torch.inference_mode():
            scatter_calls = [kv_scatter_b200(y[:, C:2 * C].view(T, H, D), y[:, 2 * C:].view(T, H, D),
                                             self.pool, self.slots, layer, prepare=True)
                             for layer in range(self.LAYERS)]
        turn = [0]

        def unfused(scatter):
            layer = turn[0] % self.LAYERS
            turn[0] += 1
            torch.matmul(self.x, self.ws[layer].t(), out=y)
            if scatter:
                scatter_calls[layer]()

        def graph_ms(fn, calls=12, reps=20):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(3):
                    fn()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(calls):
                    fn()
            graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / (reps * calls)
            del graph
            return ms

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
                torch.cuda.synchronize(dev)
                ms = e0.elapsed_time(e1) / steps
                key = "cublas_matmul_plus_scatter" if scatter else "cublas_matmul_alone"
                res[key] = {"ms_per_step": ms,
                            "value": self.work() / (ms * 1e-3) / (1e12 if self.bound == "tensor" else 1e9),
                            "unit": self.unit}
            res["cuda_graph"] = {"fused_ms_per_call": graph_ms(self.step),
                                 "cublas_matmul_alone_ms_per_call": graph_ms(lambda: unfused(False)),
                                 "cublas_matmul_plus_scatter_ms_per_call": graph_ms(lambda: unfused(True))}
        res["fused_ms_per_step"] = ms_max / steps
        return {"unfused_comparison": res}


def make_workload(name, rank, device, args, extra=False):
    """The workload of ``name``; ``extra`` builds it at its default size
    (the sub-objects of the default run ignore --batch / --ctx / --kv-dtype)."""
    if name in ("cfg4", "cfg3", "cfg3-f32"):
        kv = "f32" if name == "cfg3-f32" else ("bf16" if extra else args.kv_dtype)
        batch = None if extra else args.batch
        ctx = None if extra else args.ctx
        wl = DecodeWorkload(name.split("-")[0], rank, device, batch, ctx, kv)
        # ncu traffic: configuration 3's captured DRAM/algorithmic ratio (bf16
        # KV, any batch); configuration 4's full-size bytes (its default shape).
        if name.startswith("cfg3"):
            wl.traffic_key = "cfg3" if kv == "bf16" else None
        else:
            wl.traffic_key = "cfg4" if kv == "bf16" and wl.B == 64 and wl.lens[0] == 32768 \
                else None
        return wl
    if name == "cfg5-t512":
        return PrefillWorkload(512, rank, device)
    if name == "cfg5-t64":
        return PrefillWorkload(64, rank, device)
    if name == "scatter":
        return ScatterWorkload(rank, device)
    if name in ("qkv-prefill", "qkv-decode"):
        wl = QkvWorkload(name, rank, device)
        wl.traffic_key = name
        return wl
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
        """Opens a new timed window (one per workload); summary() reports
        the most recent one."""
        self._t0 = time.perf_counter()
        self._t1 = None

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


def traffic_from_profile(workload: str | None, algorithmic: float) -> float | None:
    """ncu DRAM bytes per launch of a workload at its full size, from the
    committed profile summary, or None when none was captured for it.  A
    summary holds either the full-size figure or the ratio of captured DRAM
    bytes to algorithmic bytes (applied to this launch's algorithmic bytes)."""
    if workload not in TRAFFIC_FILES:
        return None
    p = REPO / "profiles" / TRAFFIC_FILES[workload]
    try:
        d = json.loads(p.read_text())
        if "dram_over_algorithmic" in d:
            return float(d["dram_over_algorithmic"]) * algorithmic
        return float(d["dram_bytes_per_launch_full_size"])
    except Exception:
        return None


class RuntimeWorkload:
    """Request-sharded serving through the runtime harness (decode tokens/s).

    64 requests in all (1024-token prompts of random ids, 128 greedy outputs
    each) over a random-init MiniGPT with 8 heads of 128 dims, 4 layers,
    fp32 weights and KV, TF32 off; rank r serves requests r, r + N, ... with
    its own scheduler, block manager and KV pool, device block tables and
    CUDA-graph decode steps.  The timed region runs from the first request's
    admission to the end of the NCCL all-gather of every rank's finished
    token ids (b200attn.harness.sharded.serve_shard), on the device clock,
    max over ranks.
    """

    def __init__(self, rank, world, device, requests=64, prompt=1024, output=128, heads=8,
                 layers=4, vocab=256, block_size=16, token_budget=2048):
        from b200attn.harness import MiniGPT, SequenceState, init_weights

        self.rank, self.world, self.device = rank, world, device
        self.requests, self.prompt, self.output = requests, prompt, output
        self.heads, self.layers, self.block_size = heads, layers, block_size
        self.token_budget = token_budget
        torch.backends.cuda.matmul.allow_tf32 = False
        self.model = MiniGPT(n_embd=heads * 128, n_head=heads, vocab_size=vocab,
                             block_size=prompt + output + 1, n_layer=layers).eval()
        init_weights(self.model, seed=0)
        self.model.to(device)
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, vocab, (prompt,), generator=g).tolist()
                   for _ in range(requests)]
        self.idx = list(range(requests))[rank::world]
        self.local = [SequenceState(seq_id=f"r{i}", prompt_tokens=prompts[i],
                                    max_tokens=prompt + output) for i in self.idx]
        self.desc = (f"sharded runtime: {requests} requests in all x {prompt}-token prompts ->"
                     f" {output} outputs, MiniGPT {heads} heads x 128 dims, {layers} layers, fp32,"
                     " device block tables + CUDA-graph decode, NCCL all-gather of token ids")

    def _runtime(self, n_local):
        from b200attn.harness import build_runtime

        per_req = -(-(self.prompt + self.output) // self.block_size)
        rt = build_runtime(self.model, num_blocks=per_req * max(n_local, 1),
                           block_size=self.block_size, max_running=max(n_local, 1),
                           token_budget=self.token_budget, policy="conservative",
                           n_head=self.heads, head_dim=128, device_tables=True, graphs=True)
        rt.sync_cuda_timing = True
        return rt

    def run(self) -> dict:
        import hashlib
        import torch.distributed as dist
        from b200attn.harness import SequenceState
        from b200attn.harness.sharded import serve_shard

        rt = self._runtime(len(self.local))
        with torch.inference_mode():
            rt.runner.graphs.capture_all()
            # Warm-up: two short requests through the same runtime (cuBLAS
            # handles, allocator); their blocks return to the free list.
            warm = [SequenceState(seq_id=f"w{i}", prompt_tokens=[1 + i] * 40, max_tokens=48)
                    for i in range(2)]
            for r in warm:
                rt.add_request(r)
            rt.run_to_completion(warm)
        rt.records.clear()
        # One untimed all-gather of the timed one's shape: NCCL sets up a
        # collective's connections on its first use, a one-time cost that
        # is not the steady-state gather.
        from b200attn.harness.sharded import gather_outputs
        gather_outputs({i: [0] * self.output for i in self.idx}, self.world, self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier()
        tokens, m = serve_shard(rt, self.local, self.idx, self.rank, self.world, self.device,
                                status_timeout_s=120.0, tag="bench")
        dec = [x for x in rt.records if x.decode_tokens > 0]
        launches = sum(self.layers for x in rt.records if x.decode_tokens > 0) + \
            sum(2 * self.layers * x.prefill_requests for x in rt.records)
        local = torch.tensor([m["wall_s"] * 1e3, m["run_ms"], m["handshake_ms"], m["gather_ms"],
                              sum(x.decode_ms for x in dec)], dtype=torch.float64,
                             device=self.device)
        counts = torch.tensor([m["output_tokens"], m["decode_tokens"], m["prefill_tokens"],
                               launches], dtype=torch.float64, device=self.device)
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        total_ms, run_ms, handshake_ms, gather_ms, dec_ms = (float(x) for x in local)
        out_tok, dec_tok, pre_tok, launches = (float(x) for x in counts)
        digest = hashlib.sha256(json.dumps([tokens[i] for i in sorted(tokens)]).encode())
        return {
            "workload": self.desc,
            "decode_tokens_per_s": dec_tok / (dec_ms * 1e-3) if dec_ms else None,
            "output_tokens_per_s": out_tok / (total_ms * 1e-3),
            "timed_ms": total_ms, "run_ms_max": run_ms, "handshake_ms_max": handshake_ms,
            "gather_ms_max": gather_ms,
            "decode_phase_ms_max": dec_ms, "output_tokens": out_tok, "decode_tokens": dec_tok,
            "prefill_tokens": pre_tok, "requests_per_gpu": len(self.local),
            "gpu_launches": int(launches),
            "tokens_sha256": digest.hexdigest(), "requests_finished": len(tokens),
            "timing": "device events on the serving stream, max over ranks; decode_phase_ms is"
                      " the runtime's per-step decode phases (host clock around a device sync)",
        }


def _barrier(dist_on: bool) -> None:
    if dist_on:
        import torch.distributed as dist
        dist.barrier()


def time_workload(wl, args, dev, clocks) -> dict:
    """Warm-up, K device-timed steps and K end-to-end steps of one workload;
    the times are reduced MAX and the work SUM over ranks."""
    import torch.distributed as dist

    stream = torch.cuda.current_stream(dev)
    wl.prepare()
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize(dev)
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
    clk = clocks.summary()
    dist.barrier()
    # End to end through the public API: H2D of the step's inputs from pinned
    # memory, the call, D2H of the result, a host synchronisation per step.
    for _ in range(2):
        wl.e2e_step()
    stream.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        wl.e2e_step()
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    dist.all_reduce(times, op=dist.ReduceOp.MAX)
    work = torch.tensor([wl.work()], dtype=torch.float64, device=dev)
    dist.all_reduce(work, op=dist.ReduceOp.SUM)
    return {"ms": ms, "ms_max": float(times[0]), "e2e_ms_max": float(times[1]),
            "work_sum": float(work[0]), "clocks": clk}


def summarize(wl, r: dict, args, world: int) -> dict:
    """The JSON fields of one timed workload."""
    K = args.steps
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = r["work_sum"] * K / (r["ms_max"] * 1e-3) / scale
    e2e_value = r["work_sum"] * K / (r["e2e_ms_max"] * 1e-3) / scale
    per_launch_s = r["ms"] * 1e-3 / K  # this rank's own kernel time
    if wl.bound == "tensor":
        peak, src = measured_peak("bf16_tflops")
        achieved, r_unit = wl.flops() / per_launch_s / 1e12, "TFLOP/s"
    else:
        peak, src = measured_peak("hbm_gbs")
        nbytes = wl.bytes() if hasattr(wl, "bytes") else wl.work()
        achieved, r_unit = nbytes / per_launch_s / 1e9, "GB/s"
    return {
        "value": value, "unit": wl.unit, "ms_per_step": r["ms_max"] / K,
        "config": wl.config(world), **wl.extra(value, r["ms_max"], world, K),
        "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": r_unit,
                     "frac": achieved / peak, "peak_source": src,
                     "traffic": traffic_from_profile(getattr(wl, "traffic_key", None), wl.work()),
                     "algorithmic_per_launch": wl.work()},
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes(),
                "d2h_bytes_per_step": wl.d2h_bytes(), "ms_per_step": r["e2e_ms_max"] / K},
        "clocks": r["clocks"], "gpu_launches": K,
    }


# The workloads the default run times besides the headline one, each reported
# as a sub-object of the JSON line: configuration 3 (batch 256, bf16 and fp32
# KV), configuration 5 (chunks 512 and 64), the prefill scatter and the fused
# QKV projection at prefill and decode sizes.
EXTRA_WORKLOADS = ("cfg3", "cfg3-f32", "cfg5-t512", "cfg5-t64", "scatter", "qkv-prefill",
                   "qkv-decode")


def _free(dev) -> None:
    import gc
    gc.collect()
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    # One process group at every N (a single-rank one at N=1), so that every
    # N runs the same code: barriers, the MAX/SUM reductions of the timings
    # and the runtime's NCCL token gather.
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    else:
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                timeout=timedelta(seconds=180), device_id=dev)
    with torch.inference_mode(), ClockSampler(gpu_indices(world)) as clocks:
        wl = make_workload(args.workload, rank, dev, args)
        head = summarize(wl, time_workload(wl, args, dev, clocks), args, world)
        head_desc = wl.config(world)
        del wl
        _free(dev)
        extras = {}
        if not args.only:
            if args.workload == "cfg4":
                # Configuration 4 as specified: 64 requests in all, rank r
                # owning requests r, r + N, ... (strong scaling).
                if world > 1:
                    wl = DecodeWorkload("cfg4", rank, dev, batch=args.batch, ctx=args.ctx,
                                        kv_dtype=args.kv_dtype, world=world, strong=True)
                    strong = summarize(wl, time_workload(wl, args, dev, clocks), args, world)
                    del wl
                    _free(dev)
                else:
                    strong = {k: head[k] for k in ("value", "unit", "ms_per_step", "e2e")}
                    strong["same_as_headline"] = True
                strong["scaling"] = "strong"
                extras["strong_scaling"] = strong
            for name in EXTRA_WORKLOADS:
                if name == args.workload and args.kv_dtype == "bf16":
                    continue
                wl = make_workload(name, rank, dev, args, extra=True)
                extras.setdefault("workloads", {})[name] = \
                    summarize(wl, time_workload(wl, args, dev, clocks), args, world)
                del wl
                _free(dev)
            rw = RuntimeWorkload(rank, world, dev)
            extras["runtime"] = rw.run()
            del rw
            _free(dev)
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
        line = {
            "metric": metric_name(args.workload, head["unit"]), "value": head["value"],
            "unit": head["unit"], "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.kv_dtype if args.workload in ("cfg4", "cfg3")
            else "bf16", "data": "synthetic", "config": head_desc,
            **{k: v for k, v in head.items() if k not in ("value", "unit", "ms_per_step",
                                                          "config")},
            "cpu_baseline": cpu,
            **extras,
        }
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--only", action="store_true",
                    help="time the named workload alone (no sub-workloads, strong-scaling or"
                         " runtime objects)")
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
