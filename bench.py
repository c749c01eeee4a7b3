"""Benchmark of the sm_100a paged decode attention (fused KV write + split-K).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg4|cfg3]

One step = one launch of the fused KV-write + batched paged decode attention
kernel over one batch (one layer) of the workload:

* cfg4 (default): configuration 4 -- bf16 KV, 64 requests per GPU, every
  context 32768 tokens, 32 heads x 128 dims, block size 16, randomly
  permuted block tables; 34.4 GB of KV per GPU (larger than the 126 MB L2,
  so no flush is needed between steps).  Requests are sharded across GPUs
  (weak scaling: each rank owns 64 requests of the global 64*N batch).
* cfg3: configuration 3 at batch 256 -- ragged contexts ~U[1, 4096].

Under torchrun (N>1) each rank runs its shard on its own GPU; the only
collective is the all-reduce(MAX) of the timing.  Rank 0 prints one JSON
line.  ``--impl reference`` times the reference algorithm's CPU restatement
(oracle/, paged_attention_batch_online_v1 of minivllm) on the host cores
instead; under torchrun only rank 0 runs it.
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
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "mini-gpt-inference_b200"))

METRIC = ("paged decode attn HBM GB/s (% of 8 TB/s); decode tokens/sec at 1/2/4/8 B200")
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ workload
class Workload:
    def __init__(self, name: str, rank: int, world: int, device: torch.device,
                 batch: int | None = None, ctx: int | None = None):
        self.name = name
        self.H, self.D, self.S = 32, 128, 16
        self.kv_dtype = torch.bfloat16
        self.q_dtype = torch.bfloat16
        if name == "cfg4":
            self.B = batch or 64
            lens = [ctx or 32768] * self.B
            self.desc = (f"config 4: long-context split-K decode, bf16 KV, {self.B} requests/GPU "
                         f"x {lens[0]} tokens, H=32, D=128, S=16, fused KV write")
        elif name == "cfg3":
            self.B = batch or 256
            g = torch.Generator().manual_seed(1000 + rank)
            lens = torch.randint(1, 4097, (self.B,), generator=g).tolist()
            lens[0] = 1
            if lens[-1] % self.S == 0:
                lens[-1] -= 1
            self.desc = (f"config 3: ragged decode, bf16 KV, batch {self.B}/GPU, contexts "
                         "~U[1,4096], H=32, D=128, S=16, fused KV write")
        else:
            raise SystemExit(f"unknown workload {name}")
        self.lens = lens
        counts = [math.ceil(n / self.S) for n in lens]
        self.counts = counts
        P = sum(counts) + max(1, sum(counts) // 100)
        self.P = P
        g = torch.Generator(device=device).manual_seed(20260000 + rank)
        shape = (1, P, self.S, self.H, self.D)
        self.k = torch.empty(shape, dtype=self.kv_dtype, device=device)
        self.v = torch.empty(shape, dtype=self.kv_dtype, device=device)
        self.k.normal_(generator=g)
        self.v.normal_(generator=g)
        perm = torch.randperm(P, generator=g, device=device).cpu()
        M = max(counts)
        tables = torch.full((self.B, M), -1, dtype=torch.int64)
        nxt = 0
        for b, c in enumerate(counts):
            tables[b, :c] = perm[nxt:nxt + c]
            nxt += c
        self.tables_h = tables.pin_memory()
        self.lens_h = torch.tensor(lens, dtype=torch.int64).pin_memory()
        slots = [int(tables[b, (n - 1) // self.S]) * self.S + (n - 1) % self.S
                 for b, n in enumerate(lens)]
        self.slots_h = torch.tensor(slots, dtype=torch.int64).pin_memory()
        self.q_h = torch.randn((self.B, self.H, self.D), generator=torch.Generator().manual_seed(rank)
                               ).to(self.q_dtype).pin_memory()
        self.knew_h = torch.randn((self.B, self.H, self.D), generator=torch.Generator().manual_seed(rank + 1)
                                  ).to(self.kv_dtype).pin_memory()
        self.vnew_h = torch.randn((self.B, self.H, self.D), generator=torch.Generator().manual_seed(rank + 2)
                                  ).to(self.kv_dtype).pin_memory()
        self.tables = self.tables_h.to(device)
        self.ctx = self.lens_h.to(device)
        self.slots = self.slots_h.to(device)
        self.q = self.q_h.to(device)
        self.k_new = self.knew_h.to(device)
        self.v_new = self.vnew_h.to(device)
        self.out_h = torch.empty((self.B, self.H, self.D), dtype=self.q_dtype).pin_memory()

    @property
    def pool(self):
        from types import SimpleNamespace
        return SimpleNamespace(k=self.k, v=self.v, block_size=self.S)

    def bytes_per_step(self) -> int:
        from b200attn import decode_bytes
        return decode_bytes(self.lens, self.H, self.D, self.S, kv_bytes=2, q_bytes=2,
                            out_bytes=2, idx_bytes=8, fused_in_bytes=2)

    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.q_h, self.knew_h, self.vnew_h, self.tables_h, self.lens_h, self.slots_h))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices: list[int]):
        self.indices = indices
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.indices:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_indices(world: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(x) for x in vis.split(",") if x.strip().isdigit()]
        return ids[:world] if len(ids) >= world else ids
    return list(range(world))


# ------------------------------------------------------------------ CPU leg
def cpu_reference_sample(steps: int = 1, warmup: int = 0, requests: int = 1,
                         ctx: int = 32768) -> dict:
    """Times the reference decode algorithm (oracle port of
    paged_attention_batch_online_v1) on the host cores on a bounded sample:
    `requests` sequences of `ctx` tokens of the bench workload's shape."""
    sys.path.insert(0, str(REPO))
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    H, D, S = 32, 128, 16
    nb = math.ceil(ctx / S)
    g = torch.Generator().manual_seed(5)
    k = torch.randn((1, nb * requests, S, H, D), generator=g).to(torch.bfloat16)
    v = torch.randn((1, nb * requests, S, H, D), generator=g).to(torch.bfloat16)
    tables = torch.randperm(nb * requests, generator=g).view(requests, nb)
    lens = torch.full((requests,), ctx, dtype=torch.int64)
    q = torch.randn((requests, H, D), generator=g)
    # The reference cannot mix bf16 KV with fp32 q; the port upcasts the
    # (sample) pool to fp32 first, as the bf16 oracle does.
    kf, vf = k.float(), v.float()
    for _ in range(warmup):
        oracle.paged_decode_online(q, kf, vf, tables, lens, 0)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.paged_decode_online(q, kf, vf, tables, lens, 0)
        times.append(time.perf_counter() - t0)
    from b200attn.ops import decode_bytes
    nbytes = decode_bytes([ctx] * requests, H, D, S, kv_bytes=2, q_bytes=2, out_bytes=2)
    return {"seconds": times, "bytes": nbytes, "threads": threads,
            "sample": f"{requests} request(s) x {ctx} tokens, H=32, D=128, S=16, bf16 KV "
                      f"upcast to fp32, paged_attention_batch_online_v1 restatement (oracle/)"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    r = cpu_reference_sample(steps=args.steps, warmup=args.warmup, requests=1, ctx=32768)
    sec = sum(r["seconds"]) / len(r["seconds"])
    gbs = r["bytes"] / sec / 1e9
    line = {"metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "cfg4 sample on host CPU", "context_len": 32768,
                       "heads": 32, "head_dim": 128, "block_size": 16, "kv_dtype": "bf16"},
            "decode_tokens_per_s": 1.0 / sec,
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": r["threads"],
                             "kind": "port", "sample": r["sample"]},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg
def traffic_from_profile(workload: str) -> float | None:
    p = REPO / "profiles" / f"paged_decode_{workload}_traffic.json"
    try:
        d = json.loads(p.read_text())
        return float(d["dram_bytes_per_launch_full_size"])
    except Exception:
        return None


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch.distributed as dist
    from b200attn import paged_attention_batch_b200

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = world > 1
    if pg:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    wl = Workload(args.workload, rank, world, dev, args.batch, args.ctx)
    stream = torch.cuda.current_stream(dev)

    def step(q, k_new, v_new, tables, ctx, slots, out):
        return paged_attention_batch_b200(q, wl.pool, tables, ctx, 0, k_new=k_new, v_new=v_new,
                                          slot_mapping=slots, out=out)

    out = torch.empty((wl.B, wl.H, wl.D), dtype=wl.q_dtype, device=dev)
    with torch.inference_mode():
        for _ in range(args.warmup):
            step(wl.q, wl.k_new, wl.v_new, wl.tables, wl.ctx, wl.slots, out)
        torch.cuda.synchronize(dev)
        if pg:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(gpu_indices(world)) as clocks:
            ev0.record(stream)
            for _ in range(args.steps):
                step(wl.q, wl.k_new, wl.v_new, wl.tables, wl.ctx, wl.slots, out)
            ev1.record(stream)
            torch.cuda.synchronize(dev)
        ms = ev0.elapsed_time(ev1)
        if pg:
            dist.barrier()
        # End to end through the public API with host buffers: H2D of the
        # step's inputs from pinned memory, the call, D2H of the output and a
        # host synchronisation every step.
        torch.cuda.synchronize(dev)
        if pg:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            q = wl.q_h.to(dev, non_blocking=True)
            kn = wl.knew_h.to(dev, non_blocking=True)
            vn = wl.vnew_h.to(dev, non_blocking=True)
            tb = wl.tables_h.to(dev, non_blocking=True)
            cx = wl.lens_h.to(dev, non_blocking=True)
            sl = wl.slots_h.to(dev, non_blocking=True)
            o = step(q, kn, vn, tb, cx, sl, None)
            wl.out_h.copy_(o, non_blocking=True)
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    times = torch.tensor([ms, e2e_s * 1e3], dtype=torch.float64, device=dev)
    if pg:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms_max, e2e_ms_max = float(times[0]), float(times[1])
    clock = clocks.summary()
    bytes_step = wl.bytes_per_step()
    per_launch_ms = ms / args.steps  # this rank's own kernel time
    achieved = bytes_step / (per_launch_ms * 1e-3) / 1e9
    peak, peak_src = measured_peak()
    value = bytes_step * world * args.steps / (ms_max * 1e-3) / 1e9
    e2e_value = bytes_step * world * args.steps / (e2e_ms_max * 1e-3) / 1e9
    tok_s = wl.B * world * args.steps / (ms_max * 1e-3)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        r = cpu_reference_sample(steps=1, warmup=0, requests=1, ctx=32768)
        sec = sum(r["seconds"]) / len(r["seconds"])
        cpu = {"value": r["bytes"] / sec / 1e9, "unit": "GB/s", "cores": r["threads"],
               "kind": "port", "sample": r["sample"]}
    traffic = traffic_from_profile(args.workload)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": wl.desc, "batch_per_gpu": wl.B, "global_batch": wl.B * world,
                       "context_lens": str(wl.lens[0]) if args.workload == "cfg4" else "U[1,4096]",
                       "heads": wl.H, "head_dim": wl.D, "block_size": wl.S,
                       "kv_dtype": "bf16", "q_dtype": "bf16", "accumulate": "f32",
                       "fused_kv_write": True,
                       "l2": "inputs larger than L2 (KV pool %.1f GB per GPU), no flush"
                             % (2 * wl.k.numel() * wl.k.element_size() / 1e9),
                       "parallelism": f"request-sharded dp{world} (no data-path collective)"},
            "pct_of_8tbs": 100.0 * value / world / NOMINAL_HBM_GBS,
            "decode_tokens_per_s": tok_s,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src,
                         "traffic": traffic, "algorithmic_bytes_per_launch": bytes_step},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": wl.h2d_bytes(),
                    "d2h_bytes_per_step": wl.out_h.numel() * wl.out_h.element_size(),
                    "ms_per_step": e2e_ms_max / args.steps},
            "clocks": clock,
            "gpu_launches": args.steps,
        }
        print(json.dumps(line), flush=True)
    if pg:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("cfg4", "cfg3"), default="cfg4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="requests per GPU (default: the workload's; smaller for profiling)")
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
