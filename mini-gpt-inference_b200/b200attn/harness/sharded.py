"""Request-sharded multi-GPU serving: one process per GPU, NCCL only to gather tokens.

Decode attention has no cross-request term, so requests shard across ranks
with no data-path collective: rank r owns requests r, r + N, r + 2N, ...
and runs its own Scheduler, BlockManager and KV pool.  When its requests
finish, each rank posts its status to the process group's store and the
finished token ids are all-gathered (padded int64 tensors, NCCL on GPUs,
gloo on CPU ranks) so that rank 0 can assemble the outputs in request order.

Failure detection: a rank that fails posts "error" to the store; a rank that
dies or stalls posts nothing.  gather_outputs waits for every rank's status
with a deadline before entering the collective, so the surviving ranks
raise RuntimeError instead of blocking in the all-gather.

CLI (one process per GPU under torchrun):
    torchrun --nproc-per-node N -m b200attn.harness.sharded
runs configuration 2's requests sharded over the N GPUs and prints one JSON
line on rank 0 (per-request tokens, decode tokens/s).
"""
from __future__ import annotations

import json
import os
import time
from datetime import timedelta
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from .sequence import SequenceState

_STATUS_PREFIX = "b200attn/sharded/status"

# Calls of run_sharded / serve_shard made so far by this process.  Every rank
# makes the same calls in the same order, so the count names one call on all
# ranks; it is folded into the status keys so that a later call never sees
# the statuses an earlier call posted (a rank that dropped out of call 2
# would otherwise look alive through its "ok" of call 1).
_CALLS = 0


def _call_tag(tag: str) -> str:
    global _CALLS
    _CALLS += 1
    return f"{tag}#{_CALLS}"


def shard(items: Sequence, rank: int, world: int) -> list:
    """The items a rank owns: rank, rank + world, rank + 2*world, ..."""
    if not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    return list(items[rank::world])


def post_status(store, rank: int, ok: bool, message: str = "", tag: str = "") -> None:
    store.set(f"{_STATUS_PREFIX}{tag}/{rank}", ("ok" if ok else "error:" + message))


def wait_statuses(store, world: int, timeout_s: float, tag: str = "") -> None:
    """Raises RuntimeError naming the ranks that failed or never reported."""
    keys = [f"{_STATUS_PREFIX}{tag}/{r}" for r in range(world)]
    deadline = time.monotonic() + timeout_s
    missing = list(range(world))
    # The poll interval starts at 0.5 ms and grows to 2 ms: ranks of a
    # balanced shard finish within a few ms of each other, and every ms one
    # rank oversleeps here delays every rank's all-gather that follows (a
    # store check costs one local round trip, far less than the pause).
    pause = 0.0005
    while missing and time.monotonic() < deadline:
        still = []
        for r in missing:
            if store.check([keys[r]]):
                val = store.get(keys[r]).decode()
                if val.startswith("error:"):
                    raise RuntimeError(f"rank {r} failed: {val[6:]}")
            else:
                still.append(r)
        missing = still
        if missing:
            time.sleep(pause)
            pause = min(0.002, pause * 1.5)
    if missing:
        raise RuntimeError(f"ranks {missing} did not report within {timeout_s:.1f} s")


def gather_outputs(local: dict[int, list[int]], world: int, device: torch.device,
                   group=None) -> dict[int, list[int]]:
    """All-gathers {global request index: token ids} from every rank."""
    n_local = len(local)
    width = max((len(v) for v in local.values()), default=0)
    meta = torch.tensor([n_local, width], dtype=torch.int64, device=device)
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta, group=group)
    rows = max(int(m[0]) for m in metas)
    cols = max(int(m[1]) for m in metas)
    buf = torch.full((max(rows, 1), cols + 2), -1, dtype=torch.int64)
    for i, (idx, toks) in enumerate(sorted(local.items())):
        buf[i, 0] = idx
        buf[i, 1] = len(toks)
        buf[i, 2:2 + len(toks)] = torch.tensor(toks, dtype=torch.int64)
    buf = buf.to(device)
    bufs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf, group=group)
    out: dict[int, list[int]] = {}
    for b in bufs:
        b = b.cpu()
        for row in b:
            if int(row[0]) < 0:
                continue
            out[int(row[0])] = row[2:2 + int(row[1])].tolist()
    return out


class _Clock:
    """Phase timestamps: CUDA events on the device's current stream for a
    CUDA device (the device's own clock), perf_counter on the CPU."""

    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        self.device = device
        self.marks: list = []

    def mark(self) -> None:
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.marks.append(ev)
        else:
            self.marks.append(time.perf_counter())

    def ms(self, i: int, j: int) -> float:
        if self.cuda:
            torch.cuda.synchronize(self.device)
            return self.marks[i].elapsed_time(self.marks[j])
        return (self.marks[j] - self.marks[i]) * 1e3


def serve_shard(rt, local: Sequence[SequenceState], idx: Sequence[int], rank: int, world: int,
                device: torch.device, status_timeout_s: float = 60.0,
                tag: str = "") -> tuple[dict[int, list[int]], dict]:
    """Runs a built runtime over this rank's requests, then the status
    handshake and the token all-gather.

    local[i] is global request idx[i].  The returned metrics carry the
    runtime's metrics_summary plus ``run_ms`` (requests added until the
    last one finished), ``handshake_ms`` (the status handshake: waiting for
    every rank to finish) and ``gather_ms`` (the token all-gather), timed on
    the device for a CUDA device.
    """
    store = dist.distributed_c10d._get_default_store()
    tag = _call_tag(tag)
    clock = _Clock(device)
    metrics: dict = {}
    try:
        clock.mark()
        for r in local:
            rt.add_request(r)
        with torch.inference_mode():
            rt.run_to_completion(list(local))
        clock.mark()
        metrics = dict(rt.metrics_summary())
    except Exception as exc:
        post_status(store, rank, False, f"{type(exc).__name__}: {exc}", tag)
        raise
    post_status(store, rank, True, tag=tag)
    wait_statuses(store, world, status_timeout_s, tag)
    clock.mark()
    tokens = gather_outputs({i: list(r.generated_tokens) for i, r in zip(idx, local)}, world,
                            device)
    clock.mark()
    metrics["run_ms"] = clock.ms(0, 1)
    metrics["handshake_ms"] = clock.ms(1, 2)  # waiting for the slowest rank to finish
    metrics["gather_ms"] = clock.ms(2, 3)     # the all-gather itself
    metrics["wall_s"] = clock.ms(0, 3) / 1e3
    return tokens, metrics


def run_sharded(requests: Sequence[SequenceState], make_runtime: Callable[[list], object],
                rank: int, world: int, device: torch.device, status_timeout_s: float = 60.0,
                tag: str = "") -> tuple[dict[int, list[int]] | None, dict]:
    """Runs this rank's shard to completion and gathers every rank's tokens.

    make_runtime(local_requests) returns a MiniRuntime-like object with
    add_request / run_to_completion / metrics_summary.  Returns (tokens by
    global request index on every rank, local metrics).
    """
    idx = list(range(len(requests)))[rank::world]
    local = [requests[i] for i in idx]
    try:
        rt = make_runtime(local)
    except Exception as exc:
        store = dist.distributed_c10d._get_default_store()
        post_status(store, rank, False, f"{type(exc).__name__}: {exc}", _call_tag(tag))
        raise
    return serve_shard(rt, local, idx, rank, world, device, status_timeout_s, tag)


def _cfg2_main() -> None:
    from .model import MiniGPT, init_weights
    from .runtime import build_runtime

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator().manual_seed(0)
    lens = [128, 256, 128, 256]
    prompts = [torch.randint(0, 256, (p,), generator=g).tolist() for p in lens]
    reqs = [SequenceState(seq_id=f"r{i}", prompt_tokens=p, max_tokens=len(p) + 8)
            for i, p in enumerate(prompts)]
    model = MiniGPT(n_embd=256, n_head=8, vocab_size=256, block_size=296, n_layer=4).eval()
    init_weights(model, seed=0)
    model.to(dev)

    def make_runtime(local):
        blocks = sum(-(-(r.max_tokens - 1) // 16) for r in local)
        return build_runtime(model, num_blocks=max(blocks, 1), block_size=16,
                             max_running=max(len(local), 1), token_budget=64,
                             policy="conservative", n_head=8, head_dim=32)

    tokens, metrics = run_sharded(reqs, make_runtime, rank, world, dev)
    t = torch.tensor([metrics.get("wall_s", 0.0), float(metrics.get("output_tokens", 0))],
                     dtype=torch.float64, device=dev)
    wall = t.clone()
    dist.all_reduce(wall, op=dist.ReduceOp.MAX)
    total_out = t.clone()
    dist.all_reduce(total_out, op=dist.ReduceOp.SUM)
    if rank == 0:
        print(json.dumps({"world": world,
                          "tokens": {f"r{i}": tokens[i] for i in sorted(tokens)},
                          "output_tok_s": float(total_out[1]) / float(wall[0]),
                          "wall_s_max": float(wall[0])}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _cfg2_main()
