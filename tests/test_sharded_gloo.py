"""Request sharding across ranks, on CPU gloo ranks (world size 2).

Each rank runs its shard of configuration 2 through the runtime harness
(oracle attention backend) with its own scheduler / block manager / pool,
then the finished token ids are all-gathered; the assembled outputs must
equal the reference runtime's golden tokens.  Failure detection is tested
on the host: a rank that raises, and a rank that exits without reporting,
must make the surviving rank raise instead of hanging.
"""
from __future__ import annotations

import json
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, out_dir: str) -> None:
    from b200attn.harness import MiniGPT, SequenceState, build_runtime, init_weights
    from b200attn.harness.sharded import run_sharded
    from e2e_common import CFG2, prompts
    from oracle_backend import OracleBackend

    torch.set_num_threads(2)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=30))
    reqs = [SequenceState(seq_id=f"r{i}", prompt_tokens=p, max_tokens=len(p) + CFG2["output_len"])
            for i, p in enumerate(prompts())]
    model = MiniGPT(n_embd=CFG2["n_embd"], n_head=CFG2["n_head"], vocab_size=CFG2["vocab"],
                    block_size=CFG2["pos"], n_layer=CFG2["n_layer"], backend=OracleBackend()).eval()
    init_weights(model, seed=0)

    def make_runtime(local):
        if mode == "raise" and rank == 1:
            raise ValueError("injected failure on rank 1")
        if mode == "vanish" and rank == 1:
            os._exit(0)  # exits without reporting, between steps
        blocks = sum(-(-(r.max_tokens - 1) // CFG2["block_size"]) for r in local)
        return build_runtime(model, num_blocks=blocks, block_size=CFG2["block_size"],
                             max_running=len(local), token_budget=CFG2["token_budget"],
                             policy="conservative", n_head=CFG2["n_head"],
                             head_dim=CFG2["n_embd"] // CFG2["n_head"])

    result = {}
    try:
        if mode == "drop_second":
            # A first call that every rank completes; rank 1 then leaves
            # before the second call.  Its "ok" from the first call must not
            # count for the second.
            reqs2 = [SequenceState(seq_id=r.seq_id, prompt_tokens=list(r.prompt_tokens),
                                   max_tokens=r.max_tokens) for r in reqs]
            run_sharded(reqs2, make_runtime, rank, world, torch.device("cpu"),
                        status_timeout_s=5.0)
            if rank == 1:
                os._exit(0)
        tokens, metrics = run_sharded(reqs, make_runtime, rank, world, torch.device("cpu"),
                                      status_timeout_s=5.0)
        result = {"tokens": {f"r{i}": t for i, t in tokens.items()}, "metrics": metrics}
    except Exception as exc:  # recorded for the parent to check
        result = {"error": f"{type(exc).__name__}: {exc}"}
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps(result))
    if "error" not in result:
        dist.destroy_process_group()


def _launch(mode: str, tmp_path) -> dict:
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    out = {}
    for r in range(2):
        f = Path(tmp_path, f"rank{r}.json")
        if f.exists():
            out[r] = json.loads(f.read_text())
    return out


def test_sharded_tokens_match_single_process_reference(tmp_path):
    from e2e_common import GOLDEN

    out = _launch("ok", tmp_path)
    want = GOLDEN["ample/sdpa_v2"]["tokens"]
    for r in (0, 1):
        assert out[r]["tokens"] == want, f"rank {r}"
    # Shards: rank 0 ran r0, r2; rank 1 ran r1, r3 (8 output tokens each).
    assert out[0]["metrics"]["output_tokens"] == 16 and out[1]["metrics"]["output_tokens"] == 16


def test_rank_failure_is_reported(tmp_path):
    out = _launch("raise", tmp_path)
    assert "injected failure" in out[1]["error"]
    assert "rank 1 failed" in out[0]["error"]


def test_vanished_rank_is_detected(tmp_path):
    out = _launch("vanish", tmp_path)
    assert 1 not in out
    assert "did not report" in out[0]["error"]


def test_rank_leaving_before_a_second_call_is_detected(tmp_path):
    out = _launch("drop_second", tmp_path)
    assert 1 not in out
    assert "did not report" in out[0]["error"]


def test_shard_assignment():
    from b200attn.harness.sharded import shard

    assert shard(list(range(10)), 1, 4) == [1, 5, 9]
    with pytest.raises(ValueError):
        shard([1, 2], 2, 2)
