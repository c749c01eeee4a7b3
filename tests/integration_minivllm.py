"""Runs minivllm itself with the sm100 host diff applied -- TEST INFRASTRUCTURE.

    python tests/integration_minivllm.py --reference <minivllm checkout> --workdir <tmp dir>

Copies the checkout's ``minivllm`` package into the work directory, applies
``mini-gpt-inference_b200/integration/minivllm_sm100.patch`` to the copy
(insertion-only hunks, applied here without external tools) and imports the
patched package.  The b200attn entry points the diff calls are replaced by
CPU stand-ins built on the oracle, which also check how the diff calls them:

* decode: q/k_new/v_new are [B, H, D]; the reference's own KV index_put
  (attention.py:382-392) has NOT run before the call (the rows at the slots
  do not hold k_new yet); the stand-in writes k_new/v_new at the slots and
  attends with the online-softmax restatement;
* prefill: the scatter gets [T, H, D] k/v and T slots; the chunk attention
  gets [T, H, D] q and reads the chunk's own K/V back from the pool (so a
  scatter that did not run first gives wrong tokens).

Configuration 2 then runs through the reference's own MiniGPT, ModelRunner,
Scheduler, BlockManager and MiniRuntime (fp32, CPU, ample and capped KV,
recompute preemption) with the backends under test, and one JSON object with
the greedy tokens, lifecycle counts and stand-in call counts per run is
printed.  tests/test_integration_minivllm.py compares it with the golden
tokens and counts the reference produced with its own backends.
"""
from __future__ import annotations

import argparse
import json
import re
import shutil
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[1]
PATCH = REPO / "mini-gpt-inference_b200" / "integration" / "minivllm_sm100.patch"


def apply_insertions(patch_text: str, root: Path) -> int:
    """Applies a unified diff whose hunks only insert lines (zero context,
    ``@@ -N,0 +M,K @@``: K lines after old line N).  Returns the hunk count."""
    files: dict[str, list[tuple[int, list[str]]]] = {}
    current = None
    hunk = None
    for line in patch_text.splitlines():
        if line.startswith("+++ "):
            current = line[4:].strip()
            current = current[2:] if current.startswith("b/") else current
            files[current] = []
        elif line.startswith("@@"):
            m = re.match(r"@@ -(\d+),0 \+\d+,(\d+) @@", line)
            if m is None:
                raise ValueError(f"not an insertion-only hunk: {line}")
            hunk = (int(m.group(1)), [])
            files[current].append(hunk)
        elif hunk is not None and line.startswith("+") and not line.startswith("+++"):
            hunk[1].append(line[1:])
    count = 0
    for rel, hunks in files.items():
        path = root / rel
        lines = path.read_text().split("\n")
        for after, block in sorted(hunks, key=lambda h: -h[0]):  # bottom-up
            lines[after:after] = block
            count += 1
        path.write_text("\n".join(lines))
    return count


class StandIns:
    """Oracle-backed CPU stand-ins for the b200attn entry points."""

    def __init__(self, oracle):
        self.oracle = oracle
        self.calls = {"decode": 0, "scatter": 0, "prefill": 0}

    def paged_attention_batch_b200(self, q, pool, block_tables, context_lengths, layer_idx, *,
                                   k_new=None, v_new=None, slot_mapping=None, **_):
        self.calls["decode"] += 1
        B, H, D = q.shape
        assert pool.k.shape[2:] == (pool.block_size, H, D)
        assert block_tables.shape[0] == B and context_lengths.shape == (B,)
        assert k_new is not None and v_new is not None and slot_mapping is not None, \
            "the sm100 decode branch must hand the new K/V to the kernel"
        assert k_new.shape == v_new.shape == (B, H, D) and slot_mapping.shape == (B,)
        S = pool.block_size
        for b, slot in enumerate(slot_mapping.tolist()):
            pos = int(context_lengths[b]) - 1  # the new token is the last context position
            assert slot == int(block_tables[b, pos // S]) * S + pos % S
            assert not torch.equal(pool.k[layer_idx, slot // S, slot % S], k_new[b]), \
                "the reference's KV index_put ran before the sm100 call"
        self.oracle.kv_scatter(pool.k, pool.v, k_new, v_new, slot_mapping, layer_idx)
        return self.oracle.paged_decode_online(q, pool.k, pool.v, block_tables,
                                               context_lengths, layer_idx).to(q.dtype)

    def kv_scatter_b200(self, k, v, pool, slot_mapping, layer_idx, **_):
        self.calls["scatter"] += 1
        N, H, D = k.shape
        assert v.shape == (N, H, D) and pool.k.shape[3:] == (H, D)
        assert len(slot_mapping) == N
        self.oracle.kv_scatter(pool.k, pool.v, k, v, slot_mapping, layer_idx)

    def chunked_prefill_b200(self, q, pool, block_table, prefix_len, layer_idx, **_):
        self.calls["prefill"] += 1
        T, H, D = q.shape
        table = [int(x) for x in block_table]
        assert len(table) * pool.block_size >= prefix_len + T
        return self.oracle.prefix_prefill_from_pool(q, pool.k, pool.v, table, prefix_len,
                                                    layer_idx).to(q.dtype)


RUNS = [("ample", "sm100", "sm100"), ("capped", "sm100", "sm100"),
        ("capped", "sm100", "reference"), ("capped", "sdpa_v2", "sm100")]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--workdir", required=True)
    a = ap.parse_args()
    work = Path(a.workdir)
    shutil.copytree(Path(a.reference) / "minivllm", work / "minivllm")
    hunks = apply_insertions(PATCH.read_text(), work)
    for p in (REPO / "tests", REPO / "mini-gpt-inference_b200", REPO, work):
        sys.path.insert(0, str(p))
    import b200attn
    import oracle
    from e2e_common import CFG2, prompts
    from b200attn.harness.model import init_weights
    from minivllm.block_manager import BlockManager
    from minivllm.kv_block_pool import KVBlockPool
    from minivllm.mini_runtime import MiniRuntime
    from minivllm.model import MiniGPT
    from minivllm.model_runner import ModelRunner
    from minivllm.scheduler import Scheduler
    from minivllm.sequence import SequenceState, Status

    assert Path(sys.modules["minivllm"].__file__).resolve().is_relative_to(work.resolve())
    torch.set_num_threads(4)
    torch.backends.cuda.matmul.allow_tf32 = False
    stand = StandIns(oracle)
    for name in ("paged_attention_batch_b200", "kv_scatter_b200", "chunked_prefill_b200"):
        setattr(b200attn, name, getattr(stand, name))
    model = MiniGPT(n_embd=CFG2["n_embd"], n_head=CFG2["n_head"], vocab_size=CFG2["vocab"],
                    block_size=CFG2["pos"], dropout=0.0, n_layer=CFG2["n_layer"]).eval()
    init_weights(model, seed=0)
    out = {"hunks": hunks, "runs": {}}
    for run_name, prefill_mode, decode_backend in RUNS:
        run = CFG2["runs"][run_name]
        model.set_prefill_fastpath_mode(prefill_mode)
        model.set_decode_attention_backend(decode_backend)
        bm = BlockManager(run["num_blocks"], CFG2["block_size"])
        pool = KVBlockPool(CFG2["n_layer"], run["num_blocks"], CFG2["block_size"], CFG2["n_head"],
                           CFG2["n_embd"] // CFG2["n_head"])
        pool.k.fill_(float("nan"))  # unwritten KV must never be read
        pool.v.fill_(float("nan"))
        # Built as the reference's own tests build a small runtime
        # (MiniRuntime.__init__ makes its own fixed-size model).
        rt = MiniRuntime.__new__(MiniRuntime)
        rt.block_manager = bm
        rt.scheduler = Scheduler(bm, max_running=CFG2["max_running"],
                                 max_num_batched_tokens=CFG2["token_budget"],
                                 preemption_policy=run["policy"])
        rt.runner = ModelRunner(model, pool, bm)
        rt.iteration = 0
        rt.records = []
        rt.sync_cuda_timing = False
        rt.verbose = False
        rt._kv_high_watermark = {}
        reqs = [SequenceState(seq_id=f"r{i}", prompt_tokens=p,
                              max_tokens=len(p) + CFG2["output_len"])
                for i, p in enumerate(prompts())]
        for r in reqs:
            rt.add_request(r)
        before = dict(stand.calls)
        with torch.inference_mode():
            for _ in range(1000):
                if all(r.status is Status.FINISHED for r in reqs):
                    break
                rt.step()
        bm.check_invariants(reqs)
        summ = rt.metrics_summary()
        out["runs"][f"{run_name}/{prefill_mode}/{decode_backend}"] = {
            "tokens": {r.seq_id: list(r.generated_tokens) for r in reqs},
            "counts": {k: summ[k] for k in ("iterations", "scheduled_tokens", "prefill_tokens",
                                            "decode_tokens", "output_tokens", "preemptions",
                                            "repeated_kv_tokens")},
            "calls": {k: stand.calls[k] - before[k] for k in stand.calls},
        }
    print(json.dumps(out))


if __name__ == "__main__":
    main()
