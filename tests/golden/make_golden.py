"""Generates the golden fixtures of the parity tests from the reference itself.

Run in a container where the reference checkout (zyyh-ops/mini-gpt-inference)
is importable:

    python tests/golden/make_golden.py --reference /path/to/mini-gpt-inference

It imports the reference's own functions -- paged_attention_batch_online_v1,
paged_attention_batch_reference, dense_gold, build_case and
KVCacheCausalSelfAttention.forward_prefill_chunk -- runs them on the
deterministic inputs of tests/golden/cases.py and writes
  decode_golden.npz / decode_golden.json    (decode outputs + input digests)
  prefill_golden.npz / prefill_golden.json  (prefill outputs, pool digests)
  e2e_golden.json                           (MiniRuntime greedy tokens and counts,
                                             configuration 2, ample and capped KV)
  qkv_golden.json / qkv_golden.npz          (pool digests and written K/V rows after
                                             the attention's own qkv projection + KV write)
It also checks that cases.py reproduces the reference's input builders
bit for bit.  The GPU box never runs this script; it only reads the files.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def decode_fixtures(ref) -> tuple[dict, dict]:
    from minivllm.paged_attention_batch import (paged_attention_batch_online_v1,
                                                paged_attention_batch_reference)
    from experiments.gpu_day6_fused_decode_ab import build_case, dense_gold
    from minivllm.kv_block_pool import KVBlockPool

    arrays, meta = {}, {}

    def record(c: cases.DecodeCase, with_reference: bool):
        pool = KVBlockPool(c.pool.k.shape[0], c.pool.k.shape[1], c.pool.block_size,
                           c.pool.k.shape[3], c.pool.k.shape[4])
        pool.k, pool.v = c.pool.k.clone(), c.pool.v.clone()
        with torch.inference_mode():
            online = paged_attention_batch_online_v1(c.q, pool, c.block_tables,
                                                     c.context_lengths, c.layer_idx)
            dense = dense_gold(c.q, pool, c.block_tables, c.context_lengths, c.layer_idx)
            arrays[f"{c.name}/online"] = online.numpy()
            arrays[f"{c.name}/dense"] = dense.numpy()
            if with_reference:
                per_req = paged_attention_batch_reference(c.q, pool, c.block_tables,
                                                          c.context_lengths, c.layer_idx)
                arrays[f"{c.name}/reference"] = per_req.numpy()
        meta[c.name] = {"digest": cases.case_digest(c)}

    # 1. unit-pool cases: the seed-2026 global-RNG setUp restated with a generator.
    torch.manual_seed(2026)
    pool = KVBlockPool(1, 4, 4, 2, 4)
    pool.k.copy_(torch.randn_like(pool.k))
    pool.v.copy_(torch.randn_like(pool.v))
    q = torch.randn(2, 2, 4)
    mine = cases.unit_pool_cases()
    assert cases.digest(q, pool.k, pool.v) == cases.digest(mine[2].q, mine[2].pool.k, mine[2].pool.v), \
        "unit_pool_cases does not reproduce tests/test_paged_attention.py inputs"
    for c in mine:
        record(c, True)

    # 2. NaN padding case (seed 11).
    torch.manual_seed(11)
    p2 = KVBlockPool(n_layer=1, num_blocks=3, block_size=4, n_head=2, head_dim=8)
    p2.k.fill_(float("nan"))
    p2.v.fill_(float("nan"))
    p2.k[0, 0, :2] = torch.randn(2, 2, 8)
    p2.v[0, 0, :2] = torch.randn(2, 2, 8)
    p2.k[0, 1, :4] = torch.randn(4, 2, 8)
    p2.v[0, 1, :4] = torch.randn(4, 2, 8)
    p2.k[0, 2, :1] = torch.randn(1, 2, 8)
    p2.v[0, 2, :1] = torch.randn(1, 2, 8)
    q2 = torch.randn(2, 2, 8)
    c = cases.nan_padding_case()
    assert cases.digest(q2, p2.k, p2.v) == cases.digest(c.q, c.pool.k, c.pool.v), \
        "nan_padding_case does not reproduce tests/test_paged_attention_padding.py inputs"
    record(c, True)

    # 3. build_case restatement: bit-exact against the reference builder.
    def ragged(**kw):
        mine = cases.ragged_case(**kw)
        q, p, t, l, layer = build_case(torch.device("cpu"), kw["batch"], kw["length"],
                                       kw["heads"], kw["dim"], kw["block_size"], kw["layout"],
                                       seed=kw["seed"], scale=kw["scale"])
        assert cases.digest(q, p.k, p.v, t, l) == cases.case_digest(mine), \
            f"ragged_case diverges from build_case for {kw}"
        assert layer == mine.layer_idx and q.stride() == mine.q.stride()
        return mine

    for bs, length in cases.RAGGED_CPU_SHAPES:
        record(ragged(batch=3, length=length, heads=4, dim=8, block_size=bs, layout="mixed",
                      seed=20261030, scale=0.3), False)
    for bs, length, batch, dim in cases.RAGGED_GPU_SHAPES:
        record(ragged(batch=batch, length=length, heads=8, dim=dim, block_size=bs,
                      layout="mixed", seed=20261030, scale=0.3), False)
    record(ragged(batch=2, length=65, heads=4, dim=32, block_size=16, layout="mixed",
                  seed=20261030, scale=8.0), False)
    for batch, length in cases.RAGGED_CORRECTNESS:
        record(ragged(batch=batch, length=length, heads=8, dim=32, block_size=16,
                      layout="mixed", seed=20261030 + batch + length, scale=0.3), False)

    # 4. configuration 1.
    record(cases.cfg1_case(), True)
    return arrays, meta


class _Fixed(torch.nn.Module):
    """Stands in for the fused QKV projection: returns a prepared [q|k|v]."""

    def __init__(self, qkv: torch.Tensor):
        super().__init__()
        self.out = qkv

    def forward(self, x):
        return self.out


def prefill_fixtures(ref) -> tuple[dict, dict]:
    from minivllm.attention import KVCacheCausalSelfAttention
    from minivllm.kv_block_pool import KVBlockPool
    from minivllm.kv_runtime import PrefillChunkContext
    from minivllm.sequence import SequenceState

    arrays, meta = {}, {}

    def run(c: cases.PrefillCase, mode: str):
        T, H, D = c.q.shape
        C = H * D
        attn = KVCacheCausalSelfAttention(C, H, block_size=4096).eval()
        attn.prefill_fastpath_enabled = mode != "reference"
        attn.prefill_prefix_fastpath_enabled = mode == "sdpa_v2"
        # [1, T, 3C] with q, k, v laid out as the module's chunk/view expects.
        qkv = torch.cat([c.q.reshape(T, C), c.k.reshape(T, C), c.v.reshape(T, C)], dim=-1)[None]
        attn.qkv = _Fixed(qkv)
        attn.project = torch.nn.Identity()
        pool = KVBlockPool(c.pool.k.shape[0], c.pool.k.shape[1], c.pool.block_size, H, D)
        pool.k, pool.v = c.pool.k.clone(), c.pool.v.clone()
        seq = SequenceState(seq_id="s", max_tokens=10**6, prompt_tokens=[0])
        seq.block_table = list(c.block_table)
        ctx = PrefillChunkContext(seq_state=seq, kv_pool=pool, layer_idx=c.layer_idx,
                                  start_pos=c.prefix_len, num_tokens=T, slot_mapping=c.slots)
        with torch.inference_mode():
            out = attn.forward_prefill_chunk(torch.zeros(1, T, C), ctx)
        return out.reshape(T, H, D), pool

    seed = 500
    shapes = [(4, 8, 4)] + [(8, 32, 16)]
    for H, D, S in shapes:
        for pieces in cases.PREFILL_PIECES:
            for prefix, T in cases.chunk_boundaries(pieces):
                seed += 1
                c = cases.prefill_case(prefix, T, H, D, S, seed)
                name = f"{c.name}_seed{seed}"
                if name in meta:
                    continue
                fast_mode = "sdpa_v2" if prefix > 0 else "sdpa_v1"
                out_fast, pool_after = run(c, fast_mode)
                out_ref, pool_after_ref = run(c, "reference")
                assert cases.digest(pool_after.k, pool_after.v) == \
                    cases.digest(pool_after_ref.k, pool_after_ref.v)
                arrays[f"{name}/sdpa"] = out_fast.numpy()
                arrays[f"{name}/reference"] = out_ref.numpy()
                meta[name] = {"prefix_len": prefix, "T": T, "H": H, "D": D, "S": S,
                              "seed": seed, "fast_mode": fast_mode,
                              "input_digest": cases.digest(c.q, c.k, c.v, c.pool.k, c.pool.v),
                              "pool_after_digest": cases.digest(pool_after.k, pool_after.v)}
    return arrays, meta


def qkv_fixtures(ref) -> dict:
    """Pool contents after the reference's own projection + KV write:
    KVCacheCausalSelfAttention.forward_prefill_chunk with its real qkv Linear
    (weights set from the case) on a first chunk (attention.py:177-208)."""
    from minivllm.attention import KVCacheCausalSelfAttention
    from minivllm.kv_block_pool import KVBlockPool
    from minivllm.kv_runtime import PrefillChunkContext
    from minivllm.sequence import SequenceState

    meta, arrays = {}, {}
    for T, H, D, S, seed in cases.QKV_CASES:
        c = cases.qkv_case(T, H, D, S, seed)
        C = H * D
        attn = KVCacheCausalSelfAttention(C, H, block_size=4096).eval()
        with torch.no_grad():
            attn.qkv.weight.copy_(c.w)
        attn.project = torch.nn.Identity()
        pool = KVBlockPool(c.pool.k.shape[0], c.pool.k.shape[1], S, H, D)
        pool.k, pool.v = c.pool.k.clone(), c.pool.v.clone()
        seq = SequenceState(seq_id="s", max_tokens=10**6, prompt_tokens=[0])
        seq.block_table = list(c.table)
        ctx = PrefillChunkContext(seq_state=seq, kv_pool=pool, layer_idx=c.layer_idx, start_pos=0,
                                  num_tokens=T, slot_mapping=c.slots)
        with torch.inference_mode():
            attn.forward_prefill_chunk(c.x[None], ctx)
        meta[c.name] = {"T": T, "H": H, "D": D, "S": S, "seed": seed,
                        "input_digest": cases.digest(c.x, c.w, c.pool.k, c.pool.v),
                        "pool_after_digest": cases.digest(pool.k, pool.v)}
        # The written rows themselves: fp32 matmul bits differ between host
        # CPUs, so the tests compare these values within fp32 tolerance.
        rows = torch.tensor(c.slots)
        arrays[f"{c.name}/k_rows"] = pool.k[c.layer_idx].reshape(-1, C)[rows].numpy()
        arrays[f"{c.name}/v_rows"] = pool.v[c.layer_idx].reshape(-1, C)[rows].numpy()
    return meta, arrays


CFG2 = {"n_embd": 256, "n_head": 8, "n_layer": 4, "vocab": 256, "pos": 296,
        "prompts": [128, 256, 128, 256], "output_len": 8, "block_size": 16,
        "token_budget": 64, "max_running": 4,
        "runs": {"ample": {"num_blocks": 52, "policy": "conservative"},
                 "capped": {"num_blocks": 26, "policy": "recompute"}}}


def cfg2_prompts() -> list[list[int]]:
    """Configuration 2 prompts: randint(0, 256) with one seed-0 generator."""
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, CFG2["vocab"], (p,), generator=g).tolist() for p in CFG2["prompts"]]


def e2e_fixtures(ref) -> dict:
    """Runs the reference MiniRuntime on configuration 2 (fp32, CPU)."""
    sys.path.insert(0, str(HERE.parents[1] / "mini-gpt-inference_b200"))
    from b200attn.harness.model import init_weights
    from minivllm.block_manager import BlockManager
    from minivllm.kv_block_pool import KVBlockPool
    from minivllm.mini_runtime import MiniRuntime
    from minivllm.model import MiniGPT
    from minivllm.model_runner import ModelRunner
    from minivllm.scheduler import Scheduler
    from minivllm.sequence import SequenceState, Status

    model = MiniGPT(n_embd=CFG2["n_embd"], n_head=CFG2["n_head"], vocab_size=CFG2["vocab"],
                    block_size=CFG2["pos"], dropout=0.0, n_layer=CFG2["n_layer"]).eval()
    init_weights(model, seed=0)
    prompts = cfg2_prompts()
    out = {"config": CFG2, "prompt_digest": cases.digest(*[torch.tensor(p) for p in prompts])}
    for run_name, run in CFG2["runs"].items():
        for prefill_mode in ("sdpa_v2", "reference"):
            model.set_prefill_fastpath_mode(prefill_mode)
            model.set_decode_attention_backend("reference")
            bm = BlockManager(run["num_blocks"], CFG2["block_size"])
            pool = KVBlockPool(CFG2["n_layer"], run["num_blocks"], CFG2["block_size"],
                               CFG2["n_head"], CFG2["n_embd"] // CFG2["n_head"])
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
            margins = []
            orig = rt.runner.decode_batch

            def probe(seqs, _orig=orig):
                logits, toks = _orig(seqs)
                top = torch.topk(logits, 2, dim=-1).values
                margins.extend((top[:, 0] - top[:, 1]).tolist())
                return logits, toks

            rt.runner.decode_batch = probe
            reqs = [SequenceState(seq_id=f"r{i}", prompt_tokens=p,
                                  max_tokens=len(p) + CFG2["output_len"])
                    for i, p in enumerate(prompts)]
            for r in reqs:
                rt.add_request(r)
            with torch.inference_mode():
                for _ in range(1000):
                    if all(r.status is Status.FINISHED for r in reqs):
                        break
                    rt.step()
            bm.check_invariants(reqs)
            summ = rt.metrics_summary()
            key = f"{run_name}/{prefill_mode}"
            out[key] = {
                "tokens": {r.seq_id: list(r.generated_tokens) for r in reqs},
                "counts": {k: summ[k] for k in ("iterations", "scheduled_tokens",
                                                "prefill_tokens", "decode_tokens",
                                                "output_tokens", "preemptions",
                                                "repeated_kv_tokens")},
                "min_decode_logit_margin": min(margins),
            }
            print(key, out[key]["counts"], "min margin", round(min(margins), 5))
        assert out[f"{run_name}/sdpa_v2"]["tokens"] == out[f"{run_name}/reference"]["tokens"]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", choices=("all", "qkv"), default="all",
                    help="regenerate every fixture, or only qkv_golden.json")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import minivllm  # noqa: F401  (fail early when the path is wrong)

    torch.set_num_threads(1)
    out = Path(args.out)
    qkv, qkv_arrays = qkv_fixtures(args.reference)
    (out / "qkv_golden.json").write_text(json.dumps(qkv, indent=1, sort_keys=True))
    np.savez_compressed(out / "qkv_golden.npz", **qkv_arrays)
    if args.only == "qkv":
        print("wrote", out / "qkv_golden.json")
        return
    arrays, meta = decode_fixtures(args.reference)
    np.savez_compressed(out / "decode_golden.npz", **arrays)
    (out / "decode_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    arrays, meta = prefill_fixtures(args.reference)
    np.savez_compressed(out / "prefill_golden.npz", **arrays)
    (out / "prefill_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    e2e = e2e_fixtures(args.reference)
    (out / "e2e_golden.json").write_text(json.dumps(e2e, indent=1, sort_keys=True))
    print("wrote fixtures to", out)


if __name__ == "__main__":
    main()
