"""Decode throughput of the runtime harness on one GPU.

    python -m b200attn.harness.bench_runtime [--requests 64] [--prompt 1024]
        [--output 128] [--modes eager,device_tables,graphs]

Runs the same seeded workload through MiniRuntime once per mode (host-built
decode metadata, persistent device block tables, CUDA-graph decode) and
prints one JSON line per mode: decode tokens/s = decode tokens / summed
decode-phase wall time (the runtime synchronises the device around each
phase), the mean decode step time, and whether the greedy tokens equal the
first mode's.  Model: MiniGPT with n_embd = heads * 128 (head_dim 128), fp32
weights N(0, 0.02), fp32 KV, TF32 off; prompts are random token ids.
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from .model import MiniGPT, init_weights
from .runtime import build_runtime
from .sequence import SequenceState


def run_mode(mode: str, a) -> dict:
    torch.manual_seed(0)
    n_embd = a.heads * 128
    model = MiniGPT(n_embd=n_embd, n_head=a.heads, vocab_size=a.vocab,
                    block_size=a.prompt + a.output + 1, n_layer=a.layers).eval()
    init_weights(model, seed=0)
    model.to("cuda")
    g = torch.Generator().manual_seed(0)
    reqs = [SequenceState(seq_id=f"r{i}",
                          prompt_tokens=torch.randint(0, a.vocab, (a.prompt,), generator=g).tolist(),
                          max_tokens=a.prompt + a.output)
            for i in range(a.requests)]
    per_req = -(-(a.prompt + a.output) // a.block_size)
    rt = build_runtime(model, num_blocks=per_req * a.requests, block_size=a.block_size,
                       max_running=a.requests, token_budget=a.token_budget,
                       policy="conservative", n_head=a.heads, head_dim=128,
                       device_tables=mode != "eager", graphs=mode == "graphs")
    rt.sync_cuda_timing = True
    for r in reqs:
        rt.add_request(r)
    with torch.inference_mode():
        if mode == "graphs":
            rt.runner.graphs.capture_all()  # capture outside the timed steps
        t0 = time.perf_counter()
        rt.run_to_completion(reqs, max_steps=100_000)
    wall = time.perf_counter() - t0
    dec = [x for x in rt.records if x.decode_tokens > 0]
    dec_ms = sum(x.decode_ms for x in dec)
    dec_tok = sum(x.decode_tokens for x in dec)
    return {"mode": mode, "decode_tok_s": dec_tok / (dec_ms / 1e3) if dec_ms else 0.0,
            "decode_step_ms": dec_ms / max(len(dec), 1), "decode_steps": len(dec),
            "decode_tokens": dec_tok, "wall_s": wall,
            "tokens": [list(r.generated_tokens) for r in reqs]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=256)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--token-budget", type=int, default=2048)
    ap.add_argument("--modes", default="eager,device_tables,graphs")
    a = ap.parse_args()
    torch.backends.cuda.matmul.allow_tf32 = False
    first = None
    for mode in a.modes.split(","):
        r = run_mode(mode, a)
        toks = r.pop("tokens")
        first = toks if first is None else first
        r["tokens_equal_first_mode"] = toks == first
        r["config"] = {k: getattr(a, k) for k in ("requests", "prompt", "output", "heads",
                                                  "layers", "block_size")}
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
