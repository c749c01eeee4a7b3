"""Configuration-2 end-to-end workload shared by the CPU and GPU harness tests."""
from __future__ import annotations

import json
from pathlib import Path

import torch

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "e2e_golden.json").read_text())
CFG2 = GOLDEN["config"]


def prompts() -> list[list[int]]:
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, CFG2["vocab"], (p,), generator=g).tolist() for p in CFG2["prompts"]]


def run_cfg2(run_name: str, device: str, backend=None, mode: str = "eager",
             dtype: torch.dtype = torch.float32):
    """Runs configuration 2 through the harness; returns (tokens, counts, runtime).

    mode: "eager" (host-built metadata per step), "device_tables" (persistent
    device block tables) or "graphs" (device tables + CUDA-graph decode).
    dtype: weights and KV pool (the configuration is specified in fp32)."""
    if mode not in ("eager", "device_tables", "graphs"):
        raise ValueError(mode)
    from b200attn.harness import MiniGPT, SequenceState, build_runtime, init_weights

    model = MiniGPT(n_embd=CFG2["n_embd"], n_head=CFG2["n_head"], vocab_size=CFG2["vocab"],
                    block_size=CFG2["pos"], n_layer=CFG2["n_layer"], backend=backend).eval()
    init_weights(model, seed=0)
    model.to(device=device, dtype=dtype)
    run = CFG2["runs"][run_name]
    rt = build_runtime(model, num_blocks=run["num_blocks"], block_size=CFG2["block_size"],
                       max_running=CFG2["max_running"], token_budget=CFG2["token_budget"],
                       policy=run["policy"], n_head=CFG2["n_head"],
                       head_dim=CFG2["n_embd"] // CFG2["n_head"], kv_dtype=dtype,
                       device_tables=mode != "eager", graphs=mode == "graphs")
    rt.runner.kv_pool.k.fill_(float("nan"))  # unwritten KV must never be read
    rt.runner.kv_pool.v.fill_(float("nan"))
    reqs = [SequenceState(seq_id=f"r{i}", prompt_tokens=p, max_tokens=len(p) + CFG2["output_len"])
            for i, p in enumerate(prompts())]
    for r in reqs:
        rt.add_request(r)
    with torch.inference_mode():
        rt.run_to_completion(reqs, max_steps=1000)
    rt.block_manager.check_invariants(reqs)
    assert not rt.block_manager.block_owner and len(rt.block_manager.free_blocks) == run["num_blocks"]
    summ = rt.metrics_summary()
    counts = {k: summ[k] for k in GOLDEN[f"{run_name}/sdpa_v2"]["counts"]}
    return {r.seq_id: list(r.generated_tokens) for r in reqs}, counts, rt
