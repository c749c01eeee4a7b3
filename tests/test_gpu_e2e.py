"""End to end on the GPU: configuration 2 through the runtime harness with the
sm_100a kernels (fused KV-write decode, scatter, chunked prefill), fp32 with
TF32 off.  Greedy tokens and lifecycle counts must equal the reference
MiniRuntime's, with ample KV and with capped KV (recompute preemption), for
host-built decode metadata, persistent device block tables, and CUDA-graph
replay of the decode step."""
from __future__ import annotations

import pytest
import torch

from e2e_common import GOLDEN, run_cfg2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["eager", "device_tables", "graphs"])
@pytest.mark.parametrize("run_name", ["ample", "capped"])
def test_cfg2_token_exact_on_gpu(run_name, mode):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    tokens, counts, rt = run_cfg2(run_name, "cuda", mode=mode)
    want = GOLDEN[f"{run_name}/sdpa_v2"]
    assert tokens == want["tokens"]
    assert counts == want["counts"]
    if mode != "eager":
        assert not rt.runner.state.row_of
    if mode == "graphs":
        assert rt.runner.graphs.replays == sum(r.decode_requests > 0 for r in rt.records)



def test_fused_qkv_backend_model_outputs_match_unfused():
    """One bf16 model, two backends: the QKV projection + KV write fused in
    one tcgen05 GEMM against torch's projection followed by the separate
    write.  Prefill of a first chunk, a second chunk over its prefix, then a
    decode step: logits and the KV written agree to bf16 rounding."""
    from types import SimpleNamespace

    from b200attn.harness import MiniGPT, init_weights
    from b200attn.harness.kv_pool import DecodeBatchMetadata
    from b200attn.harness.model import B200Backend, B200FusedQKVBackend

    d = torch.device("cuda", 0)
    n_embd, n_head, S, L = 256, 8, 16, 2
    model = MiniGPT(n_embd=n_embd, n_head=n_head, vocab_size=256, block_size=296,
                    n_layer=L).eval()
    init_weights(model, seed=0)
    model.to(device=d, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 256, (1, 96), generator=g).to(d)
    table = torch.randperm(12, generator=g)[:7].to(d)  # 96 + 1 tokens -> 7 blocks
    slots = (table[torch.arange(97, device=d) // S] * S + torch.arange(97, device=d) % S)
    outs = []
    for backend in (B200Backend(), B200FusedQKVBackend(decode=True)):
        model.backend = backend
        pool = SimpleNamespace(
            k=torch.full((L, 12, S, n_head, n_embd // n_head), float("nan"), dtype=torch.bfloat16,
                         device=d), block_size=S)
        pool.v = torch.full_like(pool.k, float("nan"))
        with torch.inference_mode():
            a = model.prefill_chunk(ids[:, :64], pool, 0, table, slots[:64])
            b = model.prefill_chunk(ids[:, 64:], pool, 64, table, slots[64:96])
            meta = DecodeBatchMetadata(positions=torch.tensor([96], device=d),
                                       context_lengths=torch.tensor([97], device=d),
                                       block_tables=table.view(1, -1),
                                       slot_mapping=slots[96:97])
            c = model.decode_batch(ids[:, 95:96], meta, pool)
        torch.cuda.synchronize()
        outs.append((a.float(), b.float(), c.float(), pool))
    for x, y, what in zip(outs[0][:3], outs[1][:3], ("chunk 1", "chunk 2", "decode")):
        err = (x - y).abs().max().item()
        assert err <= 0.05 * x.abs().max().item(), f"{what}: logits differ by {err:.3e}"
    used = table.long()
    for t in ("k", "v"):
        p0 = getattr(outs[0][3], t)[:, used].float()
        p1 = getattr(outs[1][3], t)[:, used].float()
        written = ~torch.isnan(p0)
        assert torch.equal(written, ~torch.isnan(p1))
        assert ((p0 - p1).abs()[written] <= p0.abs()[written] * 0.03 + 0.02).all()


@pytest.mark.parametrize("fused_decode", [False, True])
@pytest.mark.parametrize("mode", ["eager", "graphs"])
def test_cfg2_bf16_fused_qkv_runtime(mode, fused_decode):
    """Configuration 2's requests on a bf16 model through the runtime with the
    fused-QKV backend (capped KV: recompute preemption replays prefills
    through the fused GEMM; with fused_decode the decode steps too).
    Lifecycle counts equal the reference's; the greedy tokens equal those of
    the same bf16 model on the unfused backend."""
    from b200attn.harness.model import B200Backend, B200FusedQKVBackend

    t_ref, c_ref, _ = run_cfg2("capped", "cuda", backend=B200Backend(), mode=mode,
                               dtype=torch.bfloat16)
    t_fused, c_fused, rt = run_cfg2("capped", "cuda",
                                    backend=B200FusedQKVBackend(decode=fused_decode), mode=mode,
                                    dtype=torch.bfloat16)
    assert c_fused == GOLDEN["capped/sdpa_v2"]["counts"] == c_ref
    same = sum(a == b for r in t_ref for a, b in zip(t_ref[r], t_fused[r]))
    total = sum(len(t) for t in t_ref.values())
    assert same == total, f"{total - same} of {total} greedy tokens differ"
