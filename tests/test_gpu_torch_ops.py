"""torch.ops.b200attn.* on the GPU give exactly what the direct ops give."""
from __future__ import annotations

import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality (the NaN-poisoned pools compare unequal as floats)."""
    it = {2: torch.int16, 4: torch.int32}[a.element_size()]
    return torch.equal(a.view(it), b.view(it))


def test_torch_ops_match_direct_calls():
    from b200attn import chunked_prefill_b200, kv_scatter_b200, paged_attention_batch_b200

    d = torch.device("cuda")
    # Decode with the fused write (configuration 1 shapes, fp32).
    c = cases.cfg1_case()
    B, H, D = c.q.shape
    S = c.pool.block_size
    g = torch.Generator().manual_seed(7)
    k_new = torch.randn((B, H, D), generator=g).to(d)
    v_new = torch.randn((B, H, D), generator=g).to(d)
    slots = torch.tensor([int(c.block_tables[b, (int(n) - 1) // S]) * S + (int(n) - 1) % S
                          for b, n in enumerate(c.context_lengths)], device=d)
    q, bt, cl = c.q.to(d), c.block_tables.to(d), c.context_lengths.to(d)
    k1, v1 = c.pool.k.to(d), c.pool.v.to(d)
    k2, v2 = k1.clone(), v1.clone()
    want = paged_attention_batch_b200(q, cases.Pool(k1, v1, S), bt, cl, 0, k_new=k_new,
                                      v_new=v_new, slot_mapping=slots)
    got = torch.ops.b200attn.paged_decode(q, k2, v2, bt, cl, 0, k_new, v_new, slots)
    torch.cuda.synchronize()
    assert torch.equal(want, got) and _same_bits(k1, k2) and _same_bits(v1, v2)

    # Prefill: scatter the chunk, then attend (bf16 pool, tensor-core path).
    pc = cases.prefill_case(40, 70, 4, 128, 16, 11, dtype=torch.bfloat16, n_layer=2, layer_idx=1)
    kp1, vp1 = pc.pool.k.to(d), pc.pool.v.to(d)
    kp2, vp2 = kp1.clone(), vp1.clone()
    sl = torch.tensor(pc.slots, device=d)
    table = torch.tensor(pc.block_table, device=d)
    kv_scatter_b200(pc.k.to(d), pc.v.to(d), cases.Pool(kp1, vp1, 16), sl, 1)
    want = chunked_prefill_b200(pc.q.to(d), cases.Pool(kp1, vp1, 16), table, 40, 1)
    got = torch.ops.b200attn.chunked_prefill(pc.q.to(d), pc.k.to(d), pc.v.to(d), kp2, vp2, table,
                                             sl, 40, 1)
    torch.cuda.synchronize()
    assert torch.equal(want, got) and _same_bits(kp1, kp2) and _same_bits(vp1, vp2)

    # Scatter alone.
    kp3, vp3 = pc.pool.k.to(d), pc.pool.v.to(d)
    torch.ops.b200attn.kv_scatter(pc.k.to(d), pc.v.to(d), kp3, vp3, sl, 1)
    torch.cuda.synchronize()
    assert _same_bits(kp1, kp3) and _same_bits(vp1, vp3)
