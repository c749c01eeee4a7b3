"""torch.ops.b200attn.*: registration, schemas and fake (meta) shapes, on CPU."""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensorMode


def test_ops_registered_with_schemas():
    import b200attn  # noqa: F401  (registers the ops)

    sch = {n: str(getattr(torch.ops.b200attn, n).default._schema)
           for n in ("paged_decode", "kv_scatter", "chunked_prefill", "qkv_kv_write")}
    assert "Tensor(a1!) k_pool, Tensor(a2!) v_pool" in sch["paged_decode"]
    assert sch["paged_decode"].endswith("Tensor? slot_mapping=None) -> Tensor")
    assert sch["kv_scatter"].endswith("SymInt layer_idx) -> ()")
    assert "Tensor slot_mapping, SymInt prefix_len, SymInt layer_idx) -> Tensor" in sch["chunked_prefill"]
    assert "Tensor(a2!) k_pool, Tensor(a3!) v_pool, Tensor slot_mapping, SymInt layer_idx) -> Tensor" in sch["qkv_kv_write"]


def test_fake_implementations_give_output_shapes():
    import b200attn  # noqa: F401

    with FakeTensorMode():
        q = torch.empty(4, 8, 32, device="cuda")
        kp = torch.empty(2, 16, 16, 8, 32, device="cuda")
        vp = torch.empty_like(kp)
        bt = torch.zeros(4, 3, dtype=torch.int64, device="cuda")
        cl = torch.ones(4, dtype=torch.int64, device="cuda")
        out = torch.ops.b200attn.paged_decode(q, kp, vp, bt, cl, 1, None, None, None)
        assert out.shape == q.shape and out.dtype == q.dtype
        k = torch.empty(10, 8, 32, device="cuda")
        sm = torch.zeros(10, dtype=torch.int64, device="cuda")
        torch.ops.b200attn.kv_scatter(k, k, kp, vp, sm, 0)
        o = torch.ops.b200attn.chunked_prefill(torch.empty(10, 8, 32, device="cuda"), k, k, kp, vp,
                                               torch.zeros(3, dtype=torch.int64, device="cuda"), sm,
                                               5, 0)
        assert o.shape == (10, 8, 32)
        x = torch.empty(10, 256, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(768, 256, dtype=torch.bfloat16, device="cuda")
        q = torch.ops.b200attn.qkv_kv_write(x, w, kp, vp, sm, 0)
        assert q.shape == (10, 8, 32) and q.dtype == torch.bfloat16
