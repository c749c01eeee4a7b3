"""KV scatter and chunked-prefill parity on the GPU, through the C ABI.

The scatter is integer/byte work: the pool after it must be bit-identical to
the reference's write loop (pool digests in tests/golden/prefill_golden.json).
The fp32 prefill must match the reference's SDPA v1/v2 and per-token outputs
(max abs error <= 1e-4); bf16 prefill matches the fp32 oracle on the upcast
inputs within 2e-2.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
PRE_META = json.loads((GOLDEN / "prefill_golden.json").read_text())


def _dev():
    return torch.device("cuda", 0)


def _case(name):
    m = PRE_META[name]
    return cases.prefill_case(m["prefix_len"], m["T"], m["H"], m["D"], m["S"], m["seed"])


@pytest.mark.parametrize("name", sorted(PRE_META))
def test_scatter_and_prefill_match_reference(name):
    from b200attn import chunked_prefill_b200, kv_scatter_b200

    golden = np.load(GOLDEN / "prefill_golden.npz")
    c = _case(name)
    d = _dev()
    pool = c.pool.to(d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    with torch.inference_mode():
        kv_scatter_b200(c.k.to(d), c.v.to(d), pool, c.slots, c.layer_idx, status=status)
        out = chunked_prefill_b200(c.q.to(d), pool, c.block_table, c.prefix_len, c.layer_idx,
                                   status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert cases.digest(pool.k.cpu(), pool.v.cpu()) == PRE_META[name]["pool_after_digest"]
    got = out.cpu()
    for key in ("sdpa", "reference"):
        want = torch.from_numpy(golden[f"{name}/{key}"])
        err = (got - want).abs().max().item()
        assert err <= 1e-4, f"{name} vs reference {key}: {err:.3e}"


def test_scatter_strided_inputs_and_bf16_rounding():
    from b200attn import kv_scatter_b200

    d = _dev()
    g = torch.Generator().manual_seed(3)
    L, P, S, H, D, N = 2, 9, 16, 8, 32, 37
    kp = torch.full((L, P, S, H, D), float("nan"), dtype=torch.bfloat16)
    vp = kp.clone()
    qkv = torch.randn((N, 3 * H * D), generator=g)  # k/v as strided views of a fused QKV
    k = qkv[:, H * D:2 * H * D].view(N, H, D)
    v = qkv[:, 2 * H * D:].view(N, H, D)
    slots = torch.randperm(P * S, generator=g)[:N]
    want_k, want_v = kp.clone(), vp.clone()
    oracle.kv_scatter(want_k, want_v, k.to(torch.bfloat16), v.to(torch.bfloat16), slots, 1)
    pool = cases.Pool(kp.to(d), vp.to(d), S)
    kv_scatter_b200(k.to(d), v.to(d), pool, slots.to(d), 1)
    torch.cuda.synchronize()
    assert cases.digest(pool.k.cpu(), pool.v.cpu()) == cases.digest(want_k, want_v)
    # Non-unit innermost stride takes the element path.
    kt = torch.randn((N, D, H), generator=g).transpose(1, 2)
    pool32 = cases.Pool(torch.zeros((1, P, S, H, D), device=d), torch.zeros((1, P, S, H, D), device=d), S)
    kv_scatter_b200(kt.to(d), kt.to(d), pool32, slots.tolist(), 0)
    want32 = torch.zeros((1, P, S, H, D))
    oracle.kv_scatter(want32, want32.clone(), kt, kt, slots, 0)
    torch.cuda.synchronize()
    assert torch.equal(pool32.k.cpu(), want32)


def test_scatter_bad_slot_is_flagged_not_written():
    from b200attn import _lib, kv_scatter_b200

    d = _dev()
    pool = cases.Pool(torch.zeros((1, 4, 4, 2, 8), device=d), torch.zeros((1, 4, 4, 2, 8), device=d), 4)
    k = torch.ones((2, 2, 8), device=d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    kv_scatter_b200(k, k, pool, [3, 4 * 4 + 2], 0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.DEV_BAD_SLOT
    assert float(pool.k.sum()) == 16.0  # only the valid slot was written


@pytest.mark.parametrize("prefix,T,seed", [(0, 64, 1), (16, 64, 2), (37, 5, 3), (1000, 64, 4),
                                           (256, 200, 5), (4032, 64, 6), (96, 512, 7)])
def test_prefill_bf16_kv_against_oracle(prefix, T, seed):
    from b200attn import chunked_prefill_b200, kv_scatter_b200

    c = cases.prefill_case(prefix, T, 32, 128, 16, seed, dtype=torch.bfloat16, n_layer=1,
                           layer_idx=0)
    d = _dev()
    pool = c.pool.to(d)
    kv_scatter_b200(c.k.to(d), c.v.to(d), pool, c.slots, 0)
    out = chunked_prefill_b200(c.q.to(d), pool, c.block_table, prefix, 0)
    torch.cuda.synchronize()
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(kp, vp, c.k, c.v, c.slots, 0)
    want = oracle.prefix_prefill_from_pool(c.q.float(), kp.float(), vp.float(), c.block_table,
                                           prefix, 0, compute_dtype=torch.float64).float()
    err = (out.float().cpu() - want).abs().max().item()
    assert err <= 2e-2, f"max abs {err:.3e}"


# One query tile with >= 2 key tiles takes the key split (the two softmax
# groups alternate key tiles and merge at the end): (1000, 64), (600, 300)'s
# last tile, (100, 64) where rows 0-27 see no key of group 1's first tile,
# and (200, 100) with an odd key-tile count.
@pytest.mark.parametrize("dim,bs,heads,prefix,T", [(64, 16, 4, 300, 130), (128, 8, 2, 40, 129),
                                                   (128, 32, 3, 1000, 64), (128, 256, 2, 600, 300),
                                                   (64, 64, 5, 0, 1), (128, 16, 1, 127, 1),
                                                   (128, 16, 2, 100, 64), (64, 16, 3, 200, 100),
                                                   (128, 8, 2, 129, 127)])
@pytest.mark.parametrize("q_kind", ["f32", "bf16_strided"])
def test_prefill_tensor_core_shapes(dim, bs, heads, prefix, T, q_kind):
    """fp32 q takes the thread-loaded Q path; bf16 q, here a strided view of a
    fused [T, 3, H, D] projection, takes the TMA-loaded Q path."""
    from b200attn import chunked_prefill_b200, kv_scatter_b200

    c = cases.prefill_case(prefix, T, heads, dim, bs, 900 + dim + bs + T, dtype=torch.bfloat16,
                           n_layer=2, layer_idx=1)
    d = _dev()
    pool = c.pool.to(d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    kv_scatter_b200(c.k.to(d), c.v.to(d), pool, c.slots, 1)
    if q_kind == "f32":
        q = c.q.float().to(d)
    else:
        fused = torch.zeros((T, 3, heads, dim), dtype=torch.bfloat16, device=d)
        fused[:, 1] = c.q.to(d)
        q = fused[:, 1]
    out = chunked_prefill_b200(q, pool, c.block_table, prefix, 1, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(kp, vp, c.k, c.v, c.slots, 1)
    want = oracle.prefix_prefill_from_pool(c.q.float(), kp.float(), vp.float(), c.block_table,
                                           prefix, 1, compute_dtype=torch.float64).float()
    err = (out.float().cpu() - want).abs().max().item()
    assert err <= 2e-2, f"max abs {err:.3e}"


def test_prefill_batch_matches_single_calls():
    from b200attn import chunked_prefill_b200, chunked_prefill_batch_b200, kv_scatter_b200

    d = _dev()
    specs = [(0, 64, 11), (48, 64, 12), (500, 17, 13)]
    cs = [cases.prefill_case(p, t, 32, 128, 16, s, dtype=torch.bfloat16, n_layer=1,
                             layer_idx=0) for p, t, s in specs]
    # One shared pool: give each sequence its own block range.
    S, H, D = 16, 32, 128
    sizes = [c.pool.k.shape[1] for c in cs]
    kp = torch.cat([c.pool.k for c in cs], dim=1).to(d)
    vp = torch.cat([c.pool.v for c in cs], dim=1).to(d)
    pool = cases.Pool(kp, vp, S)
    tables, qs, offs = [], [], 0
    for c, n in zip(cs, sizes):
        table = [x + offs for x in c.block_table]
        slots = [s + offs * S for s in c.slots]
        kv_scatter_b200(c.k.to(d), c.v.to(d), pool, slots, 0)
        tables.append(table)
        qs.append(c.q.to(d))
        offs += n
    outs = chunked_prefill_batch_b200(qs, pool, tables, [c.prefix_len for c in cs], 0)
    for q, t, c, o in zip(qs, tables, cs, outs):
        single = chunked_prefill_b200(q, pool, t, c.prefix_len, 0)
        torch.cuda.synchronize()
        assert torch.equal(single.cpu(), o.cpu())


def test_prefill_batch_mixed_chunk_lengths_against_oracle():
    """A batch holding a chunk longer than one query tile runs every sequence
    with 64-key tiles and double-buffered S; a batch of short chunks runs
    128-key tiles.  Both must match the fp32 oracle."""
    from b200attn import chunked_prefill_batch_b200, kv_scatter_b200

    d = _dev()
    for specs in ([(100, 64, 21), (640, 300, 22), (0, 129, 23)], [(100, 64, 24), (33, 1, 25)]):
        cs = [cases.prefill_case(p, t, 4, 128, 16, s, dtype=torch.bfloat16, n_layer=1,
                                 layer_idx=0) for p, t, s in specs]
        S = 16
        sizes = [c.pool.k.shape[1] for c in cs]
        kp = torch.cat([c.pool.k for c in cs], dim=1)
        vp = torch.cat([c.pool.v for c in cs], dim=1)
        pool = cases.Pool(kp.to(d), vp.to(d), S)
        tables, qs, offs, wants = [], [], 0, []
        for c, n in zip(cs, sizes):
            table = [x + offs for x in c.block_table]
            slots = [s + offs * S for s in c.slots]
            kv_scatter_b200(c.k.to(d), c.v.to(d), pool, slots, 0)
            k2, v2 = c.pool.k.clone(), c.pool.v.clone()
            oracle.kv_scatter(k2, v2, c.k, c.v, c.slots, 0)
            wants.append(oracle.prefix_prefill_from_pool(c.q.float(), k2.float(), v2.float(),
                                                         c.block_table, c.prefix_len, 0,
                                                         compute_dtype=torch.float64).float())
            tables.append(table)
            qs.append(c.q.to(d))
            offs += n
        outs = chunked_prefill_batch_b200(qs, pool, tables, [c.prefix_len for c in cs], 0)
        torch.cuda.synchronize()
        for o, want in zip(outs, wants):
            err = (o.float().cpu() - want).abs().max().item()
            assert err <= 2e-2, f"max abs {err:.3e}"


@pytest.mark.parametrize("prefix,T", [(32768, 300), (32768, 64)])
def test_prefill_long_prefix(prefix, T):
    """A 32k-token prefix: hundreds of key tiles streamed through one CTA's
    rings (64-key double-buffered tiles for T=300, 128-key key-split tiles
    for T=64), against the float64 oracle."""
    from b200attn import chunked_prefill_b200, kv_scatter_b200

    c = cases.prefill_case(prefix, T, 2, 128, 16, 31 + T, dtype=torch.bfloat16, n_layer=1,
                           layer_idx=0)
    d = _dev()
    pool = c.pool.to(d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    kv_scatter_b200(c.k.to(d), c.v.to(d), pool, c.slots, 0)
    out = chunked_prefill_b200(c.q.to(d), pool, c.block_table, prefix, 0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(kp, vp, c.k, c.v, c.slots, 0)
    want = oracle.prefix_prefill_from_pool(c.q.float(), kp.float(), vp.float(), c.block_table,
                                           prefix, 0, compute_dtype=torch.float64).float()
    err = (out.float().cpu() - want).abs().max().item()
    assert err <= 2e-2, f"max abs {err:.3e}"


@pytest.mark.parametrize("prefix,T,heads", [(4032, 64, 32), (4032, 512, 32), (8000, 1, 8)])
def test_prefill_key_split_over_ctas_matches_unsplit(prefix, T, heads):
    """A launch of fewer CTAs than SMs (one sequence) splits each chunk's
    keys over several CTAs when the caller's workspace holds their partial
    rows, and the last CTA of each (query pair, head) combines them.  Its
    output equals the unsplit launch's (the C ABI without a workspace) and
    the float64 oracle's within the bf16 tolerance."""
    import ctypes

    from b200attn import _lib, chunked_prefill_b200, kv_scatter_b200, ops

    c = cases.prefill_case(prefix, T, heads, 128, 16, 4100 + T, dtype=torch.bfloat16, n_layer=1,
                           layer_idx=0)
    d = _dev()
    pool = c.pool.to(d)
    kv_scatter_b200(c.k.to(d), c.v.to(d), pool, c.slots, 0)
    lib = _lib.load()
    table = ops._index_tensor(c.block_table, d, "block_table")
    assert lib.b200_chunked_prefill_workspace_size(T, heads, 128, table.shape[0], 16,
                                                   _lib.DTYPE_BF16) > 0  # the launch splits
    status = torch.zeros(1, dtype=torch.int32, device=d)
    q = c.q.to(d)
    split = chunked_prefill_b200(q, pool, c.block_table, prefix, 0, status=status)
    unsplit = torch.empty_like(split)
    a = ops._prefill_struct(q, pool, ops._pool_struct(pool), table, prefix, 0, unsplit, status)
    a.workspace = None
    a.workspace_bytes = 0
    _lib.check(lib.b200_chunked_prefill(ctypes.byref(a), ops._stream_ptr(d)), "prefill")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert (split.float() - unsplit.float()).abs().max().item() <= 2e-2
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    oracle.kv_scatter(kp, vp, c.k, c.v, c.slots, 0)
    want = oracle.prefix_prefill_from_pool(c.q.float(), kp.float(), vp.float(), c.block_table,
                                           prefix, 0, compute_dtype=torch.float64).float()
    err = (split.float().cpu() - want).abs().max().item()
    assert err <= 2e-2, f"max abs {err:.3e}"
