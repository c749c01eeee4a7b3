"""Fused QKV projection + KV write (b200_qkv_kv_write) on the GPU, through the C ABI.

The reference computes ``q, k, v = self.qkv(x).chunk(3, -1)`` and writes k and
v at each token's slot (minivllm/attention.py:177-208, :360-392).  The kernel
is a bf16 tcgen05 GEMM with f32 accumulation and one bf16 rounding per
output, so it is checked against the same product in fp32 (torch, on the
upcast bf16 operands): every output must be the fp32 value rounded to bf16
up to the accumulation order, i.e. |got - ref| <= 2^-8 |ref| + 1e-4 (unit
roundoff of bf16 plus f32 summation-order slack).  Pool rows that no slot
names must keep their bits (the pool is NaN-poisoned first).
"""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_U = 2.0 ** -8


def _dev():
    return torch.device("cuda", 0)


def _make(T, C, H, S, L, layer, seed, slot_dtype=torch.int64, x_pad=0, P=None):
    g = torch.Generator().manual_seed(seed)
    D = C // H
    need = -(-T // S) + 2
    P = P or max(need * 2, 4)
    x_full = torch.randn(T, C + x_pad, generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * C, C, generator=g) / C ** 0.5).to(torch.bfloat16)
    slots = torch.randperm(P * S, generator=g)[:T].to(slot_dtype)
    d = _dev()
    pool = SimpleNamespace(
        k=torch.full((L, P, S, H, D), float("nan"), dtype=torch.bfloat16, device=d),
        v=torch.full((L, P, S, H, D), float("nan"), dtype=torch.bfloat16, device=d),
        block_size=S)
    x = x_full.to(d)[:, :C]
    return SimpleNamespace(x=x, w=w.to(d), slots=slots.to(d), pool=pool, T=T, C=C, H=H, D=D,
                           S=S, L=L, P=P, layer=layer)


def _ref(c):
    return c.x.float() @ c.w.float().t()  # [T, 3C] in fp32 (products of bf16 are exact)


def _assert_rounded(got, ref, what):
    err = (got.float() - ref).abs()
    bound = ref.abs() * BF16_U + 1e-4
    bad = (err > bound).sum().item()
    assert bad == 0, f"{what}: {bad} elements beyond bf16 rounding, max err {err.max().item():.3e}"


def _check_pool(c, y, status_bits=0):
    """k/v rows at the slots equal y's thirds; every other row is untouched."""
    C = c.C
    kf = c.pool.k.view(c.L, c.P * c.S, C)
    vf = c.pool.v.view(c.L, c.P * c.S, C)
    slots = c.slots.long()
    valid = (slots >= 0) & (slots < c.P * c.S)
    rows = slots[valid]
    _assert_rounded(kf[c.layer, rows], y[valid, C:2 * C], "k rows")
    _assert_rounded(vf[c.layer, rows], y[valid, 2 * C:], "v rows")
    written = torch.zeros(c.L, c.P * c.S, dtype=torch.bool, device=kf.device)
    written[c.layer, rows] = True
    assert torch.isnan(kf[~written].float()).all() and torch.isnan(vf[~written].float()).all()


@pytest.mark.parametrize("T,C,H,S,L,layer", [
    (1, 256, 8, 16, 2, 1),       # one decode token, cfg2-sized model (H=8, D=32)
    (5, 256, 8, 16, 1, 0),
    (64, 4096, 32, 16, 1, 0),    # decode batch at H=32, D=128 (split-K clusters)
    (96, 4096, 32, 16, 1, 0),    # split-K clusters, 48 rows owned per cluster rank
    (77, 4096, 32, 16, 1, 0),    # split-K clusters, ragged owned rows (39 + 38)
    (1, 1664, 13, 16, 1, 0),     # split-K clusters of 3 CTAs (hidden 1664, 112-wide tiles)
    (37, 3584, 28, 16, 2, 1),    # clusters of 3 CTAs, ragged owned rows (240-wide tiles)
    (37, 2048, 16, 16, 1, 0),    # hidden 2048: 96-wide tiles over 2 splits
    (128, 2048, 16, 16, 1, 0),   # hidden 2048: 64-wide single CTAs, one wave
    (192, 2048, 16, 16, 1, 0),   # hidden 2048: 128-wide single CTAs, two token tiles, one wave
    (1, 4096, 32, 16, 1, 0),     # one token, split-K: most cluster ranks own no row
    (90, 1024, 8, 16, 1, 0),     # split-K clusters at hidden 1024 (16 k-steps)
    (104, 4096, 32, 16, 1, 0),   # single CTAs, x box of the 104 live rows (rows past them stale)
    (129, 4096, 32, 16, 2, 1),   # CTA pairs (192-wide tiles), 72 + 57 token rows per pair
    (161, 4096, 32, 16, 1, 0),   # CTA pairs, 88 + 73 token rows (rows past them stale, not stored)
    (128, 4096, 32, 16, 1, 0),   # single CTAs, 128-wide tiles, one wave
    (256, 4096, 32, 16, 1, 0),   # CTA pairs, 192-wide tiles, one wave
    (300, 512, 4, 16, 1, 0),     # single CTAs, 64-wide tiles
    (1000, 4096, 32, 16, 1, 0),  # prefill chunk (CTA pairs, 256 x 256 tiles)
    (600, 2048, 16, 16, 2, 1),   # CTA pairs; the second CTA of the last pair has no rows
    (77, 64, 1, 8, 1, 0),        # smallest hidden size: one k-step, ragged 128-wide tile
    (200, 192, 3, 32, 1, 0),     # three heads of 64, block size 32
    (200, 3136, 49, 16, 1, 0),   # hidden 3136 (49 heads of 64): 148 single-CTA tiles in one wave
    (200, 4160, 65, 16, 1, 0),   # CTA pairs, 192-wide tiles, 65 pairs
    (200, 6400, 50, 16, 1, 0),   # no layout in one wave: persistent CTA pairs, 100 tiles over 74 pairs
    (1000, 4160, 65, 16, 1, 0),  # CTA pairs, 3C = 48.75 tiles: ragged last output tile
])
def test_qkv_kv_write_matches_fp32_projection(T, C, H, S, L, layer):
    from b200attn import qkv_kv_write_b200

    c = _make(T, C, H, S, L, layer, seed=T * 7 + C)
    status = torch.zeros(1, dtype=torch.int32, device=_dev())
    with torch.inference_mode():
        q = qkv_kv_write_b200(c.x, c.w, c.pool, c.slots, layer, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert q.shape == (T, H, C // H) and q.dtype == torch.bfloat16
    y = _ref(c)
    _assert_rounded(q.reshape(T, C), y[:, :C], "q")
    _check_pool(c, y)


def test_qkv_kv_write_agrees_with_cublas_within_one_ulp():
    """Against torch's bf16 matmul (cuBLAS, f32 accumulation, one rounding):
    the two differ only where the f32 sums straddle a bf16 rounding point."""
    from b200attn import qkv_kv_write_b200

    c = _make(512, 4096, 32, 16, 1, 0, seed=3)
    with torch.inference_mode():
        q = qkv_kv_write_b200(c.x, c.w, c.pool, c.slots, 0)
        y = c.x @ c.w.t()
    torch.cuda.synchronize()
    diff = (q.reshape(512, 4096).float() - y[:, :4096].float()).abs()
    assert (diff <= y[:, :4096].float().abs() * 2 * BF16_U + 1e-4).all()
    same = (q.reshape(512, 4096) == y[:, :4096]).float().mean().item()
    assert same > 0.95, f"only {same:.3f} of q equals cuBLAS bit for bit"


def test_qkv_kv_write_strided_x_int32_slots():
    from b200attn import qkv_kv_write_b200

    c = _make(150, 512, 8, 16, 1, 0, seed=11, slot_dtype=torch.int32, x_pad=64)
    assert c.x.stride(0) == 576
    with torch.inference_mode():
        q = qkv_kv_write_b200(c.x, c.w, c.pool, c.slots, 0)
    torch.cuda.synchronize()
    y = _ref(c)
    _assert_rounded(q.reshape(150, 512), y[:, :512], "q")
    _check_pool(c, y)


@pytest.mark.parametrize("T,C,H", [
    (40, 256, 8),      # split-K clusters
    (104, 4096, 32),   # single CTAs, one short token tile
    (300, 512, 4),     # single CTAs, several tiles per CTA
    (160, 4096, 32),   # CTA pairs, 80 + 80 token rows
    (1000, 4096, 32),  # CTA pairs, several token tiles
])
def test_qkv_kv_write_bad_slots_are_flagged_and_skipped(T, C, H):
    """A slot outside the pool sets the status bit and skips that token's k
    and v rows; its q row and every other token are still written."""
    from b200attn import _lib, qkv_kv_write_b200

    c = _make(T, C, H, 16, 1, 0, seed=5 + T)
    c.slots[3] = -1
    c.slots[T - 5] = c.P * c.S  # one past the pool
    status = torch.zeros(1, dtype=torch.int32, device=_dev())
    with torch.inference_mode():
        q = qkv_kv_write_b200(c.x, c.w, c.pool, c.slots, 0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.DEV_BAD_SLOT
    y = _ref(c)
    _assert_rounded(q.reshape(T, C), y[:, :C], "q (all rows, bad slots included)")
    _check_pool(c, y)


def test_qkv_kv_write_q_out_buffer_and_prepared_call():
    from b200attn import qkv_kv_write_b200

    c = _make(33, 256, 8, 16, 1, 0, seed=9)
    q_out = torch.empty(33, 256, dtype=torch.bfloat16, device=_dev())
    with torch.inference_mode():
        call = qkv_kv_write_b200(c.x, c.w, c.pool, c.slots, 0, q_out=q_out, prepare=True)
        q1 = call()
        q1c = q1.clone()
        q2 = call()
    torch.cuda.synchronize()
    assert q1.data_ptr() == q_out.data_ptr() and torch.equal(q2, q1c)
    _assert_rounded(q_out, _ref(c)[:, :256], "q")


def test_torch_op_qkv_kv_write():
    import b200attn  # noqa: F401  (registers torch.ops.b200attn.*)

    c = _make(20, 256, 8, 16, 1, 0, seed=21)
    with torch.inference_mode():
        q = torch.ops.b200attn.qkv_kv_write(c.x, c.w, c.pool.k, c.pool.v, c.slots, 0)
    torch.cuda.synchronize()
    y = _ref(c)
    _assert_rounded(q.reshape(20, 256), y[:, :256], "q")
    _check_pool(c, y)


@pytest.mark.parametrize("shape", [c for c in __import__("cases").QKV_CASES])
def test_qkv_kv_write_matches_pinned_oracle(shape):
    """The golden projection cases (whose oracle result is pinned to the
    reference's own qkv Linear + write loop, within the reference's fp32
    tolerance): the kernel on the bf16-rounded operands against the oracle on
    the same operands."""
    import cases
    import oracle
    from b200attn import qkv_kv_write_b200

    T, H, D, S, seed = shape
    c = cases.qkv_case(T, H, D, S, seed)
    x, w = c.x.to(torch.bfloat16), c.w.to(torch.bfloat16)
    kp, vp = c.pool.k.clone(), c.pool.v.clone()
    want_q = oracle.qkv_project_kv_write(x, w, kp, vp, c.slots, c.layer_idx)
    d = _dev()
    pool = SimpleNamespace(k=c.pool.k.to(torch.bfloat16).to(d), v=c.pool.v.to(torch.bfloat16).to(d),
                           block_size=S)
    with torch.inference_mode():
        q = qkv_kv_write_b200(x.to(d), w.to(d), pool, c.slots, c.layer_idx)
    torch.cuda.synchronize()
    _assert_rounded(q.reshape(T, H * D).cpu(), want_q.reshape(T, H * D), "q")
    for got, want, what in ((pool.k, kp, "k"), (pool.v, vp, "v")):
        got = got.float().cpu()
        written = ~torch.isnan(want)
        assert torch.equal(written, ~torch.isnan(got)), f"{what}: written rows differ"
        _assert_rounded(got[written], want[written], what)


def test_qkv_kv_write_full_size_against_cublas():
    """The bench's prefill shape (8192 tokens, hidden 4096, CTA pairs): every
    q element within one bf16 ulp of cuBLAS's bf16 GEMM, and a sample of 512
    tokens' pool rows likewise."""
    from b200attn import qkv_kv_write_b200

    T, C, H, S = 8192, 4096, 32, 16
    d = _dev()
    g = torch.Generator(device=d).manual_seed(77)
    x = torch.randn((T, C), generator=g, device=d).to(torch.bfloat16)
    w = (torch.randn((3 * C, C), generator=g, device=d) / C ** 0.5).to(torch.bfloat16)
    P = T // S + 8
    slots = torch.randperm(P * S, generator=g, device=d)[:T]
    pool = SimpleNamespace(k=torch.zeros((1, P, S, H, C // H), dtype=torch.bfloat16, device=d),
                           v=torch.zeros((1, P, S, H, C // H), dtype=torch.bfloat16, device=d),
                           block_size=S)
    with torch.inference_mode():
        q = qkv_kv_write_b200(x, w, pool, slots, 0)
        y = x @ w.t()
    torch.cuda.synchronize()
    ulp = 2.0 * BF16_U
    diff = (q.reshape(T, C).float() - y[:, :C].float()).abs()
    assert (diff <= y[:, :C].float().abs() * ulp + 1e-3).all()
    sample = torch.randperm(T, device=d)[:512]
    kf = pool.k.view(P * S, C)[slots[sample]].float()
    vf = pool.v.view(P * S, C)[slots[sample]].float()
    yk, yv = y[sample, C:2 * C].float(), y[sample, 2 * C:].float()
    assert ((kf - yk).abs() <= yk.abs() * ulp + 1e-3).all()
    assert ((vf - yv).abs() <= yv.abs() * ulp + 1e-3).all()


@pytest.mark.parametrize("T,C", [(1, 1664), (37, 3584)])
def test_qkv_plan_splits_over_more_than_two_ctas(T, C):
    """The parity cases at hidden 1664 and 3584 reach split-K clusters of 3+ CTAs."""
    import ctypes

    from b200attn import _lib

    lib = _lib.load()
    k, n, s = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert lib.b200_qkv_kv_write_plan(T, C, ctypes.byref(k), ctypes.byref(n), ctypes.byref(s)) == 0
    assert k.value == 2 and s.value >= 3, (k.value, n.value, s.value)


@pytest.mark.parametrize("T,C,kind", [
    (1, 4096, 2), (64, 4096, 2), (96, 4096, 2), (104, 4096, 0), (120, 4096, 0), (90, 1024, 2), (128, 4096, 0),
    (129, 4096, 1), (37, 2048, 2), (128, 2048, 0), (192, 2048, 0), (192, 8192, 1),
    (256, 4096, 1), (200, 6400, 1), (300, 512, 0), (384, 4096, 0), (512, 4096, 1),
    (1000, 4096, 1), (8192, 4096, 1),
])
def test_qkv_plan_covers_each_kernel(T, C, kind):
    """The shapes of the parity tests reach the kernel their comments name:
    0 single CTAs, 1 CTA pairs, 2 split-K clusters."""
    import ctypes

    from b200attn import _lib

    lib = _lib.load()
    k, n, s = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert lib.b200_qkv_kv_write_plan(T, C, ctypes.byref(k), ctypes.byref(n), ctypes.byref(s)) == 0
    assert k.value == kind, (k.value, n.value, s.value)
    if kind == 2:
        assert 1 <= s.value <= 8 and n.value % 16 == 0
    if kind == 1:
        # 192-wide pair tiles for 129-256 tokens (more SMs), 256-wide for long runs.
        assert n.value == (192 if T <= 256 else 256), n.value
