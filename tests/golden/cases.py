"""Deterministic input builders shared by the fixture generator and the tests.

Every builder draws from its own seeded ``torch.Generator`` on the CPU, so
the same inputs come out on any machine with this torch build; the golden
fixtures store a SHA-256 of the inputs to detect generator drift.  Builders
that restate a reference fixture say which one; make_golden.py checks them
bit-for-bit against the reference's own builders.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch


@dataclass
class Pool:
    """Duck-typed stand-in for minivllm.kv_block_pool.KVBlockPool."""

    k: torch.Tensor
    v: torch.Tensor
    block_size: int

    def to(self, device) -> "Pool":
        return Pool(self.k.to(device), self.v.to(device), self.block_size)


@dataclass
class DecodeCase:
    name: str
    q: torch.Tensor
    pool: Pool
    block_tables: torch.Tensor
    context_lengths: torch.Tensor
    layer_idx: int


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().to("cpu").contiguous()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()


def case_digest(c: DecodeCase) -> str:
    return digest(c.q, c.pool.k, c.pool.v, c.block_tables, c.context_lengths)


def unit_pool_cases() -> list[DecodeCase]:
    """tests/test_paged_attention.py:11-47 (seed 2026, 4 blocks of 4 tokens)."""
    g = torch.Generator().manual_seed(2026)
    shape = (1, 4, 4, 2, 4)
    k = torch.randn(shape, generator=g)
    v = torch.randn(shape, generator=g)
    q = torch.randn((2, 2, 4), generator=g)
    pool = Pool(k, v, 4)
    t = lambda x: torch.tensor(x, dtype=torch.int64)
    return [
        DecodeCase("unit_single_block", q[:1], pool, t([[2]]), t([3]), 0),
        DecodeCase("unit_cross_block", q[:1], pool, t([[0, 1]]), t([6]), 0),
        DecodeCase("unit_variable_lengths", q, pool, t([[0, 1], [2, -1]]), t([6, 3]), 0),
    ]


def nan_padding_case() -> DecodeCase:
    """tests/test_paged_attention_padding.py:12-32 (seed 11, NaN-poisoned pool)."""
    g = torch.Generator().manual_seed(11)
    k = torch.full((1, 3, 4, 2, 8), float("nan"))
    v = torch.full((1, 3, 4, 2, 8), float("nan"))
    k[0, 0, :2] = torch.randn((2, 2, 8), generator=g)
    v[0, 0, :2] = torch.randn((2, 2, 8), generator=g)
    k[0, 1, :4] = torch.randn((4, 2, 8), generator=g)
    v[0, 1, :4] = torch.randn((4, 2, 8), generator=g)
    k[0, 2, :1] = torch.randn((1, 2, 8), generator=g)
    v[0, 2, :1] = torch.randn((1, 2, 8), generator=g)
    q = torch.randn((2, 2, 8), generator=g)
    return DecodeCase("nan_padding", q, Pool(k, v, 4),
                      torch.tensor([[0, -1], [1, 2]]), torch.tensor([2, 5]), 0)


def ragged_case(batch: int = 2, length: int = 128, heads: int = 8, dim: int = 32,
                block_size: int = 16, layout: str = "mixed", seed: int = 20261030,
                scale: float = 0.3) -> DecodeCase:
    """Restates build_case (experiments/gpu_day6_fused_decode_ab.py:35-77).

    Pre-filled paged KV over a random permutation of physical blocks, two
    layers (layer 1 used), unwritten token rows NaN, -1 table padding, and a
    stride-2 q.  The draw order of the generator matches the reference:
    randperm of the physical blocks, then per logical block the K rows and
    the V rows, then q.
    """
    g = torch.Generator().manual_seed(seed)
    if layout == "mixed":
        lengths = [max(1, length - (i % 4) * max(1, length // 7)) for i in range(batch)]
    elif layout == "fixed":
        lengths = [length] * batch
    else:
        raise ValueError("layout must be fixed/mixed")
    counts = [math.ceil(n / block_size) for n in lengths]
    n_phys = sum(counts) + 7
    layer = 1
    k = torch.full((2, n_phys, block_size, heads, dim), float("nan"))
    v = torch.full((2, n_phys, block_size, heads, dim), float("nan"))
    table = torch.full((batch, max(counts)), -1, dtype=torch.int64)
    order = torch.randperm(n_phys, generator=g).tolist()
    nxt = 0
    for b in range(batch):
        for j in range(counts[b]):
            phys = order[nxt]
            nxt += 1
            table[b, j] = phys
            rows = min(block_size, lengths[b] - j * block_size)
            k[layer, phys, :rows] = torch.randn((rows, heads, dim), generator=g) * scale
            v[layer, phys, :rows] = torch.randn((rows, heads, dim), generator=g) * scale
    q = torch.randn((batch, heads, 2 * dim), generator=g)[..., ::2].mul_(scale)
    name = f"ragged_b{batch}_l{length}_h{heads}_d{dim}_s{block_size}_{layout}_sc{scale}_seed{seed}"
    return DecodeCase(name, q, Pool(k, v, block_size), table,
                      torch.tensor(lengths, dtype=torch.int64), layer)


# (block_size, length) pairs of tests/test_triton_paged_decode.py:14-15 (CPU fixture test).
RAGGED_CPU_SHAPES = [(8, 17), (16, 1), (16, 15), (16, 16), (16, 17), (16, 31), (16, 65), (16, 129)]
# (block_size, length, batch, dim) of tests/test_triton_paged_decode.py:54-59 (CUDA kernel test).
RAGGED_GPU_SHAPES = [(16, 1, 1, 32), (16, 15, 2, 32), (16, 16, 2, 32), (16, 17, 4, 32),
                     (16, 65, 4, 32), (16, 129, 4, 32), (16, 257, 2, 32), (8, 37, 3, 16),
                     (32, 129, 3, 64), (16, 33, 2, 48)]
# Lengths of the correctness mode of experiments/gpu_day6_fused_decode_ab.py:168-169.
RAGGED_CORRECTNESS = [(1, 1), (1, 15), (1, 16), (2, 17), (4, 33), (4, 64), (4, 65), (2, 128),
                      (4, 129), (2, 256), (4, 257)]


def cfg1_case() -> DecodeCase:
    """Configuration 1: isolated fp32 decode, seed 0.

    B=4, H=8, D=32, S=16, context lengths [128, 256, 128, 256] (48 blocks),
    P=64, L=1.  Draw order: K pool ~N(0,1), V pool ~N(0,1), randperm(64), q.
    The first 48 entries of the permutation are cut, in order, into the
    four block tables (8, 16, 8, 16 blocks); shorter rows are -1 padded.
    """
    g = torch.Generator().manual_seed(0)
    B, H, D, S, P = 4, 8, 32, 16, 64
    lens = [128, 256, 128, 256]
    k = torch.randn((1, P, S, H, D), generator=g)
    v = torch.randn((1, P, S, H, D), generator=g)
    perm = torch.randperm(P, generator=g)
    q = torch.randn((B, H, D), generator=g)
    counts = [n // S for n in lens]
    table = torch.full((B, max(counts)), -1, dtype=torch.int64)
    nxt = 0
    for b, c in enumerate(counts):
        table[b, :c] = perm[nxt:nxt + c]
        nxt += c
    return DecodeCase("cfg1", q, Pool(k, v, S), table, torch.tensor(lens), 0)


def bf16_case(batch: int, heads: int, dim: int, block_size: int, max_len: int, seed: int,
              min_len: int = 1) -> DecodeCase:
    """Ragged bf16-KV decode case (configuration-3 shapes scaled down).

    Lengths ~U[min_len, max_len] with lengths[0] = min_len and one length
    forced to a non-multiple of the block size; the pool holds the needed
    blocks plus 10 % spare, tables are a random permutation with -1 tail,
    unwritten rows NaN, K/V/q ~N(0,1) (q in float32).
    """
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (batch,), generator=g)
    lens[0] = min_len
    if batch > 1 and int(lens[-1]) % block_size == 0:
        lens[-1] = max(1, int(lens[-1]) - 1)
    counts = [math.ceil(int(n) / block_size) for n in lens]
    P = math.ceil(1.1 * sum(counts)) + 1
    k = torch.full((1, P, block_size, heads, dim), float("nan"), dtype=torch.bfloat16)
    v = torch.full((1, P, block_size, heads, dim), float("nan"), dtype=torch.bfloat16)
    perm = torch.randperm(P, generator=g)
    table = torch.full((batch, max(counts)), -1, dtype=torch.int64)
    nxt = 0
    for b in range(batch):
        for j in range(counts[b]):
            phys = int(perm[nxt])
            nxt += 1
            table[b, j] = phys
            rows = min(block_size, int(lens[b]) - j * block_size)
            k[0, phys, :rows] = torch.randn((rows, heads, dim), generator=g).to(torch.bfloat16)
            v[0, phys, :rows] = torch.randn((rows, heads, dim), generator=g).to(torch.bfloat16)
    q = torch.randn((batch, heads, dim), generator=g)
    return DecodeCase(f"bf16_b{batch}_h{heads}_d{dim}_s{block_size}_l{max_len}", q,
                      Pool(k, v, block_size), table, lens.to(torch.int64), 0)


@dataclass
class PrefillCase:
    name: str
    q: torch.Tensor        # [T, H, D]
    k: torch.Tensor        # [T, H, D] chunk keys
    v: torch.Tensor
    pool: Pool             # prefix already written, chunk rows NaN
    block_table: list[int]
    prefix_len: int
    slots: list[int]
    layer_idx: int


def prefill_case(prefix_len: int, T: int, heads: int, dim: int, block_size: int, seed: int,
                 dtype: torch.dtype = torch.float32, n_layer: int = 2, layer_idx: int = 1,
                 spare_blocks: int = 5) -> PrefillCase:
    """One sequence with `prefix_len` cached tokens and a T-token chunk.

    Physical blocks are a random permutation (non-monotonic, as
    tests/test_prefill_prefix_sdpa_v2.py:20-22 forces); prefix rows ~N(0,1),
    every other row NaN; chunk q/k/v ~N(0,1); slots = the chunk positions'
    physical slots (BlockManager.reserve_slots, minivllm/block_manager.py:85-110).
    """
    g = torch.Generator().manual_seed(seed)
    total = prefix_len + T
    nb = math.ceil(total / block_size)
    P = nb + spare_blocks
    perm = torch.randperm(P, generator=g).tolist()
    table = perm[:nb]
    k = torch.full((n_layer, P, block_size, heads, dim), float("nan"), dtype=dtype)
    v = torch.full((n_layer, P, block_size, heads, dim), float("nan"), dtype=dtype)
    for pos in range(prefix_len):
        phys, off = table[pos // block_size], pos % block_size
        k[layer_idx, phys, off] = torch.randn((heads, dim), generator=g).to(dtype)
        v[layer_idx, phys, off] = torch.randn((heads, dim), generator=g).to(dtype)
    q = torch.randn((T, heads, dim), generator=g).to(dtype)
    kc = torch.randn((T, heads, dim), generator=g).to(dtype)
    vc = torch.randn((T, heads, dim), generator=g).to(dtype)
    slots = [table[(prefix_len + i) // block_size] * block_size + (prefix_len + i) % block_size
             for i in range(T)]
    name = f"prefill_p{prefix_len}_t{T}_h{heads}_d{dim}_s{block_size}_{str(dtype)[6:]}"
    return PrefillCase(name, q, kc, vc, Pool(k, v, block_size), table, prefix_len, slots,
                       layer_idx)


# (prefix_len, T) chunk boundaries of the irregular chunkings of
# tests/test_prefill_prefix_sdpa_v2.py:53-54, flattened.
def chunk_boundaries(pieces: list[int]) -> list[tuple[int, int]]:
    out, start = [], 0
    for p in pieces:
        out.append((start, p))
        start += p
    return out


PREFILL_PIECES = [[5, 7, 19], [1, 1, 9], [16, 1, 15], [8, 8, 8, 8], [3, 5, 4, 16, 11],
                  [16, 16, 16, 16], [64, 32, 32]]


@dataclass
class QkvCase:
    name: str
    x: torch.Tensor      # [T, C] activations entering the attention's qkv Linear
    w: torch.Tensor      # [3C, C] qkv.weight
    pool: Pool
    table: list
    slots: list
    layer_idx: int


def qkv_case(T: int, heads: int, dim: int, block_size: int, seed: int, n_layer: int = 2,
             layer_idx: int = 1, spare_blocks: int = 3) -> QkvCase:
    """A first prefill chunk of T tokens through the attention's projection:
    x ~N(0,1), qkv.weight ~N(0,1)/sqrt(C), a NaN-filled pool and the slots of
    positions 0..T-1 over a permuted block table."""
    g = torch.Generator().manual_seed(seed)
    C = heads * dim
    nb = math.ceil(T / block_size)
    P = nb + spare_blocks
    table = torch.randperm(P, generator=g).tolist()[:nb]
    k = torch.full((n_layer, P, block_size, heads, dim), float("nan"))
    v = torch.full((n_layer, P, block_size, heads, dim), float("nan"))
    x = torch.randn((T, C), generator=g)
    w = torch.randn((3 * C, C), generator=g) / math.sqrt(C)
    slots = [table[i // block_size] * block_size + i % block_size for i in range(T)]
    name = f"qkv_t{T}_h{heads}_d{dim}_s{block_size}_seed{seed}"
    return QkvCase(name, x, w, Pool(k, v, block_size), table, slots, layer_idx)


# (T, heads, dim, block_size, seed) of the projection fixtures.
QKV_CASES = [(5, 2, 32, 4, 901), (37, 4, 32, 8, 902), (64, 8, 32, 16, 903)]
