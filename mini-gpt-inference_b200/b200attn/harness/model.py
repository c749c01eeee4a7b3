"""MiniGPT model of the runtime harness, with the sm_100a attention backend.

Parameter names and shapes are those of minivllm's MiniGPT
(minivllm/model.py:16-61, block.py, feed_forward.py, attention.py:79-97) so
the same weights load into both; the forward passes follow
MiniGPT.prefill_chunk / decode_batch (model.py:189-248) and the pre-LN
TransformerBlock (block.py:47-93).  Attention goes through a backend object;
the default, B200Backend, is the fused KV-write + paged decode kernel and
the scatter + prefix-aware prefill kernels -- the "sm100" branches of
the reference-side host diff.  B200FusedQKVBackend (bf16 models) also moves
the QKV projection and the KV write into one tcgen05 GEMM.
"""
from __future__ import annotations

import torch
from torch import Tensor, nn

from .kv_pool import DecodeBatchMetadata, KVBlockPool


class B200Backend:
    """Attention on libb200attn.so (CUDA only; no fallback)."""

    def decode(self, q: Tensor, k: Tensor, v: Tensor, pool: KVBlockPool,
               metadata: DecodeBatchMetadata, layer_idx: int) -> Tensor:
        from ..ops import paged_attention_batch_b200

        return paged_attention_batch_b200(q, pool, metadata.block_tables,
                                          metadata.context_lengths, layer_idx, k_new=k,
                                          v_new=v, slot_mapping=metadata.slot_mapping)

    def prefill(self, q: Tensor, k: Tensor, v: Tensor, pool: KVBlockPool, block_table: Tensor,
                start_pos: int, slot_mapping: Tensor, layer_idx: int) -> Tensor:
        from ..ops import chunked_prefill_b200, kv_scatter_b200

        kv_scatter_b200(k, v, pool, slot_mapping, layer_idx)
        return chunked_prefill_b200(q, pool, block_table, start_pos, layer_idx)


class B200FusedQKVBackend(B200Backend):
    """B200Backend with the QKV projection and the KV write fused into one
    tcgen05 GEMM (b200_qkv_kv_write): the k and v thirds of the projection
    go from the GEMM epilogue straight into the pool, and attention then
    reads them from there.  Needs bf16 weights and a bf16 KV pool.

    decode=False (the default) keeps decode steps on the B200Backend path
    (torch projection, KV write fused into the attention kernel), which is
    the faster one at decode batch sizes above a few tokens; prefill chunks
    always take the fused projection."""

    fused_qkv = True

    def __init__(self, decode: bool = False):
        self.fused_qkv_decode = decode

    def decode_fused(self, x: Tensor, weight: Tensor, pool: KVBlockPool,
                     metadata: DecodeBatchMetadata, layer_idx: int) -> Tensor:
        from ..ops import paged_attention_batch_b200, qkv_kv_write_b200

        q = qkv_kv_write_b200(x, weight, pool, metadata.slot_mapping, layer_idx)
        return paged_attention_batch_b200(q, pool, metadata.block_tables,
                                          metadata.context_lengths, layer_idx)

    def prefill_fused(self, x: Tensor, weight: Tensor, pool: KVBlockPool, block_table: Tensor,
                      start_pos: int, slot_mapping: Tensor, layer_idx: int) -> Tensor:
        from ..ops import chunked_prefill_b200, qkv_kv_write_b200

        q = qkv_kv_write_b200(x, weight, pool, slot_mapping, layer_idx)
        return chunked_prefill_b200(q, pool, block_table, start_pos, layer_idx)


class Attention(nn.Module):
    def __init__(self, n_embd: int, n_head: int):
        super().__init__()
        if n_embd % n_head != 0:
            raise ValueError(f"n_embd {n_embd} is not divisible by n_head {n_head}")
        self.n_embd, self.n_head, self.head_size = n_embd, n_head, n_embd // n_head
        self.qkv = nn.Linear(n_embd, 3 * n_embd, bias=False)
        self.project = nn.Linear(n_embd, n_embd)

    def _split(self, x: Tensor, rows: int) -> tuple[Tensor, Tensor, Tensor]:
        # [rows, 3C] -> three strided [rows, H, D] views, like the reference's
        # view(...).transpose(1, 2) of the fused projection (attention.py:180-191).
        q, k, v = self.qkv(x).reshape(rows, 3 * self.n_embd).chunk(3, dim=-1)
        shape = (rows, self.n_head, self.head_size)
        return q.view(shape), k.view(shape), v.view(shape)

    def forward_decode_batch(self, x: Tensor, metadata: DecodeBatchMetadata, pool: KVBlockPool,
                             layer_idx: int, backend) -> Tensor:
        B, T, C = x.shape
        assert T == 1
        if getattr(backend, "fused_qkv_decode", False):
            out = backend.decode_fused(x.reshape(B, C), self.qkv.weight, pool, metadata, layer_idx)
        else:
            q, k, v = self._split(x, B)
            out = backend.decode(q, k, v, pool, metadata, layer_idx)
        return self.project(out.reshape(B, 1, C))

    def forward_prefill_chunk(self, x: Tensor, ctx: "PrefillChunk", backend) -> Tensor:
        B, T, C = x.shape
        assert B == 1
        if getattr(backend, "fused_qkv", False):
            out = backend.prefill_fused(x.reshape(T, C), self.qkv.weight, ctx.pool, ctx.block_table,
                                        ctx.start_pos, ctx.slot_mapping, ctx.layer_idx)
        else:
            q, k, v = self._split(x, T)
            out = backend.prefill(q, k, v, ctx.pool, ctx.block_table, ctx.start_pos,
                                  ctx.slot_mapping, ctx.layer_idx)
        return self.project(out.reshape(1, T, C))


class FeedForward(nn.Module):
    def __init__(self, n_embd: int):
        super().__init__()
        self.network = nn.Sequential(nn.Linear(n_embd, 4 * n_embd), nn.GELU(),
                                     nn.Linear(4 * n_embd, n_embd), nn.Dropout(0.0))

    def forward(self, x: Tensor) -> Tensor:
        return self.network(x)


class TransformerBlock(nn.Module):
    def __init__(self, n_embd: int, n_head: int):
        super().__init__()
        self.attn = Attention(n_embd, n_head)
        self.ffn = FeedForward(n_embd)
        self.layer_norm_1 = nn.LayerNorm(n_embd)
        self.layer_norm_2 = nn.LayerNorm(n_embd)


class PrefillChunk:
    """Per-layer prefill context: the device block table and slots of a chunk."""

    def __init__(self, pool: KVBlockPool, layer_idx: int, start_pos: int, block_table: Tensor,
                 slot_mapping: Tensor):
        self.pool, self.layer_idx, self.start_pos = pool, layer_idx, start_pos
        self.block_table, self.slot_mapping = block_table, slot_mapping


class MiniGPT(nn.Module):
    def __init__(self, n_embd: int, n_head: int, vocab_size: int, block_size: int,
                 n_layer: int = 1, backend=None):
        super().__init__()
        self.block_size, self.vocab_size, self.n_layer = block_size, vocab_size, n_layer
        self.token_embedding_table = nn.Embedding(vocab_size, n_embd)
        self.position_embedding_table = nn.Embedding(block_size, n_embd)
        self.blocks = nn.Sequential(*[TransformerBlock(n_embd, n_head) for _ in range(n_layer)])
        self.layer_norm = nn.LayerNorm(n_embd)
        self.language_model_head = nn.Linear(n_embd, vocab_size)
        self.backend = backend if backend is not None else B200Backend()

    def prefill_chunk(self, input_ids: Tensor, pool: KVBlockPool, start_pos: int,
                      block_table: Tensor, slot_mapping: Tensor) -> Tensor:
        T = input_ids.shape[1]
        pos = torch.arange(start_pos, start_pos + T, device=input_ids.device)
        x = self.token_embedding_table(input_ids) + self.position_embedding_table(pos)
        for layer_idx, blk in enumerate(self.blocks):
            ctx = PrefillChunk(pool, layer_idx, start_pos, block_table, slot_mapping)
            x = x + blk.attn.forward_prefill_chunk(blk.layer_norm_1(x), ctx, self.backend)
            x = x + blk.ffn(blk.layer_norm_2(x))
        return self.language_model_head(self.layer_norm(x))

    def decode_batch(self, input_ids: Tensor, metadata: DecodeBatchMetadata,
                     pool: KVBlockPool) -> Tensor:
        x = (self.token_embedding_table(input_ids)
             + self.position_embedding_table(metadata.positions.unsqueeze(1)))
        for layer_idx, blk in enumerate(self.blocks):
            x = x + blk.attn.forward_decode_batch(blk.layer_norm_1(x), metadata, pool, layer_idx,
                                                  self.backend)
            x = x + blk.ffn(blk.layer_norm_2(x))
        return self.language_model_head(self.layer_norm(x))


def init_weights(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Deterministic init by parameter name: 2-D weights (Linear, Embedding)
    ~N(0, std) from one CPU generator in sorted-name order, biases 0,
    LayerNorm weights 1.  Names match the reference model, so the same call
    gives both models identical weights."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
            if p.dim() >= 2:
                p.copy_(torch.empty(p.shape, dtype=torch.float32).normal_(0.0, std, generator=g))
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)
