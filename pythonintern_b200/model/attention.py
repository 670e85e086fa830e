"""Sharded GQA attention with RoPE over the paged KV cache.

Drop-in for engine/model/attention.py: ``RotaryEmbedding``, ``repeat_kv`` and
``DistributedAttention(config, layer_idx, rank, world_size, communicator)`` with
``forward(x, positions, kv_pool, block_tables, is_prefill, step_id)``.

The forward runs two or three kernels instead of the reference's per-token Python
loops and dense gather/pad/repeat copies:
  1. ``b2_linear_qkv``: one GEMM for the q, k and v projections (attention.py:156-158);
  2. ``b2_rope_kv_write``: RoPE on q and k and the paged K/V store (attention.py:161-184)
     -- for decode batches with head_dim 128 both run as one launch,
     ``b2_linear_qkv_rope_kv``, whose GEMM epilogue rotates and stores (bit-identical);
  3. ``b2_paged_attention``: the softmax attention read straight from the pool
     through the block tables, GQA heads sharing each K/V read (attention.py:186-228);
     a bf16 prefill runs ``b2_prefill_attention`` instead, every prompt token of every
     sequence of the call in one causal launch that shares each K/V block across a tile
     of tokens (attention.py:166-174,211-228);
then the row-parallel out_proj with its all-reduce (attention.py:231-232).
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.nn as nn

from pythonintern_b200 import kernels
from pythonintern_b200.config import ModelConfig
from pythonintern_b200.model.kv_cache import PhysicalKVCachePool
from pythonintern_b200.model.metadata import TokenMetadata, build_metadata
from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
from pythonintern_b200.tensor_parallel.layers import ColumnParallelLinear, RowParallelLinear
from pythonintern_b200._lib import torch_dtype


class RotaryEmbedding:
    """cos/sin tables ``[max_seq_len, dim]`` (engine/model/attention.py:25-63).

    Built on the host with the reference's float32 formula and copied to the
    device, so the tables match the reference bit for bit.
    """

    def __init__(self, dim: int, max_seq_len: int = 4096, base: float = 10000.0, device="cuda"):
        self.dim = dim
        self.max_seq_len = max_seq_len
        self.base = base
        self.device = torch.device(device)
        self._init_cos_sin_tables()

    def _init_cos_sin_tables(self):
        inv_freq = 1.0 / (self.base ** (torch.arange(0, self.dim, 2, dtype=torch.float32) / self.dim))
        t = torch.arange(self.max_seq_len, dtype=torch.float32)
        freqs = torch.outer(t, inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.cos_cached = emb.cos().to(self.device)
        self.sin_cached = emb.sin().to(self.device)

    def apply_rope(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """Standalone rotate-half RoPE on a tensor (not used by the forward, which fuses it)."""
        cos = self.cos_cached[positions].unsqueeze(-2)
        sin = self.sin_cached[positions].unsqueeze(-2)
        x1, x2 = x[..., : self.dim // 2], x[..., self.dim // 2:]
        return (x * cos) + (torch.cat((-x2, x1), dim=-1) * sin)


def repeat_kv(x: torch.Tensor, num_rep: int) -> torch.Tensor:
    """GQA head expansion (attention.py:66-76); the kernels share heads without materialising this."""
    if num_rep == 1:
        return x
    b, s, h, d = x.shape
    return x[:, :, :, None, :].expand(b, s, h, num_rep, d).reshape(b, s, h * num_rep, d)


_rope_cache = {}


def rope_for(head_dim: int, max_seq_len: int, base: float, device) -> RotaryEmbedding:
    key = (head_dim, max_seq_len, float(base), str(torch.device(device)))
    r = _rope_cache.get(key)
    if r is None:
        r = RotaryEmbedding(head_dim, max_seq_len, base, device)
        _rope_cache[key] = r
    return r


class DistributedAttention(nn.Module):
    """Tensor-parallel GQA attention (engine/model/attention.py:79-233)."""

    def __init__(self, config: ModelConfig, layer_idx: int, rank: int = 0, world_size: int = 1,
                 communicator: Optional[DistributedCommunicator] = None, device=None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.rank = rank
        self.world_size = world_size
        self.head_dim = config.head_dim
        self.communicator = communicator
        assert config.num_heads % world_size == 0
        assert config.num_kv_heads % world_size == 0
        self.local_heads = config.num_heads // world_size
        self.local_kv_heads = config.num_kv_heads // world_size
        self.num_queries_per_kv = self.local_heads // self.local_kv_heads
        dt = torch_dtype(config.dtype)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        H, hd = config.hidden_dim, self.head_dim
        self.q_proj = ColumnParallelLinear(H, config.num_heads * hd, False, rank, world_size, dtype=dt, device=dev)
        self.k_proj = ColumnParallelLinear(H, config.num_kv_heads * hd, False, rank, world_size, dtype=dt, device=dev)
        self.v_proj = ColumnParallelLinear(H, config.num_kv_heads * hd, False, rank, world_size, dtype=dt, device=dev)
        self.out_proj = RowParallelLinear(config.num_heads * hd, H, False, rank, world_size, communicator,
                                          dtype=dt, device=dev)
        self.rope = rope_for(hd, config.max_seq_len, config.rope_base, dev)

    def set_communicator(self, communicator: DistributedCommunicator):
        self.communicator = communicator
        self.out_proj.set_communicator(communicator)

    # -- fused pieces shared with the model's decode/prefill path -----------------------
    def attend(self, x2d: torch.Tensor, md: TokenMetadata, pool: PhysicalKVCachePool,
               out: Optional[torch.Tensor] = None, row_ss: Optional[torch.Tensor] = None,
               eps: float = 1e-5) -> torch.Tensor:
        """q/k/v GEMM, RoPE + KV write and paged attention; returns [T, local_heads*head_dim].

        With ``row_ss`` the input is the un-normalised ``z = h * w`` of a deferred RMSNorm
        (``kernels.linear_residual_norm``) and the q/k/v GEMM applies the row scale.
        """
        nq, nkv, hd = self.local_heads, self.local_kv_heads, self.head_dim
        wdt = self.q_proj.weight.dtype
        if x2d.dtype != wdt:
            x2d = x2d.to(wdt)
        wq, wk, wv = self.q_proj.packed_weight(), self.k_proj.packed_weight(), self.v_proj.packed_weight()
        q = torch.empty(md.n_tokens, nq * hd, dtype=wdt, device=x2d.device)
        # q|k|v GEMM with RoPE and the KV write in its epilogue where the shape allows it
        # (bit-identical to the GEMM + rope_kv_write pair below)
        if not kernels.linear_qkv_rope_kv(x2d, wq, wk, wv, nq, nkv, hd, md.rope_pos, md.store_pos, md.table_index,
                                          md.tables, self.rope.cos_cached, self.rope.sin_cached, q, pool.k_cache,
                                          pool.v_cache, self.layer_idx, row_ss=row_ss, eps=eps):
            if row_ss is not None:
                qkv = kernels.linear_qkv_rownorm(x2d, wq, wk, wv, row_ss, eps)
            else:
                qkv = kernels.linear_qkv(x2d, wq, wk, wv)
            kernels.rope_kv_write(qkv, nq, nkv, hd, md.rope_pos, md.store_pos, md.table_index, md.tables,
                                  self.rope.cos_cached, self.rope.sin_cached, q, pool.k_cache, pool.v_cache,
                                  self.layer_idx)
        if (md.is_prefill and md.seq_start is not None
                and kernels.prefill_supported(wdt, nq, nkv, hd, pool.block_size)):
            # every prompt token of every sequence in one causal launch
            return kernels.prefill_attention(q, nq, nkv, hd, pool.k_cache, pool.v_cache, self.layer_idx, md.tables,
                                             md.seq_start, md.n_seqs, 1.0 / math.sqrt(hd), seq_ctx0=md.seq_ctx0,
                                             out=out)
        splits = kernels.attention_splits(md.n_tokens, nkv, md.max_ctx, pool.block_size, x2d.device)
        return kernels.paged_attention(q, nq, nkv, hd, pool.k_cache, pool.v_cache, self.layer_idx, md.tables,
                                       md.table_index, md.ctx_lens, md.compat_pad, 1.0 / math.sqrt(hd),
                                       out=out, num_splits=splits)

    def forward(self, x: torch.Tensor, positions: torch.Tensor, kv_pool: Optional[PhysicalKVCachePool] = None,
                block_tables: Optional[List[List[int]]] = None, is_prefill: bool = True,
                step_id: int = 0) -> torch.Tensor:
        """x: [batch, seq_len, hidden_dim]; positions: [batch, seq_len] -> [batch, seq_len, hidden_dim]."""
        B, S, _ = x.shape
        with torch.no_grad():
            if kv_pool is None or block_tables is None:
                # No cache given (attention.py:204-205): attend over the in-flight k/v by staging
                # them in a scratch pool with one block run per sequence.
                bs = 16
                nblk = (S + bs - 1) // bs
                kv_pool = PhysicalKVCachePool(B * nblk, bs, self.local_kv_heads, self.head_dim,
                                              self.layer_idx + 1, device=x.device, dtype=self.q_proj.weight.dtype)
                block_tables = [list(range(b * nblk, (b + 1) * nblk)) for b in range(B)]
                if not is_prefill:
                    raise ValueError("decode without a KV cache is not meaningful")
            md = build_metadata(positions, block_tables, is_prefill, x.device,
                                masked_padding=self.config.masked_decode_padding)
            attn = self.attend(x.reshape(B * S, -1), md, kv_pool)
            step_tag = f"step_{step_id}_l{self.layer_idx}_attn"
            return self.out_proj(attn.view(B, S, -1), step_tag=step_tag)
