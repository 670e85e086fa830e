"""Sharded LLaMA / Mistral decoder (engine/model/llama.py:25-174).

``DistributedTransformerBlock`` and ``DistributedLLaMAModel`` keep the reference's
module tree and parameter names (so ``state_dict`` keys match the reference and
its WeightSharder), and the reference's forward signatures.

``DistributedLLaMAModel.forward`` runs the fused path.  The residual stream stays
float32 in HBM, and each row-parallel projection is followed by ONE kernel that finishes
the all-reduce, adds the residual and applies the NEXT RMSNorm (the post-attention norm,
the next layer's input norm, or the final norm), so a decoder layer is seven kernels:

    qkv GEMM -> RoPE + KV write -> paged attention -> o_proj GEMM
    -> all-reduce + residual + norm -> gate/up GEMM + SwiGLU -> down GEMM
    -> all-reduce + residual + norm

With world_size > 1 the residual is sharded by rows: each rank keeps the float32
residual of its own rows only, the row-parallel GEMM pushes each partial row to the rank
that owns it straight from its epilogue (NVLink stores into peer memory), and the owner
sums, normalises and pushes the normalised row to every rank (all-gather), all inside
``b2_row_parallel_linear`` + ``b2_allreduce_rmsnorm_sharded``.
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from pythonintern_b200 import kernels
from pythonintern_b200.config import ModelConfig
from pythonintern_b200.model.attention import DistributedAttention
from pythonintern_b200.model.kv_cache import PhysicalKVCachePool
from pythonintern_b200.model.metadata import TokenMetadata, build_metadata
from pythonintern_b200.model.mlp import DistributedMLP
from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
from pythonintern_b200.tensor_parallel.layers import RMSNorm, RowParallelLinear
from pythonintern_b200._lib import torch_dtype


def _row_parallel_norm(proj: RowParallelLinear, inp: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor,
                       eps: float, y: torch.Tensor):
    """``h += inp @ W``; ``y = rmsnorm(h) * norm_w`` at world_size 1 (layers.py:147-162 + llama.py:70-75)."""
    partial = kernels.linear(inp, proj.packed_weight())
    kernels.rmsnorm(partial, norm_w, eps, residual=h, h_out=h, out=y)


class DistributedTransformerBlock(nn.Module):
    """Pre-norm residual block: ``h = x + attn(norm(x)); out = h + mlp(norm(h))`` (llama.py:25-76)."""

    def __init__(self, config: ModelConfig, layer_idx: int, rank: int = 0, world_size: int = 1,
                 communicator: Optional[DistributedCommunicator] = None, device=None):
        super().__init__()
        self.layer_idx = layer_idx
        self.input_layernorm = RMSNorm(config.hidden_dim, eps=config.rms_norm_eps, device=device)
        self.self_attn = DistributedAttention(config, layer_idx, rank, world_size, communicator, device=device)
        self.post_attention_layernorm = RMSNorm(config.hidden_dim, eps=config.rms_norm_eps, device=device)
        self.mlp = DistributedMLP(config, layer_idx, rank, world_size, communicator, device=device)

    def set_communicator(self, communicator: DistributedCommunicator):
        self.self_attn.set_communicator(communicator)
        self.mlp.set_communicator(communicator)

    def forward(self, x: torch.Tensor, positions: torch.Tensor, kv_pool: Optional[PhysicalKVCachePool] = None,
                block_tables: Optional[List[List[int]]] = None, is_prefill: bool = True,
                step_id: int = 0) -> torch.Tensor:
        with torch.no_grad():
            B, S, H = x.shape
            wdt = self.self_attn.q_proj.weight.dtype
            h = x.reshape(B * S, H).to(torch.float32).contiguous()  # residual stream, float32
            xn = kernels.rmsnorm(h, self.input_layernorm.weight, self.input_layernorm.eps, out_dtype=wdt)
            attn = self.self_attn(xn.view(B, S, H), positions, kv_pool, block_tables, is_prefill, step_id)
            xn2 = kernels.rmsnorm(attn, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps,
                                  residual=h, h_out=h, out_dtype=wdt)
            mlp = self.mlp(xn2.view(B, S, H), step_id=step_id)
            kernels.residual_add(mlp, h)
            return h.view(B, S, H).to(x.dtype)


class DistributedLLaMAModel(nn.Module):
    """Embedding, N blocks, final norm, replicated lm_head (llama.py:79-174)."""

    def __init__(self, config: ModelConfig, rank: int = 0, world_size: int = 1,
                 communicator: Optional[DistributedCommunicator] = None, device="cuda"):
        super().__init__()
        self.config = config
        self.rank = rank
        self.world_size = world_size
        self.communicator = communicator
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise ValueError("DistributedLLaMAModel runs on CUDA devices only")
        self.device = dev
        dt = torch_dtype(config.dtype)
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_dim, device=dev, dtype=dt)
        self.layers = nn.ModuleList([
            DistributedTransformerBlock(config, i, rank, world_size, communicator, device=dev)
            for i in range(config.num_layers)])
        self.norm = RMSNorm(config.hidden_dim, eps=config.rms_norm_eps, device=dev)
        self.lm_head = nn.Linear(config.hidden_dim, config.vocab_size, bias=False, device=dev, dtype=dt)

    def set_communicator(self, communicator: DistributedCommunicator):
        self.communicator = communicator
        for layer in self.layers:
            layer.set_communicator(communicator)

    @property
    def dtype(self) -> torch.dtype:
        return self.embed_tokens.weight.dtype

    def _forward_hidden_sharded(self, ids: torch.Tensor, md: TokenMetadata, kv_pool: PhysicalKVCachePool,
                                trace: Optional[list]) -> torch.Tensor:
        """Tensor-parallel layers with a row-sharded residual (world_size > 1).

        Each rank keeps the float32 residual only for its rows; every row-parallel GEMM
        pushes its partial rows to their owners from its epilogue, and the owners finish
        the all-reduce, add the residual, normalise and all-gather the normalised rows
        into every rank's buffer (``b2_row_parallel_linear`` + ``b2_allreduce_rmsnorm_sharded``).
        """
        cfg, comm = self.config, self.communicator
        eps = cfg.rms_norm_eps
        T, H = md.n_tokens, cfg.hidden_dim
        wdt = self.dtype
        h_all = kernels.embedding(ids, self.embed_tokens.weight, out_dtype=torch.float32)
        xn = torch.empty(T, H, dtype=wdt, device=self.device)
        kernels.rmsnorm(h_all, self.layers[0].input_layernorm.weight, eps, out=xn)
        r0, r1, R = comm.row_slice(T)
        h = torch.zeros(R, H, dtype=torch.float32, device=self.device)
        if r1 > r0:
            h[: r1 - r0].copy_(h_all[r0:r1])
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            attn = layer.self_attn.attend(xn, md, kv_pool)
            comm.row_parallel_linear(attn, layer.self_attn.out_proj.packed_weight())
            xn = comm.allreduce_rmsnorm_sharded(T, H, wdt, h, layer.post_attention_layernorm.weight, eps)
            inter = layer.mlp.gate_up(xn)
            next_w = self.layers[i + 1].input_layernorm.weight if i + 1 < n else self.norm.weight
            comm.row_parallel_linear(inter, layer.mlp.down_proj.packed_weight())
            xn = comm.allreduce_rmsnorm_sharded(T, H, wdt, h, next_w, eps)
            if trace is not None:
                trace.append((r0, h[: r1 - r0].clone()))
        return xn

    def forward_hidden(self, token_ids: torch.Tensor, md: TokenMetadata, kv_pool: PhysicalKVCachePool,
                       trace: Optional[list] = None) -> torch.Tensor:
        """Runs every layer; returns the final-normed hidden states [T, hidden] in the model dtype.

        ``trace`` (optional list) receives a copy of the float32 residual stream after
        each layer (the reference block's output), for parity checks; with
        world_size > 1 each entry is ``(first_row, rows)`` of this rank's row slice.
        """
        if self.world_size > 1:
            if self.communicator is None:
                raise RuntimeError("world_size > 1 needs a communicator (set_communicator)")
            ids = token_ids.reshape(-1)
            if ids.device != self.device or ids.dtype != torch.int64:
                ids = ids.to(self.device, torch.int64)
            return self._forward_hidden_sharded(ids, md, kv_pool, trace)
        cfg = self.config
        eps = cfg.rms_norm_eps
        T, H = md.n_tokens, cfg.hidden_dim
        wdt = self.dtype
        ids = token_ids.reshape(-1)
        if ids.device != self.device or ids.dtype != torch.int64:
            ids = ids.to(self.device, torch.int64)
        h = kernels.embedding(ids, self.embed_tokens.weight, out_dtype=torch.float32)
        xn = torch.empty(T, H, dtype=wdt, device=self.device)
        kernels.rmsnorm(h, self.layers[0].input_layernorm.weight, eps, out=xn)
        # Deferred RMSNorm (bf16, <= 512 rows, where the GEMM gets a split-K cluster plan):
        # the row-parallel GEMM adds the residual and leaves z = h * w plus per-tile sums of
        # h^2; the next GEMM applies the row scale.
        # ready: the next GEMM's input is (z, ss) rather than the normalised xn.
        fused = wdt == torch.bfloat16 and T <= 512 and H % 128 == 0
        z = torch.empty(T, H, dtype=wdt, device=self.device) if fused else None
        ss = torch.empty(T, H // 128, dtype=torch.float32, device=self.device) if fused else None
        ready = False
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            attn = layer.self_attn.attend(z if ready else xn, md, kv_pool, row_ss=ss if ready else None, eps=eps)
            post_w = layer.post_attention_layernorm.weight
            ready = fused and kernels.linear_residual_norm(attn, layer.self_attn.out_proj.packed_weight(), h, post_w,
                                                           z, ss)
            if not ready:
                _row_parallel_norm(layer.self_attn.out_proj, attn, h, post_w, eps, xn)
            inter = layer.mlp.gate_up(z if ready else xn, row_ss=ss if ready else None, eps=eps)
            next_w = self.layers[i + 1].input_layernorm.weight if i + 1 < n else self.norm.weight
            ready = fused and i + 1 < n and kernels.linear_residual_norm(inter, layer.mlp.down_proj.packed_weight(),
                                                                         h, next_w, z, ss)
            if not ready:
                _row_parallel_norm(layer.mlp.down_proj, inter, h, next_w, eps, xn)
            if trace is not None:
                trace.append(h.clone())
        return xn

    def vocab_slice(self):
        """Vocabulary ids [start, end) whose logits this rank computes in ``greedy``.

        The lm_head weight stays replicated (llama.py:121; sharding.py:105-107), so
        checkpoints load unchanged; with world_size > 1 each rank multiplies only its
        contiguous row slice of it and the ranks exchange one (max, index) pair per row.
        """
        V, t = self.config.vocab_size, max(1, self.world_size)
        per = -(-V // t)
        start = min(V, self.rank * per)
        return start, min(V, start + per)

    def greedy(self, token_ids: torch.Tensor, positions: Optional[torch.Tensor],
               kv_pool: PhysicalKVCachePool, block_tables: Optional[List[List[int]]], is_prefill: bool = False,
               step_id: int = 0, metadata: Optional[TokenMetadata] = None):
        """Greedy next token and the first ten logits of each sequence's last position.

        Equals ``argmax(forward(...))`` and ``forward(...)[:, :10]`` (execution_engine.py:
        103-108, 131-135) without materialising the full logits on every rank.
        """
        with torch.no_grad():
            B, S = token_ids.shape
            md = metadata or build_metadata(positions, block_tables, is_prefill, self.device,
                                            masked_padding=self.config.masked_decode_padding)
            xn = self.forward_hidden(token_ids, md, kv_pool)
            if md.last_rows is not None:  # varlen prefill: gather each sequence's last row
                last = kernels.embedding(md.last_rows, xn)
            else:
                last = xn.view(B, S, -1)[:, -1, :]  # row-strided view, no copy
            w = self.lm_head.weight
            if self.world_size == 1:
                logits = kernels.linear(last, w, out_dtype=torch.float32)
                return kernels.argmax(logits), logits[:, :10]
            v0, v1 = self.vocab_slice()
            logits = kernels.linear(last, w[v0:v1], out_dtype=torch.float32)
            tok = self.communicator.argmax_allgather(logits, v0)
            if v0 == 0 and v1 >= 10:
                top = logits[:, :10]
            else:
                top = kernels.linear(last, w[:10], out_dtype=torch.float32)
            return tok, top

    def forward(self, token_ids: torch.Tensor, positions: torch.Tensor,
                kv_pool: Optional[PhysicalKVCachePool] = None, block_tables: Optional[List[List[int]]] = None,
                is_prefill: bool = True, step_id: int = 0, return_logits_last_only: bool = True,
                metadata: Optional[TokenMetadata] = None, trace: Optional[list] = None) -> torch.Tensor:
        """token_ids/positions: [batch, seq_len] -> float32 logits [batch, vocab] (last token) or [batch, seq, vocab]."""
        if kv_pool is None or block_tables is None:
            raise ValueError("the fused decoder path needs a KV pool and block tables")
        with torch.no_grad():
            B, S = token_ids.shape
            md = metadata or build_metadata(positions, block_tables, is_prefill, self.device,
                                            masked_padding=self.config.masked_decode_padding)
            xn = self.forward_hidden(token_ids, md, kv_pool, trace=trace)
            if return_logits_last_only:
                if md.last_rows is not None:
                    last = kernels.embedding(md.last_rows, xn)
                else:
                    last = xn.view(B, S, -1)[:, -1, :]  # row-strided view, no copy
                return kernels.linear(last, self.lm_head.weight, out_dtype=torch.float32)
            return kernels.linear(xn, self.lm_head.weight, out_dtype=torch.float32).view(B, S, -1)
