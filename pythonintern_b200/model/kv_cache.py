"""Paged KV cache: block tables, the HBM pool and the block allocator.

Drop-in for engine/model/kv_cache.py.  ``BlockTable`` and ``KVCacheManager`` are
host-side bookkeeping with the reference's exact semantics (FIFO free list with
``pop(0)``, kv_cache.py:150-227).  ``PhysicalKVCachePool`` keeps the reference's
layout ``[L, num_blocks, block_size, kv_heads, head_dim]`` for ``k_cache`` and
``v_cache`` (kv_cache.py:45-80) but allocates it in HBM in the model dtype.  The
decoder path writes and reads it only inside the CUDA kernels
(``b2_rope_kv_write``, ``b2_paged_attention``); ``store_kv``/``read_kv_sequence``
remain for API compatibility as device-side copies.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch

from pythonintern_b200.config import KVCacheConfig, ModelConfig
from pythonintern_b200._lib import torch_dtype


class BlockTable:
    """Logical token index -> (physical block, offset) for one sequence (kv_cache.py:13-43)."""

    def __init__(self, seq_id: str, block_size: int):
        self.seq_id = seq_id
        self.block_size = block_size
        self.physical_block_ids: List[int] = []
        self.num_tokens: int = 0

    def append_block(self, block_id: int):
        self.physical_block_ids.append(block_id)

    def num_allocated_blocks(self) -> int:
        return len(self.physical_block_ids)

    def get_physical_slot(self, logical_pos: int) -> Tuple[int, int]:
        block_idx = logical_pos // self.block_size
        offset = logical_pos % self.block_size
        assert block_idx < len(self.physical_block_ids), (
            f"sequence {self.seq_id}: token {logical_pos} falls in block {block_idx}, but only "
            f"{len(self.physical_block_ids)} blocks are allocated")
        return self.physical_block_ids[block_idx], offset


class PhysicalKVCachePool:
    """K/V pool ``[L, num_blocks, block_size, kv_heads, head_dim]`` in HBM (kv_cache.py:45-147)."""

    def __init__(self, num_blocks: int, block_size: int, num_local_kv_heads: int, head_dim: int,
                 num_layers: int, device="cuda", dtype=None):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_local_kv_heads = num_local_kv_heads
        self.head_dim = head_dim
        self.num_layers = num_layers
        self.device = torch.device(device)
        if self.device.type not in ("cuda", "meta"):
            # "meta" gives a shape-only pool for host-side bookkeeping without a GPU.
            raise ValueError("PhysicalKVCachePool lives in HBM: device must be cuda")
        dt = torch_dtype(dtype)
        shape = (num_layers, num_blocks, block_size, num_local_kv_heads, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dt, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=dt, device=self.device)

    @property
    def dtype(self) -> torch.dtype:
        return self.k_cache.dtype

    def store_kv(self, layer_idx: int, physical_block_id: int, offset: int, k: torch.Tensor, v: torch.Tensor):
        """One token's K/V ``[kv_heads, head_dim]`` into a slot (kv_cache.py:85-100)."""
        self.k_cache[layer_idx, physical_block_id, offset].copy_(k)
        self.v_cache[layer_idx, physical_block_id, offset].copy_(v)

    def store_kv_batch(self, layer_idx: int, block_ids: List[int], offsets: List[int], k: torch.Tensor,
                       v: torch.Tensor):
        """Tokens ``i`` into slots ``(block_ids[i], offsets[i])`` (kv_cache.py:102-119)."""
        b = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)
        o = torch.as_tensor(offsets, dtype=torch.long, device=self.device)
        self.k_cache[layer_idx, b, o] = k.to(self.k_cache.dtype)
        self.v_cache[layer_idx, b, o] = v.to(self.v_cache.dtype)

    def read_kv_sequence(self, layer_idx: int, block_ids: List[int], seq_len: int):
        """Gather a sequence's first ``seq_len`` K/V rows (kv_cache.py:121-147)."""
        if not block_ids:
            e = torch.empty((0, self.num_local_kv_heads, self.head_dim), dtype=self.dtype, device=self.device)
            return e, e.clone()
        idx = torch.as_tensor(block_ids, dtype=torch.long, device=self.device)
        k = self.k_cache[layer_idx].index_select(0, idx).view(-1, self.num_local_kv_heads, self.head_dim)
        v = self.v_cache[layer_idx].index_select(0, idx).view(-1, self.num_local_kv_heads, self.head_dim)
        return k[:seq_len], v[:seq_len]


class KVCacheManager:
    """Block allocation, freeing and per-sequence tables (kv_cache.py:150-227)."""

    def __init__(self, config: KVCacheConfig, model_config: ModelConfig, world_size: int):
        self.config = config
        self.block_size = config.block_size
        self.total_blocks = config.num_blocks
        self.free_blocks: List[int] = list(range(config.num_blocks))
        self.block_tables: Dict[str, BlockTable] = {}
        num_local_kv_heads = max(1, model_config.num_kv_heads // world_size)
        device = config.device if config.device not in ("cpu", None) else "cuda"
        self.pool = PhysicalKVCachePool(
            num_blocks=config.num_blocks, block_size=config.block_size, num_local_kv_heads=num_local_kv_heads,
            head_dim=model_config.head_dim, num_layers=model_config.num_layers, device=device,
            dtype=model_config.dtype)

    @property
    def free_block_count(self) -> int:
        return len(self.free_blocks)

    @property
    def allocated_block_count(self) -> int:
        return self.total_blocks - len(self.free_blocks)

    def allocate_blocks_for_sequence(self, seq_id: str, num_tokens: int) -> BlockTable:
        needed_blocks = math.ceil(num_tokens / self.block_size)
        if needed_blocks > len(self.free_blocks):
            raise MemoryError(f"sequence {seq_id} needs {needed_blocks} KV blocks; "
                              f"{len(self.free_blocks)} are free")
        if seq_id not in self.block_tables:
            self.block_tables[seq_id] = BlockTable(seq_id, self.block_size)
        table = self.block_tables[seq_id]
        for _ in range(needed_blocks - len(table.physical_block_ids)):
            table.append_block(self.free_blocks.pop(0))
        table.num_tokens = num_tokens
        return table

    def append_token(self, seq_id: str) -> Tuple[int, int]:
        table = self.block_tables[seq_id]
        new_token_pos = table.num_tokens
        block_idx = new_token_pos // self.block_size
        offset = new_token_pos % self.block_size
        if block_idx >= len(table.physical_block_ids):
            if not self.free_blocks:
                raise MemoryError(f"KV pool exhausted: no free block for the next token of sequence {seq_id}")
            table.append_block(self.free_blocks.pop(0))
        table.num_tokens += 1
        return table.physical_block_ids[block_idx], offset

    def free_sequence(self, seq_id: str) -> int:
        if seq_id not in self.block_tables:
            return 0
        table = self.block_tables.pop(seq_id)
        self.free_blocks.extend(table.physical_block_ids)
        return len(table.physical_block_ids)
