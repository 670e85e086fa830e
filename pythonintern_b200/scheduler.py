"""Coordinator-side block bookkeeping with an opt-in fix for the reference's off-by-one.

The reference's coordinator (engine/scheduler/memory_manager.py:12-87,
``ClusterMemoryManager``) hands each running sequence a block table before every
decode step.  Its ``append_token_slot`` (memory_manager.py:54-74) adds a block when
``total_length % block_size == 0``, but the worker then writes the step's token at
position ``total_length - 1`` (execution_engine.py:113-130, attention.py:177-184).  A
prompt whose length is a multiple of the block size therefore reaches its first decode
with a table one block short: the reference worker raises IndexError and the sequence
never advances.

``ClusterMemoryManager`` here keeps that behaviour by default, so a batcher built on it
schedules exactly what the reference schedules, and takes ``fixed_allocator=True`` to
allocate whenever the table does not yet cover the position the step writes
(``len(table) * block_size < total_length``).  The free list is FIFO (``pop(0)``) like
the reference's, so block ids match it step for step wherever the two agree.

``sequence`` arguments need ``seq_id``, ``prompt_token_ids`` and ``total_length``
(the reference's engine/scheduler/sequence.py:57-59: prompt plus generated tokens).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

from pythonintern_b200.config import KVCacheConfig


class ClusterMemoryManager:
    """FIFO block allocator of the coordinator (memory_manager.py:12-87)."""

    def __init__(self, kv_config: KVCacheConfig, fixed_allocator: bool = False):
        self.block_size = kv_config.block_size
        self.total_blocks = kv_config.num_blocks
        self.fixed_allocator = fixed_allocator
        self.free_blocks: List[int] = list(range(self.total_blocks))
        self.seq_block_tables: Dict[str, List[int]] = {}

    @property
    def free_block_count(self) -> int:
        return len(self.free_blocks)

    @property
    def used_block_count(self) -> int:
        return self.total_blocks - len(self.free_blocks)

    @property
    def memory_utilization(self) -> float:
        return self.used_block_count / self.total_blocks if self.total_blocks > 0 else 0.0

    def _prompt_blocks(self, sequence) -> int:
        return math.ceil(len(sequence.prompt_token_ids) / self.block_size)

    def can_allocate_prefill(self, sequence) -> bool:
        return len(self.free_blocks) >= self._prompt_blocks(sequence)

    def allocate_prefill(self, sequence) -> List[int]:
        """Blocks for the prompt (memory_manager.py:42-52)."""
        need = self._prompt_blocks(sequence)
        if need > len(self.free_blocks):
            raise MemoryError(f"prefill of {sequence.seq_id} needs {need} KV blocks, "
                              f"only {len(self.free_blocks)} are free")
        table = [self.free_blocks.pop(0) for _ in range(need)]
        self.seq_block_tables[sequence.seq_id] = table
        return table

    def _needs_block(self, sequence) -> bool:
        if self.fixed_allocator:
            # the step writes position total_length - 1: the table must cover total_length tokens
            table = self.seq_block_tables.get(sequence.seq_id, [])
            return len(table) * self.block_size < sequence.total_length
        return sequence.total_length % self.block_size == 0  # the reference's test (:58, :67)

    def can_append_token(self, sequence) -> bool:
        return bool(self.free_blocks) or not self._needs_block(sequence)

    def append_token_slot(self, sequence) -> Optional[int]:
        """Adds a block if this step needs one; returns its id, else None (memory_manager.py:54-74)."""
        if not self._needs_block(sequence):
            return None
        if not self.free_blocks:
            raise MemoryError(f"no free KV block left to extend {sequence.seq_id}")
        block = self.free_blocks.pop(0)
        self.seq_block_tables[sequence.seq_id].append(block)
        return block

    def free_sequence(self, sequence) -> List[int]:
        blocks = self.seq_block_tables.pop(sequence.seq_id, [])
        self.free_blocks.extend(blocks)
        return blocks

    def get_block_table(self, seq_id: str) -> List[int]:
        return self.seq_block_tables.get(seq_id, [])
