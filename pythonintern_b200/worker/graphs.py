"""CUDA-graph capture of the batched decode step.

A decode step launches five kernels per decoder layer at world size 1 (seven with
tensor parallelism) plus the embedding, the norms, the lm_head and the greedy
sampling.  Launching them one by one from Python costs more host time than the GPU
needs for a small batch, so each (batch, table width) bucket captures the whole step
once and replays it.

Everything the step reads that changes between steps lives in ONE static device
buffer (token ids, positions, context lengths, padded block tables), refreshed by a
single copy from pinned host memory before each replay (``upload_host``; only the
block-table rows that changed since the previous step are repacked).  Kernel
arguments baked into the graph (tensor maps, split counts, communicator buffers) stay
valid because every buffer the step touches is either static here, part of the model,
or allocated from the graph's private memory pool during capture; the tensor-parallel
exchange slots rotate on a device-side epoch, so replays need no host bookkeeping.
"""

from __future__ import annotations

from typing import Dict, Optional, Sequence, Tuple

import numpy as np
import torch

from pythonintern_b200.model.metadata import TokenMetadata


def _layout(batch: int, width: int):
    """Byte offsets of the packed step inputs: tok int64, pos int64, ctx int32, tables int32."""
    def up16(x):
        return (x + 15) // 16 * 16
    o_tok = 0
    o_pos = up16(o_tok + 8 * batch)
    o_ctx = up16(o_pos + 8 * batch)
    o_tab = up16(o_ctx + 4 * batch)
    total = up16(o_tab + 4 * batch * width)
    return o_tok, o_pos, o_ctx, o_tab, total


def table_bucket(width: int) -> int:
    """Block-table widths are padded to a multiple of 32 blocks (512 tokens) per bucket."""
    return max(32, (width + 31) // 32 * 32)


class DecodeGraph:
    """One captured decode step for a fixed batch size and padded block-table width."""

    def __init__(self, model, pool, batch: int, width: int, masked_padding: bool = False):
        self.model = model
        self.pool = pool
        self.batch = batch
        self.width = width
        self.device = model.device
        o_tok, o_pos, o_ctx, o_tab, total = _layout(batch, width)
        self.nbytes = total
        self.meta = torch.zeros(total, dtype=torch.uint8, device=self.device)
        self.tok = self.meta[o_tok:o_tok + 8 * batch].view(torch.int64).view(batch, 1)
        self.pos = self.meta[o_pos:o_pos + 8 * batch].view(torch.int64)
        self.ctx = self.meta[o_ctx:o_ctx + 4 * batch].view(torch.int32)
        self.tables = self.meta[o_tab:o_tab + 4 * batch * width].view(torch.int32).view(batch, width)
        self.md = TokenMetadata(n_tokens=batch, is_prefill=False, rope_pos=self.pos, store_pos=None,
                                table_index=None, tables=self.tables, ctx_lens=self.ctx, max_ctx=width * 16,
                                compat_pad=not masked_padding)
        self.host = [torch.zeros(total, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        # Host copy of the packed block tables and the rows they were built from: a
        # decode step usually changes a few rows (a sequence crossing into a new block),
        # so only rows that differ from the previous step are converted again.
        self._tab = np.full((batch, width), -1, dtype=np.int32)
        self._rows: list = [None] * batch
        self.host_events = [None, None]
        self.host_i = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.top: Optional[torch.Tensor] = None
        self.next_tok: Optional[torch.Tensor] = None

    # -- packing -------------------------------------------------------------------
    def pack(self, tokens: Sequence[int], positions: Sequence[int], tables: Sequence[Sequence[int]],
             out: np.ndarray) -> np.ndarray:
        """Packs one step's host inputs into ``out`` (uint8, this graph's layout)."""
        B, W = self.batch, self.width
        o_tok, o_pos, o_ctx, o_tab, total = _layout(B, W)
        pos = np.asarray(positions, dtype=np.int64).reshape(B)
        out[o_tok:o_tok + 8 * B] = np.asarray(tokens, dtype=np.int64).reshape(B).view(np.uint8)
        out[o_pos:o_pos + 8 * B] = pos.view(np.uint8)
        out[o_ctx:o_ctx + 4 * B] = (pos + 1).astype(np.int32).view(np.uint8)
        tab, rows = self._tab, self._rows
        if len(tables) != B:
            raise ValueError(f"{len(tables)} block tables for a graph of batch {B}")
        for b, t in enumerate(tables):
            row = t if isinstance(t, list) else [int(x) for x in t]
            if rows[b] is not None and row == rows[b]:
                continue
            if len(row) > W:
                raise ValueError(f"block table of {len(row)} entries exceeds the graph's width {W}")
            row = list(row)
            tab[b, :len(row)] = row
            tab[b, len(row):] = -1
            rows[b] = row
        out[o_tab:o_tab + 4 * B * W] = tab.view(np.uint8).reshape(-1)
        return out

    def upload_host(self, tokens, positions, tables):
        """Pinned host staging -> the static device buffer (one asynchronous copy)."""
        k = self.host_i
        self.host_i ^= 1
        if self.host_events[k] is not None:
            self.host_events[k].synchronize()
        self.pack(tokens, positions, tables, self.host[k].numpy())
        self.meta.copy_(self.host[k], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.host_events[k] = ev

    # -- capture / replay -------------------------------------------------------------
    def _step(self):
        return self.model.greedy(self.tok, None, self.pool, [[]] * self.batch, False, 0, metadata=self.md)

    def capture(self):
        """Runs the step once eagerly (sizes workspaces, sets kernel attributes), then captures it.

        The static buffer must already hold a valid step (its KV slots are written by
        the eager run and rewritten identically by the first replay).
        """
        with torch.no_grad():
            self._step()
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.next_tok, self.top = self._step()
        self.graph = g

    def replay(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Runs the captured step; returns (greedy tokens [batch], first ten logits [batch, 10])."""
        self.graph.replay()
        return self.next_tok, self.top


class DecodeGraphCache:
    """Decode graphs keyed by (batch size, padded table width)."""

    def __init__(self, model, pool, masked_padding: bool = False, max_graphs: int = 16):
        self.model = model
        self.pool = pool
        self.masked = masked_padding
        self.max_graphs = max_graphs
        self.graphs: Dict[Tuple[int, int], DecodeGraph] = {}

    def get(self, batch: int, width: int) -> Tuple[DecodeGraph, bool]:
        key = (batch, table_bucket(width))
        g = self.graphs.get(key)
        if g is not None:
            return g, False
        if len(self.graphs) >= self.max_graphs:
            self.graphs.pop(next(iter(self.graphs)))
        g = DecodeGraph(self.model, self.pool, key[0], key[1], self.masked)
        self.graphs[key] = g
        return g, True

    def clear(self):
        self.graphs.clear()
