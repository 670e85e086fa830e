"""Per-call token metadata for the paged attention kernels.

The reference walks Python lists per token (engine/model/attention.py:166-203).
Here one call's positions, block tables and context lengths become a few small
device arrays, built on the host with numpy and copied in one go:

* decode (one token per sequence): row b stores and attends at
  ``positions[b]``; ``ctx_lens[b] = positions[b] + 1``; the batch is padded to its
  longest context without a mask in compat mode (attention.py:190-203).
* prefill (S tokens per sequence, equal lengths like the reference's batch):
  token (b, t) is rotated at ``positions[b, t]``, stored at logical slot ``t``
  (attention.py:168-173) and attends causally to slots ``0..t``
  (attention.py:219-222), i.e. ``ctx = t + 1`` without padding.
* varlen prefill (``build_prefill_metadata``): the prompts of several sequences of
  different lengths concatenated into one call; ``seq_start`` delimits them and
  ``last_rows`` picks each sequence's last token for the lm_head.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch


@dataclass
class TokenMetadata:
    n_tokens: int
    is_prefill: bool
    rope_pos: torch.Tensor            # int64 [T]
    store_pos: Optional[torch.Tensor]  # int64 [T] (None: same as rope_pos)
    table_index: Optional[torch.Tensor]  # int32 [T] token -> block-table row (None: identity)
    tables: torch.Tensor              # int32 [R, W], -1 padded
    ctx_lens: torch.Tensor            # int32 [T]
    max_ctx: int
    compat_pad: bool
    # Prefill only: rows [seq_start[s], seq_start[s+1]) are sequence s (int32 [n_seqs + 1]),
    # at positions seq_ctx0[s] + (row - seq_start[s]) (seq_ctx0 None: 0).
    seq_start: Optional[torch.Tensor] = None
    n_seqs: int = 0
    seq_ctx0: Optional[torch.Tensor] = None
    # Varlen prefill: the row of each sequence's last token (int64 [n_seqs]).
    last_rows: Optional[torch.Tensor] = None


def pad_tables(block_tables: Sequence[Sequence[int]], min_width: int = 1) -> np.ndarray:
    width = max([min_width] + [len(t) for t in block_tables])
    out = np.full((max(1, len(block_tables)), width), -1, dtype=np.int32)
    for i, t in enumerate(block_tables):
        if len(t):
            out[i, :len(t)] = np.asarray(t, dtype=np.int32)
    return out


class PinnedStager:
    """Ring of pinned host buffers: packs a call's small arrays and uploads them with one copy.

    Each slot is reused only after the copy issued from it has completed (CUDA event),
    so uploads are asynchronous and the host never writes a buffer still in flight.
    """

    def __init__(self, device, slots: int = 4, nbytes: int = 1 << 20):
        self.device = torch.device(device)
        self.slots = [None] * slots
        self.events = [None] * slots
        self.nbytes = [0] * slots
        self.i = 0
        self.last_bytes = 0
        self._grow_all(nbytes)

    def _grow_all(self, nbytes):
        for k in range(len(self.slots)):
            self.slots[k] = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            self.nbytes[k] = nbytes

    def upload(self, arrays):
        """Copy numpy arrays to the device in one transfer; returns device tensors (same order)."""
        offs, total = [], 0
        for a in arrays:
            if a is None:
                offs.append(None)
                continue
            total = (total + 15) // 16 * 16
            offs.append(total)
            total += a.nbytes
        k = self.i
        self.i = (self.i + 1) % len(self.slots)
        if self.events[k] is not None:
            self.events[k].synchronize()
        if total > self.nbytes[k]:
            self.slots[k] = torch.empty(max(total, 2 * self.nbytes[k]), dtype=torch.uint8, pin_memory=True)
            self.nbytes[k] = self.slots[k].numel()
        host = self.slots[k].numpy()
        for a, o in zip(arrays, offs):
            if a is not None:
                host[o:o + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
        dev = self.slots[k][:max(total, 16)].to(self.device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.events[k] = ev
        self.last_bytes = total
        out = []
        for a, o in zip(arrays, offs):
            if a is None:
                out.append(None)
            else:
                out.append(dev[o:o + a.nbytes].view(torch.from_numpy(a[:0]).dtype).view(*a.shape))
        return out


def build_metadata(positions, block_tables: Sequence[Sequence[int]], is_prefill: bool, device,
                   masked_padding: bool = False, stager: Optional[PinnedStager] = None,
                   extra=None) -> TokenMetadata:
    """Device metadata for ``DistributedAttention.forward``-style arguments.

    positions: [B, S] (tensor on any device, or array-like); block_tables: B lists.
    With a ``stager`` all arrays (plus ``extra``, e.g. the token ids, returned as
    ``metadata.extra``) go up in one pinned asynchronous copy.
    """
    if isinstance(positions, torch.Tensor):
        pos = positions.detach().to("cpu", torch.int64).numpy()
    else:
        pos = np.asarray(positions, dtype=np.int64)
    if pos.ndim == 1:
        pos = pos[:, None]
    B, S = pos.shape
    tables = pad_tables(block_tables)
    seq_start = None
    if is_prefill:
        store = np.tile(np.arange(S, dtype=np.int64), B)
        tidx = np.repeat(np.arange(B, dtype=np.int32), S)
        ctx = (store + 1).astype(np.int32)
        rope = pos.reshape(-1)
        compat = False
        seq_start = (np.arange(B + 1, dtype=np.int32) * S).astype(np.int32)
    else:
        assert S == 1, "decode takes one token per sequence"
        rope = pos[:, 0]
        store = None
        tidx = None
        ctx = (rope + 1).astype(np.int32)
        compat = not masked_padding
    dev = torch.device(device)
    arrays = [rope.astype(np.int64), None if store is None else store.astype(np.int64), tidx, tables,
              ctx, extra, seq_start]
    if stager is not None:
        d = stager.upload(arrays)
    else:
        d = [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays]
    md = TokenMetadata(n_tokens=B * S, is_prefill=is_prefill, rope_pos=d[0], store_pos=d[1], table_index=d[2],
                       tables=d[3], ctx_lens=d[4], max_ctx=int(ctx.max()) if ctx.size else 0, compat_pad=compat,
                       seq_start=d[6], n_seqs=B if is_prefill else 0)
    md.extra = d[5]
    return md


def prefill_layout(prompt_lens: Sequence[int], ctx0: Optional[Sequence[int]] = None):
    """Host arrays of a varlen prefill: (rope/store positions int64 [T], table row int32 [T],
    ctx int32 [T], seq_start int32 [n+1], last rows int64 [n], ctx0 int32 [n] or None)."""
    lens = np.asarray(prompt_lens, dtype=np.int64).reshape(-1)
    if lens.size == 0 or (lens <= 0).any():
        raise ValueError(f"varlen prefill needs prompts of at least one token, got lengths {lens.tolist()}")
    n = lens.size
    c0 = np.zeros(n, dtype=np.int64) if ctx0 is None else np.asarray(ctx0, dtype=np.int64).reshape(n)
    if (c0 < 0).any():
        raise ValueError("seq_ctx0 must be >= 0")
    seq_start = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=seq_start[1:])
    T = int(seq_start[-1])
    tidx = np.repeat(np.arange(n, dtype=np.int32), lens)
    pos = np.arange(T, dtype=np.int64) - np.repeat(seq_start[:-1], lens) + np.repeat(c0, lens)
    ctx = (pos + 1).astype(np.int32)
    last = (seq_start[1:] - 1).astype(np.int64)
    return pos, tidx, ctx, seq_start.astype(np.int32), last, (None if ctx0 is None else c0.astype(np.int32))


def build_prefill_metadata(prompt_lens: Sequence[int], block_tables: Sequence[Sequence[int]], device,
                           stager: Optional[PinnedStager] = None, extra=None,
                           ctx0: Optional[Sequence[int]] = None) -> TokenMetadata:
    """Metadata of one prefill call over several prompts of different lengths.

    Sequence s contributes ``prompt_lens[s]`` consecutive rows at positions
    ``ctx0[s] + arange(prompt_lens[s])`` (the reference's ``arange(P)`` when ctx0 is
    None, execution_engine.py:88-93), stored through block-table row s.  ``extra``
    (e.g. the concatenated token ids) rides along in the same upload.
    """
    if len(block_tables) != len(prompt_lens):
        raise ValueError(f"{len(block_tables)} block tables for {len(prompt_lens)} prompts")
    pos, tidx, ctx, seq_start, last, c0 = prefill_layout(prompt_lens, ctx0)
    tables = pad_tables(block_tables)
    arrays = [pos, None, tidx, tables, ctx, extra, seq_start, last, c0]
    if stager is not None:
        d = stager.upload(arrays)
    else:
        dev = torch.device(device)
        d = [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays]
    md = TokenMetadata(n_tokens=int(pos.size), is_prefill=True, rope_pos=d[0], store_pos=d[0], table_index=d[2],
                       tables=d[3], ctx_lens=d[4], max_ctx=int(ctx.max()), compat_pad=False, seq_start=d[6],
                       n_seqs=len(prompt_lens), seq_ctx0=d[8], last_rows=d[7])
    md.extra = d[5]
    return md
