"""Numpy restatement of the reference's tensor-parallel decoder-layer forward.

TEST INFRASTRUCTURE ONLY (the checker and the timed CPU stand-in for the
reference); the product path in ``pythonintern_b200`` never imports this module.

Every function cites the reference file:line it restates.  Paths are relative to
the reference project root (kmadasamy212-tech/pythonintern).  Arithmetic is done
in float64 on float32 (or bf16-rounded) inputs, so the oracle is at least as
accurate as the reference's float32 PyTorch path; the KV pool stores float32 like
the reference's ``PhysicalKVCachePool`` (engine/model/kv_cache.py:70-80).

Tensor-parallel ranks are simulated in lock step: every rank computes its partial
row-parallel output and the all-reduce sums the partials in rank order 0..t-1
(engine/tensor_parallel/comm.py:114-116 sums local-then-arrival order; for t=2
the two-term sum is order independent).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

ACC = np.float64


def set_precision(dtype):
    """Arithmetic type of every oracle function (float64 for checking, float32 to time
    the reference's float32 arithmetic)."""
    global ACC
    ACC = np.dtype(dtype).type


# --------------------------------------------------------------------------------------
# Elementwise pieces
# --------------------------------------------------------------------------------------

def rope_tables(head_dim: int, max_seq_len: int, base: float = 10000.0):
    """cos/sin tables of shape [max_seq_len, head_dim], float32.

    engine/model/attention.py:35-44: ``inv_freq = 1/base**(arange(0,d,2)/d)``,
    ``freqs = outer(t, inv_freq)``, ``emb = cat(freqs, freqs)``.  Note that the
    reference builds its RotaryEmbedding without ``base=`` (attention.py:129), so
    the model always uses base 10000 whatever ``rope_theta`` says.
    """
    expo = (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)).astype(np.float64)
    # base**x rounded to float32, then a float32 reciprocal: the same rounding steps
    # as the reference's float32 tensor arithmetic.
    inv_freq = (np.float32(1.0) / (float(base) ** expo).astype(np.float32)).astype(np.float32)
    t = np.arange(max_seq_len, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x: np.ndarray, positions: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE, engine/model/attention.py:46-63.

    x: [..., S, heads, hd]; positions: [..., S] integer.  Returns float64.
    """
    hd = x.shape[-1]
    c = cos[positions][..., None, :].astype(ACC)
    s = sin[positions][..., None, :].astype(ACC)
    x = np.asarray(x, dtype=ACC)
    rot = np.concatenate([-x[..., hd // 2:], x[..., : hd // 2]], axis=-1)
    return x * c + rot * s


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """engine/tensor_parallel/layers.py:179-184: ``x * rsqrt(mean(x^2) + eps) * w``."""
    x = np.asarray(x, dtype=ACC)
    var = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(var + eps) * np.asarray(w, dtype=ACC)


def silu(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.silu as used at engine/model/mlp.py:82."""
    x = np.asarray(x, dtype=ACC)
    return x / (1.0 + np.exp(-x))


def softmax(s: np.ndarray, axis: int = -1) -> np.ndarray:
    m = np.max(s, axis=axis, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def column_parallel_linear(x: np.ndarray, w_in_out: np.ndarray, bias: Optional[np.ndarray] = None):
    """engine/tensor_parallel/layers.py:78-86: ``Y = X @ W (+ b)`` with W stored [in, out/t]."""
    y = np.asarray(x, dtype=ACC) @ np.asarray(w_in_out, dtype=ACC)
    if bias is not None:
        y = y + np.asarray(bias, dtype=ACC)
    return y


def all_reduce_sum(partials: Sequence[np.ndarray]) -> np.ndarray:
    """engine/tensor_parallel/comm.py:72-118 (result ``local + sum(peers)``), fixed rank order."""
    out = np.array(partials[0], dtype=ACC, copy=True)
    for p in partials[1:]:
        out = out + p
    return out


def row_parallel_linear(xs: Sequence[np.ndarray], ws: Sequence[np.ndarray], bias=None):
    """engine/tensor_parallel/layers.py:147-162: per-rank partial ``X_r @ W_r``, all-reduce, ``+b``."""
    out = all_reduce_sum([np.asarray(x, dtype=ACC) @ np.asarray(w, dtype=ACC) for x, w in zip(xs, ws)])
    if bias is not None:
        out = out + bias
    return out


# --------------------------------------------------------------------------------------
# Paged KV pool and block tables
# --------------------------------------------------------------------------------------

def physical_slot(block_table: Sequence[int], logical_pos: int, block_size: int):
    """engine/model/kv_cache.py:35-43 (``BlockTable.get_physical_slot``)."""
    block_idx = logical_pos // block_size
    if block_idx >= len(block_table):
        raise IndexError(f"position {logical_pos} exceeds allocated blocks ({len(block_table)})")
    return int(block_table[block_idx]), logical_pos % block_size


class KVPool:
    """engine/model/kv_cache.py:45-147 (``PhysicalKVCachePool``): [L, NB, bs, kvh, hd] x2."""

    def __init__(self, num_layers, num_blocks, block_size, kv_heads, head_dim, dtype=np.float32):
        shape = (num_layers, num_blocks, block_size, kv_heads, head_dim)
        self.k = np.zeros(shape, dtype=dtype)
        self.v = np.zeros(shape, dtype=dtype)
        self.block_size = block_size
        self.kv_heads = kv_heads
        self.head_dim = head_dim

    def store(self, layer, block_id, offset, k, v):
        """kv_cache.py:85-100."""
        self.k[layer, block_id, offset] = k
        self.v[layer, block_id, offset] = v

    def read_sequence(self, layer, block_ids, seq_len):
        """kv_cache.py:121-147: gather whole blocks, flatten, keep the first ``seq_len`` rows."""
        if len(block_ids) == 0:
            e = np.zeros((0, self.kv_heads, self.head_dim), dtype=self.k.dtype)
            return e, e.copy()
        kb = self.k[layer, list(block_ids)].reshape(-1, self.kv_heads, self.head_dim)
        vb = self.v[layer, list(block_ids)].reshape(-1, self.kv_heads, self.head_dim)
        return kb[:seq_len], vb[:seq_len]


class FifoBlockAllocator:
    """engine/model/kv_cache.py:150-218 (``KVCacheManager``): FIFO free list, ``pop(0)``."""

    def __init__(self, num_blocks: int, block_size: int):
        self.free = list(range(num_blocks))
        self.block_size = block_size
        self.tables: Dict[str, List[int]] = {}
        self.num_tokens: Dict[str, int] = {}

    def allocate(self, seq_id: str, num_tokens: int) -> List[int]:
        """kv_cache.py:180-199."""
        need = math.ceil(num_tokens / self.block_size)
        if need > len(self.free):
            raise MemoryError(f"sequence {seq_id} needs {need} blocks")
        table = self.tables.setdefault(seq_id, [])
        while len(table) < need:
            table.append(self.free.pop(0))
        self.num_tokens[seq_id] = num_tokens
        return table

    def append_token(self, seq_id: str):
        """kv_cache.py:201-218."""
        table = self.tables[seq_id]
        pos = self.num_tokens[seq_id]
        idx, off = pos // self.block_size, pos % self.block_size
        if idx >= len(table):
            if not self.free:
                raise MemoryError("no free block left")
            table.append(self.free.pop(0))
        self.num_tokens[seq_id] += 1
        return table[idx], off


# --------------------------------------------------------------------------------------
# Attention
# --------------------------------------------------------------------------------------

def decode_attention(q, k_new, v_new, positions, pool: KVPool, layer, block_tables,
                     scale: float, compat_pad: bool = True):
    """Single-token decode over the paged cache, engine/model/attention.py:175-228.

    q: [B, nq, hd] (after RoPE); k_new/v_new: [B, nkv, hd] (k after RoPE);
    positions: [B].  Stores the new token at ``positions[b]`` (attention.py:180-184),
    gathers the sequence (kv_cache.py:121-147) and, like the reference, zero-pads
    every sequence to the batch's longest context WITHOUT a mask
    (attention.py:190-203), so padded keys score 0 and still enter the softmax
    denominator.  ``compat_pad=False`` gives the masked (per-sequence) result.
    Returns [B, nq*hd] float64.
    """
    B, nq, hd = q.shape
    nkv = k_new.shape[1]
    rep = nq // nkv
    bs = pool.block_size
    ks, vs = [], []
    for b in range(B):
        pos = int(positions[b])
        blk, off = physical_slot(block_tables[b], pos, bs)
        pool.store(layer, blk, off, k_new[b], v_new[b])
        k_seq, v_seq = pool.read_sequence(layer, block_tables[b], pos + 1)
        ks.append(np.asarray(k_seq, dtype=ACC))
        vs.append(np.asarray(v_seq, dtype=ACC))
    max_len = max(k.shape[0] for k in ks)
    out = np.zeros((B, nq, hd), dtype=ACC)
    for b in range(B):
        ctx = ks[b].shape[0]
        for h in range(nq):
            g = h // rep  # repeat_kv, attention.py:66-76
            s = (ks[b][:, g, :] @ np.asarray(q[b, h], dtype=ACC)) * scale
            if compat_pad and ctx < max_len:
                s = np.concatenate([s, np.zeros(max_len - ctx, dtype=ACC)])
            p = softmax(s)
            out[b, h] = p[:ctx] @ vs[b][:, g, :]
    return out.reshape(B, nq * hd)


def prefill_attention(q, k, v, pool: Optional[KVPool], layer, block_tables, scale: float):
    """Prompt attention, engine/model/attention.py:166-174 and :211-228.

    q: [B, S, nq, hd], k/v: [B, S, nkv, hd] (q, k after RoPE).  Every prompt token
    is stored at logical position ``t`` (attention.py:170-173); attention uses the
    in-flight k/v with a causal mask.  Returns [B, S, nq*hd] float64.
    """
    B, S, nq, hd = q.shape
    nkv = k.shape[2]
    rep = nq // nkv
    if pool is not None and block_tables is not None:
        for b in range(B):
            for t in range(S):
                blk, off = physical_slot(block_tables[b], t, pool.block_size)
                pool.store(layer, blk, off, k[b, t], v[b, t])
    out = np.zeros((B, S, nq, hd), dtype=ACC)
    causal = np.triu(np.full((S, S), -np.inf), k=1)
    for b in range(B):
        for h in range(nq):
            g = h // rep
            s = (q[b, :, h, :].astype(ACC) @ k[b, :, g, :].astype(ACC).T) * scale + causal
            out[b, :, h, :] = softmax(s) @ v[b, :, g, :].astype(ACC)
    return out.reshape(B, S, nq * hd)


# --------------------------------------------------------------------------------------
# Model
# --------------------------------------------------------------------------------------

@dataclass
class OracleConfig:
    """engine/config.py:13-37 (``ModelConfig``), the fields the forward reads."""
    vocab_size: int
    hidden_dim: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    intermediate_dim: int
    max_seq_len: int = 2048
    rms_norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads


def shard_state_dict(full: Dict[str, np.ndarray], rank: int, world_size: int) -> Dict[str, np.ndarray]:
    """engine/tensor_parallel/sharding.py:96-107 (``WeightSharder.shard_full_model_state_dict``).

    Column-parallel weights ([in, out]) are sliced along dim 1, row-parallel along
    dim 0; every other tensor is replicated.
    """
    out = {}
    for key, t in full.items():
        if any(s in key for s in ("q_proj.weight", "k_proj.weight", "v_proj.weight",
                                  "gate_proj.weight", "up_proj.weight")):
            c = t.shape[1] // world_size
            out[key] = t[:, rank * c:(rank + 1) * c]
        elif "out_proj.weight" in key or "down_proj.weight" in key:
            c = t.shape[0] // world_size
            out[key] = t[rank * c:(rank + 1) * c, :]
        else:
            out[key] = t
    return out


class OracleModel:
    """``DistributedLLaMAModel`` across ``world_size`` simulated ranks (engine/model/llama.py:79-174).

    ``shards[r]`` is rank r's state dict (reference key names, [in, out] linear
    weights, nn.Linear ``lm_head.weight`` [V, H]).  ``pools[r]`` is rank r's KV pool.
    """

    def __init__(self, cfg: OracleConfig, shards: List[Dict[str, np.ndarray]], pools: List[KVPool],
                 rope_base: float = 10000.0, compat_pad: bool = True, cos=None, sin=None):
        self.cfg = cfg
        self.shards = shards
        self.pools = pools
        self.world_size = len(shards)
        if cos is None:
            cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, rope_base)
        self.cos, self.sin = cos, sin
        self.compat_pad = compat_pad

    # engine/model/attention.py:135-233 for one rank
    def _attention_rank(self, r, layer, x, positions, block_tables, is_prefill):
        cfg = self.cfg
        w = self.shards[r]
        pre = f"layers.{layer}.self_attn."
        B, S, _ = x.shape
        hd = cfg.head_dim
        nq = cfg.num_heads // self.world_size
        nkv = cfg.num_kv_heads // self.world_size
        q = column_parallel_linear(x, w[pre + "q_proj.weight"]).reshape(B, S, nq, hd)
        k = column_parallel_linear(x, w[pre + "k_proj.weight"]).reshape(B, S, nkv, hd)
        v = column_parallel_linear(x, w[pre + "v_proj.weight"]).reshape(B, S, nkv, hd)
        q = apply_rope(q, positions, self.cos, self.sin)
        k = apply_rope(k, positions, self.cos, self.sin)
        scale = 1.0 / math.sqrt(hd)
        if is_prefill:
            a = prefill_attention(q, k, v, self.pools[r], layer, block_tables, scale)
        else:
            assert S == 1
            a = decode_attention(q[:, 0], k[:, 0], v[:, 0], positions[:, 0], self.pools[r], layer,
                                 block_tables, scale, self.compat_pad)[:, None, :]
        return a @ np.asarray(w[pre + "out_proj.weight"], dtype=ACC)

    # engine/model/mlp.py:72-86 for one rank
    def _mlp_rank(self, r, layer, x):
        w = self.shards[r]
        pre = f"layers.{layer}.mlp."
        g = column_parallel_linear(x, w[pre + "gate_proj.weight"])
        u = column_parallel_linear(x, w[pre + "up_proj.weight"])
        return (silu(g) * u) @ np.asarray(w[pre + "down_proj.weight"], dtype=ACC)

    def block(self, layer, h, positions, block_tables, is_prefill):
        """engine/model/llama.py:48-76 (pre-norm residual block)."""
        w0 = self.shards[0]
        eps = self.cfg.rms_norm_eps
        x = rmsnorm(h, w0[f"layers.{layer}.input_layernorm.weight"], eps)
        attn = all_reduce_sum([self._attention_rank(r, layer, x, positions, block_tables, is_prefill)
                               for r in range(self.world_size)])
        h = h + attn
        x2 = rmsnorm(h, w0[f"layers.{layer}.post_attention_layernorm.weight"], eps)
        mlp = all_reduce_sum([self._mlp_rank(r, layer, x2) for r in range(self.world_size)])
        return h + mlp

    def forward(self, token_ids, positions, block_tables, is_prefill, trace: Optional[list] = None,
                last_only: bool = True):
        """engine/model/llama.py:131-174; returns float64 logits [B, V] (last token)."""
        w0 = self.shards[0]
        token_ids = np.asarray(token_ids)
        positions = np.asarray(positions)
        h = np.asarray(w0["embed_tokens.weight"][token_ids], dtype=ACC)
        for layer in range(self.cfg.num_layers):
            h = self.block(layer, h, positions, block_tables, is_prefill)
            if trace is not None:
                trace.append(h.copy())
        h = rmsnorm(h, w0["norm.weight"], self.cfg.rms_norm_eps)
        hl = h[:, -1, :] if last_only else h
        return hl @ np.asarray(w0["lm_head.weight"], dtype=ACC).T


# --------------------------------------------------------------------------------------
# Worker step
# --------------------------------------------------------------------------------------

@dataclass
class Slot:
    """Fields of ``SequenceSlotProto`` read by the worker (protos/distributed_inference.proto:49-57)."""
    seq_id: str
    is_prefill: bool
    prompt_token_ids: List[int] = field(default_factory=list)
    current_token_id: int = 0
    current_len: int = 0
    block_table: List[int] = field(default_factory=list)


def execute_step(model: OracleModel, slots: List[Slot]):
    """engine/worker/execution_engine.py:63-154.

    Each prefill runs as its own batch-1 forward with positions ``arange(P)``;
    decodes run as one batch with positions ``current_len - 1``.  The sampled
    token is the rank-local greedy argmax; ``top_logits`` are the first ten logits.
    Returns a list of (seq_id, token_id, top_logits[10]) in the reference's order
    (all prefills, then all decodes).
    """
    out = []
    full = []  # every row's full logits, kept on the model as ``last_logits`` for margin checks
    for s in (s for s in slots if s.is_prefill):
        toks = np.asarray([s.prompt_token_ids], dtype=np.int64)
        pos = np.arange(toks.shape[1], dtype=np.int64)[None, :]
        logits = model.forward(toks, pos, [list(s.block_table)], True)
        out.append((s.seq_id, int(np.argmax(logits[0])), logits[0][:10].copy()))
        full.append(logits[0])
    dec = [s for s in slots if not s.is_prefill]
    if dec:
        toks = np.asarray([[s.current_token_id] for s in dec], dtype=np.int64)
        pos = np.asarray([[s.current_len - 1] for s in dec], dtype=np.int64)
        logits = model.forward(toks, pos, [list(s.block_table) for s in dec], False)
        for i, s in enumerate(dec):
            out.append((s.seq_id, int(np.argmax(logits[i])), logits[i][:10].copy()))
            full.append(logits[i])
    model.last_logits = np.stack(full) if full else None
    return out


def run_greedy(model: OracleModel, prompts: List[List[int]], num_tokens: int, num_blocks: int,
               block_size: int = 16):
    """Greedy generation driver used for the Tiny LLaMA workload.

    Step 0 prefills every request (each as its own forward, like
    execution_engine.py:85-111); steps 1..num_tokens-1 decode all requests as one
    batch.  Blocks come from a FIFO allocator that mirrors
    ``KVCacheManager.allocate_blocks_for_sequence`` / ``append_token``
    (kv_cache.py:180-218) and always holds the slot a step writes.
    Returns (tokens [num_tokens, R], top_logits [num_tokens, R, 10], tables).
    """
    alloc = FifoBlockAllocator(num_blocks, block_size)
    ids = [f"req_{i}" for i in range(len(prompts))]
    slots = []
    for sid, p in zip(ids, prompts):
        table = alloc.allocate(sid, len(p))
        slots.append(Slot(sid, True, list(p), 0, len(p), list(table)))
    res = execute_step(model, slots)
    toks = [[t for _, t, _ in res]]
    tops = [[tl for _, _, tl in res]]
    cur = {sid: t for sid, t, _ in res}
    lens = {sid: len(p) for sid, p in zip(ids, prompts)}
    for _ in range(1, num_tokens):
        slots = []
        for sid in ids:
            alloc.append_token(sid)
            lens[sid] += 1
            slots.append(Slot(sid, False, [], cur[sid], lens[sid], list(alloc.tables[sid])))
        res = execute_step(model, slots)
        toks.append([t for _, t, _ in res])
        tops.append([tl for _, _, tl in res])
        cur = {sid: t for sid, t, _ in res}
    return np.asarray(toks), np.asarray(tops), {k: list(v) for k, v in alloc.tables.items()}
