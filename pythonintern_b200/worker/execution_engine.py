"""Worker step driver (engine/worker/execution_engine.py:24-160).

``WorkerExecutionEngine(model_config, shard_config, kv_config, communicator,
device).execute_step(step_request)`` keeps the reference's semantics: each
prefill sequence is computed at positions ``arange(P)`` and attends causally to its
own tokens only; all decodes run as one batch with positions ``current_len - 1``;
the sampled token is the rank-local greedy argmax and ``top_logits`` the first ten
logits of the row.

What changes is where the work runs: the model is the fused CUDA path, the
argmax is a kernel, and the whole step costs one host synchronisation (one
device-to-host copy of every sampled token and its ten logits, plus the kernel
status word).  The reference runs one forward per prefill sequence
(execution_engine.py:85-111); here the step's prompts are concatenated into as few
forwards as the token cap allows (``batch_prefills``), so the weights are read once
for all of them and the attention is one varlen causal launch per layer.
"""

from __future__ import annotations

import time
from typing import List, Optional

import numpy as np
import torch

from pythonintern_b200 import _lib
from pythonintern_b200.config import KVCacheConfig, ModelConfig, ShardConfig
from pythonintern_b200.model.kv_cache import KVCacheManager
from pythonintern_b200.model.llama import DistributedLLaMAModel
from pythonintern_b200.model.metadata import PinnedStager, build_metadata, build_prefill_metadata
from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
from pythonintern_b200.worker.graphs import DecodeGraphCache
from pythonintern_b200.worker.messages import SampledToken, StepResponse


def group_prefills(prompt_lens: List[int], max_tokens: int, batch: bool = True) -> List[List[int]]:
    """Indices of consecutive prefill slots packed into groups of at most ``max_tokens``
    prompt tokens (a longer prompt forms a group of its own); ``batch=False`` gives one
    group per prompt, the reference's loop (execution_engine.py:85-111)."""
    if not batch:
        return [[i] for i in range(len(prompt_lens))]
    groups: List[List[int]] = []
    cur: List[int] = []
    n = 0
    for i, P in enumerate(prompt_lens):
        if cur and n + P > max_tokens:
            groups.append(cur)
            cur, n = [], 0
        cur.append(i)
        n += P
    if cur:
        groups.append(cur)
    return groups


class WorkerExecutionEngine:
    def __init__(self, model_config: ModelConfig, shard_config: ShardConfig, kv_config: KVCacheConfig,
                 communicator: Optional[DistributedCommunicator] = None, device="cuda",
                 use_cuda_graphs: bool = True, batch_prefills: bool = True,
                 max_prefill_tokens: Optional[int] = None):
        self.model_config = model_config
        self.shard_config = shard_config
        self.kv_config = kv_config
        self.communicator = communicator
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        if kv_config.device in ("cpu", "cuda"):
            kv_config.device = str(dev)
        self.kv_manager = KVCacheManager(config=kv_config, model_config=model_config,
                                         world_size=shard_config.world_size)
        self.model = DistributedLLaMAModel(config=model_config, rank=shard_config.rank,
                                           world_size=shard_config.world_size, communicator=communicator, device=dev)
        self.stager = PinnedStager(dev)
        self.use_cuda_graphs = use_cuda_graphs
        self.batch_prefills = batch_prefills
        if max_prefill_tokens is None:
            max_prefill_tokens = 16384
            if shard_config.world_size > 1 and communicator is not None:
                # a row-parallel partial [tokens, hidden] must fit the communicator's buffer
                esz = torch.tensor([], dtype=self.model.dtype).element_size()
                max_prefill_tokens = min(max_prefill_tokens,
                                         communicator.max_bytes // (model_config.hidden_dim * esz))
        self.max_prefill_tokens = max(1, int(max_prefill_tokens))
        self.graphs = DecodeGraphCache(self.model, self.kv_manager.pool, model_config.masked_decode_padding)
        self._pin_tok: Optional[torch.Tensor] = None  # pinned read-back buffers (_read_back)
        self._pin_top: Optional[torch.Tensor] = None
        self._pin_status = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.total_steps_executed = 0
        self.total_latency_ms = 0.0
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    def _read_back(self, toks: List[torch.Tensor], tops: List[torch.Tensor], step_id: int):
        """Sampled tokens, first ten logits and the kernels' error word in one synchronisation.

        Asynchronous copies into pinned host buffers, then one stream synchronise; a set
        error word is cleared and raised after the wait.
        """
        tok = toks[0] if len(toks) == 1 else torch.cat(toks)
        top = tops[0] if len(tops) == 1 else torch.cat(tops)
        n = tok.shape[0]
        if self._pin_tok is None or self._pin_tok.shape[0] < n:
            self._pin_tok = torch.empty(n, dtype=torch.int64, pin_memory=True)
            self._pin_top = torch.empty(n, 10, dtype=torch.float32, pin_memory=True)
        st = _lib.device_state(self.device).status
        self._pin_tok[:n].copy_(tok, non_blocking=True)
        self._pin_top[:n].copy_(top, non_blocking=True)
        self._pin_status.copy_(st, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        v = int(self._pin_status[0])
        if v:
            st.zero_()
            _lib.raise_for_status(v, f"step {step_id}")
        return self._pin_tok[:n].numpy(), self._pin_top[:n].numpy()

    def _prefill_groups(self, slots) -> List[list]:
        """The step's prefill slots in groups of at most ``max_prefill_tokens`` prompt tokens."""
        idx = group_prefills([len(s.prompt_token_ids) for s in slots], self.max_prefill_tokens, self.batch_prefills)
        return [[slots[i] for i in g] for g in idx]

    def execute_step(self, step_request) -> StepResponse:
        start = time.perf_counter()
        step_id = step_request.step_id
        prefill_slots = [s for s in step_request.active_sequences if s.is_prefill]
        decode_slots = [s for s in step_request.active_sequences if not s.is_prefill]
        pool = self.kv_manager.pool
        toks: List[torch.Tensor] = []
        tops: List[torch.Tensor] = []
        ids: List[str] = []
        h2d = 0
        with torch.no_grad(), torch.cuda.device(self.device):
            for group in self._prefill_groups(prefill_slots):
                prompts = [np.asarray(list(s.prompt_token_ids), dtype=np.int64) for s in group]
                tables = [list(s.block_table) for s in group]
                ids_cat = np.concatenate(prompts)[None, :]
                md = build_prefill_metadata([p.size for p in prompts], tables, self.device, stager=self.stager,
                                            extra=ids_cat)
                h2d += self.stager.last_bytes
                t, tl = self.model.greedy(md.extra, None, pool, tables, True, step_id, metadata=md)
                toks.append(t)
                tops.append(tl)
                ids.extend(s.seq_id for s in group)
            if decode_slots:
                tok_ids = np.asarray([[s.current_token_id] for s in decode_slots], dtype=np.int64)
                pos = np.asarray([[s.current_len - 1] for s in decode_slots], dtype=np.int64)
                if self.use_cuda_graphs:
                    tables = [s.block_table for s in decode_slots]  # packed row by row, only where changed
                    # One graph replay per step (worker/graphs.py); captured on first use.
                    g, new = self.graphs.get(len(decode_slots), max(len(t) for t in tables))
                    g.upload_host(tok_ids.reshape(-1), pos.reshape(-1), tables)
                    h2d += g.nbytes
                    if new:
                        g.capture()
                    t, tl = g.replay()
                else:
                    tables = [list(s.block_table) for s in decode_slots]
                    md = build_metadata(pos, tables, False, self.device,
                                        masked_padding=self.model_config.masked_decode_padding,
                                        stager=self.stager, extra=tok_ids)
                    h2d += self.stager.last_bytes
                    t, tl = self.model.greedy(md.extra, None, pool, tables, False, step_id, metadata=md)
                toks.append(t)
                tops.append(tl)
                ids.extend(s.seq_id for s in decode_slots)
            sampled = []
            if toks:
                tok_host, top_host = self._read_back(toks, tops, step_id)
                self.last_d2h_bytes = tok_host.nbytes + top_host.nbytes
                tok_list, top_list = tok_host.tolist(), top_host.tolist()
                sampled = [SampledToken(seq_id=sid, token_id=tok_list[i], top_logits=top_list[i])
                           for i, sid in enumerate(ids)]
        self.last_h2d_bytes = h2d
        elapsed_ms = (time.perf_counter() - start) * 1000.0
        self.total_steps_executed += 1
        self.total_latency_ms += elapsed_ms
        return StepResponse(step_id=step_id, rank=self.shard_config.rank, success=True, sampled_tokens=sampled,
                            step_latency_ms=elapsed_ms, active_blocks=self.kv_manager.allocated_block_count,
                            free_blocks=self.kv_manager.free_block_count)

    def evict_sequences(self, seq_ids: List[str]) -> int:
        return sum(self.kv_manager.free_sequence(sid) for sid in seq_ids)
