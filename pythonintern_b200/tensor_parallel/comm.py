"""All-reduce(SUM) for the row-parallel layers over NVLink peer memory.

Drop-in for engine/tensor_parallel/comm.py: ``DistributedCommunicator(rank,
world_size, peer_addresses)`` with ``all_reduce_sum(tensor, step_tag,
timeout_sec=15.0)`` returning a new tensor (raising ``TimeoutError`` like
comm.py:99-107), ``register_peer_stub``, ``register_in_memory_peer`` and
``cleanup``.  The transport is not gRPC: each rank owns a device buffer pair and
flag array exported by CUDA IPC (libb2tp ``b2_comm_*``), peers read each other's
partials directly inside the reduction kernel, and the sum runs in rank order
0..world-1 so that every rank gets bit-identical results.

Peers are connected in one of two ways:
* one process per GPU: ``connect(group)`` exchanges the IPC handles once over a
  ``torch.distributed`` group (any backend; gloo or nccl), or ``connect_store``
  over a ``torch.distributed`` Store;
* one thread per GPU in one process (the reference's in-memory test harness):
  ``register_in_memory_peer`` for every peer, on distinct GPUs.

The tensor-parallel decode path uses ``row_parallel_linear`` (the row-parallel GEMM
pushes each output row to the rank that owns it from its epilogue),
``allreduce_rmsnorm_sharded`` (sum in rank order + residual + next RMSNorm +
all-gather, flag free) and ``argmax_allgather`` (greedy token over a vocab-parallel
lm_head), all without host synchronisation; errors surface at the step's status
check.  ``all_reduce_sum`` / ``allreduce_rmsnorm`` keep the reference's one-shot
semantics for the module-level API.
"""

from __future__ import annotations

import ctypes
import threading
from typing import Dict, List, Optional

import torch

from pythonintern_b200 import _lib
from pythonintern_b200._lib import check, dtype_code, ptr, status_ptr, stream_ptr

DEFAULT_MAX_BYTES = 64 << 20


class _DevicePointer:
    """Exposes a raw device range through __cuda_array_interface__ so torch can alias it."""

    def __init__(self, address: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (address, False),
                                         "version": 3, "strides": None, "stream": None}


def exchange_handles(mine: bytes, world_size: int, group=None) -> List[bytes]:
    """All-gather every rank's handle bytes over a torch.distributed group, in rank order."""
    import torch.distributed as dist
    out: List[Optional[bytes]] = [None] * world_size
    dist.all_gather_object(out, mine, group=group)
    return [bytes(b) for b in out]


def exchange_handles_store(store, prefix: str, rank: int, world_size: int, mine: bytes,
                           timeout_sec: float = 60.0) -> List[bytes]:
    """Exchange handle bytes through a torch.distributed Store (TCPStore, FileStore, ...)."""
    store.set(f"{prefix}/{rank}", mine)
    keys = [f"{prefix}/{r}" for r in range(world_size)]
    store.wait(keys)
    return [bytes(store.get(k)) for k in keys]


_local_lock = threading.Lock()


class DistributedCommunicator:
    """NVLink all-reduce with the reference's interface (engine/tensor_parallel/comm.py:27-166)."""

    def __init__(self, rank: int, world_size: int, peer_addresses: Optional[List[str]] = None,
                 device=None, max_bytes: int = DEFAULT_MAX_BYTES):
        self.rank = rank
        self.world_size = world_size
        self.peer_addresses = peer_addresses or []
        self.max_bytes = int(max_bytes)
        self.device = torch.device(device) if device is not None else None
        self._stubs: Dict[int, object] = {}
        self._in_memory_peers: Dict[int, "DistributedCommunicator"] = {}
        self._comm = ctypes.c_void_p()
        self._opened = world_size <= 1
        self._calls = 0
        self._views: Dict[tuple, torch.Tensor] = {}

    # ------------------------------------------------------------------ setup
    def _ensure_created(self):
        if self._comm.value:
            return
        if self.device is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            check(_lib.lib().b2_comm_create(self.rank, self.world_size, self.max_bytes, ctypes.byref(self._comm)),
                  "b2_comm_create")

    def handle_bytes(self) -> bytes:
        self._ensure_created()
        n = _lib.lib().b2_comm_handle_bytes()
        buf = ctypes.create_string_buffer(n)
        check(_lib.lib().b2_comm_export_handle(self._comm, buf, n), "b2_comm_export_handle")
        return buf.raw

    def open_peers(self, handles: List[bytes]):
        self._ensure_created()
        blob = b"".join(handles)
        with torch.cuda.device(self.device):
            check(_lib.lib().b2_comm_open_peers(self._comm, blob, len(blob)), "b2_comm_open_peers")
        self._opened = True

    def connect(self, group=None):
        """Exchange IPC handles over torch.distributed (one process per GPU) and map the peers."""
        if self.world_size > 1 and not self._opened:
            self.open_peers(exchange_handles(self.handle_bytes(), self.world_size, group))
        else:
            self._ensure_created()
        return self

    def connect_store(self, store, prefix: str = "b2tp_comm"):
        """Exchange IPC handles through a torch.distributed Store and map the peers."""
        if self.world_size > 1 and not self._opened:
            self.open_peers(exchange_handles_store(store, prefix, self.rank, self.world_size, self.handle_bytes()))
        else:
            self._ensure_created()
        return self

    def register_peer_stub(self, peer_rank: int, stub):
        """Kept for API compatibility with comm.py:47-49; the NVLink path does not use gRPC stubs."""
        self._stubs[peer_rank] = stub

    def register_in_memory_peer(self, peer_rank: int, peer_comm: "DistributedCommunicator"):
        """In-process peer (comm.py:51-53).  Ranks must sit on distinct GPUs."""
        self._in_memory_peers[peer_rank] = peer_comm

    def _wire_in_memory(self):
        with _local_lock:
            if self._opened:
                return
            group = dict(self._in_memory_peers)
            group[self.rank] = self
            if sorted(group) != list(range(self.world_size)):
                raise RuntimeError(f"[Rank {self.rank}] in-memory peers {sorted(group)} do not cover the world")
            comms = [group[r] for r in range(self.world_size)]
            for c in comms:
                if c.device is None:
                    raise RuntimeError("in-memory peers need an explicit device=cuda:<i> per rank")
                c._ensure_created()
            arr = (ctypes.c_void_p * self.world_size)(*[c._comm.value for c in comms])
            check(_lib.lib().b2_comm_open_local(arr, self.world_size), "b2_comm_open_local")
            for c in comms:
                c._opened = True

    @property
    def ready(self) -> bool:
        return self._opened

    def _require_open(self):
        if self.world_size <= 1:
            self._ensure_created()
            return
        if not self._opened:
            if self._in_memory_peers:
                self._wire_in_memory()
            else:
                raise RuntimeError(f"[Rank {self.rank}] communicator not connected; call connect() first")

    # ------------------------------------------------------------------ buffers
    def next_parity(self) -> int:
        p = self._calls & 1
        self._calls += 1
        return p

    def buffer_address(self, parity: int) -> int:
        self._ensure_created()
        out = ctypes.c_void_p()
        check(_lib.lib().b2_comm_buffer(self._comm, parity, ctypes.byref(out)), "b2_comm_buffer")
        return out.value

    def partial_buffer(self, parity: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """This rank's symmetric buffer ``parity`` viewed as a tensor of ``shape`` (the GEMM writes here)."""
        shape = tuple(int(s) for s in shape)
        key = (parity, shape, dtype)
        view = self._views.get(key)
        if view is None:
            n = 1
            for s in shape:
                n *= s
            nbytes = n * torch.tensor([], dtype=dtype).element_size()
            if nbytes > self.max_bytes:
                raise ValueError(f"all-reduce payload of {nbytes} bytes exceeds the {self.max_bytes}-byte buffer")
            raw = torch.as_tensor(_DevicePointer(self.buffer_address(parity), nbytes), device=self.device)
            view = raw.view(dtype).view(*shape)
            self._views[key] = view
        return view

    def row_slice(self, rows: int):
        """Rows [start, end) of a [rows, dim] activation this rank owns in the sharded all-reduce."""
        R = (rows + self.world_size - 1) // self.world_size
        start = min(rows, self.rank * R)
        return start, min(rows, start + R), R

    # ------------------------------------------------------------------ collectives
    def all_reduce_sum(self, tensor: torch.Tensor, step_tag: str = "", timeout_sec: float = 15.0) -> torch.Tensor:
        """Synchronous all-reduce(SUM); returns a new tensor (comm.py:72-118)."""
        if self.world_size <= 1:
            return tensor
        self._require_open()
        _lib.require_cuda(tensor, "tensor")
        dt = tensor.dtype
        n = tensor.numel()
        n8 = (n + 7) // 8 * 8
        parity = self.next_parity()
        with torch.cuda.device(self.device):
            buf = self.partial_buffer(parity, (n8,), dt)
            buf[:n].copy_(tensor.reshape(-1))
            if n8 > n:
                buf[n:].zero_()
            out = torch.empty(n8, dtype=dt, device=self.device)
            check(_lib.lib().b2_allreduce_sum(self._comm, parity, n8, dtype_code(dt), ptr(out),
                                              int(timeout_sec * 1e9), status_ptr(self.device),
                                              stream_ptr(self.device)), "b2_allreduce_sum")
            try:
                _lib.check_device_status(self.device, f"[Rank {self.rank}] All-Reduce on tag '{step_tag}'")
            except TimeoutError as e:
                raise TimeoutError(f"[Rank {self.rank}] All-Reduce timeout on tag '{step_tag}'. "
                                   f"Expected {self.world_size - 1} peers.") from e
        return out[:n].view(tensor.shape)

    def allreduce_rmsnorm(self, parity: int, rows: int, dim: int, dtype: torch.dtype, residual: torch.Tensor,
                          h_out: torch.Tensor, norm_w: torch.Tensor, eps: float, y: torch.Tensor,
                          timeout_sec: float = 15.0):
        """Fused ``h = residual + sum_r partial_r``; ``y = rmsnorm(h) * norm_w`` (no host sync)."""
        self._require_open()
        check(_lib.lib().b2_allreduce_rmsnorm(self._comm, parity, rows, dim, dtype_code(dtype), ptr(residual),
                                              ptr(h_out), ptr(norm_w), float(eps), ptr(y), dtype_code(y.dtype),
                                              int(timeout_sec * 1e9), status_ptr(self.device),
                                              stream_ptr(self.device)), "b2_allreduce_rmsnorm")

    def row_parallel_linear(self, x: torch.Tensor, w_packed: torch.Tensor):
        """Row-parallel GEMM whose epilogue pushes each output row to the rank that owns it."""
        self._require_open()
        K = x.shape[-1]
        x2 = x if (x.dim() == 2 and x.stride(1) == 1) else x.reshape(-1, K).contiguous()
        M, N = x2.shape[0], w_packed.shape[0]
        dc = dtype_code(w_packed.dtype)
        nbytes = _lib.lib().b2_linear_workspace_bytes(M, N, K, dc)
        ws = _lib.workspace(self.device, "linear", nbytes)
        check(_lib.lib().b2_row_parallel_linear(self._comm, ptr(x2), x2.stride(0), M, K, ptr(w_packed), N, dc,
                                                ptr(ws), nbytes, status_ptr(self.device),
                                                stream_ptr(self.device)), "b2_row_parallel_linear")

    def allreduce_rmsnorm_sharded(self, rows: int, dim: int, dtype: torch.dtype, h_slice: torch.Tensor,
                                  norm_w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
                                  timeout_sec: float = 15.0) -> torch.Tensor:
        """Completes ``row_parallel_linear``: residual slice += sum of partials, normalise, all-gather.

        Returns the [rows, dim] normalised activations (every rank gets all rows).
        """
        self._require_open()
        if out is None:
            out = torch.empty(rows, dim, dtype=dtype, device=self.device)
        check(_lib.lib().b2_allreduce_rmsnorm_sharded(self._comm, rows, dim, dtype_code(dtype), ptr(h_slice),
                                                      ptr(norm_w), float(eps), ptr(out), int(timeout_sec * 1e9),
                                                      status_ptr(self.device), stream_ptr(self.device)),
              "b2_allreduce_rmsnorm_sharded")
        return out

    def argmax_allgather(self, logits: torch.Tensor, vocab_offset: int, out: Optional[torch.Tensor] = None,
                         timeout_sec: float = 15.0) -> torch.Tensor:
        """Greedy token per row when each rank holds the logits of one vocabulary slice.

        ``logits`` [rows, cols] float32 are this rank's logits for ids
        [vocab_offset, vocab_offset + cols); returns the global argmax [rows] int64 on every
        rank, equal to torch.argmax over the full row (execution_engine.py:103,133).
        """
        self._require_open()
        _lib.require_cuda(logits, "logits")
        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("argmax_allgather: logits must be a row-major [rows, cols] float32 tensor")
        rows, cols = logits.shape
        if out is None:
            out = torch.empty(rows, dtype=torch.int64, device=self.device)
        check(_lib.lib().b2_argmax_allgather(self._comm, ptr(logits), logits.stride(0), rows, cols, int(vocab_offset),
                                             ptr(out), int(timeout_sec * 1e9), status_ptr(self.device),
                                             stream_ptr(self.device)), "b2_argmax_allgather")
        return out

    def cleanup(self):
        """Release the symmetric buffers and peer mappings (comm.py:156-166)."""
        self._views.clear()
        if self._comm.value:
            _lib.lib().b2_comm_destroy(self._comm)
            self._comm = ctypes.c_void_p()
        self._opened = self.world_size <= 1
        self._stubs.clear()
        self._in_memory_peers.clear()

    def __del__(self):  # pragma: no cover - best effort at interpreter exit
        try:
            self.cleanup()
        except Exception:
            pass
