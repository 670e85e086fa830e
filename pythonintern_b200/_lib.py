"""ctypes binding of libb2tp.so (the C ABI declared in include/b2tp.h).

The library is the only compute path of this package: there is no CPU or PyTorch
fallback.  If ``libb2tp.so`` is missing, or no CUDA device is present, every
compute call raises.  Build it with ``python -m pythonintern_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libb2tp.so")

B2_OK, B2_EINVAL, B2_ETIMEOUT, B2_ECUDA, B2_ENOTSUP, B2_ERANGE = 0, 1, 2, 3, 4, 5
B2_F32, B2_BF16 = 0, 1
B2_DEV_RANGE, B2_DEV_PIPE_TIMEOUT, B2_DEV_PEER_TIMEOUT = 1, 2, 4

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float

# name -> (restype, argtypes); mirrors include/b2tp.h
_SIGS = {
    "b2_abi_version": (_c_int, []),
    "b2_status_name": (ctypes.c_char_p, [_c_int]),
    "b2_last_error": (_c_int, [ctypes.c_char_p, _c_size]),
    "b2_embedding": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_int,
                              _c_void_p, _c_void_p]),
    "b2_rmsnorm": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_void_p, _c_int, _c_void_p, _c_float,
                            _c_void_p, _c_int, _c_int, _c_int, _c_void_p]),
    "b2_linear_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "b2_linear": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p,
                           _c_i64, _c_int, _c_int, _c_void_p, _c_size, _c_void_p, _c_void_p]),
    "b2_linear_qkv": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_int,
                               _c_void_p, _c_int, _c_void_p, _c_i64, _c_int, _c_void_p, _c_size, _c_void_p,
                               _c_void_p]),
    "b2_linear_swiglu": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p,
                                  _c_i64, _c_int, _c_void_p, _c_size, _c_void_p, _c_void_p]),
    "b2_rope_kv_write": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                  _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_int,
                                  _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p]),
    "b2_paged_attention_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "b2_paged_attention": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                    _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                    _c_float, _c_void_p, _c_i64, _c_int, _c_void_p, _c_size, _c_int,
                                    _c_void_p, _c_void_p]),
    "b2_paged_attention_noalloc": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_void_p,
                                            _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p,
                                            _c_void_p, _c_int, _c_float, _c_void_p, _c_i64, _c_int, _c_int,
                                            _c_void_p, _c_void_p]),
    "b2_prefill_attention": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                      _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                      _c_float, _c_void_p, _c_i64, _c_int, _c_void_p, _c_void_p]),
    "b2_prefill_attention_tc": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                         _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                         _c_float, _c_void_p, _c_i64, _c_int, _c_void_p, _c_void_p]),
    "b2_argmax": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p]),
    "b2_comm_handle_bytes": (_c_size, []),
    "b2_comm_create": (_c_int, [_c_int, _c_int, _c_size, ctypes.POINTER(_c_void_p)]),
    "b2_comm_export_handle": (_c_int, [_c_void_p, _c_void_p, _c_size]),
    "b2_comm_open_peers": (_c_int, [_c_void_p, _c_void_p, _c_size]),
    "b2_comm_open_local": (_c_int, [ctypes.POINTER(_c_void_p), _c_int]),
    "b2_comm_buffer": (_c_int, [_c_void_p, _c_int, ctypes.POINTER(_c_void_p)]),
    "b2_comm_destroy": (_c_int, [_c_void_p]),
    "b2_allreduce_sum": (_c_int, [_c_void_p, _c_int, _c_size, _c_int, _c_void_p, _c_i64, _c_void_p, _c_void_p]),
    "b2_allreduce_rmsnorm": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                      _c_void_p, _c_float, _c_void_p, _c_int, _c_i64, _c_void_p, _c_void_p]),
    "b2_row_parallel_linear": (_c_int, [_c_void_p, _c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_int,
                                        _c_int, _c_void_p, _c_size, _c_void_p, _c_void_p]),
    "b2_allreduce_rmsnorm_sharded": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                              _c_float, _c_void_p, _c_i64, _c_void_p, _c_void_p]),
    "b2_argmax_allgather": (_c_int, [_c_void_p, _c_void_p, _c_i64, _c_int, _c_int, _c_i64, _c_void_p, _c_i64,
                                     _c_void_p, _c_void_p]),
    "b2_linear_residual_norm": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_i64,
                                         _c_void_p, _c_void_p, _c_i64, _c_void_p, _c_void_p, _c_size,
                                         _c_void_p, _c_void_p]),
    "b2_linear_qkv_rownorm": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_int, _c_void_p, _c_int,
                                       _c_void_p, _c_int, _c_void_p, _c_i64, _c_void_p, _c_int, _c_int, _c_float,
                                       _c_void_p, _c_size, _c_void_p, _c_void_p]),
    "b2_linear_swiglu_rownorm": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p, _c_int,
                                          _c_void_p, _c_i64, _c_void_p, _c_int, _c_int, _c_float, _c_void_p,
                                          _c_size, _c_void_p, _c_void_p]),
    "b2_linear_qkv_rope_kv": (_c_int, [_c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
                                       _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_int, _c_float,
                                       _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int,
                                       _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int,
                                       _c_void_p, _c_size, _c_void_p, _c_void_p]),
}

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


class B2Error(RuntimeError):
    """A libb2tp call failed (bad argument, CUDA error, unsupported shape, range error)."""


def exported_symbols():
    """Names of every entry point the binding declares (the C ABI of include/b2tp.h)."""
    return list(_SIGS)


def lib() -> ctypes.CDLL:
    """Load libb2tp.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise B2Error(f"{LIB_PATH} is not built; run `python -m pythonintern_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().b2_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


# Kernel launches issued through this binding (every launching entry point is
# checked through ``check``); bench.py reads it to report its launch count.
launch_count = 0
_LAUNCHING = {"b2_embedding", "b2_rmsnorm", "b2_linear", "b2_linear_qkv", "b2_linear_swiglu",
              "b2_rope_kv_write", "b2_paged_attention", "b2_argmax", "b2_allreduce_sum", "b2_allreduce_rmsnorm",
              "b2_row_parallel_linear", "b2_allreduce_rmsnorm_sharded", "b2_paged_attention_noalloc",
              "b2_argmax_allgather", "b2_linear_residual_norm", "b2_linear_qkv_rownorm", "b2_linear_swiglu_rownorm",
              "b2_linear_qkv_rope_kv", "b2_prefill_attention", "b2_prefill_attention_tc"}


def check(rc: int, what: str = ""):
    global launch_count
    if rc == B2_OK:
        if what in _LAUNCHING:
            launch_count += 1
        return
    msg = f"{what}: {lib().b2_status_name(rc).decode()}: {last_error()}"
    if rc == B2_ETIMEOUT:
        raise TimeoutError(msg)
    if rc == B2_ERANGE:
        raise IndexError(msg)
    raise B2Error(msg)


def require_cuda(t: torch.Tensor, name: str = "tensor"):
    if not t.is_cuda:
        raise B2Error(f"{name} must be a CUDA tensor (this package has no CPU path)")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return B2_F32
    if dt == torch.bfloat16:
        return B2_BF16
    raise B2Error(f"unsupported dtype {dt}; use torch.float32 or torch.bfloat16")


def torch_dtype(name) -> torch.dtype:
    if isinstance(name, torch.dtype):
        return name
    if name in (None, "float32", "fp32"):
        return torch.float32
    if name in ("bfloat16", "bf16"):
        return torch.bfloat16
    raise B2Error(f"unsupported dtype {name!r}; use 'float32' or 'bfloat16'")


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ------------------------------------------------------------------ per-device state
class _DeviceState:
    def __init__(self, device: torch.device):
        self.device = device
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.ws: Dict[str, torch.Tensor] = {}


_states: Dict[int, _DeviceState] = {}


def device_state(device) -> _DeviceState:
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _states.get(idx)
    if st is None:
        st = _DeviceState(torch.device("cuda", idx))
        _states[idx] = st
    return st


def workspace(device, key: str, nbytes: int) -> Optional[torch.Tensor]:
    """Zero-initialised scratch owned by this module, grown on demand (never shrunk)."""
    if nbytes <= 0:
        return None
    st = device_state(device)
    buf = st.ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=st.device)
        st.ws[key] = buf
    return buf


def status_ptr(device) -> int:
    return device_state(device).status.data_ptr()


def raise_for_status(v: int, what: str = "kernel"):
    """Raises the exception a kernel error word stands for (nothing when it is 0)."""
    if v:
        if v & B2_DEV_PEER_TIMEOUT:
            raise TimeoutError(f"{what}: a tensor-parallel peer did not arrive before the all-reduce timeout")
        if v & B2_DEV_RANGE:
            raise IndexError(f"{what}: position, block-table entry or token id out of range")
        raise B2Error(f"{what}: device error bits {v:#x}")


def check_device_status(device, what: str = "kernel"):
    """Synchronise the device, read and clear the kernel error word, raise on error."""
    st = device_state(device)
    v = int(st.status.item())
    if v:
        st.status.zero_()
        raise_for_status(v, what)
