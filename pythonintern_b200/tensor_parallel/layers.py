"""Tensor-parallel linears and RMSNorm with the reference's Python API.

Drop-in for engine/tensor_parallel/layers.py: same class names, constructor
arguments, parameter names and shapes ([in, out/ws] for ColumnParallelLinear,
[in/ws, out] for RowParallelLinear, float32 ``ones`` for RMSNorm), same forward
signatures.  The parameter tensor is a transposed VIEW of a packed [out, in]
(K-contiguous) device buffer, which is the layout the tcgen05 / FFMA kernels read;
``load_state_dict``, ``copy_`` and the reference's WeightSharder all write through
the view, so no second copy of the weights exists.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from pythonintern_b200 import kernels
from pythonintern_b200._lib import torch_dtype
from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator


def _default_device(device):
    return torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())


def packed_parameter(in_features: int, out_features: int, dtype, device) -> nn.Parameter:
    """A Parameter of shape [in, out] whose storage is a contiguous [out, in] buffer."""
    buf = torch.empty(out_features, in_features, dtype=dtype, device=device)
    return nn.Parameter(buf.t())


def packed_view(param: nn.Parameter) -> torch.Tensor:
    """The [out, in] K-contiguous buffer behind an [in, out] parameter (re-packs if replaced)."""
    w = param.detach().t()
    if not w.is_contiguous():
        param.data = param.data.t().contiguous().t()
        w = param.detach().t()
    return w


def _kaiming(param: nn.Parameter):
    # The reference applies kaiming_uniform_(a=sqrt(5)) to its [in, out] tensor
    # (engine/tensor_parallel/layers.py:70-76, :136-142).
    nn.init.kaiming_uniform_(param, a=math.sqrt(5))


class ColumnParallelLinear(nn.Module):
    """``Y_local = X @ W_local (+ b_local)``, W_local = [in, out/ws] (engine/tensor_parallel/layers.py:23-86)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, rank: int = 0,
                 world_size: int = 1, gather_output: bool = False, dtype=None, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.rank = rank
        self.world_size = world_size
        self.gather_output = gather_output  # accepted and unused, like the reference (layers.py:38,47)
        assert out_features % world_size == 0, (
            f"out_features ({out_features}) must be divisible by world_size ({world_size})")
        self.out_features_per_partition = out_features // world_size
        dt = torch_dtype(dtype)
        dev = _default_device(device)
        self.weight = packed_parameter(in_features, self.out_features_per_partition, dt, dev)
        if bias:
            self.bias = nn.Parameter(torch.empty(self.out_features_per_partition, dtype=dt, device=dev))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self):
        with torch.no_grad():
            _kaiming(self.weight)
            if self.bias is not None:
                fan_in = self.weight.shape[1]
                bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
                nn.init.uniform_(self.bias, -bound, bound)

    def packed_weight(self) -> torch.Tensor:
        return packed_view(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: [batch, seq_len, in_features] -> [batch, seq_len, out_features_per_partition]."""
        with torch.no_grad():
            return kernels.linear(x, self.packed_weight(), self.bias)


class RowParallelLinear(nn.Module):
    """``Y = AllReduce(X_local @ W_local) + b``, W_local = [in/ws, out] (engine/tensor_parallel/layers.py:89-162)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, rank: int = 0,
                 world_size: int = 1, communicator: Optional[DistributedCommunicator] = None, dtype=None,
                 device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.rank = rank
        self.world_size = world_size
        self.communicator = communicator
        assert in_features % world_size == 0, (
            f"in_features ({in_features}) must be divisible by world_size ({world_size})")
        self.in_features_per_partition = in_features // world_size
        dt = torch_dtype(dtype)
        dev = _default_device(device)
        self.weight = packed_parameter(self.in_features_per_partition, out_features, dt, dev)
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=dt, device=dev))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self):
        with torch.no_grad():
            _kaiming(self.weight)
            if self.bias is not None:
                fan_in = self.weight.shape[1]
                bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
                nn.init.uniform_(self.bias, -bound, bound)

    def set_communicator(self, communicator: DistributedCommunicator):
        self.communicator = communicator

    def packed_weight(self) -> torch.Tensor:
        return packed_view(self.weight)

    def forward(self, x: torch.Tensor, step_tag: str = "") -> torch.Tensor:
        """x: [batch, seq_len, in_features_per_partition] -> [batch, seq_len, out_features]."""
        with torch.no_grad():
            partial = kernels.linear(x, self.packed_weight())
            if self.world_size > 1 and self.communicator is not None:
                output = self.communicator.all_reduce_sum(partial, step_tag=step_tag)
            else:
                output = partial
            if self.bias is not None:
                output = output + self.bias
            return output


class RMSNorm(nn.Module):
    """``x * rsqrt(mean(x^2) + eps) * weight`` with a float32 ``ones`` weight (engine/tensor_parallel/layers.py:165-184)."""

    def __init__(self, dim: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=_default_device(device)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # torch promotes x * float32 weight to float32 for bf16 inputs; so do we.
        out_dtype = torch.promote_types(x.dtype, self.weight.dtype)
        with torch.no_grad():
            return kernels.rmsnorm(x, self.weight, self.eps, out_dtype=out_dtype)
