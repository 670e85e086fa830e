"""Sharded SwiGLU MLP (engine/model/mlp.py:22-86).

``gate_proj``/``up_proj`` are ColumnParallelLinear and ``down_proj`` is
RowParallelLinear, exactly as in the reference.  The forward runs the gate and up
GEMMs as ONE tensor-core kernel whose epilogue writes ``silu(g) * u``
(``b2_linear_swiglu``; ``b2_linear_swiglu_rownorm`` when it also finishes a deferred
RMSNorm of its input rows), then the row-parallel down projection and its all-reduce.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from pythonintern_b200 import kernels
from pythonintern_b200.config import ModelConfig
from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
from pythonintern_b200.tensor_parallel.layers import ColumnParallelLinear, RowParallelLinear
from pythonintern_b200._lib import torch_dtype


class DistributedMLP(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int, rank: int = 0, world_size: int = 1,
                 communicator: Optional[DistributedCommunicator] = None, device=None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.rank = rank
        self.world_size = world_size
        self.communicator = communicator
        assert config.intermediate_dim % world_size == 0, (
            f"intermediate_dim {config.intermediate_dim} must be divisible by world_size {world_size}")
        dt = torch_dtype(config.dtype)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        H, inter = config.hidden_dim, config.intermediate_dim
        self.gate_proj = ColumnParallelLinear(H, inter, False, rank, world_size, dtype=dt, device=dev)
        self.up_proj = ColumnParallelLinear(H, inter, False, rank, world_size, dtype=dt, device=dev)
        self.down_proj = RowParallelLinear(inter, H, False, rank, world_size, communicator, dtype=dt, device=dev)

    def set_communicator(self, communicator: DistributedCommunicator):
        self.communicator = communicator
        self.down_proj.set_communicator(communicator)

    def gate_up(self, x2d: torch.Tensor, out: Optional[torch.Tensor] = None, row_ss: Optional[torch.Tensor] = None,
                eps: float = 1e-5) -> torch.Tensor:
        """``silu(x Wg) * (x Wu)`` for [T, hidden] rows (mlp.py:80-82); with ``row_ss`` the rows
        are a deferred RMSNorm's ``z = h * w`` and the row scale is applied in the GEMM."""
        if row_ss is not None:
            return kernels.linear_swiglu_rownorm(x2d, self.gate_proj.packed_weight(), self.up_proj.packed_weight(),
                                                 row_ss, eps, out=out)
        return kernels.linear_swiglu(x2d, self.gate_proj.packed_weight(), self.up_proj.packed_weight(), out=out)

    def forward(self, x: torch.Tensor, step_id: int = 0) -> torch.Tensor:
        with torch.no_grad():
            inter = self.gate_up(x)
            return self.down_proj(inter, step_tag=f"step_{step_id}_l{self.layer_idx}_mlp")
