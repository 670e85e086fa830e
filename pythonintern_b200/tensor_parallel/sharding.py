"""Slice a full state dict into tensor-parallel shards (engine/tensor_parallel/sharding.py:19-108).

Same routing as the reference's ``WeightSharder.shard_full_model_state_dict``:
q/k/v/gate/up weights ([in, out]) are split along dim 1, out_proj/down weights
along dim 0, everything else (embedding, norms, lm_head) is replicated.  Host-side
tensor slicing only; the shards are then loaded with ``load_state_dict``.
"""

from typing import Any, Dict

import torch

from pythonintern_b200.config import ModelConfig


class WeightSharder:
    def __init__(self, model_config: ModelConfig, world_size: int):
        self.config = model_config
        self.world_size = world_size
        self.heads_per_rank = model_config.num_heads // world_size
        self.kv_heads_per_rank = model_config.num_kv_heads // world_size
        self.inter_dim_per_rank = model_config.intermediate_dim // world_size

    def shard_column_parallel_weight(self, weight: torch.Tensor, rank: int) -> torch.Tensor:
        c = weight.shape[1] // self.world_size
        return weight[:, rank * c:(rank + 1) * c].clone()

    def shard_row_parallel_weight(self, weight: torch.Tensor, rank: int) -> torch.Tensor:
        c = weight.shape[0] // self.world_size
        return weight[rank * c:(rank + 1) * c, :].clone()

    def shard_attention_weights(self, q_weight, k_weight, v_weight, o_weight, rank: int):
        return (self.shard_column_parallel_weight(q_weight, rank), self.shard_column_parallel_weight(k_weight, rank),
                self.shard_column_parallel_weight(v_weight, rank), self.shard_row_parallel_weight(o_weight, rank))

    def shard_mlp_weights(self, gate_weight, up_weight, down_weight, rank: int):
        return (self.shard_column_parallel_weight(gate_weight, rank),
                self.shard_column_parallel_weight(up_weight, rank),
                self.shard_row_parallel_weight(down_weight, rank))

    def shard_full_model_state_dict(self, full_state_dict: Dict[str, Any], rank: int) -> Dict[str, Any]:
        out = {}
        for key, t in full_state_dict.items():
            if "q_proj.weight" in key or "k_proj.weight" in key or "v_proj.weight" in key:
                out[key] = self.shard_column_parallel_weight(t, rank)
            elif "out_proj.weight" in key:
                out[key] = self.shard_row_parallel_weight(t, rank)
            elif "gate_proj.weight" in key or "up_proj.weight" in key:
                out[key] = self.shard_column_parallel_weight(t, rank)
            elif "down_proj.weight" in key:
                out[key] = self.shard_row_parallel_weight(t, rank)
            else:
                out[key] = t.clone()
        return out
