"""Configuration dataclasses, field for field the reference's engine/config.py.

``ModelConfig`` (engine/config.py:13-37), ``ShardConfig`` (:40-52),
``KVCacheConfig`` (:55-64), ``SchedulerConfig`` (:67-73) and ``ClusterConfig``
(:76-87) keep their names, fields and defaults so that code written against the
reference constructs them unchanged.  Two behaviours are worth stating:

* ``ModelConfig.rope_theta`` is NOT read by the reference model, whose
  ``RotaryEmbedding`` is always built with base 10000 (engine/model/attention.py:129).
  This package reproduces that by default; ``ModelConfig.honor_rope_theta = True``
  opts into the configured base.
* ``KVCacheConfig.device`` defaults to ``"cuda"`` here: the pool lives in HBM.
"""

from dataclasses import dataclass, field
from typing import List


@dataclass
class ModelConfig:
    vocab_size: int = 32000
    hidden_dim: int = 1024
    num_layers: int = 8
    num_heads: int = 16
    num_kv_heads: int = 4
    intermediate_dim: int = 2816
    max_seq_len: int = 2048
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    dtype: str = "float32"  # "float32" or "bfloat16"
    # Behaviour switches (defaults reproduce the reference exactly).
    honor_rope_theta: bool = False      # reference ignores rope_theta (attention.py:129)
    masked_decode_padding: bool = False  # reference pads decode K/V with zeros and no mask

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads

    @property
    def num_queries_per_kv(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def rope_base(self) -> float:
        return float(self.rope_theta) if self.honor_rope_theta else 10000.0

    def validate(self):
        assert self.hidden_dim % self.num_heads == 0, "hidden_dim must be divisible by num_heads"
        assert self.num_heads % self.num_kv_heads == 0, "num_heads must be divisible by num_kv_heads"


@dataclass
class ShardConfig:
    rank: int = 0
    world_size: int = 1
    host: str = "127.0.0.1"
    port: int = 50051
    peer_addresses: List[str] = field(default_factory=list)
    timeout_seconds: float = 30.0

    @property
    def address(self) -> str:
        return f"{self.host}:{self.port}"


@dataclass
class KVCacheConfig:
    block_size: int = 16
    num_blocks: int = 256
    device: str = "cuda"

    @property
    def total_token_capacity(self) -> int:
        return self.block_size * self.num_blocks


@dataclass
class SchedulerConfig:
    max_batch_size: int = 16
    max_tokens_per_step: int = 512
    step_timeout_sec: float = 10.0
    preemption_mode: str = "recompute"


@dataclass
class ClusterConfig:
    coordinator_host: str = "127.0.0.1"
    coordinator_port: int = 50050
    worker_endpoints: List[str] = field(default_factory=lambda: ["127.0.0.1:50051", "127.0.0.1:50052"])
    model: ModelConfig = field(default_factory=ModelConfig)
    kv_cache: KVCacheConfig = field(default_factory=KVCacheConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)

    @property
    def world_size(self) -> int:
        return len(self.worker_endpoints)
