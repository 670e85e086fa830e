"""Seeded synthetic weights and inputs for the reference's benchmark configurations.

There are no checkpoints or datasets for this engine: the reference initialises
every shard randomly (engine/worker/worker_node.py:51-57) and its README quotes no
dataset.  These helpers produce the deterministic stand-ins used by the tests and
the benchmark:

* ``tiny_config`` / ``reference_init_state_dict``: the Tiny LLaMA configuration
  (hidden 256, 4 layers, 8/2 heads, intermediate 688, vocab 1024) with the exact
  parameter initialisation the reference performs under ``torch.manual_seed(0)``
  (nn.Embedding normal init, kaiming-uniform(a=sqrt 5) for every linear, ones
  for the norms), replayed in the reference's module-construction order
  (engine/model/llama.py:101-121, attention.py:111-127, mlp.py:52-66).
* ``synthetic_state_dict``: N(0, 0.02) weights for the larger shapes, drawn key
  by key from one seeded generator (the reference has no such init).
* ``tiny_prompts``: 8 prompts whose lengths are ``randint(16, 64)`` and tokens
  ``randrange(1024)`` drawn interleaved from ``random.Random(0)``.
"""

from __future__ import annotations

import math
import random
from typing import Dict, List

import torch

from pythonintern_b200.config import ModelConfig


def tiny_config() -> ModelConfig:
    """Tiny LLaMA: hidden 256, 4 layers, 8 q / 2 kv heads (head_dim 32), SwiGLU 688, vocab 1024."""
    return ModelConfig(vocab_size=1024, hidden_dim=256, num_layers=4, num_heads=8, num_kv_heads=2,
                       intermediate_dim=688, max_seq_len=2048, rms_norm_eps=1e-5, rope_theta=10000.0,
                       dtype="float32")


def tinyllama_config(num_layers: int = 22) -> ModelConfig:
    """TinyLlama 1.1B shape: hidden 2048, 32 q / 4 kv heads, intermediate 5632, vocab 32000."""
    return ModelConfig(vocab_size=32000, hidden_dim=2048, num_layers=num_layers, num_heads=32,
                       num_kv_heads=4, intermediate_dim=5632, max_seq_len=2048, rms_norm_eps=1e-5,
                       rope_theta=10000.0, dtype="bfloat16")


def llama3_8b_config(num_layers: int = 32, max_seq_len: int = 4096) -> ModelConfig:
    """Llama-3-8B shape: hidden 4096, 32 q / 8 kv heads, intermediate 14336, vocab 128256."""
    return ModelConfig(vocab_size=128256, hidden_dim=4096, num_layers=num_layers, num_heads=32,
                       num_kv_heads=8, intermediate_dim=14336, max_seq_len=max_seq_len,
                       rms_norm_eps=1e-5, rope_theta=500000.0, dtype="bfloat16")


def mistral_7b_config(num_layers: int = 32, max_seq_len: int = 8448) -> ModelConfig:
    """Mistral-7B shape with GQA: hidden 4096, 32 q / 8 kv heads, intermediate 14336, vocab 32000."""
    return ModelConfig(vocab_size=32000, hidden_dim=4096, num_layers=num_layers, num_heads=32,
                       num_kv_heads=8, intermediate_dim=14336, max_seq_len=max_seq_len,
                       rms_norm_eps=1e-5, rope_theta=10000.0, dtype="bfloat16")


def state_dict_shapes(cfg: ModelConfig):
    """Full (world_size 1) parameter shapes in the reference's state_dict key order.

    Linear weights are [in, out] (engine/tensor_parallel/layers.py:55-61, :123-129);
    ``lm_head.weight`` is an nn.Linear weight [vocab, hidden] (llama.py:121).
    """
    H, hd = cfg.hidden_dim, cfg.head_dim
    nq, nkv, inter, V = cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_dim, cfg.vocab_size
    shapes = [("embed_tokens.weight", (V, H), "embedding")]
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        shapes += [
            (p + "input_layernorm.weight", (H,), "ones"),
            (p + "self_attn.q_proj.weight", (H, nq * hd), "linear"),
            (p + "self_attn.k_proj.weight", (H, nkv * hd), "linear"),
            (p + "self_attn.v_proj.weight", (H, nkv * hd), "linear"),
            (p + "self_attn.out_proj.weight", (nq * hd, H), "linear"),
            (p + "post_attention_layernorm.weight", (H,), "ones"),
            (p + "mlp.gate_proj.weight", (H, inter), "linear"),
            (p + "mlp.up_proj.weight", (H, inter), "linear"),
            (p + "mlp.down_proj.weight", (inter, H), "linear"),
        ]
    shapes += [("norm.weight", (H,), "ones"), ("lm_head.weight", (V, H), "linear")]
    return shapes


def reference_init_state_dict(cfg: ModelConfig, seed: int = 0) -> Dict[str, torch.Tensor]:
    """The float32 state dict the reference builds after ``torch.manual_seed(seed)`` (CPU RNG).

    The random stream is consumed in module-construction order: nn.Embedding's
    ``normal_``, then per layer q, k, v, out_proj, gate, up, down with
    ``kaiming_uniform_(a=sqrt(5))`` on the [in, out] tensors, then the lm_head.
    """
    torch.manual_seed(seed)
    sd = {}
    for key, shape, kind in state_dict_shapes(cfg):
        if kind == "embedding":
            sd[key] = torch.nn.init.normal_(torch.empty(shape))
        elif kind == "ones":
            sd[key] = torch.ones(shape)
        else:
            sd[key] = torch.nn.init.kaiming_uniform_(torch.empty(shape), a=math.sqrt(5))
    return sd


def synthetic_state_dict(cfg: ModelConfig, seed: int = 0, std: float = 0.02, device="cpu",
                         dtype=torch.bfloat16, layers=None) -> Dict[str, torch.Tensor]:
    """N(0, std) weights (norms = 1) for the bf16 configurations, key by key from one generator.

    ``layers`` restricts generation to those layer indices (the others are omitted).
    Values are drawn in float32 and rounded to ``dtype``.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    sd = {}
    for key, shape, kind in state_dict_shapes(cfg):
        if layers is not None and key.startswith("layers."):
            if int(key.split(".")[1]) not in layers:
                continue
        if kind == "ones":
            sd[key] = torch.ones(shape, device=device, dtype=torch.float32)
        else:
            t = torch.empty(shape, device=device, dtype=torch.float32)
            t.normal_(0.0, std, generator=g)
            sd[key] = t.to(dtype)
    return sd


def tiny_prompts(num_requests: int = 8, vocab: int = 1024, lo: int = 16, hi: int = 64,
                 seed: int = 0) -> List[List[int]]:
    """Prompt token lists: lengths ``randint(lo, hi)``, tokens ``randrange(vocab)``, interleaved."""
    rng = random.Random(seed)
    prompts = []
    for _ in range(num_requests):
        n = rng.randint(lo, hi)
        prompts.append([rng.randrange(vocab) for _ in range(n)])
    return prompts
