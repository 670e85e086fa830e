"""Generate the Llama-3-8B-shape layer parity fixture from the oracle.

``llama3_8b_layer_parity.npz`` holds what the numpy oracle (float64 arithmetic on
the bf16-rounded weights) computes for one Llama-3-8B-shape decoder layer (hidden
4096, 32 q / 8 kv heads, head_dim 128, intermediate 14336; vocabulary cut to 4096)
with the N(0, 0.02) weights of ``workloads.synthetic_state_dict(cfg, seed=21)``:

* step 0: two prompts (40 and 13 tokens, seeded) prefilled the reference's way, one
  forward per prompt at positions ``arange(P)`` (engine/worker/execution_engine.py:85-111);
* steps 1 and 2: both sequences decoded as one batch at positions ``current_len - 1``
  (execution_engine.py:113-135), fed the oracle's own greedy tokens of the step before.

Stored per step: the residual stream after the layer (the reference block's output,
engine/model/llama.py:48-76; float16 to keep the file small, a relative rounding of at
most 2**-11, far below the 2e-2 bf16 tolerance it is compared at), the float32 logits
of each sequence's last position, the greedy tokens and their top-1 minus top-2 logit
margins.  ``bench.py`` (its tensor-parallel parity leg) and ``tests/test_tp_gpu.py``
compare the CUDA path at TP = 1, 2, 4 and 8 against it; the TP degree does not change
the oracle's result beyond float64 summation order.

Usage:  python tests/golden/make_tp_parity.py      (CPU only, about half a minute)
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

OUT = os.path.join(HERE, "llama3_8b_layer_parity.npz")
SEED_WEIGHTS = 21
PROMPT_LENS = (40, 13)
TABLES = ((3, 9, 1, 12), (5, 0))
NUM_BLOCKS = 16
VOCAB = 4096
DECODE_STEPS = 2


def parity_config():
    """The layer's ModelConfig: Llama-3-8B shape, one layer, vocabulary 4096."""
    from pythonintern_b200 import workloads
    cfg = workloads.llama3_8b_config(num_layers=1, max_seq_len=512)
    cfg.vocab_size = VOCAB
    return cfg


def prompts():
    rng = np.random.default_rng(5)
    return [rng.integers(0, VOCAB, size=n).astype(np.int64) for n in PROMPT_LENS]


def compute():
    """The fixture's arrays, recomputed with the oracle."""
    import oracle
    from pythonintern_b200 import workloads
    cfg = parity_config()
    sd = {k: v.float().numpy() for k, v in workloads.synthetic_state_dict(cfg, seed=SEED_WEIGHTS).items()}
    ocfg = oracle.OracleConfig(cfg.vocab_size, cfg.hidden_dim, 1, cfg.num_heads, cfg.num_kv_heads,
                               cfg.intermediate_dim, cfg.max_seq_len, cfg.rms_norm_eps)
    om = oracle.OracleModel(ocfg, [sd], [oracle.KVPool(1, NUM_BLOCKS, 16, cfg.num_kv_heads, cfg.head_dim)])
    ps = prompts()
    hidden, logits = [], []
    for p, table in zip(ps, TABLES):
        tr = []
        lg = om.forward(p[None], np.arange(p.size)[None], [list(table)], True, trace=tr)
        hidden.append(tr[0][0])
        logits.append(lg[0])
    steps_hidden = [np.concatenate(hidden)]
    steps_logits = [np.stack(logits)]
    lens = np.asarray(PROMPT_LENS, dtype=np.int64)
    for _ in range(DECODE_STEPS):
        toks = np.argmax(steps_logits[-1], axis=1)
        tr = []
        lg = om.forward(toks[:, None], lens[:, None], [list(t) for t in TABLES], False, trace=tr)
        steps_hidden.append(tr[0][:, 0])
        steps_logits.append(lg)
        lens = lens + 1
    lg = np.stack(steps_logits)                         # [steps, 2, V]
    srt = np.sort(lg, axis=-1)
    return dict(
        prompt0=ps[0], prompt1=ps[1],
        hidden_prefill=steps_hidden[0].astype(np.float16),
        hidden_decode=np.stack(steps_hidden[1:]).astype(np.float16),
        logits=lg.astype(np.float32),
        tokens=np.argmax(lg, axis=-1).astype(np.int64),
        margins=(srt[..., -1] - srt[..., -2]).astype(np.float32),
    )


def main():
    out = compute()
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, "tokens", out["tokens"].tolist(), "margins", np.round(out["margins"], 4).tolist())


if __name__ == "__main__":
    main()
