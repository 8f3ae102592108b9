"""Generate the golden vectors that pin the CPU oracle to the reference's eager path.

Run from the repository root:  python tests/golden/make_golden.py

The reference's ground truth is native Transformers ``Qwen3ForCausalLM`` in
eager bf16 with SDPA (``dryft/tests/test_decode.py:106,149``,
``dryft/agent/benchmark_gpu.py:136-153``); its baseline engine is the greedy
``DynamicCache`` loop of ``dryft/OPTIMIZATION_GUIDE.md:316-368``. This script
runs exactly that on seeded random-init weights and writes small fixtures:

* ``qwen3_0p6b_greedy.json``: the 0.6B shape, weights seed 0, a 32-token
  uniform random prompt (seed 1), 128 greedy tokens, and per step the top-64
  bf16 logits (values, ids), the top-1/top-2 margin and fp64 sum / sum of
  squares of the whole logit row. Also the noise floor of the reference
  itself: cached-decode vs full-prefix logits on the first 8 steps.
* ``qwen3_0p6b_greedy_notie.json``: the same for a second 32-token prompt
  (seed 81) chosen because no step of its 128 has a top-1/top-2 margin below
  0.0625 (4 bf16 ulps at the logits' scale), so every token can be required
  identical; the seed-1 prompt holds an exact tie at step 14. Prompt seeds
  from 2 upward were scanned in order: 81 is the first whose stream changes
  token and has no margin below 0.0625 (most seeds hold exact ties).
* ``qwen3_small_greedy.npz``: the small test shape (seed 0 weights, seed 1
  prompt of 16), 24 greedy tokens with the full bf16 logit rows.
* ``attention_sdpa.npz``: fp32 SDPA outputs (the reference's attention check,
  ``dryft/tests/test_fused_kernels.py:390-401``) for GQA 32/8, D 128, L 512,
  1 and 5 causal query rows, on Q/K/V drawn from seed 2.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from hackthenorth_b200.config import QWEN3_0P6B, QWEN3_SMALL  # noqa: E402
from hackthenorth_b200.weights import random_state_dict  # noqa: E402
from oracle import hf_eager  # noqa: E402
from oracle.qwen3_oracle import sdpa_reference  # noqa: E402


def prompt_ids(vocab: int, n: int, seed: int = 1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g).tolist()


def attention_inputs(L: int, queries: int, seed: int = 2, hq: int = 32, hkv: int = 8, d: int = 128):
    """Q [hq, queries, d], K/V [hkv, L, d] ~ N(0,1) bf16; query rows sit at the
    last ``queries`` positions of the cache."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(hq, queries, d, generator=g).to(torch.bfloat16)
    k = torch.randn(hkv, L, d, generator=g).to(torch.bfloat16)
    v = torch.randn(hkv, L, d, generator=g).to(torch.bfloat16)
    positions = list(range(L - queries, L))
    return q, k, v, positions


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)


def write_0p6b_greedy(model, cfg, prompt_seed: int, filename: str):
    """128 native greedy tokens for a 32-token prompt, per-step top-64 logits,
    margins, row sums, and the native cached vs full-prefix noise floor."""
    prompt = prompt_ids(cfg.vocab, 32, seed=prompt_seed)
    logits = []
    tokens = hf_eager.greedy(model, prompt, 128, logits)
    steps = []
    for row in logits:
        f = row.float()
        top = f.topk(64)
        steps.append({
            "top_ids": top.indices.tolist(),
            "top_vals": top.values.tolist(),
            "margin": float(top.values[0] - top.values[1]),
            "sum": float(f.double().sum()),
            "sumsq": float(f.double().pow(2).sum()),
        })
    tf = hf_eager.teacher_forced_logits(model, prompt + tokens[:8], len(prompt) - 1)
    floor = [float((a.float() - b.float()).abs().max()) for a, b in zip(logits[:8], tf[:8])]
    with open(os.path.join(HERE, filename), "w") as f:
        json.dump({
            "config": cfg.name, "weights_seed": 0, "prompt_seed": prompt_seed,
            "transformers": __import__("transformers").__version__,
            "prompt": prompt, "tokens": tokens, "steps": steps,
            "self_noise_cached_vs_full_prefix": floor,
        }, f)


def main(only_notie: bool = False):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    # --- 0.6B greedy, 128 steps -------------------------------------------------
    cfg = QWEN3_0P6B
    state = random_state_dict(cfg, seed=0)
    model = hf_eager.build_hf_model(cfg, state)
    if not only_notie:
        write_0p6b_greedy(model, cfg, 1, "qwen3_0p6b_greedy.json")
    write_0p6b_greedy(model, cfg, 81, "qwen3_0p6b_greedy_notie.json")
    del model, state
    if only_notie:
        return

    # --- small shape, full logits ----------------------------------------------
    cfg = QWEN3_SMALL
    state = random_state_dict(cfg, seed=0)
    model = hf_eager.build_hf_model(cfg, state)
    prompt = prompt_ids(cfg.vocab, 16)
    logits = []
    tokens = hf_eager.greedy(model, prompt, 24, logits)
    np.savez_compressed(os.path.join(HERE, "qwen3_small_greedy.npz"),
                        prompt=np.array(prompt, np.int64), tokens=np.array(tokens, np.int64),
                        logits_bf16=np.stack([bf16_bits(r) for r in logits]))

    # --- attention op -------------------------------------------------------------
    out = {}
    for queries in (1, 5):
        q, k, v, positions = attention_inputs(512, queries)
        out[f"q{queries}"] = sdpa_reference(q, k, v, positions).numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "attention_sdpa.npz"), **out)
    print("wrote golden fixtures to", HERE)


if __name__ == "__main__":
    main(only_notie="--notie" in sys.argv)
