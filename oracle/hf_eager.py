"""The reference's eager PyTorch path: Transformers ``Qwen3ForCausalLM`` on the CPU.

TEST INFRASTRUCTURE ONLY (pins the oracle, generates golden vectors, and is the
timed CPU baseline of ``bench.py --impl reference``). Never used by the engine.

The reference treats native Transformers Qwen3 as ground truth: its tests
compare against ``model(prefix, use_cache=False)`` (``dryft/tests/test_decode.py:106,149``),
its judge replays teacher-forced (``dryft/agent/benchmark_gpu.py:136-153``),
and its baseline engine is a greedy ``DynamicCache`` loop
(``dryft/OPTIMIZATION_GUIDE.md:316-368``). Transformers is a third-party
dependency: the reference pins 4.51.3 (``dryft/requirements.txt:9``); this
image has 5.5.0, whose Qwen3 arithmetic (RMSNorm cast placement, fp32 rotary,
SiLU-gated MLP, pre-norm residuals) is the same.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

BF16 = torch.bfloat16


def build_hf_model(cfg, state: Optional[Dict[str, torch.Tensor]] = None):
    """A bf16, SDPA, eval-mode ``Qwen3ForCausalLM`` holding ``state`` (or
    uninitialised storage when ``state`` is None, for timing only).

    ``model.to(bf16)`` would also cast the rotary ``inv_freq`` buffer to bf16;
    the rotary module is rebuilt afterwards so it stays fp32, as in a
    checkpoint loaded with ``torch_dtype=bfloat16``.
    """
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    hf = cfg.to_hf()
    hf.pop("architectures", None)
    hf.pop("model_type", None)
    hf.pop("torch_dtype", None)
    config = Qwen3Config(**hf)
    config._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(config)
    if state is None:
        model = model.to_empty(device="cpu").to(BF16)
    else:
        sd = {k: v.to("cpu", BF16) for k, v in state.items()}
        if cfg.tied:
            sd.pop("lm_head.weight", None)
        missing, unexpected = model.load_state_dict(sd, strict=False, assign=True)
        missing = [m for m in missing if not (cfg.tied and m == "lm_head.weight")]
        if missing or unexpected:
            raise ValueError(f"state mismatch: missing={missing} unexpected={unexpected}")
        if cfg.tied:
            model.lm_head.weight = model.model.embed_tokens.weight
    model.model.rotary_emb = Qwen3RotaryEmbedding(config=config, device="cpu")
    return model.eval()


@torch.inference_mode()
def greedy(model, prompt: Sequence[int], n_new: int, logits_out: Optional[List] = None) -> List[int]:
    """The reference's baseline greedy loop with a ``DynamicCache``
    (``dryft/OPTIMIZATION_GUIDE.md:316-368``): prefill the prompt, then one
    token per forward, argmax of the bf16 logits."""
    from transformers import DynamicCache

    cache = DynamicCache()
    current = torch.tensor([list(prompt)], dtype=torch.int64)
    out = []
    for _ in range(n_new):
        res = model(input_ids=current, past_key_values=cache, use_cache=True, logits_to_keep=1)
        cache = res.past_key_values
        logits = res.logits[0, -1]
        if logits_out is not None:
            logits_out.append(logits.clone())
        tok = int(logits.float().argmax())
        out.append(tok)
        current = torch.tensor([[tok]], dtype=torch.int64)
    return out


@torch.inference_mode()
def teacher_forced_logits(model, ids: Sequence[int], start: int) -> torch.Tensor:
    """Full-prefix forward with ``use_cache=False``; logits predicting
    ids[start+1:] and beyond, i.e. rows start..len(ids)-1 (bf16 [n, V])."""
    x = torch.tensor([list(ids)], dtype=torch.int64)
    res = model(input_ids=x, use_cache=False)
    return res.logits[0, start:]
