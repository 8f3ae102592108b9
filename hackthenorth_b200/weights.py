"""Seeded random-init Qwen3 weights, the engine's packed HBM layout, and HF checkpoints.

The benchmark runs on synthetic weights: every linear and embedding matrix is
N(0, 0.02) drawn in fp32 from one seeded ``torch.Generator`` in a fixed
parameter order, then rounded to bf16; RMSNorm gains are 1 (Transformers'
default init). ``save_checkpoint`` writes a Hugging Face directory
(``config.json`` + ``model.safetensors``) so ``Engine(model_path)`` and the
native ``Qwen3ForCausalLM`` read the same bytes, as the reference's engine does
with the pinned checkpoint (``dryft/engine/engine.py:180-189``).

Packed layout (built once at load, like the reference's ``GroupedAttention``
q/k/v concatenation, ``dryft/engine/attention.py:51-63``, and ``FusedMLP``
gate/up concatenation, ``dryft/engine/engine.py:40-48``):

* ``qkv``  ``[Hq*D + 2*Hkv*D, H]``: q rows, then k rows, then v rows.
* ``gu``   ``[2*F, H]``: gate and up rows **interleaved** (row 2j = gate j,
  row 2j+1 = up j) so one CTA's contiguous row range holds whole SwiGLU pairs.
  The reference stacks gate rows then up rows instead; only the order differs.
* ``o`` ``[H, Hq*D]`` and ``down`` ``[H, F]`` keep the HF row-major layout.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterator, Tuple

import torch

from .config import ModelConfig

INIT_STD = 0.02


def param_specs(cfg: ModelConfig) -> Iterator[Tuple[str, tuple, str]]:
    """(HF name, shape, init kind) in the fixed generation order."""
    H, D, F = cfg.hidden, cfg.head_dim, cfg.ffn
    yield "model.embed_tokens.weight", (cfg.vocab, H), "normal"
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        yield p + "input_layernorm.weight", (H,), "ones"
        yield p + "self_attn.q_proj.weight", (cfg.q_width, H), "normal"
        yield p + "self_attn.k_proj.weight", (cfg.kv_width, H), "normal"
        yield p + "self_attn.v_proj.weight", (cfg.kv_width, H), "normal"
        yield p + "self_attn.o_proj.weight", (H, cfg.q_width), "normal"
        yield p + "self_attn.q_norm.weight", (D,), "ones"
        yield p + "self_attn.k_norm.weight", (D,), "ones"
        yield p + "post_attention_layernorm.weight", (H,), "ones"
        yield p + "mlp.gate_proj.weight", (F, H), "normal"
        yield p + "mlp.up_proj.weight", (F, H), "normal"
        yield p + "mlp.down_proj.weight", (H, F), "normal"
    yield "model.norm.weight", (H,), "ones"
    if not cfg.tied:
        yield "lm_head.weight", (cfg.vocab, H), "normal"


def random_state_dict(cfg: ModelConfig, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    """HF-named bf16 state dict drawn from ``torch.Generator(device).manual_seed(seed)``.

    CPU and CUDA generators produce different streams; parity runs draw on the
    CPU (the oracle's device) and copy, throughput runs may draw on the GPU.
    """
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = {}
    for name, shape, kind in param_specs(cfg):
        if kind == "ones":
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            t = torch.randn(shape, generator=gen, dtype=torch.float32, device=device)
            out[name] = t.mul_(INIT_STD).to(torch.bfloat16)
            del t
    return out


def save_checkpoint(path: str, cfg: ModelConfig, state: Dict[str, torch.Tensor]) -> None:
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg.to_hf(), f, indent=1)
    tensors = {k: v.detach().to("cpu").contiguous() for k, v in state.items()}
    save_file(tensors, os.path.join(path, "model.safetensors"), metadata={"format": "pt"})


def load_checkpoint(path: str, device="cpu") -> Tuple[ModelConfig, Dict[str, torch.Tensor]]:
    from safetensors.torch import load_file

    cfg = ModelConfig.from_dir(path)
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors file in {path}")
    state = {}
    for f in files:
        state.update(load_file(os.path.join(path, f), device=str(device)))
    for k in list(state):
        if state[k].dtype != torch.bfloat16:
            state[k] = state[k].to(torch.bfloat16)
    return cfg, state


class PackedWeights:
    """Device-resident weights in the engine's layout (see module docstring).

    With ``tp_size > 1`` only rank ``tp_rank``'s shard is kept (Megatron-style):
    KV heads [r*Hkv/n, (r+1)*Hkv/n) with their query heads (q/k/v rows of qkv,
    the matching input columns of o), FFN columns [r*F/n, (r+1)*F/n) (gate/up
    rows, down input columns) and vocabulary rows [r*V/n, (r+1)*V/n) of the
    head; the embedding and the norm gains stay whole. The block prefill's
    column-parallel projections also keep output rows [r*H/n, (r+1)*H/n) of o
    and down over every input column (``o_rows``, ``down_rows``: 2 (H/n)(Hq*D +
    F) bytes per layer more).
    """

    def __init__(self, cfg: ModelConfig, state: Dict[str, torch.Tensor], device="cuda:0",
                 tp_rank: int = 0, tp_size: int = 1):
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        dev = torch.device(device)
        n, r = tp_size, tp_rank
        D = cfg.head_dim
        if cfg.n_kv_heads % n or cfg.ffn % n or cfg.vocab % n:
            raise ValueError("n_kv_heads, ffn and vocab must divide by tp_size")
        hq, hkv, f, v = cfg.n_heads // n, cfg.n_kv_heads // n, cfg.ffn // n, cfg.vocab // n
        qs, ks, fs = slice(r * hq * D, (r + 1) * hq * D), slice(r * hkv * D, (r + 1) * hkv * D), slice(r * f, (r + 1) * f)

        def get(name):
            return state[name].to(device=dev, dtype=torch.bfloat16).contiguous()

        def dev_bf16(t):
            return t.to(device=dev, dtype=torch.bfloat16).contiguous()

        self.embed = get("model.embed_tokens.weight")
        self.final_norm = get("model.norm.weight")
        head = state.get("lm_head.weight")
        full_head = state["model.embed_tokens.weight"] if (cfg.tied or head is None) else head
        if n == 1:
            self.lm_head = self.embed if (cfg.tied or head is None) else get("lm_head.weight")
        else:
            self.lm_head = dev_bf16(full_head[r * v:(r + 1) * v])
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"model.layers.{i}."
            q, k, vv = (state[p + f"self_attn.{nm}_proj.weight"] for nm in "qkv")
            gate, up = state[p + "mlp.gate_proj.weight"], state[p + "mlp.up_proj.weight"]
            o, down = state[p + "self_attn.o_proj.weight"], state[p + "mlp.down_proj.weight"]
            self.layers.append({
                "input_norm": get(p + "input_layernorm.weight"),
                "qkv": dev_bf16(torch.cat((q[qs], k[ks], vv[ks]))),
                "q_norm": get(p + "self_attn.q_norm.weight"),
                "k_norm": get(p + "self_attn.k_norm.weight"),
                "o": dev_bf16(o[:, qs]) if n > 1 else get(p + "self_attn.o_proj.weight"),
                "post_norm": get(p + "post_attention_layernorm.weight"),
                "gu": dev_bf16(interleave_gate_up(gate[fs], up[fs])),
                "down": dev_bf16(down[:, fs]) if n > 1 else get(p + "mlp.down_proj.weight"),
            })
            if n > 1:
                hs = slice(r * (cfg.hidden // n), (r + 1) * (cfg.hidden // n))
                self.layers[-1]["o_rows"] = dev_bf16(o[hs])
                self.layers[-1]["down_rows"] = dev_bf16(down[hs])

    def nbytes(self) -> int:
        seen, total = set(), 0
        tensors = [self.embed, self.final_norm, self.lm_head]
        for layer in self.layers:
            tensors.extend(layer.values())
        for t in tensors:
            if t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                total += t.numel() * t.element_size()
        return total


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F,H] gate and up -> [2F,H] with gate j at row 2j and up j at row 2j+1."""
    if gate.shape != up.shape:
        raise ValueError("gate and up projections must have the same shape")
    return torch.stack((gate, up), dim=1).reshape(2 * gate.shape[0], gate.shape[1])


def rotary_table(cfg: ModelConfig, capacity: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin rows for positions [0, capacity), computed on the CPU in fp32.

    Same arithmetic as the installed ``Qwen3RotaryEmbedding.forward`` with its
    ``inv_freq`` kept in fp32: inv_freq = 1 / theta^(arange(0, D, 2)/D), angle =
    inv_freq * position (one fp32 product), cos/sin of cat(angle, angle) in fp32,
    then one rounding to bf16. The reference caches exactly these rows
    (``dryft/engine/decode.py:49-67``) and selects them by device position.
    """
    D = cfg.head_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    pos = torch.arange(capacity, dtype=torch.float32)
    freqs = (inv_freq[:, None] @ pos[None, :]).transpose(0, 1)  # [cap, D/2]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
