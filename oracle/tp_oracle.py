"""CPU restatement of the tensor-parallel decode path over torch.distributed.

TEST INFRASTRUCTURE ONLY (checks the shard layout and the reduction order of
the multi-GPU engine; never used by the engine). The reference has no
multi-GPU path; this splits its single-GPU arithmetic (``qwen3_oracle``) the
way ``hackthenorth_b200.weights.PackedWeights`` shards the weights:

* rank r owns KV heads [r*Hkv/n, (r+1)*Hkv/n) and their query heads, FFN
  columns [r*F/n, (r+1)*F/n) and vocabulary rows [r*V/n, (r+1)*V/n);
* o-proj and down produce fp32 partial sums, all-reduced across ranks, then
  rounded to bf16 once and added to the residual (the single rounding of
  ``dryft/engine/kernels/projection.py:65`` and ``kernels/down.py:283``);
* the greedy token is the largest bf16 logit over all shards, lowest index on
  ties (``dryft/engine/kernels/greedy.py:27-31``).
"""
from __future__ import annotations

from typing import Dict, Sequence

import torch
import torch.distributed as dist

from .qwen3_oracle import BF16, grouped_attention, linear, norm_rope, rms_norm, swiglu


class OracleQwen3TP:
    def __init__(self, cfg, state: Dict[str, torch.Tensor], capacity: int, rank: int, world: int):
        from hackthenorth_b200.weights import rotary_table

        self.cfg, self.rank, self.world = cfg, rank, world
        n, r, D = world, rank, cfg.head_dim
        self.hq, self.hkv, self.f, self.v = cfg.n_heads // n, cfg.n_kv_heads // n, cfg.ffn // n, cfg.vocab // n
        qs = slice(r * self.hq * D, (r + 1) * self.hq * D)
        ks = slice(r * self.hkv * D, (r + 1) * self.hkv * D)
        fs = slice(r * self.f, (r + 1) * self.f)
        w = {k: t.to("cpu", BF16) for k, t in state.items()}
        self.embed = w["model.embed_tokens.weight"]
        self.final_norm = w["model.norm.weight"]
        head = w.get("lm_head.weight", self.embed)
        self.head = head[r * self.v:(r + 1) * self.v]
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"model.layers.{i}."
            self.layers.append({
                "in": w[p + "input_layernorm.weight"], "post": w[p + "post_attention_layernorm.weight"],
                "q": w[p + "self_attn.q_proj.weight"][qs], "k": w[p + "self_attn.k_proj.weight"][ks],
                "v": w[p + "self_attn.v_proj.weight"][ks], "o": w[p + "self_attn.o_proj.weight"][:, qs],
                "qn": w[p + "self_attn.q_norm.weight"], "kn": w[p + "self_attn.k_norm.weight"],
                "gate": w[p + "mlp.gate_proj.weight"][fs], "up": w[p + "mlp.up_proj.weight"][fs],
                "down": w[p + "mlp.down_proj.weight"][:, fs],
            })
        self.keys = torch.zeros(cfg.n_layers, self.hkv, capacity, D, dtype=BF16)
        self.values = torch.zeros_like(self.keys)
        self.cos, self.sin = rotary_table(cfg, capacity)

    def _reduce(self, partial: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(partial)  # fp32 sum over ranks
        return partial

    def forward_rows(self, tokens: Sequence[int], first_position: int):
        cfg, D, eps = self.cfg, self.cfg.head_dim, self.cfg.rms_eps
        Q = len(tokens)
        positions = list(range(first_position, first_position + Q))
        x = self.embed[torch.as_tensor(list(tokens))]
        cos = self.cos[positions][:, None, :]
        sin = self.sin[positions][:, None, :]
        for l, L in enumerate(self.layers):
            nrm = rms_norm(x, L["in"], eps)
            q = norm_rope(linear(nrm, L["q"]).view(Q, self.hq, D), L["qn"], eps, cos, sin)
            k = norm_rope(linear(nrm, L["k"]).view(Q, self.hkv, D), L["kn"], eps, cos, sin)
            v = linear(nrm, L["v"]).view(Q, self.hkv, D)
            self.keys[l][:, positions] = k.transpose(0, 1)
            self.values[l][:, positions] = v.transpose(0, 1)
            a = grouped_attention(q.transpose(0, 1), self.keys[l], self.values[l], positions)
            a = a.transpose(0, 1).reshape(Q, self.hq * D)
            o = self._reduce(a.float() @ L["o"].float().T)
            h = o.to(BF16) + x
            n2 = rms_norm(h, L["post"], eps)
            m = swiglu(linear(n2, L["gate"]), linear(n2, L["up"]))
            d = self._reduce(m.float() @ L["down"].float().T)
            x = d.to(BF16) + h
        xn = rms_norm(x, self.final_norm, eps)
        logits = linear(xn, self.head)                        # [Q, V/n] bf16
        gathered = [torch.empty_like(logits) for _ in range(self.world)]
        dist.all_gather(gathered, logits)
        full = torch.cat(gathered, dim=-1)
        return full, full.float().argmax(-1)
