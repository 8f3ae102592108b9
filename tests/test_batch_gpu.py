"""Batched decode (B > 1 sequences on one GPU) against the CPU oracle.

The reference's DecodeState takes a batch dimension (KV cache [B, Hkv, cap, D]
per layer, dryft/engine/decode.py:25-67,102-138) and tuned B4/B16 variants of
its kernels (dryft/engine/fused_layer.py:171-185). Here B <= 8 sequences share
one pass of the rows kernels per step; every sequence keeps its own cache slice
and position. Parity is per sequence: each row's logits against the oracle's
single-sequence forward, and the greedy stream against the oracle's."""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda:0"
LOGIT_ATOL = 0.0625


@pytest.mark.parametrize("shape", ["small", "8b-layer"])
def test_batched_step_distinct_positions_matches_oracle(built_lib, cpu_threads, shape):
    """Three sequences with seeded N(0, 1) cache prefixes of different lengths:
    one batched step appends each sequence's K/V at its own position, its
    logits match the oracle's single-sequence step within LOGIT_ATOL (the
    greedy token too, unless the oracle holds a near tie), and every position
    advances by one."""
    from hackthenorth_b200.config import QWEN3_8B, QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = QWEN3_SMALL if shape == "small" else dataclasses.replace(QWEN3_8B, n_layers=1)
    state = random_state_dict(cfg, 6)
    engine = Engine(None, DEV, cfg=cfg, state=state)
    positions, tokens = [100, 37, 250], [17, 5, 900]
    B, cap = len(positions), 300
    st = engine.new_state(1, 4, capacity=cap, batch=B, keep_logits=True)
    g = torch.Generator().manual_seed(12)
    prefixes = []
    for b, p in enumerate(positions):
        kp = torch.randn(cfg.n_layers, cfg.n_kv_heads, p, cfg.head_dim, generator=g).to(BF16)
        vp = torch.randn(cfg.n_layers, cfg.n_kv_heads, p, cfg.head_dim, generator=g).to(BF16)
        st.keys[:, b, :, :p] = kp.to(DEV)
        st.values[:, b, :, :p] = vp.to(DEV)
        prefixes.append((kp, vp))
    st.token.copy_(torch.tensor(tokens))
    st.position.copy_(torch.tensor(positions))
    st.step_eager()
    st.check()
    assert st.position.tolist() == [p + 1 for p in positions]
    got_tok = st.read_token()
    logits = st.logits.float().cpu()
    for b, p in enumerate(positions):
        o = OracleQwen3(cfg, state, cap)
        o.keys[:, :, :p], o.values[:, :, :p] = prefixes[b]
        ref, ref_tok = o.forward_rows([tokens[b]], p)
        ref = ref[0].float()
        d = (logits[b] - ref).abs()
        assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (b, float(d.max()), float(d.mean()))
        if got_tok[b] != int(ref_tok[0]):
            top2 = ref.topk(2).values
            assert float(top2[0] - top2[1]) <= LOGIT_ATOL, f"sequence {b}"
        torch.testing.assert_close(st.keys[:, b, :, p].float().cpu(), o.keys[:, :, p].float(), atol=0.0625,
                                   rtol=0.02)
        torch.testing.assert_close(st.values[:, b, :, p].float().cpu(), o.values[:, :, p].float(), atol=0.0625,
                                   rtol=0.02)


@pytest.mark.parametrize("B", [2, 5, 8, 12, 17])
def test_batched_generate_matches_oracle_greedy(built_lib, cpu_threads, B):
    """Engine.generate over B prompts of 16 tokens (teacher-forced batched
    prefill, then the captured batched step; above 8 sequences, chunks of 8
    on contexts sharing the weights): every sequence's stream equals the
    oracle's greedy continuation of that prompt up to the first step where
    the oracle's top-2 logits lie within LOGIT_ATOL."""
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg, n_new, P = QWEN3_SMALL, 12, 16
    state = random_state_dict(cfg, 0)
    engine = Engine(None, DEV, cfg=cfg, state=state)
    g = torch.Generator().manual_seed(40 + B)
    prompts = torch.randint(0, cfg.vocab, (B, P), generator=g).tolist()
    steps = list(engine.generate(prompts, n_new))
    engine.state.check()
    assert len(steps) == n_new and all(len(s) == B for s in steps)
    for b in range(B):
        got = [s[b] for s in steps]
        o = OracleQwen3(cfg, state, P + n_new)
        logits, toks = o.forward_rows(prompts[b], 0)
        last, tok, pos = logits[-1].float(), int(toks[-1]), P
        for i in range(n_new):
            if got[i] != tok:
                top2 = last.topk(2).values
                assert float(top2[0] - top2[1]) <= LOGIT_ATOL, f"sequence {b} step {i}"
                break
            logits, toks = o.forward_rows([tok], pos)
            last, tok, pos = logits[0].float(), int(toks[0]), pos + 1


def test_batched_state_rejects_verify_and_bad_shapes(built_lib):
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    engine = Engine.from_random(QWEN3_SMALL, seed=0)
    st = engine.new_state(4, 4, batch=2)
    with pytest.raises(ValueError):
        st.verify(1, [2, 3])
    with pytest.raises(ValueError):
        st.prefill(torch.zeros(3, 4, dtype=torch.int64, device=DEV))
    with pytest.raises(ValueError):
        engine.new_state(4, 4, batch=9)
    with pytest.raises(ValueError):
        list(engine.generate([[1, 2, 3], [4, 5]], 2))
