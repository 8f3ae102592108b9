"""Speculative verify pass (qb_verify / DecodeState.verify) against the CPU
oracle and the plain greedy path.

The reference's verify (dryft/engine/decode.py:168-206) runs the current
token and k draft tokens at consecutive positions through every layer and the
LM head; its tests require the emitted stream to equal plain greedy decoding
(dryft/tests/test_speculate.py: accepted prefixes never change the output).
"""
import dataclasses
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
LOGIT_ATOL = 0.0625


def _verify_rows(engine, state, current, proposal):
    """Run one verify pass without applying it; returns (predictions, logits)."""
    from hackthenorth_b200 import _lib

    n = len(proposal) + 1
    dev = engine.device
    ids = torch.tensor([current, *proposal], dtype=torch.int64, device=dev)
    preds = torch.zeros(n, dtype=torch.int64, device=dev)
    logits = torch.zeros(n, engine.cfg.vocab, dtype=BF16, device=dev)
    L = _lib.load()
    _lib.check(L.qb_verify(engine.ctx, ids.data_ptr(), n, state.position.data_ptr(), preds.data_ptr(),
                           logits.data_ptr(), _lib.stream_handle()), engine.ctx)
    state.check()
    return preds.cpu().tolist(), logits.float().cpu()


@pytest.mark.parametrize("shape", ["small", "8b-layer"])
@pytest.mark.parametrize("n_rows", [2, 5, 8])
def test_verify_rows_match_oracle(built_lib, cpu_threads, shape, n_rows):
    from hackthenorth_b200.config import QWEN3_8B, QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = QWEN3_SMALL if shape == "small" else dataclasses.replace(QWEN3_8B, n_layers=1)
    state = random_state_dict(cfg, 5)
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    rng = torch.Generator().manual_seed(17 + n_rows)
    prompt = torch.randint(0, cfg.vocab, (37,), generator=rng).tolist()
    drafts = torch.randint(0, cfg.vocab, (n_rows - 1,), generator=rng).tolist()
    st = engine.new_state(len(prompt), 4, draft_tokens=8)
    st.prefill(torch.tensor(prompt, device=engine.device))
    current = st.read_token()[0]
    preds, logits = _verify_rows(engine, st, current, drafts)
    assert int(st.position.item()) == len(prompt)  # verify leaves the position to the caller

    o = OracleQwen3(cfg, state, st.capacity)
    o.forward_rows(prompt, 0)
    ref, ref_tok = o.forward_rows([current, *drafts], len(prompt))
    ref = ref.float()
    d = (logits - ref).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    for i in range(n_rows):
        if preds[i] != int(ref_tok[i]):
            top2 = ref[i].topk(2).values
            assert float(top2[0] - top2[1]) <= LOGIT_ATOL, f"row {i}"
    # the rows' K/V are in the cache at positions len(prompt) ..
    p0 = len(prompt)
    for l in range(cfg.n_layers):
        torch.testing.assert_close(st.keys[l, :, p0:p0 + n_rows].float().cpu(), o.keys[l, :, p0:p0 + n_rows].float(),
                                   atol=0.0625, rtol=0.02)
        torch.testing.assert_close(st.values[l, :, p0:p0 + n_rows].float().cpu(),
                                   o.values[l, :, p0:p0 + n_rows].float(), atol=0.0625, rtol=0.02)


def test_verify_row0_matches_decode_step(built_lib):
    """Row 0 of a verify pass is the decode step of the same token: same
    greedy token, logits within LOGIT_ATOL (different summation order)."""
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    engine = Engine.from_random(QWEN3_SMALL, seed=2)
    prompt = list(range(3, 40))
    st = engine.new_state(len(prompt), 4, draft_tokens=4, keep_logits=True)
    st.prefill(torch.tensor(prompt, device=engine.device))
    current = st.read_token()[0]
    preds, logits = _verify_rows(engine, st, current, [5, 6, 7])
    st.step_eager()
    st.check()
    assert st.read_token()[0] == preds[0]
    assert (st.logits.float().cpu() - logits[0]).abs().max() <= LOGIT_ATOL


def test_speculative_generate_equals_plain_greedy(built_lib):
    """Synthetic drafts (target continuation with p = 0.7, else uniform) and
    prompt lookup: the emitted stream is the golden greedy stream, every
    length is exact, and proposals were actually verified."""
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.speculate import PromptLookup, SyntheticDraft

    g = np.load(os.path.join(GOLDEN, "qwen3_small_greedy.npz"))
    prompt, gold = g["prompt"].tolist(), g["tokens"].tolist()
    engine = Engine.from_random(QWEN3_SMALL, seed=0)
    for k in (1, 4, 7):
        draft = SyntheticDraft(gold, QWEN3_SMALL.vocab, p=0.7, seed=3, draft_length=k)
        out = [s[0] for s in engine.generate([prompt], len(gold), draft_tokens=k, drafter=draft)]
        assert out == gold, f"k={k}"
        assert engine.state._verify_n == k + 1
    # prompt lookup on a repetitive prompt proposes continuations
    rep = (prompt[:6] * 5)[:30]
    plain = [s[0] for s in engine.generate([rep], 24, draft_tokens=0)]
    spec = [s[0] for s in engine.generate([rep], 24, draft_tokens=4, drafter=PromptLookup(rep, draft_length=4))]
    assert spec == plain
    # the default, as the reference's generate (dryft/engine/engine.py:214-249):
    # prompt lookup with draft_width(24) = 7 draft tokens, verified 8 rows at a time
    default = [s[0] for s in engine.generate([rep], 24)]
    assert default == plain and engine.state._verify_n == 8
    for n in (1, 2, 3):
        assert len(list(engine.generate([rep], n, draft_tokens=4))) == n


def test_default_speculation_width_with_four_query_heads_per_kv_head(built_lib):
    """With 4 query heads per KV head (the 4B and 8B shapes) the default
    prompt-lookup speculation proposes at most 5 tokens, so every verify pass
    holds at most 6 rows (24 rows per KV head, the rows attention kernel), and
    the emitted stream is the plain greedy one."""
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    cfg = dataclasses.replace(QWEN3_SMALL, name="qwen3-small-g4", n_kv_heads=2)
    engine = Engine.from_random(cfg, seed=0)
    g = torch.Generator().manual_seed(5)
    rep = (torch.randint(0, cfg.vocab, (6,), generator=g).tolist() * 5)[:30]
    plain = [s[0] for s in engine.generate([rep], 24, draft_tokens=0)]
    default = [s[0] for s in engine.generate([rep], 24)]
    assert default == plain
    assert 2 <= engine.state._verify_n <= 6


def test_verify_rejects_bad_arguments(built_lib):
    from hackthenorth_b200 import _lib
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    engine = Engine.from_random(QWEN3_SMALL, seed=0)
    st = engine.new_state(8, 4, draft_tokens=8)
    ids = torch.zeros(9, dtype=torch.int64, device=engine.device)
    preds = torch.zeros(9, dtype=torch.int64, device=engine.device)
    L = _lib.load()
    assert L.qb_verify(engine.ctx, ids.data_ptr(), 9, st.position.data_ptr(), preds.data_ptr(), None,
                       _lib.stream_handle()) == _lib.QB_ERR_UNSUPPORTED
    assert L.qb_verify(engine.ctx, ids.data_ptr(), 0, st.position.data_ptr(), preds.data_ptr(), None,
                       _lib.stream_handle()) == _lib.QB_ERR_UNSUPPORTED
    assert L.qb_replay_verify(engine.ctx, _lib.stream_handle()) == _lib.QB_ERR_STATE
    # a verify past the capacity is reported on the device, not faulted
    st.position.fill_(st.capacity - 2)
    assert L.qb_verify(engine.ctx, ids.data_ptr(), 5, st.position.data_ptr(), preds.data_ptr(), None,
                       _lib.stream_handle()) == 0
    with pytest.raises(ValueError, match="capacity"):
        st.check()


@pytest.mark.parametrize("hkv,context", [(8, 9000), (2, 15000), (1, 30000), (2, 8188), (1, 8188)])
def test_verify_long_context_matches_oracle(built_lib, cpu_threads, hkv, context):
    """From a capacity of 8192 keys the verify attention runs several clusters
    per KV head, merged through global partial rows (8 KV heads: 4 clusters of
    4 CTAs on a B200; 2 heads: 7 of 8; 1 head: 7 of 16). Five rows over a seeded
    N(0, 1) cache prefix: every row's logits within LOGIT_ATOL of the oracle
    (mean below 0.01), predictions equal up to near ties, K/V rows appended.

    Context 8188 (rows at positions 8188..8192, 8193 live keys): 33 splits of
    256 keys, the last holding key 8192 alone; at these cluster shapes
    (16 CTAs x C >= 3, 8 CTAs x C >= 5) that split is the only one of the
    last working cluster, and every row but the last cannot see it. Those
    rows take the merge branch where a cluster has no visible key
    (log-sum-exp -inf, weight 0)."""
    from hackthenorth_b200.config import ModelConfig
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = ModelConfig(f"kv{hkv}", hidden=1024, n_heads=4 * hkv, n_kv_heads=hkv, head_dim=128, ffn=2048,
                      n_layers=1, vocab=4096, rope_theta=1e6)
    state = random_state_dict(cfg, 8)
    g = torch.Generator().manual_seed(14)
    kp = torch.randn(1, hkv, context, 128, generator=g).to(BF16)
    vp = torch.randn(1, hkv, context, 128, generator=g).to(BF16)
    current, drafts = 29, [3, 77, 1000, 5]
    o = OracleQwen3(cfg, state, context + 16)
    o.keys[:, :, :context] = kp
    o.values[:, :, :context] = vp
    ref, ref_tok = o.forward_rows([current, *drafts], context)
    ref = ref.float()
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    st = engine.new_state(context, 4, draft_tokens=8)
    assert st.capacity >= 8192
    st.keys[:, :, :context] = kp.to(engine.device)
    st.values[:, :, :context] = vp.to(engine.device)
    st.position.fill_(context)
    preds, logits = _verify_rows(engine, st, current, drafts)
    d = (logits - ref).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    for i in range(len(drafts) + 1):
        if preds[i] != int(ref_tok[i]):
            top2 = ref[i].topk(2).values
            assert float(top2[0] - top2[1]) <= LOGIT_ATOL, f"row {i}"
    n = len(drafts) + 1
    torch.testing.assert_close(st.keys[0, :, context:context + n].float().cpu(),
                               o.keys[0, :, context:context + n].float(), atol=0.0625, rtol=0.02)
