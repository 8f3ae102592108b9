"""End-to-end decode through the Engine / C-ABI vs the reference's eager path
(golden vectors) and the CPU oracle. Tolerances as in test_oracle.py."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
LOGIT_ATOL = 0.0625


def _bits_to_bf16(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


@pytest.fixture(scope="module")
def small_engine(built_lib):
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine

    return Engine.from_random(QWEN3_SMALL, seed=0)


def _teacher_forced(engine, prompt, tokens, keep_logits=True):
    """Prefill, then force each golden token and collect the step logits."""
    state = engine.new_state(len(prompt), len(tokens), keep_logits=keep_logits)
    state.prefill(torch.tensor(prompt, dtype=torch.int64, device=engine.device))
    rows = [state.logits.float().cpu().clone()]
    for t in tokens[:-1]:
        state.token.fill_(t)
        state.step()
        rows.append(state.logits.float().cpu().clone())
    state.check()
    return torch.stack(rows)


def test_small_engine_matches_golden_tokens_and_logits(small_engine):
    g = np.load(os.path.join(GOLDEN, "qwen3_small_greedy.npz"))
    prompt, gold = g["prompt"].tolist(), g["tokens"].tolist()
    out = [s[0] for s in small_engine.generate([prompt], len(gold))]
    assert out == gold
    got = _teacher_forced(small_engine, prompt, gold)
    ref = _bits_to_bf16(g["logits_bf16"]).float()
    assert (got - ref).abs().max() <= LOGIT_ATOL
    assert torch.nn.functional.cosine_similarity(got, ref, dim=1).min() >= 0.999


def test_generate_contract_and_repeated_prompts(small_engine):
    # exactly N yields of one id; fresh prompt state on every call
    # (dryft/tests/test_decode.py:170-183, dryft/tests/test_prefill.py:27-60)
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    assert list(small_engine.generate([[5, 6, 7]], 0)) == []
    oracle_state = random_state_dict(QWEN3_SMALL, 0)
    rng = torch.Generator().manual_seed(5)
    for n_new in (1, 2, 9):
        for _ in range(2):
            prompt = torch.randint(0, QWEN3_SMALL.vocab, (12,), generator=rng).tolist()
            out = list(small_engine.generate([prompt], n_new))
            assert len(out) == n_new and all(len(s) == 1 for s in out)
            o = OracleQwen3(QWEN3_SMALL, oracle_state, 12 + n_new)
            assert [s[0] for s in out] == o.greedy(prompt, n_new)
    # equal-length prompts decode as one batch, more than 8 in chunks of 8
    # (test_batch_gpu.py); unequal prompt lengths are a contract violation
    with pytest.raises(ValueError):
        list(small_engine.generate([[1, 2], [3]], 2))
    nine = list(small_engine.generate([[1, 2]] * 9, 3))
    assert len(nine) == 3 and all(len(s) == 9 and len(set(s)) == 1 for s in nine)


def test_stale_cache_slots_are_never_read(small_engine):
    # dryft/tests/test_decode.py:92-115: poison unused storage with +-1000 and NaN
    g = np.load(os.path.join(GOLDEN, "qwen3_small_greedy.npz"))
    prompt, gold = g["prompt"].tolist(), g["tokens"].tolist()
    for poison in (1000.0, -1000.0, float("nan")):
        state = small_engine.new_state(len(prompt), len(gold))
        state.keys.fill_(poison)
        state.values.fill_(poison)
        state.prefill(torch.tensor(prompt, device=small_engine.device))
        toks = state.read_token()
        for _ in range(len(gold) - 1):
            state.step()
            toks += state.read_token()
        state.check()
        assert toks == gold


def test_bad_token_is_reported_not_faulted(small_engine):
    state = small_engine.new_state(4, 4)
    state.prefill(torch.tensor([1, 2, 3, 4], device=small_engine.device))
    state.check()
    state.token.fill_(10 ** 9)
    state.step_eager()
    with pytest.raises(ValueError, match="vocabulary"):
        state.check()


GOLDEN_0P6B = ["qwen3_0p6b_greedy.json", "qwen3_0p6b_greedy_notie.json"]


@pytest.mark.slow
@pytest.mark.parametrize("golden", GOLDEN_0P6B)
def test_0p6b_engine_matches_native_greedy_128(built_lib, cpu_threads, golden):
    """0.6B shape, 32-token prompt, 128 greedy steps, against native
    Transformers (the reference's ground truth).

    1. Teacher-forced on the native tokens: the top-64 logits of every step
       within LOGIT_ATOL and the native token within LOGIT_ATOL of our max;
       the full logit rows against native teacher-forced rows: max abs within
       LOGIT_ATOL, cosine >= 0.999 (both printed).
    2. Free-running plain decode: identical tokens up to the first step where
       the native logits themselves hold an exact top-1/top-2 tie (seed-1
       prompt: step 14, 2.828125 for ids 5664 and 64516; past a genuine tie
       any other summation order may pick the other id). The second prompt
       (``*_notie.json``) has no step with a top-2 margin below 0.0625, so all
       128 tokens must be identical.
    3. All 128 free-running tokens of plain decode and of the default
       generate (speculative with prompt lookup, as the reference's) pass the
       reference judge's rule (dryft/QWEN_ENGINE_CONTRACT.md:105-121) with a
       margin of LOGIT_ATOL instead of 2.0: replayed teacher-forced through
       native Transformers on our own prefix, each token is the argmax or
       within LOGIT_ATOL of it.
    """
    from hackthenorth_b200.config import QWEN3_0P6B
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle import hf_eager

    with open(os.path.join(GOLDEN, golden)) as f:
        g = json.load(f)
    state = random_state_dict(QWEN3_0P6B, 0)
    engine = Engine(None, "cuda:0", cfg=QWEN3_0P6B, state=state)
    got = _teacher_forced(engine, g["prompt"], g["tokens"])
    worst = 0.0
    for i, (row, s) in enumerate(zip(got, g["steps"])):
        ids = torch.tensor(s["top_ids"])
        worst = max(worst, float((row[ids] - torch.tensor(s["top_vals"])).abs().max()))
        assert row.max() - row[g["tokens"][i]] <= LOGIT_ATOL
    assert worst <= LOGIT_ATOL

    model = hf_eager.build_hf_model(QWEN3_0P6B, state)
    native_tf = hf_eager.teacher_forced_logits(model, g["prompt"] + g["tokens"][:-1], len(g["prompt"]) - 1).float()
    step_abs = (got - native_tf).abs().max(-1).values
    step_cos = torch.nn.functional.cosine_similarity(got, native_tf, dim=1)
    print(f"\n[{golden}] per-step logits vs native teacher-forced: max abs {float(step_abs.max()):.4f} "
          f"(median {float(step_abs.median()):.4f}, steps above 0.02: {int((step_abs > 0.02).sum())}/128), "
          f"min cosine {float(step_cos.min()):.6f}; native self-noise (cached vs full prefix) "
          f"{max(g['self_noise_cached_vs_full_prefix']):.4f}")
    assert float(step_abs.max()) <= LOGIT_ATOL and float(step_cos.min()) >= 0.999

    free = [s[0] for s in engine.generate([g["prompt"]], 128, draft_tokens=0)]
    first_tie = next((i for i, s in enumerate(g["steps"]) if s["margin"] == 0.0), 128)
    if golden.endswith("_notie.json"):
        assert first_tie == 128 and min(s["margin"] for s in g["steps"]) >= LOGIT_ATOL
    assert free[:first_tie] == g["tokens"][:first_tie]
    default = [s[0] for s in engine.generate([g["prompt"]], 128)]
    if first_tie == 128:
        assert default == g["tokens"]

    for stream in (free, default):
        native = hf_eager.teacher_forced_logits(model, g["prompt"] + stream[:-1], len(g["prompt"]) - 1).float()
        deficits = native.max(-1).values - native[torch.arange(128), torch.tensor(stream)]
        assert float(deficits.max()) <= LOGIT_ATOL, f"worst deficit {float(deficits.max())} at {int(deficits.argmax())}"


@pytest.mark.parametrize("context,capacity", [(200, None), (4096, None), (9000, None), (3000, 16384)])
def test_decode_step_matches_oracle(built_lib, cpu_threads, context, capacity):
    """One Qwen3-8B-shaped layer (full vocabulary) over a seeded N(0, 1) cache
    prefix: the decode step's logits match the CPU oracle's within LOGIT_ATOL
    (mean difference below 0.01); the greedy token matches the oracle's unless
    the oracle holds a near tie; the appended K/V rows match within bf16
    rounding of the projection.
    Context 200 runs one attention split per KV head, 4096 several (merged
    through distributed shared memory). A capacity above 8192 gives several
    clusters per KV head (four clusters of four CTAs on a B200), merged across
    clusters by the last-arriving CTA of each dim slice: context 9000 uses all
    of them, context 3000 two (8 splits)."""
    import dataclasses

    from hackthenorth_b200.config import QWEN3_8B
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = dataclasses.replace(QWEN3_8B, n_layers=1)
    state = random_state_dict(cfg, 3)
    g = torch.Generator().manual_seed(11)
    kp = torch.randn(1, cfg.n_kv_heads, context, cfg.head_dim, generator=g).to(BF16)
    vp = torch.randn(1, cfg.n_kv_heads, context, cfg.head_dim, generator=g).to(BF16)
    o = OracleQwen3(cfg, state, context + 4)
    o.keys[:, :, :context] = kp
    o.values[:, :, :context] = vp
    ref, ref_tok = o.forward_rows([17], context)
    ref = ref[0].float()
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    st = engine.new_state(context, 4, keep_logits=True, capacity=capacity)
    st.keys[:, :, :context] = kp.to(engine.device)
    st.values[:, :, :context] = vp.to(engine.device)
    st.token.fill_(17)
    st.position.fill_(context)
    st.step()
    st.check()
    got = st.logits.float().cpu()
    assert int(st.position.item()) == context + 1
    torch.testing.assert_close(st.keys[0, :, context].float().cpu(), o.keys[0, :, context].float(),
                               atol=0.0625, rtol=0.02)
    torch.testing.assert_close(st.values[0, :, context].float().cpu(), o.values[0, :, context].float(),
                               atol=0.0625, rtol=0.02)
    top2 = ref.topk(2).values
    if int(st.token.item()) != int(ref_tok[0]):
        assert float(top2[0] - top2[1]) <= LOGIT_ATOL
    d = (got - ref).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    del st, engine
    torch.cuda.empty_cache()


def test_4b_shape_prefill_and_decode_match_oracle(built_lib, cpu_threads):
    """The Qwen3-4B shape (hidden 2560, 32/8 heads, FFN 9728, full 151936
    vocabulary, rope theta 5e6) at 2 layers: a 40-token prompt through the
    dense-block prefill (tensor-core GEMMs, flash attention), then 12 decode
    steps teacher-forced on the oracle's greedy tokens. Every step's logits
    within LOGIT_ATOL of the CPU oracle (mean below 0.01), cosine >= 0.999;
    free-running tokens equal the oracle's up to a near tie."""
    import dataclasses

    from hackthenorth_b200.config import QWEN3_4B
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = dataclasses.replace(QWEN3_4B, n_layers=2)
    state = random_state_dict(cfg, 0)
    P, n_new = 40, 12
    prompt = torch.randint(0, cfg.vocab, (P,), generator=torch.Generator().manual_seed(1)).tolist()
    o = OracleQwen3(cfg, state, P + n_new)
    ref_logits = []
    ref_tokens = o.greedy(prompt, n_new, ref_logits)
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    got = _teacher_forced(engine, prompt, ref_tokens)
    ref = torch.stack([r.float() for r in ref_logits])
    d = (got - ref).abs()
    assert float(d.max()) <= LOGIT_ATOL and float(d.mean()) <= 0.01, (float(d.max()), float(d.mean()))
    assert float(torch.nn.functional.cosine_similarity(got, ref, dim=1).min()) >= 0.999
    free = [s[0] for s in engine.generate([prompt], n_new, draft_tokens=0)]
    for i, (a, b) in enumerate(zip(free, ref_tokens)):
        if a != b:
            top2 = ref[i].topk(2).values
            assert float(top2[0] - top2[1]) <= LOGIT_ATOL, f"step {i}"
            break


def test_8b_layer_decode_at_32k_matches_oracle(built_lib, cpu_threads):
    """One Qwen3-8B-shaped layer (full vocabulary) at context 32768 over a
    seeded N(0, 1) cache prefix (the configuration's long-context line): the
    decode step's logits within LOGIT_ATOL of the oracle (mean below 0.01),
    the greedy token equal unless the oracle holds a near tie, K/V appended."""
    import dataclasses

    from hackthenorth_b200.config import QWEN3_8B
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    context = 32768
    cfg = dataclasses.replace(QWEN3_8B, n_layers=1)
    state = random_state_dict(cfg, 3)
    g = torch.Generator().manual_seed(12)
    kp = torch.randn(1, cfg.n_kv_heads, context, cfg.head_dim, generator=g).to(BF16)
    vp = torch.randn(1, cfg.n_kv_heads, context, cfg.head_dim, generator=g).to(BF16)
    o = OracleQwen3(cfg, state, context + 4)
    o.keys[:, :, :context] = kp
    o.values[:, :, :context] = vp
    ref, ref_tok = o.forward_rows([17], context)
    ref = ref[0].float()
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    st = engine.new_state(context, 4, keep_logits=True)
    st.keys[:, :, :context] = kp.to(engine.device)
    st.values[:, :, :context] = vp.to(engine.device)
    st.token.fill_(17)
    st.position.fill_(context)
    st.step()
    st.check()
    got = st.logits.float().cpu()
    d = (got - ref).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    if st.read_token()[0] != int(ref_tok[0]):
        top2 = ref.topk(2).values
        assert float(top2[0] - top2[1]) <= LOGIT_ATOL
    torch.testing.assert_close(st.keys[0, :, context].float().cpu(), o.keys[0, :, context].float(), atol=0.0625,
                               rtol=0.02)
    assert torch.equal(st.values[0, :, context].cpu(), o.values[0, :, context])


@pytest.mark.parametrize("hkv,context", [(4, 8200), (2, 15000), (1, 30000)])
def test_long_context_few_kv_heads_matches_oracle(built_lib, cpu_threads, hkv, context):
    """Few KV heads at long contexts run the decode attention as many clusters
    per head (4 heads: 8 clusters of 4 CTAs; 2 heads: 7 of 8; 1 head: 7 of 16 on
    a B200). At these lengths rounding the split length up used to leave the
    last splits without keys; every split must get keys and the merged
    attention must match the oracle: one decode step over a seeded N(0, 1)
    cache prefix, logits within LOGIT_ATOL, appended K/V within bf16 rounding."""
    from hackthenorth_b200.config import ModelConfig
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.weights import random_state_dict
    from oracle.qwen3_oracle import OracleQwen3

    cfg = ModelConfig(f"kv{hkv}", hidden=1024, n_heads=4 * hkv, n_kv_heads=hkv, head_dim=128, ffn=2048,
                      n_layers=1, vocab=4096, rope_theta=1e6)
    state = random_state_dict(cfg, 8)
    g = torch.Generator().manual_seed(13)
    kp = torch.randn(1, hkv, context, 128, generator=g).to(BF16)
    vp = torch.randn(1, hkv, context, 128, generator=g).to(BF16)
    o = OracleQwen3(cfg, state, context + 4)
    o.keys[:, :, :context] = kp
    o.values[:, :, :context] = vp
    ref, ref_tok = o.forward_rows([29], context)
    ref = ref[0].float()
    engine = Engine(None, "cuda:0", cfg=cfg, state=state)
    st = engine.new_state(context, 4, keep_logits=True)
    st.keys[:, :, :context] = kp.to(engine.device)
    st.values[:, :, :context] = vp.to(engine.device)
    st.token.fill_(29)
    st.position.fill_(context)
    st.step()
    st.check()
    got = st.logits.float().cpu()
    d = (got - ref).abs()
    assert d.max() <= LOGIT_ATOL and d.mean() <= 0.01, (float(d.max()), float(d.mean()))
    if st.read_token()[0] != int(ref_tok[0]):
        top2 = ref.topk(2).values
        assert float(top2[0] - top2[1]) <= LOGIT_ATOL
    torch.testing.assert_close(st.keys[0, :, context].float().cpu(), o.keys[0, :, context].float(), atol=0.0625,
                               rtol=0.02)
