"""Draft sources and the acceptance rule (host logic; dryft/tests/test_speculate.py)."""
import random

import pytest

from hackthenorth_b200.speculate import (BackoffPromptLookup, PromptLookup, SyntheticDraft, draft_width,
                                         verified_tokens)


def test_lookup_only_proposes_previously_seen_continuations():
    lookup = PromptLookup([1, 2, 3, 4, 5, 6, 7, 8, 1, 2, 3, 4], draft_length=3)
    assert lookup.propose() == [5, 6, 7]
    lookup.append(99)
    assert lookup.propose() is None


def test_lookup_learns_verified_output_without_self_matching():
    lookup = PromptLookup([1, 2], draft_length=3)
    assert lookup.propose() is None
    for t in [3, 4, 5, 6, 7, 1, 2, 3, 4]:
        lookup.append(t)
    assert lookup.propose() == [5, 6, 7]


def test_acceptance_emits_only_correct_prefix_and_one_target_token():
    proposal = [10, 11, 12]
    for accepted in range(4):
        predictions = proposal[:accepted] + [99] + [88] * (3 - accepted)
        assert verified_tokens(proposal, predictions) == proposal[:accepted] + [99]


def test_verification_requires_bonus_prediction():
    with pytest.raises(ValueError):
        verified_tokens([1, 2, 3], [1, 2, 3])


def test_backoff_prefers_longer_match_over_more_recent_short_match():
    history = [1, 2, 3, 4, 10, 11, 12, 9, 3, 4, 20, 21, 22, 1, 2, 3, 4]
    assert BackoffPromptLookup(history, draft_length=3).propose() == [10, 11, 12]


def test_backoff_uses_short_match_and_resets_for_new_prompt():
    first = BackoffPromptLookup([8, 9, 10, 11, 12, 1, 8, 9], draft_length=3)
    assert first.propose() == [10, 11, 12]
    assert BackoffPromptLookup([1, 8, 9]).propose() is None


@pytest.mark.parametrize("width", [3, 7])
def test_backoff_matches_naive_history_search_after_every_append(width):
    rng = random.Random(1701)
    history = [rng.randrange(5) for _ in range(24)]
    lookup = BackoffPromptLookup(history, draft_length=width)
    for _ in range(200):
        expected = None
        for ngram in (4, 3, 2):
            if len(history) < ngram:
                continue
            matches = [i for i in range(len(history) - ngram - width + 1)
                       if history[i:i + ngram] == history[-ngram:]]
            if matches:
                start = matches[-1] + ngram
                expected = history[start:start + width]
                break
        assert lookup.propose() == expected
        tok = rng.randrange(5)
        history.append(tok)
        lookup.append(tok)


def test_default_width_keeps_the_verify_pass_on_the_rows_attention_kernel():
    from hackthenorth_b200.speculate import fast_verify_drafts

    assert fast_verify_drafts(32, 8) == 5     # Qwen3-4B / 8B: 6 rows x 4 heads = 24 rows per KV head
    assert fast_verify_drafts(16, 8) == 11    # Qwen3-0.6B: the reference's 7 fit
    assert fast_verify_drafts(64, 8) == 2
    assert fast_verify_drafts(32, 1) == 0     # a group of 32 leaves no room for drafts
    assert min(draft_width(100), fast_verify_drafts(16, 8)) == 7
    assert min(draft_width(100), fast_verify_drafts(32, 8)) == 5


def test_draft_width_caps_short_requests():
    assert [draft_width(n) for n in (1, 2, 3, 9, 100)] == [0, 0, 1, 7, 7]
    assert draft_width(100, 4) == 4


def test_synthetic_draft_is_seeded_and_hits_at_rate_p():
    ref = list(range(1000, 3000))
    a = SyntheticDraft(ref, vocab=151936, p=0.7, seed=3)
    b = SyntheticDraft(ref, vocab=151936, p=0.7, seed=3)
    pa = [a.propose(i * 4, 4) for i in range(400)]
    pb = [b.propose(i * 4, 4) for i in range(400)]
    assert pa == pb
    hits = sum(tok == ref[i * 4 + j] for i, p in enumerate(pa) for j, tok in enumerate(p))
    assert 0.65 < hits / 1600 < 0.75
