"""Draft sources and the exact acceptance rule for speculative decoding (host side).

Behaviour follows ``dryft/engine/speculate.py``: ``PromptLookup`` proposes the
continuation of the most recent earlier occurrence of the last n-gram
(``:11-33``), ``BackoffPromptLookup`` prefers 4-, then 3-, then 2-grams
(``:36-52``), ``verified_tokens`` accepts the longest matching prefix of the
proposal and emits one target token after it (``:55-69``), and
``draft_width`` caps the verifier width for short requests (``:6-8``).
``SyntheticDraft`` is the benchmark's draft source: the target's own greedy
token with a seeded probability, otherwise a uniform random id.
"""
from __future__ import annotations

import random
from typing import List, Optional, Sequence

DRAFT_TOKENS = 7


def draft_width(output_length: int, draft_tokens: int = DRAFT_TOKENS) -> int:
    return max(0, min(draft_tokens, output_length - 2))


# Query rows per KV head (GQA group x verify rows) that the verify pass's
# attention keeps on the cluster rows kernel; wider passes run the split kernel
# with the global merge, which at 4 query heads per KV head makes an 8-row
# verify cost 6.03 ms against 3.80 ms for 5 rows (Qwen3-8B shape, 4096 keys).
VERIFY_FAST_ROWS = 24


def fast_verify_drafts(n_heads: int, n_kv_heads: int) -> int:
    """Most draft tokens whose verify pass (drafts + 1 rows) stays on the rows
    attention kernel: 5 with 4 query heads per KV head, 11 with 2."""
    group = max(1, n_heads // max(1, n_kv_heads))
    return max(0, VERIFY_FAST_ROWS // group - 1)


class PromptLookup:
    """n-gram lookup over the request's own history (prompt + emitted tokens)."""

    def __init__(self, prompt: Sequence[int], draft_length: int = DRAFT_TOKENS, ngram: int = 4):
        self.tokens = list(prompt)
        self.draft_length = draft_length
        self.ngram = ngram
        self._indexed = 0          # next start index to add to the table
        self._table = {}           # n-gram -> index just past its latest occurrence

    def append(self, token: int) -> None:
        self.tokens.append(token)

    def propose(self) -> Optional[List[int]]:
        # Only occurrences whose continuation holds a full draft are eligible,
        # and the newest such occurrence wins.
        limit = len(self.tokens) - self.ngram - self.draft_length + 1
        while self._indexed < limit:
            i = self._indexed
            self._table[tuple(self.tokens[i:i + self.ngram])] = i + self.ngram
            self._indexed += 1
        if len(self.tokens) < self.ngram:
            return None
        start = self._table.get(tuple(self.tokens[-self.ngram:]))
        if start is None:
            return None
        return self.tokens[start:start + self.draft_length]


class BackoffPromptLookup:
    def __init__(self, prompt: Sequence[int], draft_length: int = DRAFT_TOKENS):
        self.matchers = [PromptLookup(prompt, draft_length, n) for n in (4, 3, 2)]

    def append(self, token: int) -> None:
        for m in self.matchers:
            m.append(token)

    def propose(self) -> Optional[List[int]]:
        for m in self.matchers:
            p = m.propose()
            if p is not None:
                return p
        return None


def verified_tokens(proposal: Sequence[int], predictions: Sequence[int]) -> List[int]:
    """predictions[i] is the target's greedy token after current + proposal[:i].
    Accept the matching prefix, then emit the target's token after it."""
    if len(predictions) != len(proposal) + 1:
        raise ValueError(f"{len(predictions)} predictions for {len(proposal)} draft tokens: "
                         "each draft token and the bonus position need one")
    accepted = 0
    for d, t in zip(proposal, predictions):
        if d != t:
            break
        accepted += 1
    return list(predictions[:accepted + 1])


class SyntheticDraft:
    """Draft token i = the target's greedy continuation with probability p
    (seeded Bernoulli), otherwise a uniform id in [0, vocab)."""

    def __init__(self, reference_tokens: Sequence[int], vocab: int, p: float = 0.7, seed: int = 3,
                 draft_length: int = DRAFT_TOKENS):
        self.reference = list(reference_tokens)
        self.vocab = vocab
        self.p = p
        self.rng = random.Random(seed)
        self.draft_length = draft_length
        self.emitted = 0

    def append(self, token: int) -> None:
        """Drafter interface: one more emitted token."""
        self.emitted += 1

    def propose(self, emitted: Optional[int] = None, k: Optional[int] = None) -> List[int]:
        """k draft tokens continuing after ``emitted`` already-emitted tokens.
        Without arguments (the drafter interface of ``Engine.generate``): after
        the tokens passed to ``append`` so far, ``draft_length`` tokens."""
        if emitted is None:
            emitted = self.emitted
        if k is None:
            k = self.draft_length
        out = []
        for j in range(k):
            idx = emitted + j
            if idx < len(self.reference) and self.rng.random() < self.p:
                out.append(self.reference[idx])
            else:
                out.append(self.rng.randrange(self.vocab))
        return out
