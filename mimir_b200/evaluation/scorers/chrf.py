"""Sentence-level chrF3++ (character 1..6-grams + word 1..2-grams, beta = 3), on a 0-1 scale.

Reference: ``src/mimir/evaluation/scorers/chrf.py:8-37`` (EuroEval's translation metric).
Implemented from the published definition (Popovic, "chrF++: words helping character
n-grams", WMT 2017): for each n-gram type and order, precision and recall of clipped n-gram
matches; precision and recall are averaged over the orders that occur in both hypothesis and
reference, and combined as ``F_beta = (1 + b^2) P R / (b^2 P + R)``.  Character n-grams
ignore whitespace; word n-grams split trailing/leading punctuation off tokens.  With several
references the best-scoring reference counts.
"""
from __future__ import annotations

import string
from collections import Counter

CHAR_ORDER, WORD_ORDER, BETA = 6, 2, 3.0
_PUNCT = set(string.punctuation)


def _words(text: str) -> list[str]:
    out = []
    for tok in text.split():
        if len(tok) > 1 and tok[-1] in _PUNCT:
            out += [tok[:-1], tok[-1]]
        elif len(tok) > 1 and tok[0] in _PUNCT:
            out += [tok[0], tok[1:]]
        else:
            out.append(tok)
    return out


def _ngrams(seq, n: int) -> Counter:
    return Counter(tuple(seq[i:i + n]) for i in range(len(seq) - n + 1))


def _stats(hyp: str, ref: str):
    hc, rc = "".join(hyp.split()), "".join(ref.split())
    hw, rw = _words(hyp), _words(ref)
    out = []
    for seq_h, seq_r, orders in ((hc, rc, CHAR_ORDER), (hw, rw, WORD_ORDER)):
        for n in range(1, orders + 1):
            h, r = _ngrams(seq_h, n), _ngrams(seq_r, n)
            out.append((sum(h.values()), sum(r.values()), sum((h & r).values())))
    return out


def _fscore(stats, beta: float = BETA) -> float:
    precisions, recalls = [], []
    for n_hyp, n_ref, n_match in stats:
        if n_hyp > 0 and n_ref > 0:
            precisions.append(n_match / n_hyp)
            recalls.append(n_match / n_ref)
    if not precisions:
        return 0.0
    p, r = sum(precisions) / len(precisions), sum(recalls) / len(recalls)
    b2 = beta * beta
    return (1 + b2) * p * r / (b2 * p + r) if p + r > 0 else 0.0


def compute_chrf3pp(prediction: str, references: list[str]) -> float:
    refs = [r for r in references if r]
    if not refs:
        return 0.0
    return max(_fscore(_stats(prediction, r)) for r in refs)


def chrf3pp():
    """Inspect AI scorer wrapper (requires ``inspect_ai``)."""
    from inspect_ai.scorer import Score, mean, scorer, stderr

    @scorer(metrics=[mean(), stderr()])
    def _chrf():
        async def score(state, target):
            pred = state.output.completion
            return Score(value=compute_chrf3pp(pred, [t for t in target.target if t]), answer=pred)
        return score
    return _chrf()
