"""CPU checks of the oracle's sampling rules (src/infer.py:591-609), the rules the device's
sampled decoding is compared against.

Top-p with exactly tied weights at the cutoff: the reference sorts the warped logits and drops
by sort position (exclusive cumulative mass > top_p, the first token always kept), so of two
tokens tied exactly at the cutoff it may keep one. The device keeps every token whose weight is
tied with the cutoff token's (a value threshold, no sort); the difference only exists at exact
ties, which the sampled parity tests treat as tie decisions. This pins the oracle side.
"""

from __future__ import annotations

import torch

from oracle import pulsar_oracle as O


def test_top_p_keeps_the_first_token_and_drops_by_exclusive_mass():
    lg = torch.tensor([3.0, 2.0, 1.0, 0.0])
    p = O.warped_probs(lg, 1.0, 0.5)   # softmax masses ~0.64, 0.24, 0.09, 0.03
    assert p is not None
    assert p[0] > 0 and (p[1:] == 0).all(), "first token alone covers top_p"
    p = O.warped_probs(lg, 1.0, 0.7)
    assert (p[:2] > 0).all() and (p[2:] == 0).all(), "exclusive mass 0.64 <= 0.7 keeps the second token"


def test_top_p_exact_tie_at_the_cutoff_keeps_by_sort_position():
    # tokens 1 and 2 tie exactly; the cutoff falls between them: the reference keeps at most
    # one of the tied pair (which one depends on torch.sort's order of equal keys)
    lg = torch.tensor([2.0, 1.0, 1.0, -10.0])
    w = torch.softmax(lg, 0)
    top_p = float(w[0] + 0.5 * w[1])
    p = O.warped_probs(lg, 1.0, top_p)
    kept = int((p[1:3] > 0).sum())
    assert p[0] > 0 and kept == 1, "one of the two tied tokens is dropped by position"

