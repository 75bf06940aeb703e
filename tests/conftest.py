"""Shared fixtures for the pulsar_b200 test-suite.

Markers: ``gpu`` (needs a CUDA device; run on the B200 box) and ``slow``. The CPU suite
(``-m "not gpu"``) checks the oracle against the reference's golden vectors, the host
logic and the C-ABI library's symbol table.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "pulsar-300m_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")
HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def load_golden(name: str):
    path = os.path.join(GOLDEN, f"{name}.pt")
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name}.pt not generated")
    return torch.load(path, weights_only=False)


def early_exit_model(g):
    """(state_dict, config) of an early_exit_* golden case: the synthetic weights with the
    case's sharpening (tests/golden/make_golden.py:sharpen)."""
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.weights import make_state_dict
    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    from make_golden import sharpen
    cfg = PulsarConfig(**g["cfg"])
    sd = make_state_dict(cfg, recipe=g["recipe"], seed=g["seed"], b_std=g["b_std"])
    return sharpen(sd, g["final_scale"], g["res0_scale"], g.get("zero_lora", False)), cfg


def assert_close(actual, expected, *, atol=2e-2, rtol=2e-2, msg=""):
    """Fails only when BOTH max-abs > atol and max-rel > rtol (the reference's rule,
    tests/conftest.py:118-144 of the reference)."""
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    if a.shape != e.shape:
        raise AssertionError(f"{msg}: shape mismatch {tuple(a.shape)} vs {tuple(e.shape)}")
    max_abs = (a - e).abs().max().item() if a.numel() else 0.0
    max_rel = ((a - e).abs() / e.abs().clamp_min(1e-6)).max().item() if a.numel() else 0.0
    if not (math.isfinite(max_abs) and math.isfinite(max_rel)):
        raise AssertionError(f"{msg}: non-finite values (max_abs={max_abs}, max_rel={max_rel})")
    if max_abs > atol and max_rel > rtol:
        raise AssertionError(f"{msg}: max_abs={max_abs:.3e} (atol {atol:.1e}), max_rel={max_rel:.3e} (rtol {rtol:.1e})")


@pytest.fixture
def gpu():
    if not HAS_CUDA:
        pytest.skip("CUDA not available")
    return torch.device("cuda")


# ---- sampled decoding: tie tolerances of accept decisions and inverse-CDF draws -------------
SAMPLED_ACCEPT_TIE = 1e-3   # |u1 - ratio| below this: the decision may flip (tolerance of record)
SAMPLED_DRAW_TIE = 1e-4     # draw target this close (relative) to a bucket edge may change bucket


def sampled_draw_margin(probs, u):
    """Distance of the draw target u * total from the nearest bucket edge of the chosen index,
    relative to the total (the oracle's sample_from inverse CDF)."""
    p = probs.double().numpy()
    c = np.cumsum(p)
    t = u * c[-1]
    i = min(int(np.searchsorted(c, t, side="right")), len(p) - 1)
    lo = c[i - 1] if i > 0 else 0.0
    return min(abs(t - lo), abs(c[i] - t)) / c[-1]


def sampled_safe_prefix(prefill_logits, trace, stats, gamma, T, top_p, seed, seq_id):
    """Number of leading tokens of an oracle block_spec_generate_ids run (its trace and
    stats) whose every deciding draw and accept test lies outside the tie tolerances."""
    from oracle import pulsar_oracle as O
    p0 = O.warped_probs(prefill_logits, T, top_p)
    if sampled_draw_margin(p0, O.uniforms(seed, seq_id, 0xFFFFFFFF, 0)[0]) < SAMPLED_DRAW_TIE:
        return 0
    n = 1
    log = {}
    for (rnd, j, ok, u, ratio) in stats.accept_log:
        log.setdefault(rnd, []).append((j, ok, u, ratio))
    for (rnd, toks, q_logits, P) in trace:
        for j in range(gamma):
            qp = O.warped_probs(q_logits[j], T, top_p)
            if sampled_draw_margin(qp, O.uniforms(seed, seq_id, rnd, j)[0]) < SAMPLED_DRAW_TIE:
                return n
        a, rejected = 0, None
        for (j, ok, u, ratio) in log.get(rnd, []):
            if abs(u - ratio) < SAMPLED_ACCEPT_TIE:
                return n
            if ok:
                a += 1
            else:
                rejected = j
                break
        if rejected is None:
            p = O.warped_probs(P[gamma], T, top_p)
            if sampled_draw_margin(p, O.uniforms(seed, seq_id, rnd, gamma)[2]) < SAMPLED_DRAW_TIE:
                return n
        else:
            p = O.warped_probs(P[rejected - 1], T, top_p)
            q = O.warped_probs(q_logits[rejected - 1], T, top_p)
            resid = (p - q).clamp_min(0.0)
            u2 = O.uniforms(seed, seq_id, rnd, rejected - 1)[2]
            if float(resid.sum()) > 0 and sampled_draw_margin(resid / resid.sum(), u2) < SAMPLED_DRAW_TIE:
                return n
        n += a + 1
    return n


PATH_IDS = ["megakernel", "per-op", "wide"]


def use_path(eng, path):
    """Select the pulse implementation: 0 persistent kernel (rows <= 5, else the per-op
    kernels), 1 per-op GEMV kernels, 2 the many-row GEMM path."""
    eng.set_option("wide", 1 if path == 2 else 0)
    eng.set_option("megakernel", 1 if path == 0 else 0)


# ---- oracle state taken from the device (long prompts) --------------------------------------
def oracle_kv_from_engine(eng, m, slot, T, capacity):
    """An OracleKV holding the engine's cached K/V of prompt positions [0, T) of ``slot``
    (read through pulsar_engine_read_kv), with length T: the window of the local layers (their
    last 1024 positions, all a later query can see) and every position of the global layers.
    Decoding then starts from the same state on both sides; used for prompts whose recipe-B
    prefill is chaotic (capacity dropping decided by router near-ties)."""
    from oracle import pulsar_oracle as O
    kv = O.OracleKV(m, capacity)
    for layer in range(m.L):
        lo = max(0, T - m.window) if layer in O.LOCAL_LAYERS else 0
        k, v = eng.read_kv(slot, layer, lo, T - lo)
        kv.k[layer][:, lo:T] = k
        kv.v[layer][:, lo:T] = v
    kv.length = T
    return kv


def logit_margin(lg):
    v = lg.float().reshape(-1).topk(2).values
    return float(v[0] - v[1])


def spec_stream_divergence(got, ref, first_logits, trace, gamma, tol):
    """Where a device greedy speculative stream first differs from the oracle's
    block_spec_generate_ids stream (``trace`` from that run), and whether the difference is a
    tie within ``tol``. Returns (index or None, reason).

    Every emitted token is the argmax of one verify row (or of the first logits): round r emits
    argmax(P_r[0..a]) where a counts the accepted drafts. A first difference at a token is
    explained when that row's top-1 margin is <= tol. Draft decisions (argmax of the pulse-1
    exit rows q) do not change the emitted tokens of their round, but a different draft changes
    where the device's next block starts, and so the in-block K/V every later verify row sees;
    a draft near-tie in that round or an earlier one therefore also explains a later
    difference. Any other first difference is a parity failure (the reason starts with
    'FAIL')."""
    k = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), None)
    if k is None:
        return None, "identical"
    rows = [(-1, logit_margin(first_logits))]   # (round, margin) per emitted token
    for (rnd, toks, q, P) in trace:
        a = 0
        while a < gamma and int(P[a].argmax()) == toks[a + 1]:
            a += 1
        rows.extend((rnd, logit_margin(P[j])) for j in range(a + 1))
    rnd, mg = rows[k] if k < len(rows) else (trace[-1][0], 0.0)
    if mg <= tol:
        return k, f"token {k}: verify-row tie (margin {mg:.2e})"
    draft = [(r, min(logit_margin(q[j]) for j in range(q.shape[0]))) for (r, _, q, _) in trace if r <= rnd]
    lo = min(draft, key=lambda x: x[1]) if draft else (None, float("inf"))
    if lo[1] <= tol:
        return k, f"token {k}: draft tie in round {lo[0]} (margin {lo[1]:.2e}) changed the block boundaries"
    return k, f"FAIL token {k} (round {rnd}): {got[k]} vs oracle {ref[k]}, margin {mg:.2e}, no tie"
