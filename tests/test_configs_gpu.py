"""Parity of the engine with the CPU oracle at the BASELINE configs' own shapes.

Tolerances (north_star): per-step logits max |engine - oracle| <= 2e-2; greedy tokens
identical wherever the oracle's top-1 margin exceeds 2e-2, the first difference being
explained by a tie at that decision (``spec_stream_divergence`` for speculative streams).

Two weight recipes (the same ones every other parity test uses):
  * recipe A (the reference init, BASELINE's literal weights) with the bf16 KV cache the bench
    runs: the oracle prefills the 2048-token prompt itself, so this is the bench workload
    checked end to end. Recipe A copies its input token (top-1 margins ~5), so its token
    streams are a weak check; its per-step logits are not.
  * recipe B (non-trivial acceptance; its loop adapter is live) with the fp32-KV parity mode.
    Its prefill of more than 32 tokens drops expert rows chosen by router near-ties (capacity
    dropping), which any rounding flips, so these tests start the oracle from the engine's own
    prefilled cache (``oracle_kv_from_engine``) and check the decode path from that state:
    per-step logits on the oracle's greedy token path (teacher forcing), and the speculative
    token streams.
"""

from __future__ import annotations

import time

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

from conftest import logit_margin, oracle_kv_from_engine, spec_stream_divergence, use_path

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _engine(recipe, kv, **kw):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe=recipe, seed=0)
    eng = DeviceEngine(cfg, sd, device=0, kv_dtype=kv, **kw)
    use_path(eng, 0)
    return eng, O.OracleModel(sd, cfg), cfg


def _first_diff_is_tie(got, ref, margins, what):
    for i, (g, r) in enumerate(zip(got, ref)):
        if g != r:
            assert margins[i] <= TOL, f"{what}: token {i} differs ({g} vs {r}) with oracle margin {margins[i]:.3e}"
            return i
    return len(ref)


def _teacher_forced(eng, m, okv, slot, first_logits, T, n_steps):
    """Decode n_steps tokens on the oracle's greedy path: each step's three pulses on the
    engine (R = 1, the persistent kernel) and on the oracle from the same cache state; returns
    the largest per-pulse logits difference."""
    tok, pos = int(first_logits.argmax()), T
    worst = 0.0
    for step in range(n_steps):
        h = h0 = hr = h0r = None
        for p in range(3):
            lg, h, h0 = eng.pulse(p, [(slot, pos, tok)], h, h0)
            lr, hr, h0r = O.pulse_pass(m, p, [tok], [pos], okv, hr, h0r)
            err = (lg[0].cpu() - lr[0]).abs().max().item()
            worst = max(worst, err)
            assert err <= TOL, f"step {step} (position {pos}) pulse {p}: max |logit err| = {err:.3e}"
        eng.set_length(slot, pos + 1)
        okv.length = pos + 1
        tok, pos = int(lr[0].argmax()), pos + 1
    return worst


# ------------------------------------------------------------------ config 2 (the bench workload)
def test_config2_recipeA_bench_workload_matches_oracle():
    """BASELINE config 2 exactly: 2048-token prompt, 512 new tokens, greedy, bf16 KV. The
    engine's prefill logits, its gamma = 4 stream and its sequential stream against the
    oracle's prefill and non-speculative greedy decode (src/infer.py:551-621)."""
    T, N = 2048, 512
    eng, m, cfg = _engine("A", torch.bfloat16, max_batch=1, max_seq_len=T + N + 16, max_prefill=T)
    try:
        ids = random_prompts(1, T, cfg.vocab_size, seed=0)[0].tolist()
        t0 = time.time()
        trace = []
        ref = O.stream_generate_ids(m, ids, N, trace=trace)
        oracle_s = time.time() - t0
        margins = [logit_margin(lg) for _, lg in trace]   # trace[0]: the prefill logits
        first = eng.prefill(0, ids)
        d = (first.cpu() - trace[0][1]).abs().max().item()
        assert d <= TOL, f"prefill logits differ by {d:.3e}"
        for gamma in (4, 0):
            eng.set_length(0, T)
            got, stats = eng.generate_greedy([0], first.view(1, -1), N, gamma=gamma)
            k = _first_diff_is_tie(got[0].tolist(), ref, margins, f"config 2 gamma={gamma}")
            assert k == N, f"gamma={gamma}: stream ends at a tie at token {k}"
            if gamma:
                assert stats["accepted"] == stats["drafted"], "recipe A: every draft is accepted"
        print(f"config 2 recipe A: oracle prefill + 512 greedy steps {oracle_s:.1f} s")
    finally:
        eng.close()


def test_config2_recipeB_decode_logits_teacher_forced():
    """Config 2 shape under recipe B (fp32 KV): per-pulse logits of all 512 decode steps at
    positions 2048..2559 (every local layer's ring wraps, YaRN active on the global layers)
    against the oracle started from the engine's prefilled cache."""
    T, N = 2048, 512
    eng, m, cfg = _engine("B", torch.float32, max_batch=1, max_seq_len=T + N + 16, max_prefill=T)
    try:
        ids = random_prompts(1, T, cfg.vocab_size, seed=0)[0].tolist()
        first = eng.prefill(0, ids).cpu()
        okv = oracle_kv_from_engine(eng, m, 0, T, T + N + 8)
        worst = _teacher_forced(eng, m, okv, 0, first, T, N)
        print(f"config 2 recipe B: worst per-pulse logit difference over {N} steps {worst:.2e}")
    finally:
        eng.close()


def test_config2_recipeB_speculative_streams():
    """Config 2 shape under recipe B (fp32 KV), from the engine's prefilled cache: gamma = 4
    against the oracle's block-verify loop and gamma = 0 against its sequential greedy loop
    (128 tokens each); the first difference must be a tie at the deciding row, and identical
    streams must have identical accept decisions (acceptance equal to the oracle's)."""
    T, N, gamma = 2048, 128, 4
    eng, m, cfg = _engine("B", torch.float32, max_batch=1, max_seq_len=T + N + 16, max_prefill=T)
    try:
        ids = random_prompts(1, T, cfg.vocab_size, seed=0)[0].tolist()
        first = eng.prefill(0, ids)
        fl = first.cpu()
        trace, st = [], O.SpecStats()
        okv = oracle_kv_from_engine(eng, m, 0, T, T + N + gamma + 8)
        ref = O.block_spec_generate_ids(m, ids, N, gamma=gamma, stats=st, trace=trace, kv=okv, first_logits=fl)
        got, stats = eng.generate_greedy([0], first.view(1, -1), N, gamma=gamma)
        k, why = spec_stream_divergence(got[0].tolist(), ref, fl, trace, gamma, TOL)
        assert not why.startswith("FAIL"), why
        if k is None:
            assert (stats["rounds"], stats["drafted"], stats["accepted"]) == (st.rounds, st.drafted, st.accepted)
        print(f"config 2 recipe B gamma=4: {why}; oracle accept rate {st.accepted / max(1, st.drafted):.3f}, "
              f"engine {stats['accepted'] / max(1, stats['drafted']):.3f}")
        eng.set_length(0, T)
        okv = oracle_kv_from_engine(eng, m, 0, T, T + N + 8)
        tr = []
        ref0 = O.stream_generate_ids(m, ids, N, trace=tr, kv=okv, first_logits=fl)
        margins = [logit_margin(lg) for _, lg in tr]   # tr[0]: the first logits
        got0, _ = eng.generate_greedy([0], first.view(1, -1), N, gamma=0)
        _first_diff_is_tie(got0[0].tolist(), ref0, margins, "config 2 recipe B gamma=0")
    finally:
        eng.close()


# ------------------------------------------------------------------ config 4 (32k context)
def test_config4_long_context_recipeB_matches_oracle():
    """Config 4 shape, one of its sequences: a 32768-token prompt fills the window, so the local
    layers see a wrapped 1024-key window and the global layers all 32k keys with YaRN. Per-pulse
    logits of 16 teacher-forced steps and a 32-token gamma = 4 stream against the oracle from the
    engine's prefilled cache (recipe B, fp32 KV)."""
    T, N, gamma = 32768, 32, 4
    eng, m, cfg = _engine("B", torch.float32, max_batch=1, max_seq_len=T + N + 16, max_prefill=T)
    try:
        ids = random_prompts(4, T, cfg.vocab_size, seed=0)[0].tolist()
        first = eng.prefill(0, ids)
        fl = first.cpu()
        okv = oracle_kv_from_engine(eng, m, 0, T, T + N + gamma + 8)
        _teacher_forced(eng, m, okv, 0, fl, T, 16)
        eng.set_length(0, T)
        okv = oracle_kv_from_engine(eng, m, 0, T, T + N + gamma + 8)
        trace, st = [], O.SpecStats()
        ref = O.block_spec_generate_ids(m, ids, N, gamma=gamma, stats=st, trace=trace, kv=okv, first_logits=fl)
        got, stats = eng.generate_greedy([0], first.view(1, -1), N, gamma=gamma)
        k, why = spec_stream_divergence(got[0].tolist(), ref, fl, trace, gamma, TOL)
        assert not why.startswith("FAIL"), why
        if k is None:
            assert (stats["drafted"], stats["accepted"]) == (st.drafted, st.accepted)
    finally:
        eng.close()


# ------------------------------------------------------------------ config 5 (256 sequences)
def test_config5_batch256_recipeB_matches_oracle():
    """Config 5 shape: 256 sequences of 512-token prompts decoded together (greedy, gamma = 4,
    the many-row path: 1280-row verify passes), recipe B with fp32 KV. Sequences 0, 128 and 255
    against the oracle's block-verify loop from the engine's prefilled cache (64 new tokens)."""
    B, T, N, gamma = 256, 512, 64, 4
    check = (0, 128, 255)
    eng, m, cfg = _engine("B", torch.float32, max_batch=B, max_seq_len=T + N + 16, max_prefill=T)
    try:
        P = random_prompts(B, T, cfg.vocab_size, seed=0)
        first = torch.stack([eng.prefill(b, P[b].tolist()) for b in range(B)])
        okvs = {b: oracle_kv_from_engine(eng, m, b, T, T + N + gamma + 8) for b in check}
        got, stats = eng.generate_greedy(list(range(B)), first, N, gamma=gamma)
        assert stats["rounds"] > 0
        for b in check:
            fl = first[b].cpu()
            trace = []
            ref = O.block_spec_generate_ids(m, P[b].tolist(), N, gamma=gamma, trace=trace, kv=okvs[b], first_logits=fl)
            k, why = spec_stream_divergence(got[b].tolist(), ref, fl, trace, gamma, TOL)
            assert not why.startswith("FAIL"), f"sequence {b}: {why}"
    finally:
        eng.close()
