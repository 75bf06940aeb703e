"""Repetition penalty on the device (pulsar_engine_set_repetition_penalty; src/infer.py:582-589
applied in the sequential greedy loop of src/infer.py:551-621 and to every sample of the
speculative loop, src/infer.py:658-667) against the oracle, which is pinned to the reference's
penalised greedy streams (golden ``greedy_rep115_ids``; the penalised block-verify loop emits
that stream too, tests/test_oracle_golden.py).

Tokens must be identical up to the first decision whose top-1 margin on the penalised logits
is below 2e-2 (tie tolerance, as in test_engine_gpu.py). Recipe B runs with the fp32 KV cache
and prompts of at most 32 tokens (see test_engine_gpu.py).
"""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

from conftest import PATH_IDS, early_exit_model, load_golden, sampled_safe_prefix, spec_stream_divergence, use_path

pytestmark = pytest.mark.gpu
TOL = 2e-2
PEN = 1.15
_CACHE = {}


def _setup(recipe, kv_dtype):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    key = (recipe, kv_dtype)
    if key not in _CACHE:
        for k in list(_CACHE):
            _CACHE.pop(k)[0].close()
        cfg = PulsarConfig(eos_token_id=-1)
        sd = make_state_dict(cfg, recipe=recipe, seed=0)
        eng = DeviceEngine(cfg, sd, device=0, max_batch=4, max_seq_len=512, max_prefill=256, kv_dtype=kv_dtype)
        _CACHE[key] = (eng, O.OracleModel(sd, cfg), cfg)
    eng = _CACHE[key][0]
    use_path(eng, 0)
    eng.set_repetition_penalty(1.0)
    eng.set_early_exit(None)
    return _CACHE[key]


@pytest.fixture(params=[0, 1, 2], ids=PATH_IDS)
def path(request):
    return request.param


def _safe_prefix(prompt, out, trace, penalty):
    """Leading tokens decided with a penalised top-1 margin of at least TOL."""
    for j, (_, lg) in enumerate(trace[:len(out)]):
        v = O.apply_repetition_penalty(lg, list(prompt) + out[:j], penalty).topk(2).values
        if float(v[0] - v[1]) < TOL:
            return j
    return len(out)


@pytest.mark.parametrize("recipe,kv,T", [("A", torch.bfloat16, 128), ("B", torch.float32, 32)])
def test_penalised_greedy_matches_oracle(recipe, kv, T, path):
    eng, m, cfg = _setup(recipe, kv)
    use_path(eng, path)
    ids = random_prompts(1, T, cfg.vocab_size, seed=4)[0].tolist()
    n = 32
    trace = []
    ref = O.stream_generate_ids(m, ids, n, repetition_penalty=PEN, trace=trace)
    safe = _safe_prefix(ids, ref, trace, PEN)
    eng.set_repetition_penalty(PEN)
    first = eng.prefill(0, ids)
    got, _ = eng.generate_greedy([0], first.view(1, -1), n, gamma=0)
    eng.set_repetition_penalty(1.0)
    assert got[0].tolist()[:safe] == ref[:safe], f"penalised tokens differ inside the decided prefix ({safe})"


@pytest.mark.parametrize("thr", [None, 0.3])
def test_penalty_sharpened_and_with_early_exit(thr, path):
    """The sharpened lora-free golden weights (wide top-1 margins; the penalty changes the
    stream there), alone and with early exit: the exiting pulse's logits are penalised
    (src/infer.py:549 then :582-589)."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    g = load_golden("early_exit_nolora")
    sd, cfg = early_exit_model(g)
    m = O.OracleModel(sd, cfg)
    eng = DeviceEngine(cfg, sd, device=0, max_batch=2, max_seq_len=256, max_prefill=64, kv_dtype=torch.float32)
    try:
        eng.set_option("tc_gemm", 0)   # fp32 prefill: these streams are chaotic (test_early_exit_gpu.py)
        eng.set_option("tc_attn", 0)
        use_path(eng, path)
        n = 24
        cnt, probs, trace = [0, 0, 0], [], []
        ref = O.stream_generate_ids(m, g["prompt"], n, repetition_penalty=PEN, early_exit_threshold=thr,
                                    exit_counts=cnt, exit_probs=probs, trace=trace)
        assert ref != O.stream_generate_ids(m, g["prompt"], n, early_exit_threshold=thr), "penalty without effect"
        safe = _safe_prefix(g["prompt"], ref, trace, PEN)
        assert safe >= 16, f"the case should stay decided for most of the stream ({safe})"
        near = [abs(p - thr) / thr for p in probs] if thr is not None else [1.0]
        eng.set_early_exit(thr)
        eng.set_repetition_penalty(PEN)
        first = eng.prefill(0, g["prompt"])
        got, _ = eng.generate_greedy([0], first.view(1, -1), n + 1, gamma=0)
        counts = eng.early_exit_counts()
        assert got[0].tolist()[:safe] == ref[:safe]
        if thr is not None and safe == n and min(near) > 1e-3:
            assert counts == cnt, f"exit tallies {counts} vs oracle {cnt}"
    finally:
        eng.close()


def test_penalty_batch_matches_single():
    eng, m, cfg = _setup("A", torch.bfloat16)
    P = random_prompts(2, 64, cfg.vocab_size, seed=6)
    eng.set_repetition_penalty(PEN)
    f0, f1 = eng.prefill(0, P[0].tolist()), eng.prefill(1, P[1].tolist())
    both, _ = eng.generate_greedy([0, 1], torch.stack([f0, f1]), 20, gamma=0)
    f1 = eng.prefill(1, P[1].tolist())
    one, _ = eng.generate_greedy([1], f1.view(1, -1), 20, gamma=0)
    eng.set_repetition_penalty(1.0)
    assert both[1].tolist() == one[0].tolist()


_SPEC_REF = {}


def _spec_ref(m, recipe, ids, n, gamma, **kw):
    key = (recipe, tuple(ids), n, gamma, tuple(sorted(kw.items())))
    if key not in _SPEC_REF:
        trace, st = [], O.SpecStats()
        ref = O.block_spec_generate_ids(m, ids, n, gamma=gamma, repetition_penalty=PEN, trace=trace, stats=st, **kw)
        _SPEC_REF[key] = (ref, trace, st)
    return _SPEC_REF[key]


@pytest.mark.parametrize("recipe,kv,T", [("A", torch.bfloat16, 128), ("B", torch.float32, 32)])
@pytest.mark.parametrize("gamma", [1, 4])
def test_penalised_speculative_matches_oracle(recipe, kv, T, gamma, path):
    """Greedy speculative rounds with the penalty (src/infer.py:658-667 penalises every sample):
    each draft and verify row is penalised over the slot's seen set plus the round's earlier
    drafts, against oracle.block_spec_generate_ids(repetition_penalty=1.15); the first
    difference must be explained by a tie of the penalised logits (conftest.spec_stream_divergence)."""
    eng, m, cfg = _setup(recipe, kv)
    use_path(eng, path)
    ids = random_prompts(1, T, cfg.vocab_size, seed=4)[0].tolist()
    n = 32
    ref, trace, st = _spec_ref(m, recipe, ids, n, gamma)
    eng.set_repetition_penalty(PEN)
    try:
        first = eng.prefill(0, ids)
        got, stats = eng.generate_greedy([0], first.view(1, -1), n, gamma=gamma)
    finally:
        eng.set_repetition_penalty(1.0)
    first_pen = O.apply_repetition_penalty(first.cpu().float(), ids, PEN)
    k, why = spec_stream_divergence(got[0].tolist(), ref, first_pen, trace, gamma, TOL)
    assert not why.startswith("FAIL"), why
    if k is None:
        assert stats["accepted"] == st.accepted, f"accepted drafts {stats['accepted']} vs oracle {st.accepted}"
    if recipe == "B":   # the case discriminates: without the penalty the oracle stream differs
        assert O.block_spec_generate_ids(m, ids, n, gamma=gamma) != ref


def test_penalised_speculative_differs_from_plain():
    """The penalty changes the device's speculative stream on recipe B weights (recipe A's
    random-init streams repeat one id with a top-1 margin the penalty does not overturn)."""
    eng, m, cfg = _setup("B", torch.float32)
    ids = random_prompts(1, 32, cfg.vocab_size, seed=5)[0].tolist()
    first = eng.prefill(0, ids)
    plain, _ = eng.generate_greedy([0], first.view(1, -1), 48, gamma=4)
    eng.set_repetition_penalty(PEN)
    try:
        first = eng.prefill(0, ids)
        pen, _ = eng.generate_greedy([0], first.view(1, -1), 48, gamma=4)
    finally:
        eng.set_repetition_penalty(1.0)
    assert plain[0].tolist() != pen[0].tolist()


@pytest.mark.parametrize("recipe,kv", [("A", torch.bfloat16), ("A", torch.float32)])
def test_penalised_sampled_matches_oracle(recipe, kv, path):
    """Sampled speculative rounds with the penalty: draft and verify logits penalised before
    the temperature / top-p warping, the first draw over the penalised prefill logits.
    Temperature 0.3: at 0.8 (and for recipe B at any temperature) the warped distributions keep
    ~30k tokens with buckets narrower than the draw tie tolerance, so no token is decided."""
    eng, m, cfg = _setup(recipe, kv)
    use_path(eng, path)
    temp, top_p, seed, seq_id, n, gamma = 0.3, 0.9, 11, 2, 24, 4
    ids = random_prompts(1, 32, cfg.vocab_size, seed=12)[0].tolist()
    okv = O.OracleKV(m, 64)
    pre = O.prefill(m, ids, okv)
    ref, trace, st = _spec_ref(m, recipe, ids, n, gamma, temperature=temp, top_p=top_p, seed=seed, seq_id=seq_id)
    eng.set_repetition_penalty(PEN)
    try:
        first = eng.prefill(0, ids)
        got, stats = eng.generate_sampled([0], first.view(1, -1), n, gamma, temp, top_p, seed, seq_ids=[seq_id])
    finally:
        eng.set_repetition_penalty(1.0)
    safe = sampled_safe_prefix(O.apply_repetition_penalty(pre, ids, PEN), trace, st, gamma, temp, top_p, seed, seq_id)
    k = min(safe, n)
    assert k >= 8, f"the case should stay decided for most of the stream ({k})"
    assert got[0].tolist()[:k] == ref[:k], f"penalised sampled tokens differ inside the decided prefix ({k})"


def test_penalty_argument_checks():
    eng, m, cfg = _setup("A", torch.bfloat16)
    with pytest.raises(RuntimeError, match="finite and > 0"):
        eng.set_repetition_penalty(0.0)


def test_generate_batch_penalty_api():
    """PulsarInferenceEngine.generate_batch(gamma=0, repetition_penalty=1.15)."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import PulsarInferenceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="A", seed=0)
    m = O.OracleModel(sd, cfg)
    eng = PulsarInferenceEngine((sd, cfg), device="cuda", max_batch=1, max_seq_len=256)
    ids = random_prompts(1, 64, cfg.vocab_size, seed=8)
    trace = []
    ref = O.stream_generate_ids(m, ids[0].tolist(), 16, repetition_penalty=PEN, trace=trace)
    safe = _safe_prefix(ids[0].tolist(), ref, trace, PEN)
    out = eng.generate_batch(ids, 16, gamma=0, repetition_penalty=PEN)
    assert out[0, 64:64 + safe].tolist() == ref[:safe]
    # speculative (gamma = 4) with the penalty: the oracle's penalised block-verify loop
    trace = []
    ref4 = O.block_spec_generate_ids(m, ids[0].tolist(), 16, gamma=4, repetition_penalty=PEN, trace=trace)
    out4 = eng.generate_batch(ids, 16, gamma=4, repetition_penalty=PEN)
    first_pen = O.apply_repetition_penalty(O.prefill(m, ids[0].tolist(), O.OracleKV(m, 96)), ids[0].tolist(), PEN)
    k, why = spec_stream_divergence(out4[0, 64:].tolist(), ref4, first_pen, trace, 4, TOL)
    assert not why.startswith("FAIL"), why
