"""PulsarForCausalLM.forward / generate on the engine (pulsar_engine_forward,
PulsarInferenceEngine.model_generate; src/model.py:1956-2125, 2246-2317) against the oracle,
which is pinned to the reference's own forward and generate streams (golden forward_*,
tests/test_oracle_golden.py).

The forward differs from the inference prefill in the value residual across pulses, YaRN
on the global layers, causal attention over the whole sequence on the local layers, and
softcapped logits; the tests cover a short prompt (no YaRN) and T = 1100 (YaRN on layers 3
and 7). Tolerance 2e-2 on logits as for the prefill; token streams identical up to the first
decision whose top-1 margin (after the penalty) is within 2e-2."""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu
TOL = 2e-2
_CACHE = {}


def _setup(recipe, kv):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import PulsarInferenceEngine
    key = (recipe, kv)
    if key not in _CACHE:
        for k in list(_CACHE):
            _CACHE.pop(k)[0].dev.close()
        cfg = PulsarConfig(eos_token_id=-1)
        sd = make_state_dict(cfg, recipe=recipe, seed=0)
        eng = PulsarInferenceEngine((sd, cfg), device="cuda", dtype=kv, max_batch=2, max_seq_len=2176)
        _CACHE[key] = (eng, O.OracleModel(sd, cfg), cfg)
    return _CACHE[key]


@pytest.mark.parametrize("recipe,kv,T", [("A", torch.bfloat16, 128), ("B", torch.float32, 32),
                                         ("A", torch.float32, 1100)])
def test_forward_logits_match_oracle(recipe, kv, T):
    eng, m, cfg = _setup(recipe, kv)
    ids = random_prompts(1, T, cfg.vocab_size, seed=T)[0].tolist()
    ref = O.forward_logits(m, ids)
    c = eng.new_cache()
    try:
        got = eng.dev.forward(c.slot, ids).cpu()
        assert eng.dev.get_length(c.slot) == 0, "the forward leaves its scratch slot empty"
    finally:
        c.release()
    err = (got - ref).abs().max().item()
    assert err <= TOL, f"forward logits: max |err| {err:.3e}"
    assert got.abs().max().item() <= cfg.logit_softcap + 1e-4, "softcapped"
    if T <= 128:   # the inference prefill of the same ids differs (value residual, softcap) by more than TOL
        pre = O.prefill(m, ids, O.OracleKV(m, T + 8))
        assert (pre - ref).abs().max().item() > 2 * TOL


def _decided(m, prompt, out, penalty):
    """Leading generated tokens whose (penalised) top-1 margin exceeds TOL in the oracle."""
    row = list(prompt)
    for j, tok in enumerate(out):
        lg = O.apply_repetition_penalty(O.forward_logits(m, row), row, penalty)
        v = lg.topk(2).values
        if float(v[0] - v[1]) <= TOL:
            return j
        row.append(tok)
    return len(out)


@pytest.mark.parametrize("penalty", [1.0, 1.15])
def test_model_generate_greedy_matches_oracle(penalty):
    eng, m, cfg = _setup("B", torch.float32)
    ids = random_prompts(1, 24, cfg.vocab_size, seed=5)
    n = 6
    ref = O.model_generate_ids(m, ids.tolist(), n, temperature=0.0, repetition_penalty=penalty)[0][24:]
    got = eng.model_generate(ids, n, temperature=0.0, repetition_penalty=penalty)[0, 24:].tolist()
    k = _decided(m, ids[0].tolist(), ref, penalty)
    assert got[:k] == ref[:k], f"model_generate tokens differ inside the decided prefix ({k}): {got} vs {ref}"


def test_model_generate_sampling_and_eos():
    eng, m, cfg = _setup("A", torch.bfloat16)
    ids = random_prompts(2, 16, cfg.vocab_size, seed=9)
    g = torch.Generator().manual_seed(3)
    out = eng.model_generate(ids, 5, temperature=0.8, top_k=5, top_p=0.9, generator=g)
    assert out.shape == (2, 21) and torch.equal(out[:, :16].cpu(), ids.long())
    # eos: a row whose first token is eos emits eos from then on and the loop stops when all rows finish
    first = eng.model_generate(ids[:1], 1, temperature=0.0, repetition_penalty=1.0)[0, -1].item()
    out = eng.model_generate(ids[:1], 4, temperature=0.0, repetition_penalty=1.0, eos_token_id=first)
    assert out.shape == (1, 17) and out[0, -1].item() == first
    with pytest.raises(ValueError, match="pulses"):
        eng.model_generate(ids, 1, num_pulses=2)
    c = eng.new_cache()
    try:
        with pytest.raises(RuntimeError, match="exceed"):
            eng.dev.forward(c.slot, [1] * 2100)
    finally:
        c.release()
