"""Adaptive early exit on the device (pulsar_engine_set_early_exit, the exit rule of
src/infer.py:526-549) against the reference's early-exit goldens (tests/golden/
early_exit_*.pt, reproduced exactly by the oracle in test_oracle_golden.py).
early_exit_full carries loop-adapter weights (per-op kernels); early_exit_nolora has
lora_B = 0 and so runs the persistent pulse kernel on the default path.

The rule compares a softmax max-probability with the threshold and the token is an argmax;
both are discontinuous. Tokens and tallies must be identical up to the first oracle decision
inside a tie tolerance: an examined max-probability within 1e-3 (relative) of the threshold,
or a top-1 logit margin below 2e-2. The golden cases keep every exit decision at least 4%
(relative) away from its threshold, so in practice the whole stream is compared. Recipe B
runs with the fp32 KV cache (its logits agree with the oracle to about 1e-4, see
test_engine_gpu.py) and the prefill on the fp32 SIMT GEMMs (option tc_gemm = 0): these
sharpened recipe-B streams are chaotic - a logits difference grows about a thousandfold over
25 steps - and the tensor-core GEMMs' bf16 hi/lo operand split (2^-16 relative) would carry
the stream past the tie margins before its end.

One decode step of the device loop is one reference decode_step; the reference runs a
decode_step after every emitted token (the last one's logits unused), so n_new reference
tokens carry n_new exits and correspond to n_new + 1 device tokens.
"""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.weights import random_prompts

from conftest import PATH_IDS, early_exit_model, load_golden, use_path

pytestmark = pytest.mark.gpu
PROB_TOL = 1e-3    # relative distance of an exit probability from the threshold
MARGIN_TOL = 2e-2  # top-1 logit margin of a greedy decision
_CACHE = {}


def _setup(case="early_exit_nolora"):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    if case not in _CACHE:
        g = load_golden(case)
        sd, cfg = early_exit_model(g)
        eng = DeviceEngine(cfg, sd, device=0, max_batch=4, max_seq_len=256, max_prefill=64, kv_dtype=torch.float32)
        eng.set_option("tc_gemm", 0)   # fp32 prefill (GEMMs and attention): these streams are chaotic
        eng.set_option("tc_attn", 0)
        _CACHE[case] = (eng, O.OracleModel(sd, cfg), cfg, g)
    eng = _CACHE[case][0]
    use_path(eng, 0)
    eng.set_early_exit(None)
    return _CACHE[case]


@pytest.fixture(params=[0, 1, 2], ids=PATH_IDS)
def path(request):
    return request.param


def _oracle_run(m, prompt, n, thr):
    """Oracle tokens and tallies of n decode steps, and the number of leading tokens decided
    outside the tie tolerance (step j's logits pick token j + 1)."""
    cnt = [0] * m.K
    kv = O.OracleKV(m, len(prompt) + n + 8)
    logits = O.prefill(m, prompt, kv)
    toks, pos, safe = [], len(prompt) - 1, None
    for j in range(n):
        v = logits.topk(2).values
        if safe is None and float(v[0] - v[1]) < MARGIN_TOL:
            safe = j
        toks.append(int(logits.argmax()))
        pos += 1
        probs = []
        logits = O.decode_step(m, toks[-1], pos, kv, early_exit_threshold=thr, exit_counts=cnt, exit_probs=probs)
        if safe is None and thr is not None and any(abs(p - thr) <= PROB_TOL * max(thr, 1e-12) for p in probs):
            safe = j + 1
    return toks, cnt, n if safe is None else safe


def _device_run(eng, slots, prompts, n_new, thr):
    eng.set_early_exit(thr)
    first = torch.stack([eng.prefill(s, p) for s, p in zip(slots, prompts)])
    out, _ = eng.generate_greedy(slots, first, n_new, gamma=0)
    return [r.tolist() for r in out], eng.early_exit_counts()


@pytest.mark.parametrize("case", ["early_exit_nolora", "early_exit_full"])
@pytest.mark.parametrize("run_idx", [0, 1])
def test_early_exit_matches_reference_golden(case, run_idx, path):
    eng, m, cfg, g = _setup(case)
    use_path(eng, path)
    run = g["runs"][run_idx]
    n = g["n_new"]
    ref, cnt, safe = _oracle_run(m, g["prompt"], n, run["threshold"])
    assert ref == run["ids"] and cnt == run["counts"], "oracle no longer reproduces the golden case"
    got, counts = _device_run(eng, [0], [g["prompt"]], n + 1, run["threshold"])
    assert got[0][:safe] == ref[:safe], f"tokens differ inside the decided prefix ({safe}): {got[0]} vs {ref}"
    if safe == n:
        assert counts == run["counts"], f"exit tallies {counts} vs reference {run['counts']}"


def test_early_exit_after_first_pulse_skips_the_persistent_passes():
    """Threshold 0: every token exits after the first pulse (its argmax, its K/V cached). The
    persistent second and third passes see every row exited and return at once, so they
    stream no expert weights."""
    eng, m, cfg, g = _setup()
    assert eng.get_option("loop_adapter") == 0 and eng.get_option("megakernel_grid") > 0
    n = 16
    ref, cnt, safe = _oracle_run(m, g["prompt"], n, 0.0)
    assert cnt == [n, 0, 0]
    e0 = eng.get_option("routed_experts")
    got, counts = _device_run(eng, [0], [g["prompt"]], n + 1, 0.0)
    e1 = eng.get_option("routed_experts")
    assert got[0][:safe] == ref[:safe]
    assert counts == [n, 0, 0]
    eng.set_early_exit(None)
    full, counts_off = _device_run(eng, [0], [g["prompt"]], n + 1, None)
    e2 = eng.get_option("routed_experts")
    assert counts_off == [0, 0, 0]
    # pulse-1 passes only vs all three pulses
    assert (e1 - e0) * 2 < (e2 - e1), f"early-exit run streamed {e1 - e0} experts, full run {e2 - e1}"
    ref_full, _, safe_full = _oracle_run(m, g["prompt"], n, None)
    assert full[0][:safe_full] == ref_full[:safe_full]


def test_early_exit_batch_matches_single(path):
    """Exit decisions are per sequence: two sequences in one call == each alone, and the
    tallies add up."""
    eng, m, cfg, g = _setup()
    use_path(eng, path)
    thr = g["runs"][0]["threshold"]
    P = [g["prompt"], random_prompts(1, 32, cfg.vocab_size, seed=2)[0].tolist()]
    both, cb = _device_run(eng, [0, 1], P, 24, thr)
    one0, c0 = _device_run(eng, [0], P[:1], 24, thr)
    one1, c1 = _device_run(eng, [1], P[1:], 24, thr)
    assert both[0] == one0[0] and both[1] == one1[0]
    assert cb == [a + b for a, b in zip(c0, c1)]
    assert sum(cb) == 2 * 23


def test_reference_api_early_exit_stats():
    """PulsarInferenceEngine.set_early_exit_threshold + generate_batch(gamma=0): the device
    tallies land in early_exit_counts / get_early_exit_stats (src/infer.py:211-232)."""
    from pulsar_b200.engine import PulsarInferenceEngine
    _, m, _, g = _setup()
    sd, cfg = early_exit_model(g)
    eng = PulsarInferenceEngine((sd, cfg), device="cuda", dtype=torch.float32, max_batch=1, max_seq_len=128)
    eng.dev.set_option("tc_gemm", 0)
    eng.dev.set_option("tc_attn", 0)
    run, n, T = g["runs"][0], g["n_new"], len(g["prompt"])
    _, _, safe = _oracle_run(m, g["prompt"], n, run["threshold"])
    eng.set_early_exit_threshold(run["threshold"])
    out = eng.generate_batch(torch.tensor([g["prompt"]]), n + 1, gamma=0)
    assert out[0, T:T + safe].tolist() == run["ids"][:safe]
    st = eng.get_early_exit_stats()
    assert st["total_tokens"] == n
    if safe == n:
        assert st["pulse_counts"] == run["counts"]
    eng.set_early_exit_threshold(None)
    assert eng.get_early_exit_stats() == {}
