"""Pin the CPU oracle to the reference: golden vectors made by running the reference
inference engine (tests/golden/make_golden.py) must be reproduced by oracle/."""

from __future__ import annotations

import pytest
import torch

from conftest import early_exit_model, load_golden
from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict

TINY = ["tiny_A", "tiny_B", "tiny_B_long"]
FULL = ["full_A_c1", "full_B_c1", "full_B_long"]
_MODELS = {}


def _model(g):
    key = (g["cfg"].get("d_model", 1024), g["cfg"].get("n_core", 8), g["recipe"], g["seed"], g.get("b_std", 0.09))
    if key not in _MODELS:
        cfg = PulsarConfig(**g["cfg"])
        sd = make_state_dict(cfg, recipe=g["recipe"], seed=g["seed"], b_std=g.get("b_std", 0.09))
        _MODELS.clear()
        _MODELS[key] = (O.OracleModel(sd, cfg), cfg)
    return _MODELS[key]


# Oracle and reference are both fp32 but sum in different orders (e.g. the reference adds
# the loop adapter into a merged weight on every call); recipe B amplifies such 1e-7-level
# differences about 100x, so the bound is 1e-3 - twenty times tighter than the engine's 2e-2.
ORACLE_TOL = 1e-3


def _check_logits(lg, summ, tol, what):
    lg = lg.reshape(-1).float()
    if "full" in summ:
        err = (lg - summ["full"]).abs().max().item()
    else:
        err = (lg[summ["_probe_idx"]] - summ["probe"]).abs().max().item()
    err = max(err, (lg[summ["top_idx"]] - summ["top_val"]).abs().max().item())
    assert err <= tol, f"{what}: max |oracle - reference| = {err:.3e} > {tol}"
    assert int(lg.argmax()) == summ["argmax"], f"{what}: argmax differs"
    assert abs(torch.logsumexp(lg, 0).item() - summ["lse"]) <= tol, f"{what}: logsumexp differs"


def _run_pulses(g):
    m, cfg = _model(g)
    for s in [g["prefill"]] + [p for st in g["steps"] for p in st["pulses"]]:
        s["_probe_idx"] = g["probe_idx"]
    kv = O.OracleKV(m, len(g["prompt"]) + 16)
    lg = O.prefill(m, g["prompt"], kv)
    _check_logits(lg, g["prefill"], ORACLE_TOL, f"{g['name']} prefill")
    for st in g["steps"]:
        h = h0n = None
        for p in range(m.K):
            lg, h, h0n = O.pulse_pass(m, p, [st["token"]], [st["pos"]], kv, h, h0n)
            _check_logits(lg[0], st["pulses"][p], ORACLE_TOL, f"{g['name']} pos {st['pos']} pulse {p}")
        kv.length = st["pos"] + 1


@pytest.mark.parametrize("name", TINY)
def test_oracle_pulses_tiny(name):
    _run_pulses(load_golden(name))


@pytest.mark.parametrize("name", TINY)
def test_oracle_generate_tiny(name):
    g = load_golden(name)
    m, _ = _model(g)
    assert O.stream_generate_ids(m, g["prompt"], g["n_new"]) == g["greedy_ids"]
    assert O.self_speculative_ids(m, g["prompt"], g["n_new"]) == g["spec_ids"]
    assert O.stream_generate_ids(m, g["prompt"], len(g["greedy_rep115_ids"]),
                                 repetition_penalty=1.15) == g["greedy_rep115_ids"]


@pytest.mark.slow
@pytest.mark.parametrize("name", FULL)
def test_oracle_pulses_full(name):
    _run_pulses(load_golden(name))


@pytest.mark.slow
@pytest.mark.parametrize("name", FULL)
def test_oracle_generate_full(name):
    g = load_golden(name)
    m, _ = _model(g)
    n = min(g["n_new"], 24)
    assert O.stream_generate_ids(m, g["prompt"], n) == g["greedy_ids"][:n]
    assert O.self_speculative_ids(m, g["prompt"], n) == g["spec_ids"][:n]
    r = g["greedy_rep115_ids"]
    assert O.stream_generate_ids(m, g["prompt"], len(r), repetition_penalty=1.15) == r


@pytest.mark.parametrize("name", ["early_exit_tiny", pytest.param("early_exit_full", marks=pytest.mark.slow),
                                  pytest.param("early_exit_nolora", marks=pytest.mark.slow)])
def test_oracle_early_exit(name):
    """src/infer.py:526-549 with set_early_exit_threshold: the oracle's greedy stream and
    exit tallies equal the reference's at every recorded threshold."""
    g = load_golden(name)
    sd, cfg = early_exit_model(g)
    m = O.OracleModel(sd, cfg)
    depths = set()
    for run in g["runs"]:
        cnt = [0] * m.K
        out = O.stream_generate_ids(m, g["prompt"], g["n_new"], early_exit_threshold=run["threshold"],
                                    exit_counts=cnt)
        assert out == run["ids"], f"threshold {run['threshold']}: tokens differ"
        assert cnt == run["counts"], f"threshold {run['threshold']}: exit tallies {cnt} vs {run['counts']}"
        depths |= {k for k, c in enumerate(cnt) if c}
    assert len(depths) >= 2, "the cases should exit at more than one depth"


def test_block_spec_gamma1_greedy_matches_reference_stream_on_tiny():
    """The block-verify loop with one row per verify (no in-block predecessors) commits the
    same tokens as the reference's greedy stream: every verify row sees a final prefix."""
    g = load_golden("tiny_B")
    m, _ = _model(g)
    out = O.block_spec_generate_ids(m, g["prompt"], g["n_new"], gamma=1)
    assert out[0] == g["greedy_ids"][0]
    # gamma = 1: row 0 of every verify is exact, row 1 (the bonus) sees in-block pulse-p K/V.
    assert len(out) == g["n_new"]


@pytest.mark.parametrize("gamma", [1, 2, 4])
def test_block_spec_penalised_matches_reference_stream_on_tiny(gamma):
    """Greedy block-verify decoding with the repetition penalty (each draft and verify row
    penalised over the prompt, the emitted tokens and the round's earlier drafts) emits the
    reference's own penalised greedy stream (golden greedy_rep115_ids, src/infer.py:551-621
    with repetition_penalty 1.15); without the penalty the stream differs."""
    g = load_golden("tiny_B")
    m, _ = _model(g)
    ref = g["greedy_rep115_ids"]
    assert O.block_spec_generate_ids(m, g["prompt"], len(ref), gamma=gamma, repetition_penalty=1.15) == ref
    assert O.block_spec_generate_ids(m, g["prompt"], len(ref), gamma=gamma) != ref


def test_forward_and_model_generate_tiny():
    """PulsarForCausalLM.forward / generate (src/model.py:1956-2125, 2246-2317) on the tiny
    config with a 40-token prompt (T > window and > base_seq_len): the oracle's full-sequence
    forward against the reference's softcapped logits, and its model_generate streams (greedy,
    penalised, and sampled from the same seed) against the reference's."""
    g = load_golden("forward_tiny_B")
    m, _ = _model(g)
    lg = O.forward_logits(m, g["prompt"])
    _check_logits(lg, g["forward"], ORACLE_TOL, "forward")
    n, T = g["n_new"], len(g["prompt"])
    assert O.model_generate_ids(m, [g["prompt"]], n, temperature=0.0, repetition_penalty=1.0)[0][T:] == g["greedy_ids"]
    assert O.model_generate_ids(m, [g["prompt"]], n, temperature=0.0, repetition_penalty=1.15)[0][T:] == \
        g["greedy_rep115_ids"]
    gen = torch.Generator().manual_seed(11)
    assert O.model_generate_ids(m, [g["prompt"]], n, temperature=0.8, top_k=50, top_p=0.9, repetition_penalty=1.15,
                                generator=gen)[0][T:] == g["sampled_ids"]
    # the forward is not the inference prefill (value residual, masks, softcap)
    assert (O.prefill(m, g["prompt"], O.OracleKV(m, 64)) - lg).abs().max().item() > 1e-2


def test_forward_full_yarn():
    """The production config at T = 1100 > 1024: YaRN on the global layers (3, 7) and causal
    attention over all 1100 keys on the local layers (the reference's sliding window starts
    beyond 4096 tokens)."""
    g = load_golden("forward_full_A")
    m, _ = _model(g)
    g["forward"]["_probe_idx"] = g["probe_idx"]
    lg = O.forward_logits(m, g["prompt"])
    _check_logits(lg, g["forward"], ORACLE_TOL, "forward T=1100")
    assert int(lg.argmax()) == g["greedy_ids"][0]


def test_philox_known_answer():
    """Philox4x32-10 known-answer vectors from the Random123 distribution's kat_vectors
    (counter, key) -> output, the published test values for the SC'11 generator."""
    assert O.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert O.philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert O.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_token_slots_drop_lowest_weight():
    """src/model.py:996-1054: overflow drops the lowest-weight assignments deterministically."""
    idx = torch.tensor([[0, 1], [0, 1], [0, 2], [0, 3]])
    w = torch.tensor([[0.9, 0.1], [0.2, 0.8], [0.6, 0.4], [0.7, 0.3]])
    s = O.token_slots(idx, w, 4, 2)
    # expert 0 has 4 assignments with weights .9 .2 .6 .7 -> keep .9 (slot 0) and .7 (slot 1)
    assert s[:, 0].tolist() == [0, -1, -1, 1]
    assert s[0, 1].item() == 1 and s[1, 1].item() == 0
