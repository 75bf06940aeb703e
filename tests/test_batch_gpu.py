"""Batched decoding at the BASELINE batch configs: many sequences per call, so a
speculative round's pulse passes have more than 32 rows and run on the many-row GEMM path.

Size-independent properties at (or near) the configs' sizes:
  * config 5 (256 sequences, 512-token prompts, gamma 4, greedy) and a 40-sequence case:
    each sequence of the batched call emits exactly the tokens of the same sequence decoded
    alone (recipe A, whose top-1 margins are far above the 2e-2 tie tolerance);
  * config 3 (64 sequences, gamma 6, temperature 0.8, top-p 0.95): sequences of the batched
    sampled call match the oracle's block-verify loop on their own Philox stream (seq id =
    batch index) up to the first decision inside the tie tolerances (also at temperature 0.3,
    where the decided prefix covers the stream);
  * the largest batch (1024 sequences): batched decoding equals each sequence alone;
  * config 4 (4 sequences, 32768-token prompts, gamma 4): speculative greedy decoding emits
    the tokens of sequential greedy decoding (recipe A margins), exercising the sliding window
    and the YaRN global layers on a full-window cache.
"""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

from conftest import sampled_safe_prefix, use_path

pytestmark = pytest.mark.gpu


def _engine(recipe, kv, **kw):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe=recipe, seed=0)
    return DeviceEngine(cfg, sd, device=0, kv_dtype=kv, **kw), sd, cfg


def _batched_vs_single(B, T, n, gamma, check):
    eng, sd, cfg = _engine("A", torch.bfloat16, max_batch=B, max_seq_len=T + n + 16, max_prefill=T)
    try:
        use_path(eng, 0)
        P = random_prompts(B, T, cfg.vocab_size, seed=0)
        first = torch.stack([eng.prefill(b, P[b].tolist()) for b in range(B)])
        assert eng.get_option("wide_rows") >= B * (gamma + 1)
        got, stats = eng.generate_greedy(list(range(B)), first, n, gamma=gamma)
        assert stats["rounds"] > 0
        for b in check:
            eng.prefill(b, P[b].tolist())
            one, _ = eng.generate_greedy([b], first[b].view(1, -1), n, gamma=gamma)
            assert got[b].tolist() == one[0].tolist(), f"sequence {b}: batched != alone"
    finally:
        eng.close()


def test_batch40_greedy_matches_single():
    _batched_vs_single(40, 24, 16, 4, check=(0, 17, 39))


def test_config5_batch256_greedy_matches_single():
    """Config 5 shape: 256 sequences x 512-token prompts, gamma 4 (64 of the 256 new tokens)."""
    _batched_vs_single(256, 512, 64, 4, check=(0, 255))


@pytest.mark.parametrize("recipe,kv,temp,min_decided", [("B", torch.float32, 0.8, 0), ("A", torch.float32, 0.3, 8)])
def test_config3_batch64_sampled_matches_oracle(recipe, kv, temp, min_decided):
    """Config 3 shape (reduced lengths): 64 sequences, gamma 6, top-p 0.95, Philox seed 0. At the
    config's temperature 0.8 the random-init distributions keep ~30k tokens, so few or no draws
    are outside the tie tolerance (the statistics are still checked); at 0.3 (recipe A) the
    decided prefix must cover 8+ tokens."""
    B, T, n, gamma, top_p, seed = 64, 24, 12, 6, 0.95, 0
    eng, sd, cfg = _engine(recipe, kv, max_batch=B, max_seq_len=T + n + 16, max_prefill=T)
    try:
        use_path(eng, 0)
        P = random_prompts(B, T, cfg.vocab_size, seed=0)
        first = torch.stack([eng.prefill(b, P[b].tolist()) for b in range(B)])
        got, stats = eng.generate_sampled(list(range(B)), first, n, gamma, temp, top_p, seed)
        assert stats["drafted"] == gamma * stats["rounds"]
        m = O.OracleModel(sd, cfg)
        for b in (0, 63):
            ids = P[b].tolist()
            pre = O.prefill(m, ids, O.OracleKV(m, T + 8))
            st, trace = O.SpecStats(), []
            ref = O.block_spec_generate_ids(m, ids, n, gamma=gamma, temperature=temp, top_p=top_p, seed=seed,
                                            seq_id=b, stats=st, trace=trace)
            k = min(n, sampled_safe_prefix(pre, trace, st, gamma, temp, top_p, seed, b))
            assert k >= min_decided, f"sequence {b}: only {k} decided tokens"
            assert got[b].tolist()[:k] == ref[:k], f"sequence {b}: first {k} tokens differ from the oracle"
    finally:
        eng.close()


def test_config4_long_context_spec_equals_sequential():
    """Config 4 shape: 4 sequences x 32768-token prompts; gamma 4 vs sequential greedy."""
    B, T, n = 4, 32768, 48
    eng, sd, cfg = _engine("A", torch.bfloat16, max_batch=B, max_seq_len=T + n + 16, max_prefill=T)
    try:
        use_path(eng, 0)
        P = random_prompts(B, T, cfg.vocab_size, seed=0)
        first = torch.stack([eng.prefill(b, P[b].tolist()) for b in range(B)])
        spec, _ = eng.generate_greedy(list(range(B)), first, n, gamma=4)
        for b in range(B):
            eng.set_length(b, T)
        seq, _ = eng.generate_greedy(list(range(B)), first, n, gamma=0)
        assert spec.tolist() == seq.tolist()
    finally:
        eng.close()


def test_max_batch_1024_greedy_matches_single():
    """The engine's largest batch: 1024 sequences in one call (verify passes of 5120 rows)."""
    _batched_vs_single(1024, 16, 8, 4, check=(0, 511, 1023))
