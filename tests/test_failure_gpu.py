"""Failure handling of the persistent pulse kernel, made on purpose without a GPU fault.

The test hook option ``stall_cta`` makes one CTA of the persistent kernel wait at its first
grid barrier for an arrival count the grid never reaches; with ``wait_ns`` shortened to 2 ms the
wait runs out, the kernel raises its error flag, every other CTA gives up at its next barrier
poll, and all of them return (nothing faults, traps or hangs). The host must report the failure
as PULSAR_ERR_CUDA with the bounded-wait message, and the very next call on the same engine
must decode correctly again. Host-side failures (bad rows, positions beyond the cache, a
prompt beyond max_prefill, a slot out of range) must be refused before any kernel runs.
"""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="A", seed=0)
    eng = DeviceEngine(cfg, sd, device=0, max_batch=2, max_seq_len=256, max_prefill=64)
    if eng.get_option("megakernel") != 1:
        pytest.skip("GPU cannot host the persistent kernel")
    yield eng, O.OracleModel(sd, cfg), cfg
    eng.close()


def test_stalled_wait_reports_error_and_engine_recovers(setup):
    eng, m, cfg = setup
    ids = random_prompts(1, 32, cfg.vocab_size, seed=3)[0].tolist()
    ref = O.stream_generate_ids(m, ids, 6)
    first = eng.prefill(0, ids)
    eng.set_option("wait_ns", 2_000_000)
    eng.set_option("stall_cta", 7)
    try:
        with pytest.raises(RuntimeError, match="bounded device wait ran out"):
            eng.generate_greedy([0], first.view(1, -1), 6, gamma=0)
    finally:
        eng.set_option("stall_cta", -1)
        eng.set_option("wait_ns", 2_000_000_000)
    # the same engine decodes correctly right after the failed call
    first = eng.prefill(0, ids)
    got, _ = eng.generate_greedy([0], first.view(1, -1), 6, gamma=0)
    assert got[0].tolist() == ref
    first = eng.prefill(0, ids)
    got, _ = eng.generate_greedy([0], first.view(1, -1), 6, gamma=4)
    assert got[0].tolist() == ref


def test_host_side_failures_are_refused(setup):
    eng, m, cfg = setup
    eng.prefill(1, [1, 2, 3, 4])
    with pytest.raises(RuntimeError, match="consecutive"):
        eng.pulse(0, [(1, 4, 5), (1, 6, 7)])
    with pytest.raises(RuntimeError, match="outside"):
        eng.pulse(0, [(1, 10**7, 5)])
    with pytest.raises(RuntimeError, match="token"):
        eng.pulse(0, [(1, 4, cfg.vocab_size)])
    with pytest.raises(RuntimeError, match="slot"):
        eng.pulse(0, [(5, 4, 1)])
    with pytest.raises(RuntimeError, match="max_prefill"):
        eng.prefill(1, list(range(65)))
    with pytest.raises(RuntimeError, match="max_seq_len"):
        eng.set_length(1, 10**6)
    with pytest.raises(RuntimeError, match="wait_ns"):
        eng.set_option("wait_ns", 10)
    # still usable
    lg, _, _ = eng.pulse(0, [(1, 4, 5)])
    assert torch.isfinite(lg).all()
