"""Two engines in one process on two GPUs: every kernel attribute (shared-memory size of the
persistent kernel, the tensor-core GEMM, the attention and sampling kernels) is set per device,
so both engines decode, and decode the same tokens. Skipped with fewer than two GPUs."""

from __future__ import annotations

import pytest
import torch

from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu


def test_two_engines_on_two_devices():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="A", seed=0)
    ids = random_prompts(1, 40, cfg.vocab_size, seed=2)[0].tolist()
    outs = []
    engs = [DeviceEngine(cfg, sd, device=d, max_batch=2, max_seq_len=256, max_prefill=64) for d in (0, 1)]
    try:
        for d, eng in enumerate(engs):
            with torch.cuda.device(d):
                first = eng.prefill(0, ids)
                for gamma in (0, 4):
                    eng.set_length(0, len(ids))
                    got, _ = eng.generate_greedy([0], first.view(1, -1), 12, gamma=gamma)
                    outs.append(got[0].tolist())
        assert outs[0] == outs[2] and outs[1] == outs[3]
    finally:
        for eng in engs:
            eng.close()
