"""Option "merged_adapter": per-pulse bf16 merged wqkv / wo, the reference's GPU numerics for
the loop adapter (get_merged_weight with a bf16 base weight, src/model.py:716-727), against the
oracle built with the same merge (OracleModel(merge="bf16")). Checkpoints whose lora_B is
non-zero then run the persistent pulse kernel.

Tolerances as in test_engine_gpu.py: logits max-abs <= 2e-2, greedy tokens identical up to
the first decision with a top-1 margin below 2e-2. Recipe B with the fp32 KV cache and a
32-token prompt.
"""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

from conftest import PATH_IDS, use_path

pytestmark = pytest.mark.gpu
TOL = 2e-2
_CACHE = {}


def _setup():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    if "eng" not in _CACHE:
        cfg = PulsarConfig(eos_token_id=-1)
        sd = make_state_dict(cfg, recipe="B", seed=0)
        eng = DeviceEngine(cfg, sd, device=0, max_batch=2, max_seq_len=256, max_prefill=64, kv_dtype=torch.float32)
        _CACHE["eng"] = (eng, O.OracleModel(sd, cfg, merge="bf16"), O.OracleModel(sd, cfg), cfg)
    eng = _CACHE["eng"][0]
    use_path(eng, 0)
    eng.set_option("merged_adapter", 1)
    return _CACHE["eng"]


@pytest.fixture(params=[0, 1, 2], ids=PATH_IDS)
def path(request):
    return request.param


def test_merged_adapter_matches_bf16_merge_oracle(path):
    eng, m16, m32, cfg = _setup()
    use_path(eng, path)
    assert eng.get_option("loop_adapter") == 1 and eng.get_option("merged_adapter") == 1
    ids = random_prompts(1, 32, cfg.vocab_size, seed=3)[0].tolist()
    kv = O.OracleKV(m16, 64)
    pre = O.prefill(m16, ids, kv)
    first = eng.prefill(0, ids)
    assert (first.cpu() - pre).abs().max().item() <= TOL
    tok, pos = int(pre.argmax()), len(ids)
    h = h0n = None
    dh = dz = None
    for p in range(3):
        lg, h, h0n = O.pulse_pass(m16, p, [tok], [pos], kv, h, h0n)
        lgd, dh, dz = eng.pulse(p, [(0, pos, tok)], dh, dz)
        assert (lgd.cpu()[0] - lg[0]).abs().max().item() <= TOL, f"pulse {p}"
    n = 16
    trace = []
    ref = O.stream_generate_ids(m16, ids, n, trace=trace)
    safe = next((j for j, (_, lg) in enumerate(trace[:n]) if float(lg.topk(2).values[0] - lg.topk(2).values[1]) < TOL), n)
    first = eng.prefill(0, ids)
    m0 = eng.get_option("mega_launches")
    got, _ = eng.generate_greedy([0], first.view(1, -1), n, gamma=0)
    assert got[0].tolist()[:safe] == ref[:safe]
    if path == 0:
        assert eng.get_option("mega_launches") > m0, "the persistent kernel should run the merged weights"


def test_merged_adapter_differs_from_exact_mode_and_toggles():
    """The bf16 merge is a different numerics mode from the exact fp32 adapter (the default),
    and the option switches back."""
    eng, m16, m32, cfg = _setup()
    ids = random_prompts(1, 16, cfg.vocab_size, seed=5)[0].tolist()
    a = eng.prefill(0, ids).cpu()
    eng.set_option("merged_adapter", 0)
    b = eng.prefill(0, ids).cpu()
    kv = O.OracleKV(m32, 32)
    assert (b - O.prefill(m32, ids, kv)).abs().max().item() <= TOL
    assert (a - b).abs().max().item() > 0
    eng.set_option("merged_adapter", 1)


def test_merged_adapter_is_a_no_op_without_adapter():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    eng = DeviceEngine(cfg, make_state_dict(cfg, recipe="A", seed=0), device=0, max_batch=1, max_seq_len=64,
                       max_prefill=16)
    try:
        eng.set_option("merged_adapter", 1)
        assert eng.get_option("loop_adapter") == 0 and eng.get_option("merged_adapter") == 0
    finally:
        eng.close()
