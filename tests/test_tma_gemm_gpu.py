"""The TMA-fed warp-specialised GEMM (k_tma_gemm, engine option "tma_gemm") against the
cp.async-fed kernel (k_tc_gemm). Both issue the same tcgen05 MMAs per output element in the same
order (per 64-wide K chunk, four K steps of 16, each activation hi then lo into one fp32
accumulator). Their results must therefore be bit-identical, for every epilogue (STORE, ADD,
SWIGLU, softcap LM head), for 128- and 64-column tiles, and for batched expert GEMMs. The
check runs through the prefill (M = T rows) and the many-row decode path (batched verify
passes)."""

from __future__ import annotations

import pytest
import torch

from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    e = DeviceEngine(cfg, make_state_dict(cfg, recipe="A", seed=0), device=0, max_batch=64, max_seq_len=1024,
                     max_prefill=1024)
    yield e, cfg
    e.close()


@pytest.mark.parametrize("T", [96, 1000])
def test_prefill_identical(eng, T):
    e, cfg = eng
    ids = random_prompts(1, T, cfg.vocab_size, seed=T)[0].tolist()
    assert e.get_option("tma_gemm") == 1
    a = e.prefill(0, ids).cpu()
    ka, va = e.read_kv(0, 5, 0, min(T, 64))
    try:
        e.set_option("tma_gemm", 0)
        b = e.prefill(0, ids).cpu()
        kb, vb = e.read_kv(0, 5, 0, min(T, 64))
    finally:
        e.set_option("tma_gemm", 1)
    assert torch.equal(a, b), f"prefill logits differ by {(a - b).abs().max().item():.3e}"
    assert torch.equal(ka, kb) and torch.equal(va, vb)


def test_many_row_decode_identical(eng):
    """48 sequences, gamma 4: verify passes of 240 rows run the wide path's GEMMs (QKV, Wo,
    shared and routed experts, LM head with softcap)."""
    e, cfg = eng
    P = random_prompts(48, 64, cfg.vocab_size, seed=1)
    e.set_option("wide", 1)
    try:
        outs = []
        for tma in (1, 0):
            e.set_option("tma_gemm", tma)
            first = torch.stack([e.prefill(i, P[i].tolist()) for i in range(48)])
            got, st = e.generate_greedy(list(range(48)), first, 24, gamma=4)
            outs.append((got.cpu(), first.cpu(), st))
    finally:
        e.set_option("tma_gemm", 1)
        e.set_option("wide", 0)
    assert torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][0], outs[1][0])
    assert outs[0][2] == outs[1][2]
