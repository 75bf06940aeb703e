"""The decode attention of the per-op and many-row passes (pulsar_engine_decode_attention):
the tensor-core kernel k_attn_dec_tc and the SIMT k_attn_flash against a plain fp64-accumulated
torch restatement of the op (src/infer.py:290-306 per row: softmax(q k^T / 8) v over the keys
the slot caches at positions 0..pos, the last 1024 of them on a local layer), on random queries
over the cached K/V of real prefills.

Cases: one row per block and verify blocks of 5 and 8 rows (runs of consecutive positions of
one slot; a block of 8 holding rows of two slots is cut into two runs), local layers past the
2048-entry ring (positions 2050+ read ring entries that hold positions 2..), global layers over
2300 keys, short contexts (5 keys) whose later splits see nothing, and an invalid row (output
0). Outputs are convex combinations of V rows of magnitude ~1: max abs error 1e-5 for the fp32
SIMT kernel, 5e-5 for the tensor-core kernel (Q and P enter the MMAs as bf16 hi + lo halves,
which leave 2^-16 of each unrepresented)."""

from __future__ import annotations

import pytest
import torch

from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu
LOCAL = (0, 1, 2, 4, 5, 6)
_CACHE = {}


def _setup(kv):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    if kv not in _CACHE:
        for k in list(_CACHE):
            _CACHE.pop(k)[0].close()
        cfg = PulsarConfig(eos_token_id=-1)
        eng = DeviceEngine(cfg, make_state_dict(cfg, recipe="A", seed=0), device=0, max_batch=4, max_seq_len=2304,
                           max_prefill=2048, kv_dtype=kv)
        for slot, T in ((0, 2048), (1, 300), (2, 5)):
            eng.prefill(slot, random_prompts(1, T, cfg.vocab_size, seed=slot + 1)[0].tolist())
        _CACHE[kv] = (eng, cfg)
    return _CACHE[kv]


def _torch_decode_attention(eng, layer, rows, q):
    """fp64-accumulated reference: q [R, 16, 64] unscaled; rows [(slot, pos)]."""
    out = torch.zeros_like(q)
    for r, (slot, pos) in enumerate(rows):
        if not (0 <= slot < 4 and 0 <= pos < 2304):
            continue
        lo = max(0, pos - 1023) if layer in LOCAL else 0
        K, V = eng.read_kv(slot, layer, lo, pos - lo + 1)   # [4, n, 64]
        kk = K.repeat_interleave(4, dim=0).double()          # head h reads kv head h // 4
        vv = V.repeat_interleave(4, dim=0).double()
        sc = torch.einsum("hd,hsd->hs", q[r].double() * 0.125, kk)
        out[r] = torch.einsum("hs,hsd->hd", torch.softmax(sc, dim=-1), vv).float()
    return out


CASES = {
    "one-row": (1, [(0, 2050), (0, 2303), (1, 300), (1, 150), (2, 5), (0, 1500), (1, 299), (2, 0)]),
    "verify-5": (5, [(0, 2050 + i) for i in range(5)] + [(1, 300 + i) for i in range(5)] +
                 [(2, 5 + i) for i in range(5)]),
    "verify-8-two-runs": (8, [(0, 1030 + i) for i in range(5)] + [(2, 6 + i) for i in range(3)] +
                          [(1, 296 + i) for i in range(8)]),
    "invalid-row": (5, [(1, 300), (1, 301), (9, 302), (1, 303), (1, 10**6)]),
}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("layer", [0, 3, 5, 7])
def test_decode_attention_kernels_vs_torch(case, layer):
    eng, cfg = _setup(torch.bfloat16)
    assert eng.get_option("tc_dec_attn") == 1
    rpb, rows = CASES[case]
    g = torch.Generator().manual_seed(10 * list(CASES).index(case) + layer)
    q = torch.randn(len(rows), 16, 64, generator=g) * 2.0
    ref = _torch_decode_attention(eng, layer, rows, q)
    for tc in (True, False):
        got = eng.decode_attention(layer, rows, q.cuda(), tensor_cores=tc, rows_per_block=rpb).cpu()
        err = (got - ref).abs().max().item()
        assert err <= (5e-5 if tc else 1e-5), (f"{'tensor-core' if tc else 'SIMT'} decode attention, {case}, "
                                               f"layer {layer}: max |err| {err:.3e}")
    assert eng.get_option("tc_dec_attn") == 1, "the check restores the engine option"


def test_many_rows_one_row_blocks():
    """64 rows (fewer splits per row, several chunks per split) on a global and a local layer."""
    eng, cfg = _setup(torch.bfloat16)
    rows = [(s, p) for s, p0 in ((0, 2100), (1, 250), (2, 3)) for p in range(p0, p0 + 21)] + [(0, 2303)]
    g = torch.Generator().manual_seed(7)
    q = torch.randn(len(rows), 16, 64, generator=g)
    for layer in (2, 7):
        ref = _torch_decode_attention(eng, layer, rows, q)
        got = eng.decode_attention(layer, rows, q.cuda(), tensor_cores=True).cpu()
        assert (got - ref).abs().max().item() <= 5e-5


def test_fp32_cache_takes_the_simt_kernel():
    eng, cfg = _setup(torch.float32)
    assert eng.get_option("tc_dec_attn") == 0
    rpb, rows = CASES["verify-5"]
    q = torch.randn(len(rows), 16, 64, generator=torch.Generator().manual_seed(3))
    ref = _torch_decode_attention(eng, 3, rows, q)
    got = eng.decode_attention(3, rows, q.cuda(), tensor_cores=True, rows_per_block=rpb).cpu()
    assert (got - ref).abs().max().item() <= 1e-5
