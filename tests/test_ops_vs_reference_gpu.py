"""The pulsar_cuda shim ops against the reference's own CUDA kernels, built from its
csrc/kernels.cu + csrc/pulsar_cuda.cpp for sm_100a by oracle/build_ref_ops.py. Both run on the
same B200, on the same inputs at the model's shapes: d_model 1024, 16 heads of 64, 16 routed
experts, top-4, 2048 tokens.

The reference is built with -use_fast_math, as its setup.py builds it. Its exponentials,
reciprocals and square roots therefore differ from IEEE results in the last bits. bf16 outputs
must agree within one bf16 rounding step (relative 2^-7, plus a small absolute floor). Integer
outputs (top-k ids, dispatch copies) must agree exactly. Skipped when the reference module has
not been built (no reference tree where the repository was built)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

N, D, H, DH, E, K = 2048, 1024, 16, 64, 16, 4
CAP = 640   # ceil(N * K / E * 1.25) rounded up to 32


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from oracle import build_ref_ops
    ref = build_ref_ops.load()
    if ref is None:
        pytest.skip("reference ops not built (python oracle/build_ref_ops.py)")
    import pulsar_cuda
    return pulsar_cuda, ref


def _bf16(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device="cuda", dtype=torch.bfloat16)


def _close_bf16(a, b, what, rtol=2.0 ** -7, atol=1e-2):
    a, b = a.float(), b.float()
    bad = (a - b).abs() > atol + rtol * b.abs()
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} of {b.numel()} differ, worst {(a - b).abs().max().item():.3e}"


def _routes(seed=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda()
    slots = torch.full((N, K), -1, dtype=torch.int32)
    fill = [0] * E
    for t in range(N):
        for k in range(K):
            e = int(idx[t, k])
            if fill[e] < CAP:
                slots[t, k] = fill[e]
                fill[e] += 1
    w = torch.rand(N, K, generator=g)
    return idx, slots.cuda(), (w / w.sum(-1, keepdim=True)).to("cuda", torch.bfloat16), torch.tensor(fill).cuda()


def test_rmsnorm(mods):
    pc, ref = mods
    x = _bf16(N, D, seed=2)
    w = torch.rand(D, device="cuda") + 0.5
    y1, r1 = pc.rmsnorm_forward(x, w, 1e-6)
    y2, r2 = ref.rmsnorm_forward(x, w, 1e-6)
    _close_bf16(y1, y2, "rmsnorm y")
    assert torch.allclose(r1.float().reshape(-1), r2.float().reshape(-1), rtol=1e-5, atol=0)


def test_router_topk(mods):
    pc, ref = mods
    g = torch.Generator(device="cpu").manual_seed(10)
    logits = torch.randn(N, E, generator=g).cuda()
    bias = (torch.randn(E, generator=g) * 0.1).cuda()
    i1, w1, z1, p1 = pc.moe_router_topk_forward(logits, bias, K, 1e-3)
    i2, w2, z2, p2 = ref.moe_router_topk_forward(logits, bias, K, 1e-3)
    assert torch.equal(i1.long(), i2.long()), "top-k ids differ"
    _close_bf16(w1, w2, "router weights (bf16)", atol=1e-3)
    assert torch.allclose(p1.float(), p2.float(), rtol=1e-4, atol=1e-7)
    assert torch.allclose(z1.float(), z2.float(), rtol=1e-4, atol=0)


def test_dispatch_and_combine(mods):
    pc, ref = mods
    idx, slots, tw, fill = _routes()
    x = _bf16(N, D, seed=3)
    (e1,) = pc.moe_dispatch_forward(x, idx, slots, E, CAP, fill)
    (e2,) = ref.moe_dispatch_forward(x, idx, slots, E, CAP, fill)
    assert torch.equal(e1, e2), "dispatch buffers differ"
    eo = _bf16(E, CAP, D, seed=4)
    sh = _bf16(N, D, seed=5)
    _close_bf16(pc.moe_combine_forward(eo, idx, tw, slots, sh), ref.moe_combine_forward(eo, idx, tw, slots, sh),
                "combine")
    _close_bf16(pc.moe_combine_forward(eo, idx, tw, slots), ref.moe_combine_forward(eo, idx, tw, slots),
                "combine without shared")


def test_conv_swiglu_gate(mods):
    pc, ref = mods
    x = _bf16(4, 512, D, seed=6)
    w = torch.randn(D, 4, device="cuda") * 0.3
    _close_bf16(pc.causal_depthwise_conv1d_k4_forward(x, w), ref.causal_depthwise_conv1d_k4_forward(x, w), "conv")
    gu = _bf16(N, 2 * 512, seed=7)
    _close_bf16(pc.fused_swiglu_forward(gu, 512), ref.fused_swiglu_forward(gu, 512), "swiglu")
    a = _bf16(2, H, 512, DH, seed=8)
    g = torch.randn(2, 512, H, device="cuda")
    _close_bf16(pc.fused_attn_gate_forward(a, g), ref.fused_attn_gate_forward(a, g), "attn gate")


def test_rope_and_qk_norm(mods):
    pc, ref = mods
    T = 512
    pos = torch.arange(T, device="cuda", dtype=torch.float32)
    inv = 1.0 / (10000.0 ** (torch.arange(0, DH, 2, device="cuda", dtype=torch.float32) / DH))
    ang = torch.outer(pos, inv)
    cos, sin = ang.cos(), ang.sin()
    q = _bf16(2, H, T, DH, seed=9)
    _close_bf16(pc.rope_forward(q, cos, sin), ref.rope_forward(q, cos, sin), "rope")
    wq = torch.rand(H, DH, device="cuda") + 0.5
    y1, _ = pc.qk_rmsnorm_rope_forward(q, wq, cos, sin, T, 1e-6)
    y2, _ = ref.qk_rmsnorm_rope_forward(q, wq, cos, sin, T, 1e-6)
    _close_bf16(y1, y2, "qk_rmsnorm_rope")
