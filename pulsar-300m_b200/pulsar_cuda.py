"""Drop-in ``pulsar_cuda`` module: the reference extension's forward op names and
signatures (csrc/pulsar_cuda.cpp:199-279), served by the sm_100a kernels of
``libpulsar_b200.so`` through its C ABI.

Put the directory holding this file on ``sys.path`` ahead of the reference's own build and
``src/model.py`` (``import pulsar_cuda``, src/model.py:109-113) picks these ops up
unchanged. Outputs are freshly allocated torch tensors on the input's device, kernels run
on torch's current CUDA stream, and argument errors raise ``RuntimeError`` with the
reference's TORCH_CHECK message text. Backward ops belong to training and are out of scope
for this engine: they raise ``NotImplementedError``.
"""

from __future__ import annotations

import torch

from pulsar_b200 import _lib

_lib.load()   # fail loudly at import time when the library is not built (no fallback)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def rmsnorm_forward(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """csrc/kernels.cu:224-266: (y bf16 like x, rsqrt f32 [rows])."""
    _check(x.is_cuda and x.is_contiguous(), "x must be a contiguous CUDA tensor")
    _check(x.dtype == torch.bfloat16, "x must be bfloat16")
    _check(weight.dtype == torch.float32, "weight must be float32")
    dim = x.shape[-1]
    rows = x.numel() // dim if dim else 0
    y = torch.empty_like(x)
    rs = torch.empty(rows, dtype=torch.float32, device=x.device)
    if rows:
        _lib.call("pulsar_op_rmsnorm", _p(x), _p(weight.contiguous()), rows, dim, float(eps), _p(y), _p(rs), _stream(x))
    return [y, rs]


def rope_forward(qk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """csrc/kernels.cu:935-966: half-split rotation of [B, H, T, Dh], position = row % T."""
    _check(qk.is_cuda and qk.is_contiguous(), "qk must be a contiguous CUDA tensor")
    _check(qk.dtype == torch.bfloat16, "qk must be bfloat16")
    out = torch.empty_like(qk)
    if qk.numel() == 0:
        return out
    B, Hh, T, Dh = qk.shape
    cos_f = cos.float().contiguous()
    sin_f = sin.float().contiguous()
    _lib.call("pulsar_op_rope", _p(qk), _p(cos_f), _p(sin_f), B * Hh * T, T, Dh, _p(out), _stream(qk))
    return out


def fused_swiglu_forward(gu: torch.Tensor, d_ff: int):
    """csrc/kernels.cu:825-863: silu(gu[..., :d_ff]) * gu[..., d_ff:] in fp32, bf16 out."""
    _check(gu.is_cuda and gu.is_contiguous(), "gu must be a contiguous CUDA tensor")
    _check(gu.dtype == torch.bfloat16, "gu must be bfloat16")
    sizes = list(gu.shape)
    sizes[-1] = d_ff
    out = torch.empty(sizes, dtype=gu.dtype, device=gu.device)
    if gu.numel() == 0:
        return out
    rows = gu.numel() // (2 * d_ff)
    _lib.call("pulsar_op_swiglu", _p(gu), rows, int(d_ff), _p(out), _stream(gu))
    return out


def moe_router_topk_forward(logits: torch.Tensor, expert_bias: torch.Tensor, top_k=2, z_loss_weight: float = 1e-4):
    """csrc/kernels.cu:2417-2491 (both bindings, csrc/pulsar_cuda.cpp:244-255):
    (topk_idx i64 [N,K], topk_weights bf16 [N,K], z_loss f32 [], probs_mean f32 [E])."""
    if isinstance(top_k, float):        # overload (logits, expert_bias, z_loss_weight)
        top_k, z_loss_weight = 2, top_k
    _check(logits.is_cuda, "logits must be a CUDA tensor")
    _check(expert_bias.is_cuda, "expert_bias must be a CUDA tensor")
    _check(logits.is_contiguous(), "logits must be contiguous")
    _check(expert_bias.is_contiguous(), "expert_bias must be contiguous")
    _check(logits.dim() == 2, "logits must be 2D [N, E]")
    N, E = logits.shape
    _check(E <= 32, f"moe_router_topk_forward_cuda supports E <= 32, got {E}")
    _check(0 < top_k <= 8 and top_k <= E, f"top_k must be in [1, min(8, E)], got {top_k}")
    _check(expert_bias.shape[0] == E, "expert_bias size must match E")
    _check(logits.dtype in (torch.float32, torch.bfloat16), "logits must be float32 or bfloat16")
    _check(expert_bias.dtype == torch.float32, "expert_bias must be float32")
    dev = logits.device
    idx = torch.empty(N, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(N, top_k, dtype=torch.bfloat16, device=dev)
    z = torch.zeros((), dtype=torch.float32, device=dev)
    pm = torch.zeros(E, dtype=torch.float32, device=dev)
    ws = torch.empty(max(1, N * (E + 1)), dtype=torch.float32, device=dev)
    _lib.call("pulsar_op_moe_router_topk", _p(logits), 1 if logits.dtype == torch.bfloat16 else 0, _p(expert_bias),
              N, E, int(top_k), float(z_loss_weight), _p(idx), _p(w), _p(z), _p(pm), _p(ws), _stream(logits))
    return [idx, w, z, pm]


def qk_rmsnorm_rope_forward(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, T: int,
                            eps: float = 1e-6):
    """csrc/kernels.cu:2716-2765: per-head RMSNorm then RoPE, strided input allowed
    (stride(-1) == 1), contiguous output, plus per-vector rsqrt."""
    head_dim = x.shape[-1]
    total = x.numel() // head_dim if head_dim else 0
    num_heads = weight.shape[0]
    _check(head_dim == 64, f"qk_rmsnorm_rope requires head_dim == 64, got {head_dim}")
    _check(x.stride(-1) == 1, f"qk_rmsnorm_rope requires stride(-1) == 1, got {x.stride(-1)}")
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(x.dtype == torch.bfloat16, "x must be bfloat16")
    _check(weight.is_cuda and weight.is_contiguous(), "weight must be contiguous CUDA")
    _check(weight.dtype == torch.float32, "weight must be float32")
    cos_f = cos.float().contiguous()
    sin_f = sin.float().contiguous()
    if x.dim() == 4:
        sB, sH, sT = x.stride(0), x.stride(1), x.stride(2)
    else:
        sB, sH, sT = num_heads * T * 64, T * 64, 64
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    rs = torch.empty(total, dtype=torch.float32, device=x.device)
    if total:
        _lib.call("pulsar_op_qk_rmsnorm_rope", _p(x), sB, sH, sT, total, num_heads, int(T), _p(weight), _p(cos_f),
                  _p(sin_f), float(eps), _p(y), _p(rs), _stream(x))
    return [y, rs]


def fused_attn_gate_forward(attn_out: torch.Tensor, gate_logits: torch.Tensor):
    """csrc/kernels.cu:2930-2958: out[b,t,h*64+d] = attn[b,h,t,d] * sigmoid(gate[b,t,h])."""
    B, Hh, T, Dh = attn_out.shape
    _check(Dh == 64, f"fused_attn_gate requires head_dim == 64, got {Dh}")
    _check(attn_out.is_cuda and attn_out.is_contiguous(), "attn_out must be contiguous CUDA")
    _check(attn_out.dtype == torch.bfloat16, "attn_out must be bfloat16")
    gl = gate_logits.float().contiguous()
    out = torch.empty(B, T, Hh * Dh, dtype=attn_out.dtype, device=attn_out.device)
    if out.numel():
        _lib.call("pulsar_op_attn_gate", _p(attn_out), _p(gl), B, Hh, T, _p(out), _stream(attn_out))
    return out


def causal_depthwise_conv1d_k4_forward(x: torch.Tensor, weight: torch.Tensor):
    """csrc/kernels.cu:3653-3691: y[b,t,d] = x + sum_k w[d,k] x[b,t-k,d] (zero-padded)."""
    _check(x.is_cuda and weight.is_cuda, "Inputs must be CUDA tensors")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(weight.is_contiguous(), "weight must be contiguous")
    _check(x.dtype == torch.bfloat16, "x must be bfloat16")
    _check(weight.dtype == torch.float32, "weight must be float32")
    _check(x.dim() == 3, "x must be [B, T, D]")
    _check(weight.dim() == 2 and weight.shape[1] == 4, "weight must be [D, 4]")
    B, T, Dd = x.shape
    _check(weight.shape[0] == Dd, "weight dim 0 must match D")
    y = torch.empty_like(x)
    if B * T:
        _lib.call("pulsar_op_conv1d_k4", _p(x), _p(weight), B, T, Dd, _p(y), _stream(x))
    return y


def moe_combine_forward(expert_outputs, topk_idx, topk_weights, token_to_slot, shared_out=None):
    """csrc/kernels.cu:1633-1664: out[t] = shared[t] + sum_k w_tk * expert_outputs[e_tk, slot_tk]."""
    N, K = topk_idx.shape
    E, Cc, Dd = expert_outputs.shape
    out = torch.empty(N, Dd, dtype=expert_outputs.dtype, device=expert_outputs.device)
    if N:
        sh = shared_out.contiguous() if (shared_out is not None and shared_out.numel() > 0) else None
        _lib.call("pulsar_op_moe_combine", _p(expert_outputs.contiguous()), _p(topk_idx.contiguous()),
                  _p(topk_weights.to(torch.bfloat16).contiguous()), _p(token_to_slot.contiguous()), _p(sh),
                  N, K, E, Cc, Dd, _p(out), _stream(expert_outputs))
    return out


def moe_dispatch_forward(x, topk_idx, token_to_slot, num_experts, capacity, expert_counts=None):
    """csrc/kernels.cu:1548-1605: [expert_inputs [E, C, D]] with unused slots zeroed."""
    N, Dd = x.shape
    K = topk_idx.shape[1]
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(topk_idx.is_cuda, "topk_idx must be a CUDA tensor")
    _check(token_to_slot.is_cuda, "token_to_slot must be a CUDA tensor")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(topk_idx.is_contiguous(), "topk_idx must be contiguous")
    _check(token_to_slot.is_contiguous(), "token_to_slot must be contiguous")
    _check(x.dtype == torch.bfloat16, "x must be bfloat16")
    _check(topk_idx.dtype == torch.int64, "topk_idx must be int64")
    _check(token_to_slot.dtype == torch.int32, "token_to_slot must be int32")
    _check(tuple(token_to_slot.shape) == (N, K), "token_to_slot must be [N, K]")
    _check(Dd % 8 == 0, f"D must be a multiple of 8 for vectorised dispatch, got {Dd}")
    E, Cc = int(num_experts), int(capacity)
    ei = torch.empty(E, Cc, Dd, dtype=x.dtype, device=x.device)
    if expert_counts is not None:
        _check(expert_counts.is_cuda, "expert_counts must be a CUDA tensor")
        _check(expert_counts.is_contiguous(), "expert_counts must be contiguous")
        _check(expert_counts.dtype == torch.int64, "expert_counts must be int64")
        _check(expert_counts.numel() >= E, "expert_counts must have at least E elements")
    _lib.call("pulsar_op_moe_dispatch", _p(x), _p(topk_idx), _p(token_to_slot), _p(expert_counts), N, K, E, Cc, Dd,
              _p(ei), _stream(x))
    return [ei]


def _backward_out_of_scope(name):
    def f(*args, **kwargs):
        raise NotImplementedError(f"pulsar_cuda.{name}: backward/training ops are out of scope for the decode engine")
    f.__name__ = name
    return f


for _n in ("rmsnorm_backward", "fused_add_rmsnorm_backward", "fused_swiglu_backward", "moe_dispatch_backward",
           "moe_combine_backward", "qk_rmsnorm_backward", "qk_rmsnorm_rope_backward", "fused_attn_gate_backward",
           "moe_router_topk_backward", "causal_depthwise_conv1d_k4_backward", "fused_harmonic_residual_backward",
           "fused_softcap_ce_backward", "fused_softcap_ce_backward_dev"):
    globals()[_n] = _backward_out_of_scope(_n)
