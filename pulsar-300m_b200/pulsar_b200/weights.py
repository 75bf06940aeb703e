"""Seeded synthetic Pulsar weights with the reference's state_dict names and shapes.

No trained checkpoint is available offline, so every parity test and benchmark runs on
random-init weights generated here. The generator is deterministic (CPU
``torch.Generator``), so this container and the GPU box produce bit-identical tensors.

Two recipes:

* ``"A"`` - the reference's own init distributions (src/model.py:1773-1789 for linears and
  embeddings, :1225-1233 for routed experts and router, :709-713 for the loop adapter,
  :1755-1767 for the re-injection gate). Under this init the model copies its input token
  (top-1 margin about 5), so greedy decoding is trivially stable.
* ``"B"`` - recipe A, then every >=2-D tensor whose name contains none of ``norm``,
  ``tok_emb``, ``lm_head``, ``router`` is redrawn from N(0, 0.09^2) with a second
  generator; ``stem_canon_weight`` is drawn from N(0, 0.02^2) so the decode-time
  single-token conv quirk is exercised; RMSNorm gains become 1 + N(0, 0.1^2) and the
  per-pulse expert bias N(0, 0.05^2), so per-pulse indexing mistakes cannot hide behind
  all-ones / all-zeros tensors. Draft/verify agreement is then far from 100%.

Tensors that the reference's precision policy keeps in bf16 (src/model.py:1661-1728:
>=2-D and none of the FP32 substrings) are rounded to bf16-representable values, so the
fp32 CPU oracle and the bf16 device engine start from identical weight values.
"""

from __future__ import annotations

import math
from collections import OrderedDict

import torch

from .config import PulsarConfig

# src/model.py:1661-1677
FP32_PARAM_SUBSTRINGS = (
    "norm", "bias", "router", "mix_logit", "reinject_gate", "lora_", "loop_M",
    "canon_weight", "res_scale", "routed_scale", "attn_gate", "pulse_step_emb",
    "v_resid_lambda", "q_norm_weight", "k_norm_weight",
)


def is_bf16_param(name: str, ndim: int) -> bool:
    """True when the reference casts this tensor to bf16 (src/model.py:1727-1728)."""
    if ndim <= 1:
        return False
    return not any(s in name for s in FP32_PARAM_SUBSTRINGS)


def param_specs(cfg: PulsarConfig):
    """(name, shape, init) for every tensor of the state_dict, in a fixed order.

    ``init`` is one of ("normal", std), ("zeros",), ("ones",), ("const", v), ("eye",).
    """
    D, V, P = cfg.d_model, cfg.vocab_size, cfg.max_pulses
    qkv = cfg.qkv_dim
    q = cfg.loop_lora_rank
    r = cfg.reinject_gate_rank
    E, de, ds = cfg.n_routed_experts, cfg.d_expert, cfg.d_shared
    resid_std = 0.02 / math.sqrt(2 * cfg.n_core * cfg.default_pulses)
    routed_down_std = resid_std * math.sqrt((ds / de) * cfg.top_k)
    specs = [
        ("tok_emb.weight", (V, D), ("normal", 0.006)),
        ("pulse_step_emb.weight", (P, D), ("zeros",)),
        ("pulse_state_norm.weight", (D,), ("ones",)),
        ("anchor_norm.weight", (D,), ("ones",)),
        ("stem_canon_weight", (D, cfg.canon_kernel_size), ("zeros",)),
        ("reinject_gate_down", (P, r, 2 * D), ("normal", 0.02)),
        ("reinject_gate_up", (P, D, r), ("zeros",)),
        ("reinject_gate_bias", (P, D), ("zeros",)),
        ("pulse_res_scale", (P, D), ("ones",)),
        ("final_norm.weight", (D,), ("ones",)),
    ]
    for i in range(cfg.n_core):
        b = f"core.{i}."
        specs += [
            (b + "attn_norm.weight", (P, D), ("ones",)),
            (b + "attn.q_norm_weight", (P, cfg.n_heads, cfg.head_dim), ("ones",)),
            (b + "attn.k_norm_weight", (P, cfg.n_kv_heads, cfg.head_dim), ("ones",)),
            (b + "attn.v_resid_lambda", (P,), ("const", -2.2)),
            (b + "attn.attn_gate", (P, cfg.n_heads, D), ("zeros",)),
            (b + "attn.attn_gate_bias", (P, cfg.n_heads), ("const", 2.0)),
            (b + "attn.wqkv.weight", (qkv, D), ("normal", 0.02)),
            (b + "attn.wo.weight", (D, cfg.q_dim), ("normal", resid_std)),
            (b + "attn.wqkv_adapter.lora_A", (P, q, D), ("normal", 1.0 / math.sqrt(D))),
            (b + "attn.wqkv_adapter.lora_B", (P, qkv, q), ("zeros",)),
            (b + "attn.wqkv_adapter.loop_M", (P, P), ("eye",)),
            (b + "attn.wo_adapter.lora_A", (P, q, cfg.q_dim), ("normal", 1.0 / math.sqrt(cfg.q_dim))),
            (b + "attn.wo_adapter.lora_B", (P, D, q), ("zeros",)),
            (b + "attn.wo_adapter.loop_M", (P, P), ("eye",)),
            (b + "mlp_norm.weight", (P, D), ("ones",)),
            (b + "mlp.routed_gate_up", (E, D, 2 * de), ("normal", 0.02)),
            (b + "mlp.routed_down", (E, de, D), ("normal", routed_down_std)),
            (b + "mlp.router_weight", (P, E, D), ("normal", 0.002)),
            (b + "mlp.routed_scale", (P, D), ("ones",)),
            (b + "mlp.expert_bias", (P, E) if cfg.per_pulse_bias else (E,), ("zeros",)),
            (b + "mlp.expert_counts_accum", (E,), ("zeros",)),
            (b + "mlp.expert_pulse_counts", (P, E), ("zeros",)),
            (b + "mlp.shared_expert.w_gate_up.weight", (2 * ds, D), ("normal", 0.02)),
            (b + "mlp.shared_expert.w_down.weight", (D, ds), ("normal", resid_std)),
        ]
    return specs


_NOT_REDRAWN_B = ("norm", "tok_emb", "lm_head", "router", "expert_counts", "expert_pulse_counts")


def _init(shape, init, gen):
    kind = init[0]
    if kind == "normal":
        return torch.randn(shape, generator=gen, dtype=torch.float32) * init[1]
    if kind == "zeros":
        return torch.zeros(shape, dtype=torch.float32)
    if kind == "ones":
        return torch.ones(shape, dtype=torch.float32)
    if kind == "const":
        return torch.full(shape, float(init[1]), dtype=torch.float32)
    if kind == "eye":
        return torch.eye(shape[0], shape[1], dtype=torch.float32)
    raise ValueError(init)


def make_state_dict(cfg: PulsarConfig | None = None, recipe: str = "A", seed: int = 0,
                    b_std: float = 0.09) -> "OrderedDict[str, torch.Tensor]":
    """Deterministic synthetic state_dict (fp32 tensors; bf16-class ones bf16-exact).

    ``lm_head.weight`` is the same tensor object as ``tok_emb.weight`` (weight tying,
    src/model.py:1775). ``b_std`` is recipe B's redraw scale (0.09 for the production
    shapes; small test configs need a larger one to leave the copy regime).
    """
    cfg = cfg or PulsarConfig()
    recipe = recipe.upper()
    if recipe not in ("A", "B"):
        raise ValueError(f"unknown weight recipe {recipe!r} (expected 'A' or 'B')")
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    specs = param_specs(cfg)
    sd: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    for name, shape, init in specs:
        sd[name] = _init(shape, init, g)
    if recipe == "B":
        g2 = torch.Generator(device="cpu").manual_seed(int(seed) + 1)
        for name, shape, _ in specs:
            t = sd[name]
            if name == "stem_canon_weight":
                sd[name] = torch.randn(shape, generator=g2) * 0.02
            elif t.ndim >= 2 and not any(s in name for s in _NOT_REDRAWN_B):
                sd[name] = torch.randn(shape, generator=g2) * b_std
            elif "norm" in name:
                sd[name] = 1.0 + 0.1 * torch.randn(shape, generator=g2)
            elif name.endswith("expert_bias"):
                sd[name] = 0.05 * torch.randn(shape, generator=g2)
    for name, shape, _ in specs:
        if is_bf16_param(name, len(shape)):
            sd[name] = sd[name].to(torch.bfloat16).to(torch.float32)
    sd["lm_head.weight"] = sd["tok_emb.weight"]
    return sd


def random_prompts(batch: int, length: int, vocab: int, seed: int = 0) -> torch.Tensor:
    """Uniform random token ids ``[batch, length]`` (int64), row-major from one generator."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randint(0, vocab, (batch, length), generator=g, dtype=torch.int64)


def save_checkpoint(path: str, state_dict, cfg: PulsarConfig) -> None:
    """Write ``{"model": state_dict, "config": cfg_dict}``, the layout src/infer.py:804-809 reads."""
    torch.save({"model": dict(state_dict), "config": cfg.to_dict()}, path)
