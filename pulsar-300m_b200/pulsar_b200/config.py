"""Model configuration for the Pulsar decode engine.

Field names, defaults and the warn-on-unknown-keys ``from_dict`` behaviour follow the
reference ``PulsarConfig`` (src/model.py:13-106) so that a checkpoint's ``config`` dict
loads unchanged. Only the fields the inference path reads are interpreted; the training
fields are kept so round-trips through ``to_dict`` stay lossless.
"""

from __future__ import annotations

import json
import warnings
from dataclasses import asdict, dataclass

# Attention layers that use the sliding window (src/infer.py:93, src/model.py:771).
LOCAL_LAYERS = (0, 1, 2, 4, 5, 6)


@dataclass
class PulsarConfig:
    vocab_size: int = 32768
    d_model: int = 1024
    n_heads: int = 16
    n_kv_heads: int = 4
    head_dim: int = 64
    d_expert: int = 512
    d_shared: int | None = None
    n_core: int = 8
    max_pulses: int = 8
    default_pulses: int = 3
    reinject_gate_rank: int = 8
    loop_lora_rank: int = 8
    loop_lora_alpha: float = 16.0
    use_canon_conv: bool = True
    canon_kernel_size: int = 4
    base_seq_len: int = 1024
    max_seq_len: int = 32768
    rope_theta_local: float = 10000.0
    rope_theta_global: float = 1000000.0
    sliding_window: int = 1024
    local_attn_impl: str = "auto"
    n_routed_experts: int = 16
    top_k: int = 4
    eos_token_id: int = 0
    rms_eps: float = 1e-6
    ce_chunk_size: int = 32768
    router_z_loss_weight: float = 1e-3
    router_balance_loss_weight: float = 0.01
    aux_loss_weight_1: float = 0.15
    aux_loss_weight_2: float = 0.25
    final_loss_weight: float = 0.60
    logit_softcap: float = 30.0
    moe_capacity_factor: float = 1.25
    moe_capacity_align: int = 32
    moe_grouped_mm: bool = False
    per_pulse_bias: bool = True

    def __post_init__(self):
        # src/model.py:70-72
        if self.d_shared is None:
            self.d_shared = 1024 if self.d_model >= 1024 else self.d_expert

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict, *, strict: bool = False) -> "PulsarConfig":
        """Build a config from a dict; unknown keys warn (or raise with ``strict``)."""
        valid = set(cls.__dataclass_fields__.keys())
        unknown = sorted(set(d) - valid)
        if unknown:
            msg = (f"unknown PulsarConfig key(s): {', '.join(unknown)}. "
                   f"These were previously ignored silently; the value is NOT in effect.")
            if strict:
                raise ValueError(msg)
            warnings.warn(msg, RuntimeWarning, stacklevel=2)
        return cls(**{k: v for k, v in d.items() if k in valid})

    def to_json(self, path: str):
        with open(path, "w", encoding="utf-8") as f:
            json.dump(self.to_dict(), f, indent=2)

    @classmethod
    def from_json(cls, path: str) -> "PulsarConfig":
        with open(path, "r", encoding="utf-8") as f:
            return cls.from_dict(json.load(f))

    # ---- derived sizes used by the engine ----
    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def is_local(self, layer: int) -> bool:
        return layer in LOCAL_LAYERS


def engine_supported(cfg: PulsarConfig) -> str | None:
    """Return None if the CUDA engine's compiled shapes match ``cfg``, else the reason.

    The sm_100a kernels are specialised for the Pulsar-283M shapes (the ones every
    BASELINE config uses); other shapes are served only by the CPU oracle in tests.
    """
    want = dict(d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64, d_expert=512,
                d_shared=1024, n_core=8, n_routed_experts=16, top_k=4,
                reinject_gate_rank=8, canon_kernel_size=4)
    for k, v in want.items():
        if getattr(cfg, k) != v:
            return f"{k}={getattr(cfg, k)} (engine is compiled for {k}={v})"
    if cfg.default_pulses != 3:
        return f"default_pulses={cfg.default_pulses} (engine is compiled for 3)"
    if cfg.vocab_size % 256 != 0:
        return f"vocab_size={cfg.vocab_size} must be a multiple of 256"
    if cfg.sliding_window != 1024:
        return f"sliding_window={cfg.sliding_window} (engine is compiled for 1024)"
    return None
