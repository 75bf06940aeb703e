"""Reference-compatible inference API over the sm_100a engine.

Mirrors the public surface of the reference engine (src/infer.py:64-817): the classes
``UnifiedKVCache`` and ``PulsarInferenceEngine`` with ``prefill``, ``decode_pulse_pass``,
``decode_step``, ``stream_generate``, ``self_speculative_stream_generate``, ``generate``,
the early-exit controls, and ``load_inference_model``. Every pulse runs in the CUDA
library (``libpulsar_b200.so``); there is no CPU fallback and no torch compute on the
token path except the reference's optional sampling knobs (temperature / top-p /
repetition penalty in the per-token loops, which act on device logits).

New entry point: ``generate_batch`` - batched greedy decoding, plain (gamma = 0) or
self-speculative with gamma drafts and one batched verify per round, device-resident
(CUDA graphs, no per-token host synchronisation).
"""

from __future__ import annotations

import ctypes as C
import math
import os
import re
import sys
from typing import Generator, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .config import PulsarConfig, engine_supported, LOCAL_LAYERS
from .weights import save_checkpoint  # noqa: F401  (re-export for callers)

STOP_STRINGS = ("<|im_end|>", "<|endoftext|>", "</s>")


def _rope_inv_freq(theta: float, dim: int) -> torch.Tensor:
    # src/model.py:536-543 (fp32)
    return 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))


# fp32 state_dict tensors that the bf16 weight arena replaces (pulsar_engine_arena_write)
_ARENA_SOURCE = re.compile(r"^(tok_emb\.weight|lm_head\.weight|core\.\d+\.(attn\.wqkv\.weight|attn\.wo\.weight|"
                           r"mlp\.shared_expert\.w_gate_up\.weight|mlp\.shared_expert\.w_down\.weight|"
                           r"mlp\.routed_gate_up|mlp\.routed_down))$")


class DeviceEngine:
    """Owner of one ``pulsar_engine`` handle (weights, KV slots, workspaces) on one GPU."""

    def __init__(self, cfg: PulsarConfig, state_dict, device: int | str | torch.device = 0, max_batch: int = 1,
                 max_seq_len: int = 4096, max_prefill: Optional[int] = None, kv_dtype: torch.dtype = torch.bfloat16):
        self._create(cfg, device, max_batch, max_seq_len, max_prefill, kv_dtype)
        try:
            self._upload(state_dict)
        except Exception:
            self.close()
            raise

    def _create(self, cfg, device, max_batch, max_seq_len, max_prefill, kv_dtype):
        why = engine_supported(cfg)
        if why is not None:
            raise RuntimeError(f"pulsar_b200 engine does not support this config: {why}")
        if kv_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("kv_dtype must be torch.bfloat16 or torch.float32")
        self.cfg = cfg
        dev = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        if dev.type != "cuda":
            raise RuntimeError("pulsar_b200 runs on CUDA devices only (no CPU fallback)")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.max_prefill = max_prefill or max_seq_len
        self.kv_dtype = kv_dtype
        lib = _lib.load()
        ec = _lib.EngineConfig(
            vocab_size=cfg.vocab_size, max_pulses=cfg.max_pulses, loop_lora_rank=cfg.loop_lora_rank,
            loop_lora_alpha=cfg.loop_lora_alpha, rms_eps=cfg.rms_eps, logit_softcap=cfg.logit_softcap,
            base_seq_len=cfg.base_seq_len, use_canon_conv=int(cfg.use_canon_conv), per_pulse_bias=int(cfg.per_pulse_bias),
            max_batch=max_batch, max_seq_len=max_seq_len, max_prefill=self.max_prefill,
            kv_fp32=1 if kv_dtype == torch.float32 else 0, device=self.device.index)
        h = C.c_void_p()
        _lib.check(lib.pulsar_engine_create(C.byref(ec), C.byref(h)), "pulsar_engine_create")
        self._h = h
        self._free_slots = list(range(max_batch))
        self._small = {}   # the fp32 tensors outside the bf16 arena (kept for save_repacked)

    def _upload(self, sd):
        lib = _lib.load()
        names = dict(sd)
        names.pop("lm_head.weight", None)       # tied to tok_emb (src/model.py:1775)
        for name, t in names.items():
            if name.startswith("rope_") or name.endswith(("drop_counts_accum", "demand_over_capacity_accum",
                                                          "assigned_counts_accum", "capacity_last",
                                                          "pulse_drop_accum", "pulse_assigned_accum")):
                continue
            a = t.detach().to("cpu", torch.float32).contiguous()
            _lib.check(lib.pulsar_engine_set_tensor(self._h, name.encode(), a.data_ptr(), a.numel()),
                       f"set_tensor({name})")
            if not _ARENA_SOURCE.search(name):
                self._small[name] = a
        self._finalize()

    def _finalize(self):
        lib = _lib.load()
        for key, theta in (("rope_local.inv_freq", self.cfg.rope_theta_local),
                           ("rope_global.inv_freq", self.cfg.rope_theta_global)):
            a = _rope_inv_freq(theta, self.cfg.head_dim).contiguous()
            _lib.check(lib.pulsar_engine_set_tensor(self._h, key.encode(), a.data_ptr(), a.numel()), key)
        _lib.check(lib.pulsar_engine_finalize(self._h), "pulsar_engine_finalize")

    # ---- checkpoint repack: safetensors-format file of the bf16 arena + the small fp32 tensors ----
    def save_repacked(self, path: str) -> None:
        """Write the engine's weights as a safetensors-format file (pulsar_b200.repack): the bf16
        arena tensors in the engine's layouts (BF16, 1-D) and the remaining fp32 state_dict
        tensors (F32, their shapes), the config in the header's __metadata__. Load with
        ``from_repacked``."""
        import json
        import numpy as np
        from . import repack
        lib = _lib.load()
        n = C.c_int32()
        _lib.check(lib.pulsar_engine_arena_count(self._h, C.byref(n)), "arena_count")
        tensors = []
        for i in range(n.value):
            name, numel = C.c_char_p(), C.c_int64()
            _lib.check(lib.pulsar_engine_arena_info(self._h, i, C.byref(name), C.byref(numel)), "arena_info")
            buf = np.empty(numel.value, dtype=np.uint16)
            _lib.check(lib.pulsar_engine_arena_read(self._h, name.value, buf.ctypes.data, numel.value), "arena_read")
            tensors.append((name.value.decode(), "BF16", [numel.value], buf.tobytes()))
        for name, t in self._small.items():
            tensors.append((name, "F32", list(t.shape), t.numpy().tobytes()))
        repack.write(path, tensors, {"format": repack.FORMAT, "config": json.dumps(self.cfg.to_dict())})

    @classmethod
    def from_repacked(cls, path: str, device: int | str | torch.device = 0, max_batch: int = 1,
                      max_seq_len: int = 4096, max_prefill: Optional[int] = None,
                      kv_dtype: torch.dtype = torch.bfloat16) -> "DeviceEngine":
        """An engine from a ``save_repacked`` file: bf16 arena tensors go to the device as they
        are (no fp32 staging, conversion or expert transposes)."""
        import json
        import numpy as np
        from . import repack
        header, meta, data = repack.read(path)
        cfg = PulsarConfig.from_dict(json.loads(meta["config"]))
        self = cls.__new__(cls)
        self._create(cfg, device, max_batch, max_seq_len, max_prefill, kv_dtype)
        try:
            lib = _lib.load()
            for name, h in header.items():
                b0, b1 = h["data_offsets"]
                if h["dtype"] == "BF16":
                    buf = np.frombuffer(data, dtype=np.uint16, count=(b1 - b0) // 2, offset=b0)
                    _lib.check(lib.pulsar_engine_arena_write(self._h, name.encode(), buf.ctypes.data, buf.size),
                               f"arena_write({name})")
                else:
                    a = torch.from_numpy(np.frombuffer(data, dtype=np.float32, count=(b1 - b0) // 4,
                                                       offset=b0).copy()).reshape(h["shape"])
                    _lib.check(lib.pulsar_engine_set_tensor(self._h, name.encode(), a.data_ptr(), a.numel()),
                               f"set_tensor({name})")
                    self._small[name] = a
            self._finalize()
        except Exception:
            self.close()
            raise
        return self

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.load().pulsar_engine_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ---- slots ----
    def acquire_slot(self) -> int:
        if not self._free_slots:
            raise RuntimeError(f"all {self.max_batch} sequence slots are in use")
        return self._free_slots.pop(0)

    def release_slot(self, slot: int) -> None:
        if slot not in self._free_slots:
            self._free_slots.append(slot)
            self._free_slots.sort()

    def get_length(self, slot: int) -> int:
        n = C.c_int32()
        _lib.check(_lib.load().pulsar_engine_get_length(self._h, slot, C.byref(n)), "get_length")
        return int(n.value)

    def set_length(self, slot: int, n: int) -> None:
        _lib.check(_lib.load().pulsar_engine_set_length(self._h, slot, int(n)), "set_length")

    def read_kv(self, slot: int, layer: int, pos0: int, n: int):
        """Cached keys and values of positions [pos0, pos0 + n) of one slot and layer
        (pulsar_engine_read_kv): fp32 CPU tensors K, V of shape [n_kv_heads, n, head_dim]."""
        cfg = self.cfg
        k = torch.empty(cfg.n_kv_heads, n, cfg.head_dim, dtype=torch.float32)
        v = torch.empty_like(k)
        _lib.check(_lib.load().pulsar_engine_read_kv(self._h, slot, layer, pos0, n, k.data_ptr(), v.data_ptr()),
                   "read_kv")
        return k, v

    def prefill_attention(self, slot: int, layer: int, q: torch.Tensor, tensor_cores: bool = True) -> torch.Tensor:
        """The prefill attention step of one layer (pulsar_engine_prefill_attention) over the
        slot's cached positions 0..T-1: q [T, n_heads, head_dim] fp32 on this engine's device
        (normed, rotated, unscaled) -> [T, n_heads, head_dim] fp32."""
        q = q.to(device=self.device, dtype=torch.float32).contiguous()
        out = torch.empty_like(q)
        _lib.check(_lib.load().pulsar_engine_prefill_attention(self._h, slot, layer, q.shape[0], q.data_ptr(),
                                                                out.data_ptr(), 1 if tensor_cores else 0,
                                                                self.stream()),
                   "prefill_attention")
        return out

    def decode_attention(self, layer: int, rows, q: torch.Tensor, tensor_cores: bool = True,
                         rows_per_block: int = 1) -> torch.Tensor:
        """The decode attention of one layer (pulsar_engine_decode_attention) for rows
        [(slot, pos), ...] over the keys each slot holds at positions 0..pos: q [R, n_heads,
        head_dim] fp32 (normed, rotated, unscaled) -> [R, n_heads, head_dim] fp32, without the
        head gate. rows_per_block groups consecutive rows into verify blocks (1..8)."""
        rt = torch.tensor([[s, p, 0, 0] for (s, p) in rows], dtype=torch.int32, device=self.device)
        q = q.to(device=self.device, dtype=torch.float32).contiguous()
        out = torch.empty_like(q)
        _lib.check(_lib.load().pulsar_engine_decode_attention(self._h, layer, len(rows), rt.data_ptr(), rows_per_block,
                                                               q.data_ptr(), out.data_ptr(), 1 if tensor_cores else 0,
                                                               self.stream()),
                   "decode_attention")
        return out

    def set_option(self, name: str, value: int) -> None:
        """Engine options (see include/pulsar_b200.h): "megakernel" 0/1."""
        _lib.check(_lib.load().pulsar_engine_set_option(self._h, name.encode(), int(value)), f"set_option({name})")

    def get_option(self, name: str) -> int:
        v = C.c_int64()
        _lib.check(_lib.load().pulsar_engine_get_option(self._h, name.encode(), C.byref(v)), f"get_option({name})")
        return int(v.value)

    def read_trace(self):
        """Phase stamps of the last persistent-kernel launch: uint64 [grid, 256] (ns)."""
        import numpy as np
        n = self.get_option("megakernel_grid") * 256
        buf = (C.c_uint64 * n)()
        _lib.check(_lib.load().pulsar_engine_read_trace(self._h, C.cast(buf, C.c_void_p), n), "read_trace")
        return np.frombuffer(buf, dtype=np.uint64).reshape(-1, 256).copy()

    def memory(self) -> dict:
        a, k, w = C.c_int64(), C.c_int64(), C.c_int64()
        _lib.check(_lib.load().pulsar_engine_memory(self._h, C.byref(a), C.byref(k), C.byref(w)), "memory")
        return {"arena_bytes": a.value, "kv_bytes": k.value, "work_bytes": w.value}

    # ---- compute ----
    def prefill(self, slot: int, ids) -> torch.Tensor:
        ids_t = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        logits = torch.empty(self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        _lib.check(_lib.load().pulsar_engine_prefill(self._h, slot, ids_t.data_ptr(), ids_t.numel(),
                                                     logits.data_ptr(), self.stream()), "prefill")
        return logits

    def forward(self, slot: int, ids) -> torch.Tensor:
        """pulsar_engine_forward: PulsarForCausalLM.forward's last-position softcapped logits [V]
        for ids (the training-style full-sequence pass; the slot is scratch and left empty)."""
        ids_t = torch.as_tensor(ids, dtype=torch.int32).reshape(-1).to(self.device)
        logits = torch.empty(self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        _lib.check(_lib.load().pulsar_engine_forward(self._h, slot, ids_t.data_ptr(), ids_t.numel(),
                                                     logits.data_ptr(), self.stream()), "forward")
        return logits

    def pulse(self, pulse: int, rows, h_prev=None, h0n=None, want_logits: bool = True):
        """rows: list of (slot, pos, token). Returns (logits [R,V] or None, h_out [R,D], h0n [R,D])."""
        R = len(rows)
        rt = torch.tensor([[s, p, t, 0] for (s, p, t) in rows], dtype=torch.int32, device=self.device)
        D = self.cfg.d_model
        h_out = torch.empty(R, D, dtype=torch.float32, device=self.device)
        h0n_out = torch.empty(R, D, dtype=torch.float32, device=self.device)
        logits = torch.empty(R, self.cfg.vocab_size, dtype=torch.float32, device=self.device) if want_logits else None
        hp = h_prev.float().contiguous() if h_prev is not None else None
        hz = h0n.float().contiguous() if h0n is not None else None
        _lib.check(_lib.load().pulsar_engine_pulse(
            self._h, pulse, R, rt.data_ptr(), hp.data_ptr() if hp is not None else None,
            hz.data_ptr() if hz is not None else None, h_out.data_ptr(), h0n_out.data_ptr(),
            logits.data_ptr() if logits is not None else None, self.stream()), f"pulse({pulse})")
        if pulse > 0:
            h0n_out = hz
        return logits, h_out, h0n_out

    def generate_greedy(self, slots, first_logits: torch.Tensor, n_new: int, gamma: int = 0):
        n = len(slots)
        out = torch.empty(n, n_new, dtype=torch.int32, device=self.device)
        sl = (C.c_int32 * n)(*slots)
        stats = (C.c_int64 * 3)()
        fl = first_logits.float().contiguous().reshape(n, -1)
        _lib.check(_lib.load().pulsar_engine_generate_greedy(
            self._h, n, C.cast(sl, C.c_void_p), fl.data_ptr(), n_new, gamma, out.data_ptr(), stats, self.stream()),
            "generate_greedy")
        return out, {"rounds": stats[0], "drafted": stats[1], "accepted": stats[2]}

    def set_early_exit(self, threshold: Optional[float]) -> None:
        """pulsar_engine_set_early_exit: device early exit of the gamma = 0 greedy loop (None:
        off); resets the exit tallies."""
        on = threshold is not None
        _lib.check(_lib.load().pulsar_engine_set_early_exit(self._h, int(on), float(threshold) if on else 1.0),
                   "set_early_exit")

    def set_repetition_penalty(self, penalty: float) -> None:
        """pulsar_engine_set_repetition_penalty: penalty of every generate loop (1: off)."""
        _lib.check(_lib.load().pulsar_engine_set_repetition_penalty(self._h, float(penalty)),
                   "set_repetition_penalty")

    def early_exit_counts(self) -> list[int]:
        """Tokens that exited after pulse 1, 2, 3 since the last set_early_exit."""
        c = (C.c_int64 * 3)()
        _lib.check(_lib.load().pulsar_engine_early_exit_counts(self._h, c), "early_exit_counts")
        return [int(x) for x in c]

    def generate_sampled(self, slots, first_logits: torch.Tensor, n_new: int, gamma: int, temperature: float,
                         top_p: float, seed: int, seq_ids=None):
        """Sampled self-speculative decoding (pulsar_engine_generate_sampled): Philox streams
        keyed by (seq_ids[i], round, slot) and ``seed``; seq_ids default to 0..n-1."""
        n = len(slots)
        out = torch.empty(n, n_new, dtype=torch.int32, device=self.device)
        sl = (C.c_int32 * n)(*slots)
        si = (C.c_int32 * n)(*(range(n) if seq_ids is None else seq_ids))
        stats = (C.c_int64 * 3)()
        fl = first_logits.float().contiguous().reshape(n, -1)
        _lib.check(_lib.load().pulsar_engine_generate_sampled(
            self._h, n, C.cast(sl, C.c_void_p), C.cast(si, C.c_void_p), fl.data_ptr(), n_new, gamma,
            float(temperature), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF, out.data_ptr(), stats, self.stream()),
            "generate_sampled")
        return out, {"rounds": stats[0], "drafted": stats[1], "accepted": stats[2]}


class UnifiedKVCache:
    """src/infer.py:64-178. Backed by one sequence slot of a ``DeviceEngine`` when
    created through ``PulsarInferenceEngine.new_cache`` (or implicitly by its generate
    loops); a standalone instance keeps torch tensors exactly like the reference, for
    callers that poke ``update`` directly (scripts/benchmark.py:411-417)."""

    def __init__(self, cfg: PulsarConfig, batch_size: int = 1, device="cuda", dtype: torch.dtype = torch.bfloat16,
                 engine: Optional[DeviceEngine] = None):
        self.cfg = cfg
        self.batch_size = batch_size
        self.device = torch.device(device)
        self.dtype = dtype
        self.n_core = cfg.n_core
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.head_dim
        self.sliding_window = cfg.sliding_window
        self.layers = [{"k": None, "v": None, "is_local": i in LOCAL_LAYERS} for i in range(cfg.n_core)]
        self._engine = engine
        self.slot = engine.acquire_slot() if engine is not None else None
        self._seq_len = 0

    @property
    def seq_len(self) -> int:
        return self._engine.get_length(self.slot) if self._engine is not None else self._seq_len

    @seq_len.setter
    def seq_len(self, n: int) -> None:
        if self._engine is not None:
            self._engine.set_length(self.slot, n)
        else:
            self._seq_len = n

    def release(self):
        if self._engine is not None and self.slot is not None:
            self._engine.release_slot(self.slot)
            self.slot = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def reset(self):
        for layer in self.layers:
            layer["k"] = layer["v"] = None
        self.seq_len = 0

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, pulse_idx: int = 0, is_prefill: bool = False):
        """Torch-tensor cache update with the reference's semantics (src/infer.py:108-157)."""
        if self._engine is not None:
            raise RuntimeError("update() is only available on standalone caches; engine-backed caches are written "
                               "by the device kernels")
        layer = self.layers[layer_idx]
        W = self.sliding_window
        if is_prefill or layer["k"] is None:
            if layer["is_local"] and k.shape[2] > W:
                layer["k"], layer["v"] = k[:, :, -W:].clone(), v[:, :, -W:].clone()
            else:
                layer["k"], layer["v"] = k.clone(), v.clone()
            return layer["k"], layer["v"]
        if pulse_idx == 0:
            kc = torch.cat([layer["k"], k], dim=2)
            vc = torch.cat([layer["v"], v], dim=2)
            if layer["is_local"] and kc.shape[2] > W:
                kc, vc = kc[:, :, -W:].contiguous(), vc[:, :, -W:].contiguous()
            layer["k"], layer["v"] = kc, vc
        else:
            layer["k"][:, :, -1:] = k
            layer["v"][:, :, -1:] = v
        return layer["k"], layer["v"]

    def checkpoint_state(self) -> list[int]:
        """src/infer.py:159-161: per-layer cached lengths."""
        if self._engine is None:
            return [l["k"].shape[2] if l["k"] is not None else 0 for l in self.layers]
        n = self.seq_len
        return [min(n, self.sliding_window) if l["is_local"] else n for l in self.layers]

    def restore_state(self, lengths: list[int]):
        """src/infer.py:163-168: truncate (the rollback). Engine-backed caches roll back the
        committed length to the global layers' length."""
        if self._engine is None:
            for layer, n in zip(self.layers, lengths):
                if layer["k"] is not None and layer["k"].shape[2] > n:
                    layer["k"] = layer["k"][:, :, :n].contiguous()
                    layer["v"] = layer["v"][:, :, :n].contiguous()
            return
        glob = [n for n, l in zip(lengths, self.layers) if not l["is_local"]]
        target = max(glob) if glob else max(lengths)
        if target < self.seq_len:
            self.seq_len = target

    def memory_footprint_bytes(self) -> int:
        """src/infer.py:170-178: bytes of the logical cache contents."""
        if self._engine is None:
            tot = 0
            for l in self.layers:
                for key in ("k", "v"):
                    if l[key] is not None:
                        tot += l[key].numel() * l[key].element_size()
            return tot
        esz = 4 if self._engine.kv_dtype == torch.float32 else 2
        return sum(2 * self.n_kv_heads * n * self.head_dim * esz * self.batch_size for n in self.checkpoint_state())


def _state_and_cfg(model):
    if isinstance(model, tuple):
        sd, cfg = model
    else:
        sd, cfg = model.state_dict(), model.cfg
    if not isinstance(cfg, PulsarConfig):
        cfg = PulsarConfig.from_dict(cfg.to_dict() if hasattr(cfg, "to_dict") else dict(cfg))
    return sd, cfg


class PulsarInferenceEngine:
    """src/infer.py:181-782 on the sm_100a engine.

    ``model`` is a ``PulsarForCausalLM`` (anything with ``.state_dict()`` and ``.cfg``) or a
    ``(state_dict, config)`` pair. ``dtype`` selects the KV-cache storage (bf16 default;
    ``torch.float32`` gives the fp32-KV parity mode); weights are bf16 and arithmetic fp32.
    """

    def __init__(self, model, device="cuda", dtype: torch.dtype = torch.bfloat16, max_batch: int = 4,
                 max_seq_len: Optional[int] = None, max_prefill: Optional[int] = None):
        sd, cfg = _state_and_cfg(model)
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("pulsar_b200 runs on CUDA devices only (no CPU fallback)")
        self.dtype = dtype
        self.dev = DeviceEngine(cfg, sd, device=self.device, max_batch=max_batch,
                                max_seq_len=max_seq_len or 4096, max_prefill=max_prefill,
                                kv_dtype=torch.float32 if dtype == torch.float32 else torch.bfloat16)
        self.early_exit_threshold: Optional[float] = None
        self.early_exit_counts = [0] * cfg.default_pulses
        self.stop_token_ids = {cfg.eos_token_id}
        self.last_stats: dict = {}

    # ---- early exit (src/infer.py:211-232) ----
    def set_early_exit_threshold(self, threshold: Optional[float]):
        self.early_exit_threshold = threshold
        self.early_exit_counts = [0] * self.cfg.default_pulses
        self.dev.set_early_exit(threshold)

    def get_early_exit_stats(self) -> dict:
        total = sum(self.early_exit_counts)
        if total == 0:
            return {}
        c = self.early_exit_counts
        eff = (8 * c[0] + 16 * c[1] + 24 * c[2]) / total
        return {"total_tokens": total, "pulse_counts": list(c), "pulse_pcts": [x / total * 100.0 for x in c],
                "effective_layers": eff, "compute_speedup": 24.0 / eff}

    def new_cache(self) -> UnifiedKVCache:
        return UnifiedKVCache(self.cfg, 1, self.device, self.dtype, engine=self.dev)

    def _slot(self, kv_cache: UnifiedKVCache) -> int:
        if kv_cache._engine is not self.dev:
            raise RuntimeError("kv_cache does not belong to this engine: create it with engine.new_cache()")
        return kv_cache.slot

    # ---- reference methods ----
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, kv_cache: UnifiedKVCache) -> torch.Tensor:
        """src/infer.py:353-461 -> logits [1, 1, V] (not softcapped)."""
        ids = torch.as_tensor(input_ids).reshape(-1)
        logits = self.dev.prefill(self._slot(kv_cache), ids)
        return logits.view(1, 1, -1)

    @torch.inference_mode()
    def decode_pulse_pass(self, token_id: int, pos: int, kv_cache: UnifiedKVCache, pulse_idx: int,
                          h_pulse_prev: Optional[torch.Tensor] = None, h_0_norm_cached: Optional[torch.Tensor] = None):
        """src/infer.py:463-524 -> (logits [1, V], h_pulse_out [1, 1, D], h_0_norm [1, 1, D])."""
        slot = self._slot(kv_cache)
        D = self.cfg.d_model
        hp = h_pulse_prev.reshape(1, D) if h_pulse_prev is not None else None
        hz = h_0_norm_cached.reshape(1, D) if h_0_norm_cached is not None else None
        lg, h, h0n = self.dev.pulse(pulse_idx, [(slot, int(pos), int(token_id))], hp, hz)
        return lg, h.view(1, 1, D), h0n.view(1, 1, D)

    @torch.inference_mode()
    def decode_step(self, token_id: int, pos: int, kv_cache: UnifiedKVCache) -> torch.Tensor:
        """src/infer.py:526-549: three pulses with optional early exit; commits pos + 1."""
        h = h0n = None
        logits = None
        K = self.cfg.default_pulses
        for k in range(K):
            logits, h, h0n = self.decode_pulse_pass(token_id, pos, kv_cache, k, h, h0n)
            if self.early_exit_threshold is not None and k < K - 1:
                if F.softmax(logits, dim=-1).max(dim=-1).values.item() >= self.early_exit_threshold:
                    self.early_exit_counts[k] += 1
                    break
        else:
            if self.early_exit_threshold is not None:
                self.early_exit_counts[K - 1] += 1
        kv_cache.seq_len = pos + 1
        return logits

    def _stop_ids(self, tokenizer):
        stop = {self.cfg.eos_token_id}
        for s in STOP_STRINGS:
            try:
                sid = tokenizer.convert_tokens_to_ids(s)
                if sid is not None and sid != getattr(tokenizer, "unk_token_id", None):
                    stop.add(sid)
            except Exception:
                pass
        return stop

    @staticmethod
    def _sample(lgt: torch.Tensor, seen, temperature: float, top_p: float, repetition_penalty: float) -> int:
        """src/infer.py:582-609 / 658-685 on the device logits."""
        l = lgt.reshape(1, -1).clone()
        if repetition_penalty != 1.0 and seen:
            ids = torch.tensor(sorted(set(seen)), device=l.device)
            vals = l[0, ids]
            l[0, ids] = torch.where(vals > 0, vals / repetition_penalty, vals * repetition_penalty)
        if temperature <= 1e-4:
            return int(l.argmax(dim=-1).item())
        scaled = l / max(temperature, 1e-5)
        if top_p < 1.0:
            sl, si = torch.sort(scaled, descending=True)
            cum = torch.cumsum(F.softmax(sl, dim=-1), dim=-1)
            rm = cum > top_p
            rm[..., 1:] = rm[..., :-1].clone()
            rm[..., 0] = 0
            scaled[0, si[rm]] = float("-inf")
        probs = F.softmax(scaled, dim=-1).nan_to_num(0.0)
        if probs.sum() <= 0:
            return int(l.argmax(dim=-1).item())
        probs = probs / probs.sum()
        return int(torch.multinomial(probs, num_samples=1).item())

    @torch.inference_mode()
    def stream_generate(self, tokenizer, prompt: str, max_new_tokens: int = 512, temperature: float = 0.7,
                        top_p: float = 0.9, repetition_penalty: float = 1.15) -> Generator[str, None, None]:
        """src/infer.py:551-621."""
        prompt_ids = tokenizer.encode(prompt, return_tensors="pt")
        kv = self.new_cache()
        try:
            logits = self.prefill(prompt_ids, kv)[0, -1]
            all_ids = prompt_ids.reshape(-1).tolist()
            pos = len(all_ids) - 1
            stop = self._stop_ids(tokenizer)
            for _ in range(max_new_tokens):
                tok = self._sample(logits, all_ids, temperature, top_p, repetition_penalty)
                if tok in stop:
                    break
                all_ids.append(tok)
                pos += 1
                yield tokenizer.decode([tok], skip_special_tokens=False)
                logits = self.decode_step(tok, pos, kv)[0]
        finally:
            kv.release()

    @torch.inference_mode()
    def self_speculative_stream_generate(self, tokenizer, prompt: str, max_new_tokens: int = 512,
                                         temperature: float = 0.7, top_p: float = 0.9,
                                         repetition_penalty: float = 1.15) -> Generator[str, None, None]:
        """src/infer.py:623-731: one draft from the pulse-1 exit, verified by pulses 2-3 on
        the same token, accepted on id equality, then a full decode_step."""
        prompt_ids = tokenizer.encode(prompt, return_tensors="pt")
        kv = self.new_cache()
        try:
            logits = self.prefill(prompt_ids, kv)[0, -1]
            all_ids = prompt_ids.reshape(-1).tolist()
            pos = len(all_ids) - 1
            stop = self._stop_ids(tokenizer)
            produced = 0
            samp = lambda lg: self._sample(lg, all_ids, temperature, top_p, repetition_penalty)
            while produced < max_new_tokens:
                t = samp(logits)
                if t in stop:
                    break
                all_ids.append(t)
                pos += 1
                produced += 1
                yield tokenizer.decode([t], skip_special_tokens=False)
                if produced >= max_new_tokens:
                    break
                d_lg, h0, h0n = self.decode_pulse_pass(t, pos, kv, 0)
                draft = samp(d_lg[0])
                _, h1, _ = self.decode_pulse_pass(t, pos, kv, 1, h0, h0n)
                v_lg, _, _ = self.decode_pulse_pass(t, pos, kv, 2, h1, h0n)
                kv.seq_len = pos + 1
                true = samp(v_lg[0])
                if draft == true and draft not in stop:
                    all_ids.append(draft)
                    pos += 1
                    produced += 1
                    yield tokenizer.decode([draft], skip_special_tokens=False)
                    if produced >= max_new_tokens:
                        break
                    logits = self.decode_step(draft, pos, kv)[0]
                else:
                    logits = v_lg[0]
        finally:
            kv.release()

    def generate(self, tokenizer, prompt: str, max_new_tokens: int = 512, temperature: float = 0.7,
                 top_p: float = 0.9, repetition_penalty: float = 1.15, stream: bool = False,
                 speculative: bool = False) -> str:
        """src/infer.py:733-782."""
        gen = (self.self_speculative_stream_generate if speculative else self.stream_generate)(
            tokenizer=tokenizer, prompt=prompt, max_new_tokens=max_new_tokens, temperature=temperature,
            top_p=top_p, repetition_penalty=repetition_penalty)
        acc = []
        for s in gen:
            if stream:
                sys.stdout.write(s)
                sys.stdout.flush()
            acc.append(s)
        if stream:
            sys.stdout.write("\n")
            sys.stdout.flush()
        if self.early_exit_threshold is not None:
            st = self.get_early_exit_stats()
            if st:
                print(f"\n[Adaptive Early-Exit Stats | Threshold: {self.early_exit_threshold:.2f}]")
                print(f"  Tokens: {st['total_tokens']} | P1 (8L): {st['pulse_pcts'][0]:.1f}% | "
                      f"P2 (16L): {st['pulse_pcts'][1]:.1f}% | P3 (24L): {st['pulse_pcts'][2]:.1f}%")
        return prompt + "".join(acc)

    # ---- new: batched device-resident greedy decoding ----
    @torch.inference_mode()
    def generate_batch(self, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.0,
                       top_p: float = 1.0, gamma: int = 4, seed: int = 0,
                       repetition_penalty: float = 1.0) -> torch.Tensor:
        """Decode ``input_ids`` [B, T] and return [B, T + max_new_tokens] (int64).

        gamma = 0: exact sequential greedy decoding (the reference's stream_generate with
        temperature 0 and no repetition penalty), with the adaptive early exit of
        ``set_early_exit_threshold`` decided on the device per sequence (exit depths added to
        ``early_exit_counts``). The ``repetition_penalty`` of src/infer.py:582-589 / 658-667
        applies on the device to every path: the logits choosing a token are penalised over the
        sequence's prompt, its emitted tokens and, inside a speculative round, the drafts
        before it. gamma >= 1: gamma drafts from the
        pulse-1 exit and one batched pulse-2/3 verify of the gamma+1 block per round,
        greedy acceptance (temperature <= 1e-4) or sampled acceptance (ratio test with
        residual resampling, Philox streams keyed by (sequence index, round, slot) and
        ``seed``), rollback of the rejected tail. ``self.last_stats`` receives
        {rounds, drafted, accepted, accept_rate}.
        """
        sampled = temperature > 1e-4
        if sampled and gamma < 1:
            raise ValueError("generate_batch: sampled decoding needs gamma >= 1")
        ids = torch.as_tensor(input_ids)
        if ids.dim() == 1:
            ids = ids.view(1, -1)
        B, T = ids.shape
        caches = [self.new_cache() for _ in range(B)]
        try:
            first = torch.empty(B, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
            for b in range(B):
                first[b] = self.dev.prefill(caches[b].slot, ids[b])
            slots = [c.slot for c in caches]
            self.dev.set_repetition_penalty(repetition_penalty)
            try:
                if sampled:
                    toks, stats = self.dev.generate_sampled(slots, first, max_new_tokens, gamma, temperature, top_p,
                                                            seed)
                else:
                    ee = gamma == 0 and self.early_exit_threshold is not None
                    if ee:
                        self.dev.set_early_exit(self.early_exit_threshold)   # zero the device tallies
                    toks, stats = self.dev.generate_greedy(slots, first, max_new_tokens, gamma)
            finally:
                self.dev.set_repetition_penalty(1.0)
            if not sampled:
                if ee:
                    for k, c in enumerate(self.dev.early_exit_counts()):
                        self.early_exit_counts[k] += c
        finally:
            for c in caches:
                c.release()
        stats["accept_rate"] = stats["accepted"] / max(1, stats["drafted"])
        self.last_stats = stats
        return torch.cat([ids.to(self.device, torch.int64), toks.to(torch.int64)], dim=1)

    # ---- PulsarForCausalLM.generate (src/model.py:2246-2317) on the engine ----
    @torch.no_grad()
    def model_generate(self, input_ids: torch.Tensor, max_new_tokens: int = 64, temperature: float = 0.7,
                       top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.15,
                       num_pulses: int | None = None, eos_token_id: int | None = None,
                       generator: torch.Generator | None = None) -> torch.Tensor:
        """The reference model's generate: every step recomputes the whole context (its last
        max_seq_len ids) with the training-style forward (DeviceEngine.forward, on the device),
        then on the host: repetition penalty over the row's ids, greedy argmax (temperature 0) or
        temperature, top-k, top-p and a multinomial draw (CPU generator: `generator`, else torch's
        default, as the reference's torch.multinomial); finished rows emit eos and the loop
        stops when every row has finished. Returns [B, T + n] int64 on this engine's device.
        Each row runs its own forward: the reference's batched forward shares one MoE capacity
        across a batch's rows, which couples them only when the capacity overflows."""
        K = num_pulses if num_pulses is not None else self.cfg.default_pulses
        if K != self.cfg.default_pulses:
            raise ValueError(f"model_generate: the engine runs {self.cfg.default_pulses} pulses, got num_pulses={K}")
        eos = eos_token_id if eos_token_id is not None else self.cfg.eos_token_id
        ids = torch.as_tensor(input_ids)
        if ids.dim() == 1:
            ids = ids.view(1, -1)
        rows = [r.tolist() for r in ids.cpu()]
        finished = [False] * len(rows)
        cache = self.new_cache()
        try:
            for _ in range(max_new_tokens):
                for b, row in enumerate(rows):
                    lg = self.dev.forward(cache.slot, row[-self.cfg.max_seq_len:]).float().cpu().clone()
                    if repetition_penalty != 1.0:
                        seen = torch.tensor(sorted(set(row)), dtype=torch.long)
                        vals = lg[seen]
                        lg[seen] = torch.where(vals > 0, vals / repetition_penalty, vals * repetition_penalty)
                    if temperature > 0:
                        lg = lg / temperature
                        if top_k > 0:
                            v, _ = torch.topk(lg, min(top_k, lg.numel()))
                            lg[lg < v[-1]] = float("-inf")
                        if top_p < 1.0:
                            sl, si = torch.sort(lg, descending=True)
                            cum = torch.cumsum(torch.softmax(sl, dim=-1), dim=-1)
                            rm = cum > top_p
                            rm[1:] = rm[:-1].clone()
                            rm[0] = False
                            lg[si[rm]] = float("-inf")
                        tok = int(torch.multinomial(torch.softmax(lg, dim=-1), 1, generator=generator))
                    else:
                        tok = int(lg.argmax())
                    if finished[b]:
                        tok = eos
                    row.append(tok)
                    finished[b] = finished[b] or tok == eos
                if all(finished):
                    break
        finally:
            cache.release()
        return torch.tensor(rows, dtype=torch.int64, device=self.device)

def load_inference_model(checkpoint_path: str, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                         tokenizer_path: str = "data/pulsar_tokenizer", **engine_kwargs):
    """src/infer.py:785-817: checkpoint ``{"model": state_dict, "config": dict}`` -> (engine,
    tokenizer). The tokenizer is loaded with transformers when available at
    ``tokenizer_path``; otherwise None is returned in its place."""
    if not os.path.exists(checkpoint_path):
        raise FileNotFoundError(f"Checkpoint not found at: {checkpoint_path}")
    ck = torch.load(checkpoint_path, map_location="cpu", weights_only=False)
    cfg_dict = ck.get("config") or {}
    cfg = PulsarConfig.from_dict(cfg_dict) if cfg_dict else PulsarConfig()
    engine = PulsarInferenceEngine((ck["model"], cfg), device=device, dtype=dtype, **engine_kwargs)
    tok = None
    try:
        from transformers import AutoTokenizer
        if os.path.isdir(tokenizer_path):
            tok = AutoTokenizer.from_pretrained(tokenizer_path)
    except Exception:
        tok = None
    return engine, tok
