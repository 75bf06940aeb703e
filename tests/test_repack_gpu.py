"""Checkpoint repack: DeviceEngine.save_repacked writes the engine's bf16 weight arena (in its own
layouts) and the small fp32 tensors as a safetensors-format file; DeviceEngine.from_repacked
builds an engine from it without the fp32 staging, conversion and expert transposes. The
reloaded engine must give bit-identical prefill logits and tokens.
"""

from __future__ import annotations

import json
import os
import struct

import pytest
import torch

from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts

pytestmark = pytest.mark.gpu


def test_repack_roundtrip_is_bit_identical(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="B", seed=0)   # live loop adapter: its fp32 tensors travel too
    kw = dict(device=0, max_batch=1, max_seq_len=256, max_prefill=64, kv_dtype=torch.float32)
    ids = random_prompts(1, 32, cfg.vocab_size, seed=4)[0].tolist()
    a = DeviceEngine(cfg, sd, **kw)
    la = a.prefill(0, ids)
    ta, _ = a.generate_greedy([0], la.view(1, -1), 12, gamma=2)
    path = str(tmp_path / "pulsar_arena.safetensors")
    a.save_repacked(path)
    a.close()
    with open(path, "rb") as f:
        (hl,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hl))
    assert header["__metadata__"]["format"] == "pulsar_b200.arena.v1"
    assert header["arena.0.routed_gate_up_t"]["dtype"] == "BF16"
    assert header["core.0.attn.wqkv_adapter.lora_B"]["dtype"] == "F32"
    assert "core.0.mlp.routed_gate_up" not in header and "tok_emb.weight" not in header
    fp32_bytes = sum(t.numel() * 4 for k, t in sd.items() if k != "lm_head.weight")
    assert os.path.getsize(path) < 0.6 * fp32_bytes
    b = DeviceEngine.from_repacked(path, **kw)
    try:
        assert b.get_option("loop_adapter") == 1
        lb = b.prefill(0, ids)
        assert torch.equal(la, lb)
        tb, _ = b.generate_greedy([0], lb.view(1, -1), 12, gamma=2)
        assert torch.equal(ta, tb)
    finally:
        b.close()


def test_repack_rejects_foreign_files(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from pulsar_b200.engine import DeviceEngine
    p = tmp_path / "x.safetensors"
    h = json.dumps({"__metadata__": {"format": "other"}}).encode()
    p.write_bytes(struct.pack("<Q", len(h)) + h)
    with pytest.raises(ValueError, match="not a pulsar_b200 repacked arena"):
        DeviceEngine.from_repacked(str(p))
