"""load_inference_model (src/infer.py:785-817) on a real checkpoint file: a ``.pt`` holding
``{"model": state_dict, "config": cfg.to_dict()}`` (the layout the reference saves and loads)
goes through pulsar_b200.engine.load_inference_model, and the engine it returns decodes the
oracle's tokens on both reference generate loops and the batched loop."""

from __future__ import annotations

import pytest
import torch

from oracle import pulsar_oracle as O
from pulsar_b200.config import PulsarConfig
from pulsar_b200.weights import make_state_dict, random_prompts, save_checkpoint

from conftest import logit_margin

pytestmark = pytest.mark.gpu


class _Tok:
    unk_token_id = None

    def __init__(self, ids):
        self.ids = ids

    def encode(self, prompt, return_tensors="pt"):
        return torch.tensor([self.ids])

    def decode(self, t, skip_special_tokens=False):
        return f"{t[0]},"

    def convert_tokens_to_ids(self, s):
        return None


def test_load_inference_model_from_checkpoint_file(tmp_path, gpu):
    from pulsar_b200.engine import load_inference_model
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="B", seed=0)
    path = str(tmp_path / "ckpt.pt")
    save_checkpoint(path, sd, cfg)
    eng, tok = load_inference_model(path, device="cuda", dtype=torch.float32, max_batch=2, max_seq_len=256)
    try:
        assert eng.cfg.to_dict() == cfg.to_dict()
        m = O.OracleModel(sd, cfg)
        ids = random_prompts(1, 24, cfg.vocab_size, seed=7)[0].tolist()
        trace = []
        ref = O.stream_generate_ids(m, ids, 10, trace=trace)
        margins = [logit_margin(lg) for _, lg in trace]
        # greedy: both reference loops emit the argmax of the full three-pulse logits
        assert O.self_speculative_ids(m, ids, 10) == ref
        outs = []
        for spec in (False, True):
            txt = eng.generate(_Tok(ids), "", max_new_tokens=10, temperature=0.0, repetition_penalty=1.0,
                               speculative=spec)
            outs.append([int(x) for x in txt.split(",") if x])
        outs.append(eng.generate_batch(torch.tensor([ids]), 10, gamma=0)[0, 24:].tolist())
        for got in outs:
            for i, (a, b) in enumerate(zip(got, ref)):
                if a != b:
                    assert margins[i] <= 2e-2, f"token {i}: {a} vs oracle {b} (margin {margins[i]:.2e})"
                    break
    finally:
        eng.dev.close()


def test_load_inference_model_missing_file(tmp_path):
    from pulsar_b200.engine import load_inference_model
    with pytest.raises(FileNotFoundError):
        load_inference_model(str(tmp_path / "nope.pt"))
