"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Run in a container where the reference source tree is available (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path-to-reference>

It imports the reference's own ``src.infer`` / ``src.model`` (CPU, fp32, no CUDA
extension), loads the deterministic synthetic weights of ``pulsar_b200.weights`` into
``PulsarForCausalLM``, runs the reference inference engine (prefill, decode_pulse_pass,
decode_step, stream_generate, self_speculative_stream_generate) and writes compact
summaries to ``tests/golden/*.pt``. The reference is never needed at test time.

Cases:
  tiny_*  - the reference test-suite's tiny config (tests/conftest.py:30-51): full logits.
  full_*  - the production Pulsar-283M config, recipes A and B: top-k + sampled logits.
  early_exit_* - greedy token streams and exit tallies of the reference's adaptive early
            exit (set_early_exit_threshold, src/infer.py:211-214, 536-546) at a few
            thresholds. Random-init logits are nearly flat (max-probability ~1/V), so these
            cases sharpen the model: final_norm.weight x final_scale and pulse 0's
            pulse_res_scale x res0_scale (recorded in the file), which spreads the pulses'
            max-probabilities over a range where the thresholds split exits across depths.
            early_exit_nolora also zeroes every loop-adapter lora_B (the reference's own
            initialisation of lora_B, src/model.py:710-714).
  forward_* - PulsarForCausalLM.forward / generate (the training-style full recompute that
            model.generate runs per token): last-position logits and greedy, penalised and
            sampled streams.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "pulsar-300m_b200"))

from pulsar_b200.weights import make_state_dict, random_prompts  # noqa: E402

N_PROBE = 256          # fixed probe indices per logits vector (full-size cases)
TOPK = 32


class MockTokenizer:
    """Duck-typed tokenizer for the reference loops (modelled on tests/test_model.py:518-526)."""

    unk_token_id = None

    def __init__(self, ids):
        self.ids = list(ids)

    def encode(self, prompt, return_tensors="pt"):
        return torch.tensor([self.ids], dtype=torch.long)

    def decode(self, ids, skip_special_tokens=False):
        return "".join(f"{int(i)}," for i in ids)

    def convert_tokens_to_ids(self, s):
        return None


def summarise(logits: torch.Tensor, full: bool, probe_idx: torch.Tensor):
    lg = logits.detach().float().reshape(-1)
    d = {"lse": torch.logsumexp(lg, 0).item(), "argmax": int(lg.argmax())}
    v, i = torch.topk(lg, min(TOPK, lg.numel()))
    d["top_val"], d["top_idx"] = v.clone(), i.clone()
    if full:
        d["full"] = lg.clone()
    else:
        d["probe"] = lg[probe_idx].clone()
    return d


def tiny_cfg_dict():
    return dict(vocab_size=256, d_model=64, n_heads=4, n_kv_heads=2, head_dim=16, d_expert=32,
                d_shared=64, n_core=2, n_routed_experts=4, top_k=2, max_pulses=4, default_pulses=3,
                base_seq_len=32, max_seq_len=128, sliding_window=16, ce_chunk_size=64, eos_token_id=-1)


def run_case(name, cfg_dict, recipe, seed, prompt_len, n_new, n_pulse_steps, out_dir, full_logits, b_std=0.09):
    from src.infer import PulsarInferenceEngine, UnifiedKVCache
    from src.model import PulsarConfig, PulsarForCausalLM
    from pulsar_b200.config import PulsarConfig as MyCfg

    cfg = PulsarConfig(**cfg_dict)
    my_cfg = MyCfg(**cfg_dict)
    sd = make_state_dict(my_cfg, recipe=recipe, seed=seed, b_std=b_std)
    torch.manual_seed(1234)
    model = PulsarForCausalLM(cfg)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k.startswith("rope_") for k in missing) or not missing, missing
    eng = PulsarInferenceEngine(model, device="cpu", dtype=torch.float32)
    ids = random_prompts(1, prompt_len, cfg.vocab_size, seed=seed)[0].tolist()
    probe_idx = torch.randperm(cfg.vocab_size, generator=torch.Generator().manual_seed(7))[:N_PROBE].clone()
    rec = {"name": name, "cfg": cfg_dict, "recipe": recipe, "seed": seed, "b_std": b_std, "prompt": ids,
           "n_new": n_new, "probe_idx": probe_idx}

    # Per-pulse logits of the prefill and the first decode steps (src/infer.py:353-549).
    kv = UnifiedKVCache(cfg, 1, "cpu", torch.float32)
    with torch.inference_mode():
        lg = eng.prefill(torch.tensor([ids]), kv)[0, -1]
    rec["prefill"] = summarise(lg, full_logits, probe_idx)
    steps = []
    tok = int(lg.argmax())
    pos = len(ids)
    for _ in range(n_pulse_steps):
        h = h0n = None
        pulses = []
        with torch.inference_mode():
            for p in range(cfg.default_pulses):
                lg, h, h0n = eng.decode_pulse_pass(tok, pos, kv, p, h, h0n)
                pulses.append(summarise(lg[0], full_logits, probe_idx))
        kv.seq_len = pos + 1
        steps.append({"token": tok, "pos": pos, "pulses": pulses, "kv_lengths": kv.checkpoint_state()})
        tok = pulses[-1]["argmax"]
        pos += 1
    rec["steps"] = steps

    # Token streams of the two reference generate loops (greedy, no repetition penalty).
    def run(spec):
        tk = MockTokenizer(ids)
        txt = eng.generate(tk, "", max_new_tokens=n_new, temperature=0.0, top_p=1.0,
                           repetition_penalty=1.0, stream=False, speculative=spec)
        return [int(s) for s in txt.split(",") if s != ""]

    rec["greedy_ids"] = run(False)
    rec["spec_ids"] = run(True)
    # With the reference's default repetition penalty 1.15 (src/infer.py:559).
    tk = MockTokenizer(ids)
    txt = eng.generate(tk, "", max_new_tokens=min(n_new, 16), temperature=0.0, top_p=1.0,
                       repetition_penalty=1.15, stream=False, speculative=False)
    rec["greedy_rep115_ids"] = [int(s) for s in txt.split(",") if s != ""]
    path = os.path.join(out_dir, f"{name}.pt")
    torch.save(rec, path)
    print(f"wrote {path}: greedy={rec['greedy_ids'][:12]}... spec={rec['spec_ids'][:12]}...", flush=True)


def sharpen(sd, final_scale, res0_scale, zero_lora=False):
    """The early-exit cases' weight change (applied identically by the tests)."""
    sd = dict(sd)
    if zero_lora:
        for k in list(sd):
            if k.endswith("lora_B"):
                sd[k] = torch.zeros_like(sd[k])
    sd["final_norm.weight"] = sd["final_norm.weight"] * final_scale
    rs = sd["pulse_res_scale"].clone()
    rs[0] = rs[0] * res0_scale
    sd["pulse_res_scale"] = rs
    return sd


def run_early_exit(name, cfg_dict, recipe, seed, prompt_seed, prompt_len, n_new, thresholds, final_scale, res0_scale,
                   zero_lora, out_dir, b_std=0.09):
    from src.infer import PulsarInferenceEngine
    from src.model import PulsarConfig, PulsarForCausalLM
    from pulsar_b200.config import PulsarConfig as MyCfg

    cfg = PulsarConfig(**cfg_dict)
    sd = sharpen(make_state_dict(MyCfg(**cfg_dict), recipe=recipe, seed=seed, b_std=b_std), final_scale, res0_scale,
                 zero_lora)
    torch.manual_seed(1234)
    model = PulsarForCausalLM(cfg)
    _, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    eng = PulsarInferenceEngine(model, device="cpu", dtype=torch.float32)
    ids = random_prompts(1, prompt_len, cfg.vocab_size, seed=prompt_seed)[0].tolist()
    rec = {"name": name, "cfg": cfg_dict, "recipe": recipe, "seed": seed, "b_std": b_std, "prompt": ids,
           "n_new": n_new, "final_scale": final_scale, "res0_scale": res0_scale, "zero_lora": zero_lora, "runs": []}
    for thr in thresholds:
        eng.set_early_exit_threshold(thr)
        tk = MockTokenizer(ids)
        txt = eng.generate(tk, "", max_new_tokens=n_new, temperature=0.0, top_p=1.0, repetition_penalty=1.0,
                           stream=False, speculative=False)
        toks = [int(s) for s in txt.split(",") if s != ""]
        rec["runs"].append({"threshold": thr, "ids": toks, "counts": list(eng.early_exit_counts)})
        print(f"{name} threshold {thr}: counts {eng.early_exit_counts} ids {toks[:10]}...", flush=True)
    path = os.path.join(out_dir, f"{name}.pt")
    torch.save(rec, path)
    print(f"wrote {path}", flush=True)


def run_forward(name, cfg_dict, recipe, seed, prompt_seed, prompt_len, n_new, out_dir, full_logits, sampled,
                b_std=0.09):
    """PulsarForCausalLM.forward (labels=None) and PulsarForCausalLM.generate
    (src/model.py:1956-2125, 2246-2317): last-position softcapped logits of the prompt, the
    greedy stream, the greedy stream with repetition penalty 1.15 and, when `sampled`, a
    temperature 0.8 / top-k 50 / top-p 0.9 stream drawn after torch.manual_seed(11)."""
    from src.model import PulsarConfig, PulsarForCausalLM
    from pulsar_b200.config import PulsarConfig as MyCfg

    cfg = PulsarConfig(**cfg_dict)
    sd = make_state_dict(MyCfg(**cfg_dict), recipe=recipe, seed=seed, b_std=b_std)
    torch.manual_seed(1234)
    model = PulsarForCausalLM(cfg)
    _, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    model.eval()
    ids = random_prompts(1, prompt_len, cfg.vocab_size, seed=prompt_seed)[0].tolist()
    probe_idx = torch.randperm(cfg.vocab_size, generator=torch.Generator().manual_seed(7))[:N_PROBE].clone()
    rec = {"name": name, "cfg": cfg_dict, "recipe": recipe, "seed": seed, "b_std": b_std, "prompt": ids,
           "n_new": n_new, "probe_idx": probe_idx}
    x = torch.tensor([ids])
    with torch.no_grad():
        logits, _, _ = model(x, labels=None)
    rec["forward"] = summarise(logits[0, -1], full_logits, probe_idx)
    rec["greedy_ids"] = model.generate(x, max_new_tokens=n_new, temperature=0.0, repetition_penalty=1.0)[0, len(ids):].tolist()
    rec["greedy_rep115_ids"] = model.generate(x, max_new_tokens=n_new, temperature=0.0,
                                              repetition_penalty=1.15)[0, len(ids):].tolist()
    if sampled:
        torch.manual_seed(11)
        rec["sampled_ids"] = model.generate(x, max_new_tokens=n_new, temperature=0.8, top_k=50, top_p=0.9,
                                            repetition_penalty=1.15)[0, len(ids):].tolist()
    path = os.path.join(out_dir, f"{name}.pt")
    torch.save(rec, path)
    print(f"wrote {path}: greedy={rec['greedy_ids']} rep={rec['greedy_rep115_ids']}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PULSAR_REFERENCE"),
                    help="path of the reference source tree (or set PULSAR_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or PULSAR_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    full = dict(eos_token_id=-1)
    cases = [
        ("tiny_A", tiny_cfg_dict(), "A", 0, 12, 16, 3, True),
        ("tiny_B", tiny_cfg_dict(), "B", 0, 12, 24, 3, True, 0.35),
        ("tiny_B_long", tiny_cfg_dict(), "B", 3, 40, 24, 3, True, 0.35),  # T > window and > base_seq_len
        ("full_A_c1", full, "A", 0, 128, 64, 2, False),                  # BASELINE config 1 shape
        ("full_B_c1", full, "B", 0, 128, 32, 2, False),
        ("full_B_long", full, "B", 5, 1100, 6, 2, False),                # T > 1024: local quirk + YaRN
    ]
    for c in cases:
        if args.only and c[0] != args.only:
            continue
        run_case(c[0], c[1], c[2], c[3], c[4], c[5], c[6], args.out, c[7], *c[8:])
    ee_cases = [
        # name, cfg, recipe, seed, prompt seed, prompt len, n_new, thresholds, final x, res0 x, zero lora_B, b_std
        ("early_exit_tiny", tiny_cfg_dict(), "B", 0, 0, 12, 24, [0.03, 0.04, 0.06], 16.0, 3.0, False, 0.35),
        ("early_exit_full", full, "B", 0, 1, 32, 32, [0.0075, 0.02], 8.0, 3.0, False, 0.09),
        # prompt seed 8: the router's 4th/5th score gap stays >= 1.3e-5 along both streams
        # (a near-tie there flips an expert between any two fp32 implementations)
        ("early_exit_nolora", full, "B", 0, 8, 32, 32, [0.2, 0.3], 16.0, 3.0, True, 0.09),
    ]
    for c in ee_cases:
        if args.only and c[0] != args.only:
            continue
        run_early_exit(*c[:11], args.out, *c[11:])
    fwd_cases = [
        # name, cfg, recipe, seed, prompt seed, prompt len, n_new, full logits, sampled, b_std
        ("forward_tiny_B", tiny_cfg_dict(), "B", 0, 3, 40, 8, True, True, 0.35),   # T > window, > base
        ("forward_full_A", full, "A", 0, 6, 1100, 2, False, False),                # YaRN on layers 3, 7
    ]
    for c in fwd_cases:
        if args.only and c[0] != args.only:
            continue
        run_forward(*c[:7], args.out, *c[7:])


if __name__ == "__main__":
    main()
