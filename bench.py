#!/usr/bin/env python3
"""Decode benchmark of the pulsar_b200 engine (the BASELINE.json metric on its config 2).

Workload (N = 1): Pulsar-283M, random-init weights (recipe A = the reference init, seed 0),
batch 1, a 2048-token uniform-random prompt, 512 new tokens, greedy self-speculative decode
with gamma = 4 (drafts from the pulse-1 exit, one batched pulse-2/3 verify per round).
A step = decoding the 512 new tokens from the prefilled prompt (the KV cache is rolled back
to the prompt between steps). value = new tokens / device time. The weights (~0.57 GB bf16)
are larger than the 126 MB L2, so no flush is needed between steps.

N > 1 (torchrun): independent replicas, one per GPU (seed + rank prompts), no collective on
the token path; time = max over ranks (CUDA events), value = all ranks' tokens / time.

--impl reference: the reference algorithm's CPU implementation (the oracle port of
src/infer.py, fp32 torch on the host cores), greedy decode_step loop on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pulsar-300m_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "decode tokens/sec/GPU (B=1 latency, B=256 throughput); accept rate; % HBM roof"
PROMPT, NEW, GAMMA = 2048, 512, 4


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_tflops():
    """Sustained dense bf16 TFLOP/s of MEASURED_PEAKS.json (a kernel timed inside a long run), else
    the recipe's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def bytes_per_pass(cfg, d_routed: float, kv_keys: int, rows: int, with_lm_head: bool, adapter: bool = False) -> float:
    """Algorithmic bytes of one pulse pass (the per-unit figure of the roofline): bf16
    weights read once (wqkv, wo, shared expert, d_routed distinct routed experts per
    layer), fp32 small tensors, KV keys read once per (layer, sequence) and written per
    row, LM head once, embedding gathers. adapter: the live loop adapter's fp32 factors
    (A of wqkv and wo, 24 x 1024 each, and the per-pulse Bs, 1536 x 24 and 1024 x 24)."""
    D = cfg.d_model
    attn = (cfg.qkv_dim * D + D * D) * 2
    shared = (2 * cfg.d_shared * D + D * cfg.d_shared) * 2
    routed = (2 * cfg.d_expert * D + cfg.d_expert * D) * 2
    small = (16 * D + 16 * D + 4 * D) * 4       # gate, router, norms/scales (fp32)
    lora = (2 * 24 * D + cfg.qkv_dim * 24 + D * 24) * 4 if adapter else 0
    per_layer = attn + shared + small + lora + routed * d_routed
    kv = kv_keys * 1024 + rows * 8 * 1024        # bf16 K+V: 4 heads x 64 x 2 x 2 B per key per layer
    lm = cfg.vocab_size * D * 2 if with_lm_head else 0
    return cfg.n_core * per_layer + kv + lm + rows * D * 2


def kv_keys_for(L: int) -> int:
    return 6 * min(L, 1024) + 2 * L


# The launches of one self-speculative round (gamma drafts): pulse index, rows, LM head. The
# persistent kernel k_mega_pulse runs each of them as one launch.
def round_shapes(gamma: int):
    return [("draft_lm", 0, 1, True, gamma), ("draft_nolm", 0, 1, False, 1),
            ("verify_p1", 1, gamma + 1, False, 1), ("verify_p2", 2, gamma + 1, True, 1)]


PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "k_mega_pulse_decode_shapes.txt")


def load_traffic():
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of each round shape,
    from the committed ncu summary (lines 'traffic <shape> <bytes>'); None when absent."""
    out = {}
    try:
        for line in open(PROFILE_TRAFFIC):
            f = line.split()
            if len(f) == 3 and f[0] == "traffic":
                out[f[1]] = float(f[2])
    except OSError:
        return None
    return out or None


def shape_launches(eng, cfg, gamma: int, seed: int = 1):
    """Buffers and a launcher for the round shapes through the C ABI (pulsar_engine_pulse), at
    positions PROMPT.. of slot 0 (the prompt context). Returns {shape: launch()}."""
    from pulsar_b200 import _lib
    lib = _lib.load()
    dev = eng.device
    D, V, R = cfg.d_model, cfg.vocab_size, gamma + 1
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, V, (R,), generator=g)
    rows = torch.tensor([[0, PROMPT + i, int(toks[i]), 0] for i in range(R)], dtype=torch.int32, device=dev)
    h0, z0 = torch.empty(R, D, device=dev), torch.empty(R, D, device=dev)
    h1, h2 = torch.empty(R, D, device=dev), torch.empty(R, D, device=dev)
    zo = torch.empty(R, D, device=dev)
    logits = torch.empty(R, V, device=dev)
    st = eng.stream()

    def call(p, n, hp, hz, out, lg):
        _lib.check(lib.pulsar_engine_pulse(eng.handle, p, n, rows.data_ptr(), hp.data_ptr() if hp is not None else None,
                                           hz.data_ptr() if hz is not None else None, out.data_ptr(),
                                           zo.data_ptr() if p else z0.data_ptr(),
                                           lg.data_ptr() if lg is not None else None, st), f"pulse({p})")

    call(0, R, None, None, h0, None)      # pulse-0 states of the block (the drafts' outputs)
    return {
        "draft_lm": lambda: call(0, 1, None, None, h1, logits),
        "draft_nolm": lambda: call(0, 1, None, None, h1, None),
        "verify_p1": lambda: call(1, R, h0, z0, h1, None),
        "verify_p2": lambda: call(2, R, h1, z0, h2, logits),
    }


def kernel_roofline(eng, cfg, gamma: int, recipe: str, reps: int, peak: float, peak_kind: str):
    """Roofline of the dominant kernel (k_mega_pulse): each round shape launched `reps` times
    through the C ABI on the bench's engine and context, each launch bracketed by CUDA events on
    the launching stream (option time_pulses); achieved = the round's algorithmic bytes / the
    round's summed mean launch times."""
    eng.set_length(0, PROMPT)
    launch = shape_launches(eng, cfg, gamma)
    eng.set_option("time_pulses", 1)
    for f in launch.values():          # warm-up
        f()
    torch.cuda.synchronize()
    shapes, tot_b, tot_t, tot_n = {}, 0.0, 0.0, 0
    for name, p, R, lm, n in round_shapes(gamma):
        ts = []
        e0 = eng.get_option("routed_experts")
        for _ in range(reps):
            launch[name]()
            ts.append(eng.get_option("last_pulse_ns") * 1e-9)
        t = statistics.mean(ts)
        d = (eng.get_option("routed_experts") - e0) / (reps * cfg.n_core)   # distinct experts per layer
        b = bytes_per_pass(cfg, d, kv_keys_for(PROMPT + R), R, lm, adapter=recipe == "B") + \
            (R * cfg.vocab_size * 4 if lm else 0)
        shapes[name] = {"rows": R, "lm_head": lm, "per_round": n, "us": t * 1e6, "bytes": b,
                        "experts_per_layer": d, "gbs": b / t / 1e9}
        tot_b += n * b
        tot_t += n * t
        tot_n += n
    eng.set_option("time_pulses", 0)
    achieved = tot_b / tot_t / 1e9
    traffic = load_traffic()
    tr = None
    if traffic and all(k in traffic for k in shapes):
        tr = sum(shapes[k]["per_round"] * traffic[k] for k in shapes) / tot_n
    return {"bound": "hbm", "kernel": "k_mega_pulse", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": peak_kind, "traffic": tr,
            "bytes_per_launch": tot_b / tot_n, "us_per_launch": tot_t / tot_n * 1e6,
            "timing": f"CUDA events around each launch on its stream, mean of {reps} launches per shape, "
                      "weighted by the launches of one round",
            "shapes": shapes}


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.f.name):
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx = float(c[2])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int, local: int) -> float:
    """Maximum of x over the ranks (a device tensor under NCCL, a host tensor under gloo)."""
    if world == 1:
        return x
    import torch.distributed as dist
    dev = f"cuda:{local}" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(tokens_per_rank: int, world: int, ms_max: float) -> float:
    """Whole-job tokens/s: every rank's tokens over the slowest rank's device time."""
    return tokens_per_rank * world / (ms_max / 1e3)


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_oracle_rate(n_tokens: int, prompt_len: int, seed: int = 0):
    """Greedy decode_step loop of the oracle port (src/infer.py:526-621 restated) on the host
    cores: prefill untimed, then n_tokens decode steps timed. Returns (tok/s, threads, sample)."""
    from oracle import pulsar_oracle as O
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.weights import make_state_dict, random_prompts
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe="A", seed=0)
    m = O.OracleModel(sd, cfg)
    ids = random_prompts(1, prompt_len, cfg.vocab_size, seed=seed)[0].tolist()
    kv = O.OracleKV(m, prompt_len + n_tokens + 8)
    lg = O.prefill(m, ids, kv)
    tok, pos = int(lg.argmax()), prompt_len
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        lg = O.decode_step(m, tok, pos, kv)
        tok, pos = int(lg.argmax()), pos + 1
    dt = time.perf_counter() - t0
    sample = (f"oracle port (fp32 torch, {threads} threads): prefill {prompt_len} untimed, then {n_tokens} greedy "
              f"decode_step tokens at context {prompt_len}..{prompt_len + n_tokens}")
    return n_tokens / dt, threads, sample


def arm_config(gamma: int, recipe: str, world: int) -> dict:
    """The workload both arms report (BASELINE config 2 on every GPU)."""
    return {"workload": f"pulsar-283M decode, B=1 per GPU, prompt {PROMPT}, {NEW} new tokens, greedy "
                        f"gamma={gamma} self-speculative, recipe {recipe} weights",
            "batch_per_gpu": 1, "prompt": PROMPT, "new_tokens": NEW, "gamma": gamma,
            "l2": "no flush: weights (~0.57 GB) exceed the 126 MB L2", "kv_dtype": "bf16",
            "parallelism": f"{world} independent replicas"}


def run_reference(args):
    world, rank, local = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    per_step = 4
    from oracle import pulsar_oracle as O
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.weights import make_state_dict, random_prompts
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe=args.recipe, seed=0)
    m = O.OracleModel(sd, cfg)
    ids = random_prompts(1, PROMPT, cfg.vocab_size, seed=0)[0].tolist()
    kv = O.OracleKV(m, PROMPT + (args.steps + args.warmup) * per_step + 8)
    lg = O.prefill(m, ids, kv)
    tok, pos = int(lg.argmax()), PROMPT
    times = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for _ in range(per_step):
            lg = O.decode_step(m, tok, pos, kv)
            tok, pos = int(lg.argmax()), pos + 1
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per_step * args.steps / tot
    sample = (f"oracle port of src/infer.py (fp32 torch, {threads} threads), B=1 prompt {PROMPT}: each step = "
              f"{per_step} greedy decode_step tokens of the reference's sequential loop (prefill untimed; its tokens "
              f"equal the gamma={args.gamma} loop's, and the rate is per emitted token)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": arm_config(args.gamma, args.recipe, args.gpus),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


TP_BATCH, TP_PROMPT, TP_NEW = 256, 512, 256   # BASELINE config 5 (throughput sweep), per GPU


def throughput_b256(args, world, rank, local):
    """BASELINE config 5 on this rank's GPU: 256 sequences of 512-token prompts, 256 new tokens,
    greedy gamma=4, one generate call over all sequences (the many-row path). Prefill untimed;
    decode timed with CUDA events, max over ranks; whole-job tokens/s."""
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.engine import DeviceEngine
    from pulsar_b200.weights import make_state_dict, random_prompts
    cfg = PulsarConfig(eos_token_id=-1)
    eng = DeviceEngine(cfg, make_state_dict(cfg, recipe=args.recipe, seed=0), device=local, max_batch=TP_BATCH,
                       max_seq_len=TP_PROMPT + TP_NEW + 64, max_prefill=TP_PROMPT, kv_dtype=torch.bfloat16)
    P = random_prompts(TP_BATCH, TP_PROMPT, cfg.vocab_size, seed=1000 + rank)
    first = torch.stack([eng.prefill(i, P[i].tolist()) for i in range(TP_BATCH)])
    slots = list(range(TP_BATCH))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)

    def run(n):
        for i in slots:
            eng.set_length(i, TP_PROMPT)
        return eng.generate_greedy(slots, first, n, gamma=4)

    run(16)   # graph capture and warm-up
    torch.cuda.synchronize()
    if getattr(args, "throughput_profile", False):
        # one speculative round (5 tokens) between cudaProfilerStart / Stop (ncu captures)
        torch.cuda.cudart().cudaProfilerStart()
        run(5)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        eng.close()
        return {"throughput_profile": TP_BATCH}
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _, st = run(TP_NEW)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_max = max_over_ranks(e0.elapsed_time(e1), world, local)
    eng.close()
    # roofline of one decode round of the batch (algorithmic units, mean context): gamma + 1
    # pulse-0 passes of B rows, pulse-1 and pulse-2 passes of B (gamma + 1) rows; every pass
    # streams all 16 routed experts (hundreds of rows route to every expert) and reads each
    # sequence's K/V once per layer; gamma + 1 LM heads. FLOPs: 2 x the active parameters of a
    # row (4 routed experts) per row per pass, plus the LM head rows.
    g = 4
    rounds = st["rounds"] / TP_BATCH
    L = TP_PROMPT + TP_NEW // 2
    D = cfg.d_model
    rows_pass = [TP_BATCH] * (g + 1) + [TP_BATCH * (g + 1)] * 2
    b_round = sum(bytes_per_pass(cfg, cfg.n_routed_experts, TP_BATCH * kv_keys_for(L), r, False) for r in rows_pass)
    b_round += (g + 1) * cfg.vocab_size * D * 2
    act_params = cfg.n_core * ((cfg.qkv_dim + D) * D + 3 * cfg.d_shared * D + cfg.top_k * 3 * cfg.d_expert * D)
    lm_rows = g * TP_BATCH + TP_BATCH * (g + 1)
    f_round = 2.0 * act_params * sum(rows_pass) + 2.0 * cfg.vocab_size * D * lm_rows
    bw = rounds * b_round / (ms_max / 1e3) / 1e9
    fl = rounds * f_round / (ms_max / 1e3) / 1e12
    peak, peak_kind = load_peaks()
    tf_peak, tf_kind = load_tflops()
    roof = {"bound": "hbm" if b_round / peak > f_round / 1e3 / tf_peak else "tensor",
            "achieved": bw, "peak": peak, "unit": "GB/s", "frac": bw / peak, "peak_kind": peak_kind,
            "tensor_achieved_tflops": fl, "tensor_peak_tflops": tf_peak, "tensor_frac": fl / tf_peak,
            "tensor_peak_kind": tf_kind, "bytes_per_round": b_round, "flops_per_round": f_round,
            "rounds": rounds, "scope": "per GPU: algorithmic bytes / FLOPs of the timed decode over its device time"}
    return {"value": job_rate(TP_BATCH * TP_NEW, world, ms_max), "unit": "tokens/s", "ms": ms_max,
            "roofline": roof,
            "accept_rate": st["accepted"] / max(1, st["drafted"]),
            "config": {"workload": f"BASELINE config 5: {TP_BATCH} sequences per GPU, prompt {TP_PROMPT}, {TP_NEW} new "
                                   f"tokens, greedy gamma=4, recipe {args.recipe} weights", "batch_per_gpu": TP_BATCH,
                       "timed": "decode of one generate call (prefill untimed), CUDA events, max over ranks"}}


def decode_leg(args, recipe: str, world: int, rank: int, local: int, full: bool):
    """The metric's B=1 half on one weight recipe: timed decode of the bench workload (device
    time, max over ranks), launch and expert counts, the dominant kernel's roofline and the
    path roofline; with full=True also the clocks and the end-to-end run through the C ABI."""
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.engine import DeviceEngine
    from pulsar_b200.weights import make_state_dict, random_prompts
    dev = torch.device("cuda", local)
    cfg = PulsarConfig(eos_token_id=-1)
    sd = make_state_dict(cfg, recipe=recipe, seed=0)
    eng = DeviceEngine(cfg, sd, device=local, max_batch=1, max_seq_len=PROMPT + NEW + 64, max_prefill=PROMPT,
                       kv_dtype=torch.bfloat16)
    del sd
    ids = random_prompts(1, PROMPT, cfg.vocab_size, seed=rank)[0]
    first = eng.prefill(0, ids.tolist())
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    g = args.gamma

    def step():
        eng.set_length(0, PROMPT)
        return eng.generate_greedy([0], first.view(1, -1), NEW, gamma=g)

    for _ in range(args.warmup):
        out, st = step()
    torch.cuda.synchronize()
    barrier(world)
    clk = Clocks(local) if full else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stats = {"rounds": 0, "drafted": 0, "accepted": 0}
    launches0 = eng.get_option("kernel_launches")
    mega0 = eng.get_option("mega_launches")
    experts0 = eng.get_option("routed_experts")
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        out, st = step()
        for k in stats:
            stats[k] += st[k]
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop() if clk else None
    gpu_launches = eng.get_option("kernel_launches") - launches0
    mega_launches = eng.get_option("mega_launches") - mega0
    experts_streamed = eng.get_option("routed_experts") - experts0
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, world, local)
    res = {"value": job_rate(NEW * args.steps, world, ms_max), "ms_per_step": ms_max / args.steps,
           "accept_rate": stats["accepted"] / max(1, stats["drafted"]),
           "tokens_per_round": stats["accepted"] / max(1, stats["rounds"]) + 1 if g > 0 else 1.0,
           "gpu_launches": gpu_launches, "mega_launches": mega_launches, "clocks": clocks,
           "loop_adapter": bool(eng.get_option("loop_adapter"))}
    if full:
        # ---- end-to-end through the C ABI with host buffers (prompt H2D, prefill, decode, tokens D2H)
        pinned_ids = ids.to(torch.int32).pin_memory()
        host_out = torch.empty(NEW, dtype=torch.int32).pin_memory()
        e2e_ms, pre_ms = [], []
        for s in range(args.warmup + args.steps):
            torch.cuda.synchronize()
            e0, em, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            d_ids = pinned_ids.to(dev, non_blocking=True)
            lg = eng.prefill(0, d_ids)
            em.record(stream)
            toks, _ = eng.generate_greedy([0], lg.view(1, -1), NEW, gamma=g)
            host_out.copy_(toks[0], non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize()
            if s >= args.warmup:
                e2e_ms.append(e0.elapsed_time(e1))
                pre_ms.append(e0.elapsed_time(em))
        e2e_ms_max = max_over_ranks(sum(e2e_ms) / len(e2e_ms), world, local)
        res["e2e"] = {"value": job_rate(NEW, world, e2e_ms_max), "unit": "tokens/s", "h2d_bytes_per_step": PROMPT * 4,
                      "d2h_bytes_per_step": NEW * 4, "includes": "prompt H2D, prefill, decode, tokens D2H",
                      "prefill_ms": statistics.mean(pre_ms), "ms_per_step": statistics.mean(e2e_ms)}
    # ---- roofline of the dominant kernel, then of the whole decode path
    peak, peak_kind = load_peaks()
    res["roofline"] = kernel_roofline(eng, cfg, g, recipe, args.kernel_reps, peak, peak_kind)
    # algorithmic bytes of the timed region: every launch's fixed bytes plus the routed experts
    # the kernels actually streamed (device counter), at the mean context of the step
    L = PROMPT + NEW // 2
    ad = recipe == "B"
    routed = (2 * cfg.d_expert * cfg.d_model + cfg.d_expert * cfg.d_model) * 2
    kv = kv_keys_for(L)
    if g > 0:
        n_rounds = mega_launches / (g + 3)
        fixed = n_rounds * ((g + 1) * bytes_per_pass(cfg, 0, kv, 1, False, ad) + g * cfg.vocab_size * cfg.d_model * 2
                            + bytes_per_pass(cfg, 0, kv, g + 1, False, ad) + bytes_per_pass(cfg, 0, kv, g + 1, True, ad))
    else:
        n_steps = mega_launches / 3
        fixed = n_steps * (3 * bytes_per_pass(cfg, 0, kv, 1, False, ad) + cfg.vocab_size * cfg.d_model * 2)
    path_bytes = fixed + experts_streamed * routed
    achieved = path_bytes / (ms / 1e3) / 1e9
    res["path_roofline"] = {"scope": "whole decode path: algorithmic bytes of the timed region (routed experts counted "
                                     "on the device) / device time",
                            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                            "peak_kind": peak_kind, "bytes_per_token": path_bytes / (NEW * args.steps)}
    eng.close()
    return res


def run_engine(args):
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    g = args.gamma
    a = decode_leg(args, args.recipe, world, rank, local, full=True)
    line = {"metric": METRIC, "value": a["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": a["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": arm_config(g, args.recipe, world),
            "accept_rate": a["accept_rate"], "tokens_per_round": a["tokens_per_round"],
            "e2e": a["e2e"], "roofline": a["roofline"], "path_roofline": a["path_roofline"],
            "clocks": a["clocks"], "gpu_launches": a["gpu_launches"], "mega_launches": a["mega_launches"]}
    if not args.no_recipe_b and args.recipe == "A":
        # the same workload on recipe-B weights (non-trivial acceptance, live loop adapter): its own
        # rate, acceptance, tokens per round and rooflines (same collective steps on every rank)
        b = decode_leg(args, "B", world, rank, local, full=False)
        line["recipe_b"] = {"value": b["value"], "unit": "tokens/s", "ms_per_step": b["ms_per_step"],
                            "accept_rate": b["accept_rate"], "tokens_per_round": b["tokens_per_round"],
                            "loop_adapter": b["loop_adapter"], "gpu_launches": b["gpu_launches"],
                            "roofline": b["roofline"], "path_roofline": b["path_roofline"],
                            "config": arm_config(g, "B", world)}
    if not args.no_throughput:
        # the metric's B=256 half: every rank runs its replica (same collective steps on all ranks)
        line["throughput_b256"] = throughput_b256(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, sample = cpu_oracle_rate(args.cpu_tokens, PROMPT)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_kernel_shapes(args):
    """The bench engine and prompt, then one launch of each round shape (after the pulse-0 block
    pass that feeds the verify shapes): five k_mega_pulse launches in total."""
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.engine import DeviceEngine
    from pulsar_b200.weights import make_state_dict, random_prompts
    cfg = PulsarConfig(eos_token_id=-1)
    eng = DeviceEngine(cfg, make_state_dict(cfg, recipe=args.recipe, seed=0), device=0, max_batch=1,
                       max_seq_len=PROMPT + NEW + 64, max_prefill=PROMPT, kv_dtype=torch.bfloat16)
    eng.prefill(0, random_prompts(1, PROMPT, cfg.vocab_size, seed=0)[0].tolist())
    launch = shape_launches(eng, cfg, args.gamma)
    for name, *_ in round_shapes(args.gamma):
        launch[name]()
    torch.cuda.synchronize()
    print(json.dumps({"kernel_shapes": [n for n, *_ in round_shapes(args.gamma)],
                      "mega_launches": eng.get_option("mega_launches")}), flush=True)
    eng.close()


def run_prefill_profile(args):
    """The bench engine and prompt: one warm-up prefill, then one prefill between
    cudaProfilerStart and cudaProfilerStop (ncu --profile-from-start off)."""
    from pulsar_b200.config import PulsarConfig
    from pulsar_b200.engine import DeviceEngine
    from pulsar_b200.weights import make_state_dict, random_prompts
    cfg = PulsarConfig(eos_token_id=-1)
    eng = DeviceEngine(cfg, make_state_dict(cfg, recipe=args.recipe, seed=0), device=0, max_batch=1,
                       max_seq_len=PROMPT + NEW + 64, max_prefill=PROMPT, kv_dtype=torch.bfloat16)
    ids = random_prompts(1, PROMPT, cfg.vocab_size, seed=0)[0].tolist()
    eng.prefill(0, ids)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    eng.prefill(0, ids)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"prefill_profile": PROMPT}), flush=True)
    eng.close()


def run_ops(args):
    """The drop-in op boundary: each pulsar_cuda forward op of the shim against the reference's
    own kernel (csrc/kernels.cu built for sm_100a by oracle/build_ref_ops.py), same inputs at the
    model's widths (d_model 1024, 16 heads of 64, 16 experts, top-4) over 16384 tokens (eight
    2048-token prompts: every tensor of 32-168 MB, so each launch streams from HBM), same B200. Each launch is
    timed alone with CUDA events on the current stream, after an L2 flush (a 256 MB write) and a
    device-side spin that keeps host launch overhead out of the bracket, median of
    --kernel-reps launches after 3 warm-ups. GB/s counts each op's algorithmic bytes (inputs
    read once, outputs written once)."""
    from oracle import build_ref_ops
    import pulsar_cuda as pc
    ref = build_ref_ops.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N, D, E, K, H, DH, CAP, T = 16384, 1024, 16, 4, 16, 64, 5120, 16384
    g = torch.Generator(device="cpu").manual_seed(0)
    bf = lambda *s: torch.randn(*s, generator=g).to(dev, torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).to(dev)
    slots = torch.full((N, K), -1, dtype=torch.int32)
    fill = [0] * E
    for t in range(N):
        for k in range(K):
            e = int(idx[t, k])
            if fill[e] < CAP:
                slots[t, k], fill[e] = fill[e], fill[e] + 1
    slots = slots.to(dev)
    counts = torch.tensor(fill, device=dev)
    tw = torch.rand(N, K, generator=g).to(dev, torch.bfloat16)
    x, sh, eo = bf(N, D), bf(N, D), bf(E, CAP, D)
    w = torch.rand(D, device=dev) + 0.5
    logits = torch.randn(N, E, generator=g).to(dev)
    bias = torch.zeros(E, device=dev)
    gu = bf(N, 2 * 512)
    q = bf(1, H, T, DH)
    ang = torch.outer(torch.arange(T, device=dev, dtype=torch.float32),
                      1.0 / (10000.0 ** (torch.arange(0, DH, 2, device=dev, dtype=torch.float32) / DH)))
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    wq = torch.rand(H, DH, device=dev) + 0.5
    xc, wc = bf(8, 2048, D), torch.randn(D, 4, generator=g).to(dev)
    att, gl = bf(1, H, T, DH), torch.randn(1, T, H, generator=g).to(dev)
    used = int((slots >= 0).sum())
    cases = {   # name: (call(module), algorithmic bytes)
        "moe_combine_forward": (lambda m: m.moe_combine_forward(eo, idx, tw, slots, sh),
                                used * D * 2 + 2 * N * D * 2 + N * K * (8 + 4 + 2)),
        "moe_dispatch_forward": (lambda m: m.moe_dispatch_forward(x, idx, slots, E, CAP, counts),
                                 N * D * 2 + E * CAP * D * 2 + N * K * 12),
        "moe_router_topk_forward": (lambda m: m.moe_router_topk_forward(logits, bias, K, 1e-3),
                                    N * E * 4 + N * K * 12 + E * 4),
        "rmsnorm_forward": (lambda m: m.rmsnorm_forward(x, w, 1e-6), 2 * N * D * 2 + N * 4),
        "fused_swiglu_forward": (lambda m: m.fused_swiglu_forward(gu, 512), N * 1024 * 2 + N * 512 * 2),
        "rope_forward": (lambda m: m.rope_forward(q, cos, sin), 2 * q.numel() * 2 + 2 * cos.numel() * 4),
        "qk_rmsnorm_rope_forward": (lambda m: m.qk_rmsnorm_rope_forward(q, wq, cos, sin, T, 1e-6),
                                    2 * q.numel() * 2 + 2 * cos.numel() * 4 + H * T * 4),
        "fused_attn_gate_forward": (lambda m: m.fused_attn_gate_forward(att, gl), 2 * att.numel() * 2 + gl.numel() * 4),
        "causal_depthwise_conv1d_k4_forward": (lambda m: m.causal_depthwise_conv1d_k4_forward(xc, wc),
                                               2 * xc.numel() * 2 + wc.numel() * 4),
    }
    flush = torch.empty(256 * 2 ** 20 // 4, device=dev)
    st = torch.cuda.current_stream()

    def time_once(fn):
        flush.fill_(1.0)
        # ~100 us of device-side spin after the flush: the host enqueues the op (its Python /
        # binding overhead) before the GPU reaches the start event, so the events bracket
        # device time only
        torch.cuda._sleep(200_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        b.synchronize()
        return a.elapsed_time(b) * 1e3

    out = {}
    for name, (call, nbytes) in cases.items():
        arms = [("shim", pc)] + ([("reference", ref)] if ref is not None else [])
        for _, mod in arms:
            for _ in range(3):
                call(mod)
        ts = {k: [] for k, _ in arms}
        for rep in range(max(5, args.kernel_reps)):   # the arms alternate which one runs first
            order = arms if rep % 2 == 0 else arms[::-1]
            for k, mod in order:
                ts[k].append(time_once(lambda: call(mod)))
        row = {"bytes": nbytes}
        us = statistics.median(ts["shim"])
        row["shim_us"], row["shim_gbs"] = round(us, 2), round(nbytes / us / 1e3, 1)
        if ref is not None:
            ur = statistics.median(ts["reference"])
            row["reference_us"], row["reference_gbs"] = round(ur, 2), round(nbytes / ur / 1e3, 1)
            row["speedup"] = round(ur / us, 2)
        out[name] = row
    print(json.dumps({"metric": "pulsar_cuda forward op time (median us, L2 flushed)", "unit": "us",
                      "shapes": {"tokens": N, "d_model": D, "experts": E, "top_k": K, "capacity": CAP, "heads": H},
                      "reference": "csrc/kernels.cu built for sm_100a (oracle/build_ref_ops.py)" if ref is not None
                      else "not built", "ops": out}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--gamma", type=int, default=GAMMA)
    ap.add_argument("--recipe", default="A", choices=["A", "B"])
    ap.add_argument("--cpu-tokens", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-throughput", action="store_true", help="skip the B=256 throughput measurement (config 5)")
    ap.add_argument("--no-recipe-b", action="store_true", help="skip the recipe-B decode leg")
    ap.add_argument("--throughput-profile", action="store_true",
                    help="config 5 only: one decode round between cudaProfilerStart/Stop (ncu captures)")
    ap.add_argument("--kernel-reps", type=int, default=20)
    ap.add_argument("--kernel-shapes", action="store_true",
                    help="launch each round shape of k_mega_pulse once after the prefill and exit (ncu captures)")
    ap.add_argument("--prefill-profile", action="store_true",
                    help="one profiled prefill of the bench prompt between cudaProfilerStart/Stop (ncu captures)")
    ap.add_argument("--ops", action="store_true",
                    help="time each pulsar_cuda forward op against the reference's own kernel (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.throughput_profile:
        world, rank, local = dist_setup()
        torch.cuda.set_device(local)
        print(json.dumps(throughput_b256(args, world, rank, local)), flush=True)
    elif args.kernel_shapes:
        run_kernel_shapes(args)
    elif args.prefill_profile:
        run_prefill_profile(args)
    elif args.ops:
        run_ops(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
