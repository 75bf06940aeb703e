"""CPU oracle for the Pulsar KV-cache decode path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the sm_100a engine is compared
against; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs may import it. The product path never routes through it.

It restates, in plain fp32 torch on the CPU, the algorithm of the reference inference
engine (src/infer.py) and the model pieces it calls (src/model.py). Every function cites
the reference lines it follows. Pinning: ``tests/golden/make_golden.py`` runs the real
reference here on the same synthetic weights and commits compact golden vectors;
``tests/test_oracle_golden.py`` checks this restatement against them.

Two deliberate representation choices (identical results, checked by the goldens):

* The KV cache is position-addressed (``[n_kv_heads, capacity, head_dim]`` per layer) and
  the sliding window is applied as a key-position mask, instead of physically trimming a
  growing tensor (src/infer.py:128-157). For one query per step both give the same key
  set ``[pos-1023, pos]``; position addressing also expresses rollback (a length reset,
  src/infer.py:159-168) and the block-verify rule below.
* Routed experts are evaluated per expert over the rows routed to it.

New behaviour that the reference does not have (so the goldens cannot pin it; it is
"parity unpinned" and specified here): gamma-token drafting from the pulse-1 exit,
one batched pulse-2/pulse-3 verify of the gamma+1 block with the block-verify KV rule,
greedy or ratio acceptance with residual resampling, and a Philox4x32-10 uniform stream.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

LOCAL_LAYERS = (0, 1, 2, 4, 5, 6)  # src/infer.py:93


def _cfg_get(cfg, name):
    return cfg[name] if isinstance(cfg, dict) else getattr(cfg, name)


# --------------------------------------------------------------------------------------
# Model pieces (src/model.py)
# --------------------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """src/model.py:386-392 (fp32 path): w * x * rsqrt(mean(x^2) + eps)."""
    xf = x.float()
    return w.float() * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps))


def rope_inv_freq(theta: float, dim: int) -> torch.Tensor:
    """src/model.py:532, 536-543: 1 / theta^(arange(0, dim, 2) / dim) in fp32."""
    return 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))


def rope_cos_sin(theta: float, dim: int, positions: torch.Tensor):
    """src/model.py:545-552: fp32 outer(t, inv_freq), then cos / sin, gathered at ``positions``."""
    inv = rope_inv_freq(theta, dim)
    freqs = torch.outer(positions.float(), inv)
    return freqs.cos(), freqs.sin()


def rotate_half_split(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """src/model.py:581-589: [x1 c - x2 s, x2 c + x1 s] over the two halves of head_dim.

    ``x`` is ``[..., T, dh]`` and cos/sin are ``[T, dh/2]``.
    """
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def causal_conv_k4(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """src/model.py:592-602: y[t] = x[t] + sum_k w[:, k] * x[t-k], zero-padded at the start
    of the given tensor. ``x`` is ``[T, D]``, ``w`` is ``[D, 4]``."""
    T = x.shape[0]
    y = x.clone()
    for k in range(w.shape[1]):
        if k >= T:
            break
        y[k:] = y[k:] + w[:, k] * x[: T - k]
    return y


def swiglu(gu: torch.Tensor, d_ff: int) -> torch.Tensor:
    """src/model.py:930-935: silu(gu[..., :d_ff]) * gu[..., d_ff:] in fp32."""
    return F.silu(gu[..., :d_ff]) * gu[..., d_ff:]


def merged_weight(base, lora_A, lora_B, loop_M, pulse: int, K: int, alpha: float) -> torch.Tensor:
    """src/model.py:716-727: W + (alpha/q) * sum_j M[p, j] * B_j A_j (fp32)."""
    q = lora_A.shape[1]
    d_in = lora_A.shape[2]
    d_out = lora_B.shape[1]
    A_all = lora_A[:K].reshape(K * q, d_in)
    B_perm = lora_B[:K].permute(1, 0, 2)
    B_scaled = (B_perm * (loop_M[pulse, :K] * (alpha / q)).view(1, K, 1)).reshape(d_out, K * q)
    return torch.addmm(base, B_scaled, A_all)


def merged_weight_bf16(base, lora_A, lora_B, loop_M, pulse: int, K: int, alpha: float) -> torch.Tensor:
    """src/model.py:716-727 with a bf16 base weight (the reference's GPU inference dtype):
    A_all = bf16(lora_A), B_scaled = bf16(bf16(lora_B) * bf16(loop_M[p] * alpha/q)), and the
    bf16 addmm taken as one rounding of (sum_c B_scaled[:, c] A_all[c] in fp32, in order c) +
    base. Each bf16 x bf16 product is exact in fp32, so the order fixes the value; the
    reference's GEMM may order its fp32 sum differently (last-bit differences)."""
    q = lora_A.shape[1]
    bf = torch.bfloat16
    A_all = lora_A[:K].to(bf).float().reshape(K * q, -1)
    ms = (loop_M[pulse, :K].float() * (alpha / q)).to(bf)
    B_perm = lora_B[:K].to(bf).permute(1, 0, 2)                       # [d_out][K][q]
    B_scaled = (B_perm * ms.view(1, K, 1)).float().reshape(B_perm.shape[0], K * q)
    acc = torch.zeros(B_scaled.shape[0], A_all.shape[1])
    for c in range(K * q):
        acc = acc + B_scaled[:, c:c + 1] * A_all[c:c + 1, :]
    return (acc + base.to(bf).float()).to(bf).float()


def router_topk(logits: torch.Tensor, bias: torch.Tensor, top_k: int):
    """src/infer.py:325-333 (and the fallback at src/model.py:1312-1317): centre the fp32
    logits, sigmoid, top-k of (scores + bias), weights = s_k / (sum s_k + 1e-6)."""
    logits = logits - logits.mean(dim=-1, keepdim=True)
    scores = torch.sigmoid(logits)
    _, idx = torch.topk(scores + bias, k=top_k, dim=-1)
    raw = torch.gather(scores, -1, idx)
    w = raw / (raw.sum(dim=-1, keepdim=True) + 1e-6)
    return idx, w, scores


def moe_capacity(n_tokens: int, cfg) -> int:
    """src/model.py:1339-1342."""
    avg = n_tokens * _cfg_get(cfg, "top_k") / _cfg_get(cfg, "n_routed_experts")
    raw = int(math.ceil(avg * _cfg_get(cfg, "moe_capacity_factor")))
    align = max(1, int(_cfg_get(cfg, "moe_capacity_align")))
    return max(align, ((raw + align - 1) // align) * align)


def token_slots(topk_idx: torch.Tensor, topk_w: torch.Tensor, n_experts: int, capacity: int) -> torch.Tensor:
    """src/model.py:996-1054 and :952-965: stable sort by key e - 0.5*w/(1+w) (expert
    ascending, weight descending), rank within expert, slot = rank if rank < capacity
    else -1. Returns int32 ``[N, K]``."""
    N, K = topk_idx.shape
    flat_e = topk_idx.reshape(-1).long()
    M = flat_e.numel()
    if M == 0:
        return torch.empty((N, K), dtype=torch.int32)
    flat_w = topk_w.reshape(-1).float()
    wc = flat_w.clamp_min(0.0)
    key = flat_e.to(torch.float32) - (wc / (1.0 + wc)) * 0.5
    order = torch.argsort(key, stable=True)
    e_sorted = flat_e[order]
    counts = torch.zeros(n_experts, dtype=torch.long)
    counts.index_add_(0, e_sorted, torch.ones(M, dtype=torch.long))
    start = counts.cumsum(0) - counts
    rank = torch.arange(M) - start[e_sorted]
    slot_sorted = torch.where(rank < capacity, rank.to(torch.int32), torch.full_like(rank, -1, dtype=torch.int32))
    slots = torch.empty(M, dtype=torch.int32)
    slots[order] = slot_sorted
    return slots.view(N, K)


# --------------------------------------------------------------------------------------
# Weights
# --------------------------------------------------------------------------------------

class OracleModel:
    """fp32 copies of the reference parameters, LoRA pre-merged per pulse.

    The merge result is exactly what ``get_merged_weight`` returns in fp32
    (src/model.py:716-727), which the reference recomputes on every call
    (src/infer.py:250-254, 308-312).
    """

    def __init__(self, state_dict, cfg, merge: str = "fp32"):
        """merge: "fp32" (the reference's fp32 run, the default) or "bf16" (its GPU path's
        bf16 merged weights, merged_weight_bf16)."""
        self.cfg = cfg
        g = lambda n: _cfg_get(cfg, n)
        self.D = g("d_model")
        self.H = g("n_heads")
        self.Hkv = g("n_kv_heads")
        self.dh = g("head_dim")
        self.L = g("n_core")
        self.K = g("default_pulses")
        self.E = g("n_routed_experts")
        self.top_k = g("top_k")
        self.d_expert = g("d_expert")
        self.d_shared = g("d_shared") if g("d_shared") is not None else g("d_expert")
        self.eps = g("rms_eps")
        self.window = g("sliding_window")
        self.base_seq_len = g("base_seq_len")
        self.softcap = g("logit_softcap")
        self.theta_local = g("rope_theta_local")
        self.theta_global = g("rope_theta_global")
        self.per_pulse_bias = g("per_pulse_bias")
        self.alpha = g("loop_lora_alpha")
        self.sd = {k: v.detach().float().cpu() for k, v in state_dict.items()}
        sd = self.sd
        self.tok_emb = sd["tok_emb"+".weight"]
        self.lm_head = sd.get("lm_head.weight", self.tok_emb)
        self.stem = sd.get("stem_canon_weight") if g("use_canon_conv") else None
        self.wqkv = [[None] * self.L for _ in range(self.K)]
        self.wo = [[None] * self.L for _ in range(self.K)]
        for i in range(self.L):
            b = f"core.{i}.attn."
            for p in range(self.K):
                if (b + "wqkv_adapter.lora_A") in sd and g("loop_lora_rank") > 0:
                    mw = merged_weight_bf16 if merge == "bf16" else merged_weight
                    self.wqkv[p][i] = mw(sd[b + "wqkv.weight"], sd[b + "wqkv_adapter.lora_A"],
                                         sd[b + "wqkv_adapter.lora_B"], sd[b + "wqkv_adapter.loop_M"],
                                         p, self.K, self.alpha)
                    self.wo[p][i] = mw(sd[b + "wo.weight"], sd[b + "wo_adapter.lora_A"],
                                       sd[b + "wo_adapter.lora_B"], sd[b + "wo_adapter.loop_M"],
                                       p, self.K, self.alpha)
                else:
                    self.wqkv[p][i] = sd[b + "wqkv.weight"]
                    self.wo[p][i] = sd[b + "wo.weight"]

    def p(self, name):
        return self.sd[name]

    def expert_bias(self, layer, pulse):
        b = self.sd[f"core.{layer}.mlp.expert_bias"]
        return b[pulse] if self.per_pulse_bias else b


# --------------------------------------------------------------------------------------
# KV cache
# --------------------------------------------------------------------------------------

class OracleKV:
    """Position-addressed restatement of UnifiedKVCache (src/infer.py:64-178).

    ``length`` is the number of committed positions. Keys visible to a query at position
    ``pos`` on layer ``i`` are ``[pos - window + 1, pos]`` for local layers and ``[0, pos]``
    for global layers, exactly the set the reference's trimmed cache holds at that point.
    """

    def __init__(self, model: OracleModel, capacity: int):
        self.m = model
        self.capacity = capacity
        self.k = [torch.zeros(model.Hkv, capacity, model.dh) for _ in range(model.L)]
        self.v = [torch.zeros(model.Hkv, capacity, model.dh) for _ in range(model.L)]
        self.length = 0

    def key_range(self, layer: int, pos: int):
        lo = max(0, pos - self.m.window + 1) if layer in LOCAL_LAYERS else 0
        return lo, pos + 1

    def checkpoint_state(self):
        """src/infer.py:159-161 (a single committed length covers every layer)."""
        return self.length

    def restore_state(self, length: int):
        """src/infer.py:163-168: truncate to the checkpointed length."""
        self.length = min(self.length, length)

    def memory_footprint_bytes(self, dtype_bytes: int = 2) -> int:
        """src/infer.py:170-178 for the logical cache contents of the reference."""
        total = 0
        for i in range(self.m.L):
            n = min(self.length, self.m.window) if i in LOCAL_LAYERS else self.length
            total += 2 * self.m.Hkv * n * self.m.dh * dtype_bytes
        return total


# --------------------------------------------------------------------------------------
# One pulse over a block of rows (decode: 1 row, block verify: gamma+1 rows)
# --------------------------------------------------------------------------------------

def _attention_rows(m: OracleModel, layer: int, pulse: int, a: torch.Tensor, positions: list[int],
                    kv: OracleKV, v_first, yarn: bool):
    """src/infer.py:234-314 generalised to R consecutive rows of one sequence.

    Every row writes its K/V at its position first (pulse 0 appends, later pulses
    overwrite the same slot, src/infer.py:140-155), then each row attends to its key
    range; in-block predecessors are therefore seen with their pulse-``pulse`` K/V.
    With one row this is exactly the reference step.
    """
    R = a.shape[0]
    H, Hkv, dh = m.H, m.Hkv, m.dh
    b = f"core.{layer}.attn."
    qkv = a @ m.wqkv[pulse][layer].t()
    q, k, v = qkv.split([H * dh, Hkv * dh, Hkv * dh], dim=-1)
    q = q.view(R, H, dh)
    k = k.view(R, Hkv, dh)
    v = v.view(R, Hkv, dh)
    if layer == 0 and pulse == 0:
        v_first = v
    elif v_first is not None:
        lv = torch.sigmoid(m.p(b + "v_resid_lambda")[pulse])
        v = (1.0 - lv) * v + lv * v_first
    q = m.p(b + "q_norm_weight")[pulse].view(1, H, dh) * (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + m.eps))
    k = m.p(b + "k_norm_weight")[pulse].view(1, Hkv, dh) * (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + m.eps))
    is_local = layer in LOCAL_LAYERS
    theta = m.theta_local if is_local else m.theta_global
    pos_t = torch.tensor(positions, dtype=torch.long)
    cos, sin = rope_cos_sin(theta, dh, pos_t)                 # [R, dh/2]
    q = rotate_half_split(q.transpose(0, 1), cos, sin).transpose(0, 1)   # [R, H, dh]
    k = rotate_half_split(k.transpose(0, 1), cos, sin).transpose(0, 1)
    if yarn and not is_local:
        # src/infer.py:288-291 (decode only; prefill applies none, src/infer.py:422-425)
        scales = []
        for pos in positions:
            if pos + 1 > m.base_seq_len:
                base = float(m.base_seq_len)
                scales.append(1.0 + 0.1 * math.log(max(pos + 1, base) / base))
            else:
                scales.append(1.0)
        q = q * torch.tensor(scales, dtype=torch.float32).view(R, 1, 1)
    for r, pos in enumerate(positions):
        kv.k[layer][:, pos] = k[r]
        kv.v[layer][:, pos] = v[r]
    group = H // Hkv
    out = torch.empty(R, H, dh)
    scale = 1.0 / math.sqrt(dh)
    for r, pos in enumerate(positions):
        lo, hi = kv.key_range(layer, pos)
        K_all = kv.k[layer][:, lo:hi]                          # [Hkv, S, dh]
        V_all = kv.v[layer][:, lo:hi]
        Kq = K_all.repeat_interleave(group, dim=0)             # [H, S, dh] (enable_gqa)
        Vq = V_all.repeat_interleave(group, dim=0)
        s = torch.einsum("hd,hsd->hs", q[r], Kq) * scale
        pr = torch.softmax(s, dim=-1)
        out[r] = torch.einsum("hs,hsd->hd", pr, Vq)
    gate = torch.sigmoid(a @ m.p(b + "attn_gate")[pulse].t() + m.p(b + "attn_gate_bias")[pulse])  # [R, H]
    out = (out * gate.unsqueeze(-1)).reshape(R, H * dh)
    return out @ m.wo[pulse][layer].t(), v_first


def _moe_rows(m: OracleModel, layer: int, pulse: int, x: torch.Tensor, record=None):
    """src/infer.py:316-351 for R rows: fp32 router, top-k, shared SwiGLU expert and the
    routed experts, ``shared + routed * routed_scale[p]``."""
    b = f"core.{layer}.mlp."
    logits = x @ m.p(b + "router_weight")[pulse].t()
    idx, w, _ = router_topk(logits, m.expert_bias(layer, pulse), m.top_k)
    gu = x @ m.p(b + "shared_expert.w_gate_up.weight").t()
    shared = swiglu(gu, m.d_shared) @ m.p(b + "shared_expert.w_down.weight").t()
    routed = torch.zeros_like(x)
    W_gu = m.p(b + "routed_gate_up")
    W_dn = m.p(b + "routed_down")
    for r in range(x.shape[0]):
        for kk in range(m.top_k):
            e = int(idx[r, kk])
            h = swiglu(x[r] @ W_gu[e], m.d_expert)
            routed[r] = routed[r] + (h @ W_dn[e]) * w[r, kk]
    if record is not None:
        record.append((layer, pulse, idx.clone(), w.clone()))
    return shared + routed * m.p(b + "routed_scale")[pulse]


def pulse_input(m: OracleModel, pulse: int, tokens: list[int], h_prev, h0n):
    """src/infer.py:474-501. Pulse 0 embeds and normalises the tokens; the stem conv sees
    only the current token (the single-token quirk, src/infer.py:477-479), i.e. x + w0*x.
    Later pulses mix the previous pulse output with the anchor through the rank-r gate."""
    D = m.D
    if pulse == 0:
        h0 = m.tok_emb[torch.tensor(tokens, dtype=torch.long)]
        h0n = rmsnorm(h0, m.p("anchor_norm.weight"), m.eps)
        if m.stem is not None:
            h0n = h0n + m.stem[:, 0] * h0n
        return h0n + m.p("pulse_step_emb.weight")[0], h0n
    r = rmsnorm(h_prev, m.p("pulse_state_norm.weight"), m.eps)
    wd = m.p("reinject_gate_down")[pulse]
    g = h0n @ wd[:, :D].t() + r @ wd[:, D:].t()
    mix = torch.sigmoid(g @ m.p("reinject_gate_up")[pulse].t() + m.p("reinject_gate_bias")[pulse])
    return torch.lerp(r, h0n, mix) + m.p("pulse_step_emb.weight")[pulse], h0n


def pulse_pass(m: OracleModel, pulse: int, tokens: list[int], positions: list[int], kv: OracleKV,
               h_prev=None, h0n=None, want_logits=True, record=None):
    """src/infer.py:463-524 for a block of rows: returns (softcapped logits [R, V] or
    None, h_out [R, D], h0n [R, D])."""
    h_in, h0n = pulse_input(m, pulse, tokens, h_prev, h0n)
    h = h_in
    v_first = None
    for i in range(m.L):
        a = rmsnorm(h, m.p(f"core.{i}.attn_norm.weight")[pulse], m.eps)
        att, v_first = _attention_rows(m, i, pulse, a, positions, kv, v_first, yarn=True)
        h = h + att
        x = rmsnorm(h, m.p(f"core.{i}.mlp_norm.weight")[pulse], m.eps)
        h = h + _moe_rows(m, i, pulse, x, record)
    h_out = h_in + (h - h_in) * m.p("pulse_res_scale")[pulse]
    logits = None
    if want_logits:
        logits = rmsnorm(h_out, m.p("final_norm.weight"), m.eps) @ m.lm_head.t()
        if m.softcap and m.softcap > 0:
            logits = m.softcap * torch.tanh(logits / m.softcap)
    return logits, h_out, h0n


# --------------------------------------------------------------------------------------
# Prefill (src/infer.py:353-461) with the reference's quirks
# --------------------------------------------------------------------------------------

def _prefill_moe(m: OracleModel, layer: int, pulse: int, x: torch.Tensor) -> torch.Tensor:
    """PulsarMoEMLP.forward as prefill calls it (src/model.py:1265-1493, CPU fallback
    branch): fp32 router (x.dtype), top-k, capacity ``moe_capacity`` with the
    deterministic lowest-weight drop order, routed experts with routed_scale folded into
    the down projection, combine onto the shared expert output."""
    b = f"core.{layer}.mlp."
    N = x.shape[0]
    logits = x @ m.p(b + "router_weight")[pulse].t()
    idx, w, _ = router_topk(logits, m.expert_bias(layer, pulse), m.top_k)
    gu = x @ m.p(b + "shared_expert.w_gate_up.weight").t()
    out = swiglu(gu, m.d_shared) @ m.p(b + "shared_expert.w_down.weight").t()
    cap = moe_capacity(N, m.cfg)
    slots = token_slots(idx, w, m.E, cap)
    W_gu = m.p(b + "routed_gate_up")
    W_dn = m.p(b + "routed_down") * m.p(b + "routed_scale")[pulse].view(1, 1, -1)
    for e in range(m.E):
        sel = ((idx == e) & (slots >= 0)).nonzero(as_tuple=False)
        if sel.numel() == 0:
            continue
        rows, ks = sel[:, 0], sel[:, 1]
        h = swiglu(x[rows] @ W_gu[e], m.d_expert) @ W_dn[e]
        out.index_add_(0, rows, h * w[rows, ks].unsqueeze(-1))
    return out


def prefill(m: OracleModel, ids: list[int], kv: OracleKV, record=None) -> torch.Tensor:
    """src/infer.py:353-461. Returns the last position's logits [V] (NOT softcapped,
    src/infer.py:459-461) and fills the cache with every position's final-pulse K/V.

    Quirks reproduced: no YaRN query scale (src/infer.py:422-425); on local layers with
    T > window the cache is truncated to the last ``window`` keys and SDPA's
    ``is_causal`` mask is aligned top-left, so query i sees cached keys
    0..min(i, window-1) = absolute positions T-window .. T-window+min(i, window-1)
    (src/infer.py:128-137, 433-435); value residual only in pulse 0 (src/infer.py:390,408-412)."""
    h_pulse = _full_sequence(m, ids, kv, m.K, forward=False)
    return rmsnorm(h_pulse[-1], m.p("final_norm.weight"), m.eps) @ m.lm_head.t()


def forward_logits(m: OracleModel, ids: list[int], num_pulses: int | None = None) -> torch.Tensor:
    """PulsarForCausalLM.forward with labels=None (src/model.py:1956-2125), last position:
    the training-style full-sequence pass that model.generate recomputes per token. It differs
    from the inference prefill in four ways (src/model.py:837-899, 2119-2121): the value
    residual of layer 0 / pulse 0 carries into every later pulse; global layers scale queries by
    the YaRN factor 1 + 0.1 ln(max(t + 1, base) / base) of their position; local layers attend
    causally over the whole sequence when T <= max(window, 4096) and through the sliding window
    (0 <= i - j < window) beyond; the logits are softcapped."""
    K = num_pulses if num_pulses is not None else m.K
    h_pulse = _full_sequence(m, ids, OracleKV(m, len(ids)), K, forward=True)
    logits = rmsnorm(h_pulse[-1], m.p("final_norm.weight"), m.eps) @ m.lm_head.t()
    if m.softcap and m.softcap > 0:
        logits = m.softcap * torch.tanh(logits / m.softcap)
    return logits


def _full_sequence(m: OracleModel, ids: list[int], kv: OracleKV, K: int, forward: bool) -> torch.Tensor:
    """K pulses over the whole sequence; returns the final pulse output h [T, D]. forward=False:
    the inference prefill (src/infer.py:353-461, its K/V written to ``kv``); forward=True:
    PulsarForCausalLM.forward (see forward_logits)."""
    T = len(ids)
    H, Hkv, dh = m.H, m.Hkv, m.dh
    group = H // Hkv
    scale = 1.0 / math.sqrt(dh)
    h0 = m.tok_emb[torch.tensor(ids, dtype=torch.long)]
    h0n = rmsnorm(h0, m.p("anchor_norm.weight"), m.eps)
    if m.stem is not None:
        h0n = causal_conv_k4(h0n, m.stem)
    h_pulse = h0
    positions = torch.arange(T)
    v_first = None
    for k in range(K):
        if k == 0:
            h_in = h0n + m.p("pulse_step_emb.weight")[0]
        else:
            h_in, _ = pulse_input(m, k, ids, h_pulse, h0n)
        h = h_in
        if not forward:
            v_first = None   # the inference prefill keeps the value residual inside pulse 0
        for i in range(m.L):
            b = f"core.{i}.attn."
            a = rmsnorm(h, m.p(f"core.{i}.attn_norm.weight")[k], m.eps)
            qkv = a @ m.wqkv[k][i].t()
            q, kk, v = qkv.split([H * dh, Hkv * dh, Hkv * dh], dim=-1)
            q = q.view(T, H, dh).transpose(0, 1)          # [H, T, dh]
            kk = kk.view(T, Hkv, dh).transpose(0, 1)
            v = v.view(T, Hkv, dh).transpose(0, 1)
            if i == 0 and k == 0:
                v_first = v
            elif v_first is not None:
                lv = torch.sigmoid(m.p(b + "v_resid_lambda")[k])
                v = (1.0 - lv) * v + lv * v_first
            q = m.p(b + "q_norm_weight")[k].view(H, 1, dh) * (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + m.eps))
            kk = m.p(b + "k_norm_weight")[k].view(Hkv, 1, dh) * (kk * torch.rsqrt(kk.pow(2).mean(-1, keepdim=True) + m.eps))
            is_local = i in LOCAL_LAYERS
            cos, sin = rope_cos_sin(m.theta_local if is_local else m.theta_global, dh, positions)
            q = rotate_half_split(q, cos, sin)
            kk = rotate_half_split(kk, cos, sin)
            kv.k[i][:, :T] = kk
            kv.v[i][:, :T] = v
            if forward:
                if not is_local and T > m.base_seq_len:   # YaRN per query position
                    pos1 = torch.arange(1, T + 1, dtype=torch.float32)
                    q = q * (1.0 + 0.1 * torch.log(pos1.clamp_min(m.base_seq_len) / float(m.base_seq_len))).view(1, T, 1)
                kc, vc = kk, v
                diff = positions.view(T, 1) - positions.view(1, T)
                if is_local and T > max(m.window, 4096):
                    mask = (diff >= 0) & (diff < m.window)
                else:
                    mask = diff >= 0
            else:
                if is_local and T > m.window:
                    kc, vc = kk[:, T - m.window:], v[:, T - m.window:]
                else:
                    kc, vc = kk, v
                S = kc.shape[1]
                mask = torch.ones(T, S, dtype=torch.bool).tril(diagonal=0)   # top-left aligned
            Kq = kc.repeat_interleave(group, dim=0)
            Vq = vc.repeat_interleave(group, dim=0)
            s = torch.einsum("htd,hsd->hts", q, Kq) * scale
            s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
            out = torch.einsum("hts,hsd->htd", torch.softmax(s, dim=-1), Vq)   # [H, T, dh]
            gate = torch.sigmoid(a @ m.p(b + "attn_gate")[k].t() + m.p(b + "attn_gate_bias")[k])  # [T, H]
            out = (out.transpose(0, 1) * gate.unsqueeze(-1)).reshape(T, H * dh)
            h = h + out @ m.wo[k][i].t()
            x = rmsnorm(h, m.p(f"core.{i}.mlp_norm.weight")[k], m.eps)
            h = h + _prefill_moe(m, i, k, x)
        h_pulse = h_in + (h - h_in) * m.p("pulse_res_scale")[k]
    kv.length = T
    return h_pulse


# --------------------------------------------------------------------------------------
# Decode steps and the reference generate loops
# --------------------------------------------------------------------------------------

def decode_step(m: OracleModel, token: int, pos: int, kv: OracleKV, early_exit_threshold=None,
                exit_counts=None, record=None, exit_probs=None) -> torch.Tensor:
    """src/infer.py:526-549: three pulses on one token (optional early exit on the
    softmax max); commits ``pos + 1`` positions. ``exit_probs`` (a list) receives the
    softmax max-probability of every pulse the exit rule examined."""
    h = h0n = None
    logits = None
    for k in range(m.K):
        lg, h, h0n = pulse_pass(m, k, [token], [pos], kv, h, h0n, record=record)
        logits = lg[0]
        if early_exit_threshold is not None and k < m.K - 1:
            pmax = torch.softmax(logits, dim=-1).max().item()
            if exit_probs is not None:
                exit_probs.append(pmax)
            if pmax >= early_exit_threshold:
                if exit_counts is not None:
                    exit_counts[k] += 1
                break
    else:
        if early_exit_threshold is not None and exit_counts is not None:
            exit_counts[m.K - 1] += 1
    kv.length = pos + 1
    return logits


def apply_repetition_penalty(logits: torch.Tensor, seen, penalty: float) -> torch.Tensor:
    """src/infer.py:582-589: divide positive logits of seen ids by the penalty, multiply
    the others."""
    out = logits.clone()
    if penalty != 1.0:
        for tid in set(seen):
            val = out[tid]
            out[tid] = val / penalty if val > 0 else val * penalty
    return out


def top_p_filter(scaled: torch.Tensor, top_p: float) -> torch.Tensor:
    """src/infer.py:595-602: keep the sorted prefix whose exclusive cumulative
    probability is <= top_p (the first token always kept); the rest become -inf."""
    if top_p >= 1.0:
        return scaled
    sorted_logits, sorted_idx = torch.sort(scaled, descending=True)
    cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
    remove = cum > top_p
    remove[1:] = remove[:-1].clone()
    remove[0] = False
    out = scaled.clone()
    out[sorted_idx[remove]] = float("-inf")
    return out


def warped_probs(logits: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """src/infer.py:594-608: temperature, top-p, softmax, nan_to_num, renormalise."""
    scaled = logits / max(temperature, 1e-5)
    scaled = top_p_filter(scaled, top_p)
    probs = torch.softmax(scaled, dim=-1).nan_to_num(0.0)
    s = probs.sum()
    if s <= 0:
        return None
    return probs / s


def _start(m: OracleModel, prompt: list[int], kv, first_logits, capacity: int):
    """The cache and first-token logits a generate loop starts from: a fresh prefill, or a
    given cache that already holds the prompt (its length must be len(prompt)) with the
    logits computed alongside it."""
    if kv is None:
        kv = OracleKV(m, capacity)
        return kv, prefill(m, prompt, kv)
    if first_logits is None or kv.length != len(prompt):
        raise ValueError("a given cache needs first_logits and must hold exactly the prompt's positions")
    return kv, first_logits.float().reshape(-1).cpu()


def stream_generate_ids(m: OracleModel, prompt: list[int], max_new_tokens: int, temperature: float = 0.0,
                        top_p: float = 1.0, repetition_penalty: float = 1.0, stop_ids=(), capacity=None,
                        generator: torch.Generator | None = None, trace=None, early_exit_threshold=None,
                        exit_counts=None, exit_probs=None, kv: OracleKV | None = None,
                        first_logits: torch.Tensor | None = None) -> list[int]:
    """src/infer.py:551-621 returning token ids. Greedy when temperature <= 1e-4 (ties to
    the lowest index, as torch.argmax); sampling uses torch.multinomial on ``generator``.
    ``early_exit_threshold`` / ``exit_counts`` / ``exit_probs``: the engine's adaptive early
    exit inside decode_step (src/infer.py:199-200, 536-546).
    ``kv`` + ``first_logits``: start from a cache already holding the prompt (length
    len(prompt)) and the logits that choose the first token, instead of running prefill."""
    kv, logits = _start(m, prompt, kv, first_logits, capacity or (len(prompt) + max_new_tokens + 8))
    if trace is not None:
        trace.append(("prefill", logits.clone()))
    all_ids = list(prompt)
    pos = len(prompt) - 1
    out = []
    for _ in range(max_new_tokens):
        lg = apply_repetition_penalty(logits, all_ids, repetition_penalty)
        if temperature <= 1e-4:
            tok = int(lg.argmax())
        else:
            probs = warped_probs(lg, temperature, top_p)
            tok = int(lg.argmax()) if probs is None else int(torch.multinomial(probs, 1, generator=generator))
        if tok in stop_ids:
            break
        all_ids.append(tok)
        out.append(tok)
        pos += 1
        logits = decode_step(m, tok, pos, kv, early_exit_threshold=early_exit_threshold, exit_counts=exit_counts,
                             exit_probs=exit_probs)
        if trace is not None:
            trace.append(("step", logits.clone()))
    return out


def model_generate_ids(m: OracleModel, input_ids, max_new_tokens: int = 64, temperature: float = 0.7,
                       top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.15,
                       num_pulses: int | None = None, eos_token_id: int | None = None,
                       generator: torch.Generator | None = None) -> list[list[int]]:
    """PulsarForCausalLM.generate (src/model.py:2246-2317): every step recomputes the whole
    context (the last max_seq_len ids) with forward_logits, penalises the ids of the row seen
    so far, then greedy argmax (temperature 0) or temperature, top-k (logits below the k-th
    value -> -inf), top-p over the sorted softmax (the first token always kept) and a
    multinomial draw; finished rows emit eos; the loop stops when every row has finished.
    Rows are run one at a time: the reference's batched forward shares one MoE capacity
    across the rows of a batch, which couples rows only when the capacity overflows."""
    eos = eos_token_id if eos_token_id is not None else _cfg_get(m.cfg, "eos_token_id")
    max_len = _cfg_get(m.cfg, "max_seq_len")
    rows = [list(map(int, r)) for r in input_ids]
    finished = [False] * len(rows)
    for _ in range(max_new_tokens):
        for b, row in enumerate(rows):
            lg = forward_logits(m, row[-max_len:], num_pulses).clone()
            if repetition_penalty != 1.0:
                for tok in set(row):
                    lg[tok] = lg[tok] / repetition_penalty if lg[tok] > 0 else lg[tok] * repetition_penalty
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
    return rows


def self_speculative_ids(m: OracleModel, prompt: list[int], max_new_tokens: int, temperature: float = 0.0,
                         top_p: float = 1.0, repetition_penalty: float = 1.0, stop_ids=(), capacity=None,
                         generator: torch.Generator | None = None, stats=None) -> list[int]:
    """src/infer.py:623-731: the reference's self-speculative loop (draft one token from
    the pulse-1 exit, verify with pulses 2-3 on the same token, accept on id equality,
    then a full decode_step on the accepted token)."""
    kv = OracleKV(m, capacity or (len(prompt) + max_new_tokens + 8))
    logits = prefill(m, prompt, kv)
    all_ids = list(prompt)
    pos = len(prompt) - 1
    out = []

    def sample(lg):
        lg = apply_repetition_penalty(lg, all_ids, repetition_penalty)
        if temperature <= 1e-4:
            return int(lg.argmax())
        probs = warped_probs(lg, temperature, top_p)
        if probs is None:
            return int(lg.argmax())
        return int(torch.multinomial(probs, 1, generator=generator))

    while len(out) < max_new_tokens:
        t = sample(logits)
        if t in stop_ids:
            break
        all_ids.append(t)
        out.append(t)
        pos += 1
        if len(out) >= max_new_tokens:
            break
        d_logits, h0, h0n = pulse_pass(m, 0, [t], [pos], kv)
        draft = sample(d_logits[0])
        _, h1, _ = pulse_pass(m, 1, [t], [pos], kv, h0, h0n, want_logits=False)
        v_logits, _, _ = pulse_pass(m, 2, [t], [pos], kv, h1, h0n)
        kv.length = pos + 1
        true = sample(v_logits[0])
        if stats is not None:
            stats["drafts"] = stats.get("drafts", 0) + 1
        if draft == true and draft not in stop_ids:
            if stats is not None:
                stats["accepted"] = stats.get("accepted", 0) + 1
            all_ids.append(draft)
            out.append(draft)
            pos += 1
            if len(out) >= max_new_tokens:
                break
            logits = decode_step(m, draft, pos, kv)
        else:
            logits = v_logits[0]
    return out


# --------------------------------------------------------------------------------------
# New behaviour: gamma drafting + block verify + acceptance (no reference counterpart)
# --------------------------------------------------------------------------------------

PHILOX_M0 = 0xD2511F53
PHILOX_M1 = 0xCD9E8D57
PHILOX_W0 = 0x9E3779B9
PHILOX_W1 = 0xBB67AE85


def philox4x32_10(counter, key):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11, "Parallel random numbers: as easy
    as 1, 2, 3"): ten rounds of the 4x32 S-box with multipliers 0xD2511F53 / 0xCD9E8D57
    and Weyl key increments 0x9E3779B9 / 0xBB67AE85. ``counter`` is 4 uint32, ``key`` 2."""
    c0, c1, c2, c3 = (int(x) & 0xFFFFFFFF for x in counter)
    k0, k1 = (int(x) & 0xFFFFFFFF for x in key)
    for _ in range(10):
        p0 = PHILOX_M0 * c0
        p1 = PHILOX_M1 * c2
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & 0xFFFFFFFF, lo1, (hi0 ^ c3 ^ k1) & 0xFFFFFFFF, lo0
        k0 = (k0 + PHILOX_W0) & 0xFFFFFFFF
        k1 = (k1 + PHILOX_W1) & 0xFFFFFFFF
    return c0, c1, c2, c3


def uniforms(seed: int, seq: int, rnd: int, slot: int):
    """The four uniforms in [0, 1) of stream (seq, round, slot): counter = (seq, round,
    slot, 0), key = (seed low 32 bits, seed high 32 bits); u = (x >> 8) * 2^-24."""
    x = philox4x32_10((seq, rnd, slot, 0), (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return tuple((v >> 8) * (1.0 / 16777216.0) for v in x)


def sample_from(probs: torch.Tensor, u: float) -> int:
    """Inverse-CDF draw in vocabulary order: the first index whose inclusive prefix sum
    exceeds u * total (float64 accumulation)."""
    p = probs.double().numpy()
    c = np.cumsum(p)
    t = u * c[-1]
    i = int(np.searchsorted(c, t, side="right"))
    i = min(i, len(p) - 1)
    while p[i] <= 0 and i > 0:   # never land on a zero-probability token
        i -= 1
    return i


@dataclass
class SpecStats:
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    accept_log: list = field(default_factory=list)    # (round, j, accepted, u, ratio)


def block_spec_generate_ids(m: OracleModel, prompt: list[int], max_new_tokens: int, gamma: int = 4,
                            temperature: float = 0.0, top_p: float = 1.0, seed: int = 0, seq_id: int = 0,
                            capacity=None, stats: SpecStats | None = None, trace=None, kv: OracleKV | None = None,
                            first_logits: torch.Tensor | None = None, repetition_penalty: float = 1.0) -> list[int]:
    """Self-speculative decoding with gamma drafts and one batched verify.

    Round with committed length n and pending token t0 (position n):
      1. drafts: pulse 0 on t0..t_{gamma-1} at positions n..n+gamma-1, each drafting
         d_{j+1} from its pulse-1-exit logits q_j (greedy argmax, or a warped-q draw
         with uniform u0 of stream (seq, round, j));
      2. verify: pulse 0 on d_gamma, then pulses 1 and 2 over the gamma+1 rows at once
         (block-verify KV rule: a row sees the committed prefix's final K/V and its
         in-block predecessors' K/V of the same pulse) -> verify logits P_0..P_gamma;
      3. accept d_j (j = 1..gamma) while greedy argmax(P_{j-1}) == d_j, or, sampling,
         u1 <= min(1, p_{j-1}(d_j) / q_{j-1}(d_j)) with p, q the warped distributions;
         at the first rejection the next token is argmax(P_{j-1}) / a draw from
         norm(max(0, p - q)) with u2; if all are accepted it is drawn from P_gamma;
      4. commit n..n+a (a = accepted drafts) and roll back the rest (length reset).
    The first pending token comes from the (unsoftcapped) prefill logits. ``kv`` +
    ``first_logits``: start from a cache already holding the prompt instead of prefilling.
    ``repetition_penalty``: src/infer.py:658-667 penalises every sample with the ids emitted
    before it; here the logits choosing the token at block position k (draft q_k, verify P_k)
    are penalised over the prompt, the emitted tokens (the pending t0 included) and the
    round's drafts d_1..d_k, so that greedy decoding emits the penalised sequential stream.
    The trace then holds the penalised logits (those the decisions are taken on).
    """
    greedy = temperature <= 1e-4
    kv, logits = _start(m, prompt, kv, first_logits, capacity or (len(prompt) + max_new_tokens + gamma + 8))
    n = len(prompt)
    out: list[int] = []
    rnd = 0
    seen = list(prompt)

    def penal(lg, extra):
        return apply_repetition_penalty(lg, seen + list(extra), repetition_penalty) if repetition_penalty != 1.0 else lg

    logits = penal(logits, [])
    if greedy:
        t0 = int(logits.argmax())
    else:
        probs = warped_probs(logits, temperature, top_p)
        t0 = int(logits.argmax()) if probs is None else sample_from(probs, uniforms(seed, seq_id, 0xFFFFFFFF, 0)[0])
    out.append(t0)
    seen.append(t0)
    while len(out) < max_new_tokens:
        toks = [t0]
        q_logits = []
        h_rows, h0n_rows = [], []
        for j in range(gamma):
            lg, h, h0n = pulse_pass(m, 0, [toks[j]], [n + j], kv)
            lg = penal(lg[0], toks[1:j + 1]).view(1, -1)
            q_logits.append(lg[0])
            h_rows.append(h)
            h0n_rows.append(h0n)
            if greedy:
                d = int(lg[0].argmax())
            else:
                qp = warped_probs(lg[0], temperature, top_p)
                d = int(lg[0].argmax()) if qp is None else sample_from(qp, uniforms(seed, seq_id, rnd, j)[0])
            toks.append(d)
        _, h, h0n = pulse_pass(m, 0, [toks[gamma]], [n + gamma], kv, want_logits=False)
        h_rows.append(h)
        h0n_rows.append(h0n)
        positions = list(range(n, n + gamma + 1))
        H = torch.cat(h_rows, 0)
        H0 = torch.cat(h0n_rows, 0)
        _, H, _ = pulse_pass(m, 1, toks, positions, kv, H, H0, want_logits=False)
        P, _, _ = pulse_pass(m, 2, toks, positions, kv, H, H0)
        if repetition_penalty != 1.0:
            P = torch.stack([penal(P[k], toks[1:k + 1]) for k in range(gamma + 1)])
        if trace is not None:
            trace.append((rnd, list(toks), torch.stack(q_logits), P.clone()))
        a = 0
        nxt = None
        for j in range(1, gamma + 1):
            d = toks[j]
            if greedy:
                tgt = int(P[j - 1].argmax())
                ok = tgt == d
                if not ok:
                    nxt = tgt
            else:
                u = uniforms(seed, seq_id, rnd, j - 1)
                p = warped_probs(P[j - 1], temperature, top_p)
                q = warped_probs(q_logits[j - 1], temperature, top_p)
                pd = float(p[d]) if p is not None else 0.0
                qd = float(q[d]) if q is not None else 0.0
                ratio = 1.0 if qd <= 0 else min(1.0, pd / qd)
                ok = u[1] <= ratio
                if stats is not None:
                    stats.accept_log.append((rnd, j, ok, u[1], ratio))
                if not ok:
                    resid = (p - q).clamp_min(0.0) if (p is not None and q is not None) else p
                    if resid is None or float(resid.sum()) <= 0:
                        nxt = int(P[j - 1].argmax())
                    else:
                        nxt = sample_from(resid / resid.sum(), u[2])
            if not ok:
                break
            a += 1
        if nxt is None:
            if greedy:
                nxt = int(P[gamma].argmax())
            else:
                p = warped_probs(P[gamma], temperature, top_p)
                nxt = int(P[gamma].argmax()) if p is None else sample_from(p, uniforms(seed, seq_id, rnd, gamma)[2])
        if stats is not None:
            stats.rounds += 1
            stats.drafted += gamma
            stats.accepted += a
        emitted = toks[1:1 + a] + [nxt]
        for t in emitted:
            if len(out) < max_new_tokens:
                out.append(t)
                seen.append(t)
        n = n + a + 1
        kv.length = n
        t0 = nxt
        rnd += 1
    if stats is not None:
        stats.emitted = len(out)
    return out[:max_new_tokens]
