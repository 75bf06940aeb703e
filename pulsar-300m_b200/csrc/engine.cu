// Host side of the Pulsar decode engine: weight staging and repack, the per-slot KV cache,
// workspaces, the pulse-pass / prefill drivers, the graph-captured decode loops and the
// pulsar_engine_* C ABI (include/pulsar_b200.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "capi_util.h"
#include "engine_kernels.cuh"
#include "prefill_kernels.cuh"
#include "mega_launch.h"
#include "sampling.cuh"
#include "tc_gemm.cuh"
#include "prefill_attn_tc.cuh"
#include "tma_gemm.cuh"
#include "dec_attn_tc.cuh"

using namespace pulsar;

namespace {

// ------------------------------------------------------------------ repack kernels
__global__ void k_f32_to_bf16(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16(src[i]);
}

// dst[b][c][r] = bf16(src[b][r][c]) for a batch of [rows][cols] matrices (32x32 tiles).
__global__ void k_transpose_bf16(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int rows, int cols) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const float* s = src + (int64_t)b * rows * cols;
    __nv_bfloat16* d = dst + (int64_t)b * rows * cols;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        tile[i][threadIdx.x] = (r < rows && c < cols) ? s[(int64_t)r * cols + c] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) d[(int64_t)c * rows + r] = __float2bfloat16(tile[threadIdx.x][i]);
    }
}

// Per-pulse merged weight in bf16, the reference's GPU path (get_merged_weight with a bf16
// base weight, src/model.py:716-727): A16 = bf16(lora_A[:3]) as [3q][d_in];
// Bs16[o][j*q + r] = bf16(bf16(lora_B[j][o][r]) * bf16(loop_M[p][j] * alpha / q));
// out[o][i] = bf16(sum_c Bs16[o][c] * A16[c][i] + W[o][i]): the product sum in fp32 in order
// c = 0 .. 3q-1 (each bf16 x bf16 product is exact in fp32), then the base weight added, one
// rounding (a GEMM's alpha * AB + beta * C epilogue).
__global__ void k_merge_adapter(const __nv_bfloat16* __restrict__ w, const float* __restrict__ lora_a,
                                const float* __restrict__ lora_b, const float* __restrict__ loop_m, int P, int p,
                                float scale, int d_out, int d_in, int q, __nv_bfloat16* __restrict__ out) {
    const int64_t n = (int64_t)d_out * d_in;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int o = (int)(e / d_in), i = (int)(e % d_in);
        float acc = 0.f;
        for (int j = 0; j < 3; ++j) {
            const float ms = __bfloat162float(__float2bfloat16(loop_m[p * P + j] * scale));
            for (int r = 0; r < q; ++r) {
                const float b = __bfloat162float(__float2bfloat16(
                    __bfloat162float(__float2bfloat16(lora_b[((int64_t)j * d_out + o) * q + r])) * ms));
                const float a = __bfloat162float(__float2bfloat16(lora_a[((int64_t)j * q + r) * d_in + i]));
                acc = __fadd_rn(acc, __fmul_rn(b, a));
            }
        }
        out[e] = __float2bfloat16(__fadd_rn(acc, __bfloat162float(w[e])));
    }
}

// Loop-adapter up factor for pulse p: dst[o][j*q + r] = lora_B[j][o][r] * (loop_M[p][j] * alpha / q).
__global__ void k_lora_b(const float* __restrict__ lora_b, const float* __restrict__ loop_m, int P, int p, float scale,
                         int d_out, int q, float* __restrict__ dst) {
    const int64_t n = (int64_t)d_out * 3 * q;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int o = (int)(i / (3 * q));
        const int jr = (int)(i % (3 * q));
        const int j = jr / q, r = jr % q;
        const float ms = loop_m[p * P + j] * scale;
        dst[i] = lora_b[((int64_t)j * d_out + o) * q + r] * ms;
    }
}

// RoPE tables (src/model.py:545-552): angle = fp32(pos * inv_freq[j]), cos / sin in fp32.
__global__ void k_rope_table(const float* __restrict__ inv_freq, int n, float* __restrict__ cs, float* __restrict__ sn) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)n * 32; i += (int64_t)gridDim.x * blockDim.x) {
        const int pos = (int)(i / 32), j = (int)(i % 32);
        const float a = __fmul_rn((float)pos, inv_freq[j]);
        cs[i] = cosf(a);
        sn[i] = sinf(a);
    }
}

// ------------------------------------------------------------------ decode-loop state kernels
struct SeqDev {
    int len;      // committed positions
    int pending;  // next token to process (already emitted)
    int n_out;    // tokens emitted
    int done;
    int rnd;      // speculative rounds so far (Philox stream index)
};

// Output buffer, length and sampling parameters of the running generate call; read by the
// graph kernels so a captured loop does not depend on the caller's output pointer.
struct LoopOut {
    int* out;
    int n_new;
    unsigned long long seed;   // sampled decoding: Philox key, temperature, top-p
    float temperature, top_p;
    float ee_thr;              // early exit: softmax max-probability threshold
    float rep_penalty;         // repetition penalty (1: off)
};

// Starts a generate call: sequence state, first token, and the row descriptors of round 0
// (speculative loop: toks[i][0] = first token, rows[i] = (slot, len, first)).
__global__ void k_seq_init(SeqDev* seqs, const int* lens, const int* first_tok, int n, int* out, int n_new,
                           const int* slots, int gamma, int* toks, int4* rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    seqs[i].len = lens[i];
    seqs[i].pending = first_tok[i];
    seqs[i].n_out = 1;
    seqs[i].done = n_new <= 1;
    seqs[i].rnd = 0;
    out[(int64_t)i * n_new] = first_tok[i];
    toks[i * (gamma + 1)] = first_tok[i];
    rows[i] = make_int4(slots[i], lens[i], first_tok[i], 0);
}

__global__ void k_rows_step(const SeqDev* seqs, const int* slots, int n, int4* rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) rows[i] = make_int4(slots[i], seqs[i].len, seqs[i].pending, 0);
}

// Early-exit step state (ee: [0] skip flag of the persistent kernel, [1] rows exited so far,
// [2 + i] the pulse row i exits at). rows[i].w bit 0 set = row i exited early: later pulses
// keep its cached K/V (the exiting pulse's) and their outputs for it are not used.
__global__ void k_rows_step_ee(const SeqDev* seqs, const int* slots, int n, int4* rows, int* ee) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) ee[0] = ee[1] = 0;
    if (i < n) {
        rows[i] = make_int4(slots[i], seqs[i].len, seqs[i].pending, 0);
        ee[2 + i] = NP - 1;
    }
}

// src/infer.py:536-543: after pulse `pulse` (< K - 1), row i exits when the softmax of its
// logits has max-probability >= threshold, i.e. 1 / sum_j exp(l_j - max) >= threshold.
// Finished sequences count as exited (not tallied). The last row to exit sets the skip flag,
// so a persistent pulse kernel launched afterwards returns at once.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_ee_check(const float* __restrict__ lg, int V, int n, int pulse,
                                                   const LoopOut* lo, const SeqDev* seqs, int4* rows, int* ee) {
    __shared__ float red[32];
    const int i = blockIdx.x;
    if (rows[i].w & 1) return;   // exited at an earlier pulse (uniform over the block)
    const bool done = seqs[i].done != 0;
    bool ex = done;
    if (!done) {
        const float* x = lg + (int64_t)i * V;
        float mx = -INFINITY;
        for (int j = threadIdx.x; j < V; j += SAMPLE_THREADS) mx = fmaxf(mx, x[j]);
        mx = sblock_max(mx, red);
        float z = 0.f;
        for (int j = threadIdx.x; j < V; j += SAMPLE_THREADS) z += expf(x[j] - mx);
        z = sblock_sum(z, red);
        ex = 1.f / z >= lo->ee_thr;
    }
    if (ex && threadIdx.x == 0) {
        rows[i].w |= 1;
        if (!done) ee[2 + i] = pulse;
        if (atomicAdd(&ee[1], 1) + 1 == n) ee[0] = 1;
    }
}

// Commit of an early-exit step: the token is the argmax of the exiting pulse (amax_p[k] rows).
__global__ void k_commit_ee(SeqDev* seqs, const int* amax0, const int* amax1, const int* amax2, const int* ee, int n,
                            const LoopOut* lo, unsigned long long* counts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || seqs[i].done) return;
    const int k = ee[2 + i];
    const int t = k == 0 ? amax0[i] : k == 1 ? amax1[i] : amax2[i];
    atomicAdd(&counts[k], 1ull);
    const int n_new = lo->n_new;
    lo->out[(int64_t)i * n_new + seqs[i].n_out] = t;
    seqs[i].n_out += 1;
    seqs[i].pending = t;
    seqs[i].len += 1;
    if (seqs[i].n_out >= n_new) seqs[i].done = 1;
}

// Seen-token bitmap of a slot (W = V / 32 words): cleared, then the prompt's ids set.
__global__ void k_seen_init(uint32_t* __restrict__ sb, const int* __restrict__ ids, int T, int W) {
    for (int i = threadIdx.x; i < W; i += blockDim.x) sb[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < T; i += blockDim.x) atomicOr(&sb[ids[i] >> 5], 1u << (ids[i] & 31));
}

// src/infer.py:582-589: logits of seen ids divided by the penalty when positive, multiplied
// otherwise (IEEE division, as torch's), then the argmax (ties to the lowest index) of one
// logits row per block. Every thread returns the index.
__device__ int penalized_argmax(const float* __restrict__ lg, int V, const uint32_t* __restrict__ sb, float pen,
                                float* bv, int* bi) {
    ArgMax b{-INFINITY, 1 << 30};
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
        float v = lg[j];
        if ((sb[j >> 5] >> (j & 31)) & 1u) v = v > 0.f ? v / pen : v * pen;
        b = argmax_merge(b, ArgMax{v, j});
    }
    b = warp_argmax(b);
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        bv[w] = b.v;
        bi[w] = b.i;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        ArgMax c = threadIdx.x < nw ? ArgMax{bv[threadIdx.x], bi[threadIdx.x]} : ArgMax{-INFINITY, 1 << 30};
        c = warp_argmax(c);
        if (threadIdx.x == 0) bi[0] = c.i;
    }
    __syncthreads();
    return bi[0];
}

// First token of a penalized loop: penalized argmax of the first logits (seen = the prompt),
// which then joins the seen set.
__global__ void __launch_bounds__(1024) k_first_penalized(const float* __restrict__ lg, int V, const int* slots,
                                                         uint32_t* seen, const LoopOut* lo, int* out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int i = blockIdx.x;
    uint32_t* sb = seen + (int64_t)slots[i] * (V / 32);
    const int t = penalized_argmax(lg + (int64_t)i * V, V, sb, lo->rep_penalty, bv, bi);
    if (threadIdx.x == 0) {
        out[i] = t;
        sb[t >> 5] |= 1u << (t & 31);
    }
}

// Commit of a penalized sequential step (one block per sequence): the logits row of the
// exiting pulse (ee given) or of the last pulse, penalized argmax, seen set, exit tally.
__global__ void __launch_bounds__(1024) k_commit_penalized(SeqDev* seqs, const float* lg0, const float* lg1,
                                                          const float* lg2, const int* ee, int n, int V,
                                                          const LoopOut* lo, const int* slots, uint32_t* seen,
                                                          unsigned long long* counts) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int i = blockIdx.x;
    if (seqs[i].done) return;   // uniform
    const int k = ee ? ee[2 + i] : NP - 1;
    const float* lg = (k == 0 ? lg0 : k == 1 ? lg1 : lg2) + (int64_t)i * V;
    uint32_t* sb = seen + (int64_t)slots[i] * (V / 32);
    const int t = penalized_argmax(lg, V, sb, lo->rep_penalty, bv, bi);
    if (threadIdx.x == 0) {
        if (ee) atomicAdd(&counts[k], 1ull);
        sb[t >> 5] |= 1u << (t & 31);
        const int n_new = lo->n_new;
        lo->out[(int64_t)i * n_new + seqs[i].n_out] = t;
        seqs[i].n_out += 1;
        seqs[i].pending = t;
        seqs[i].len += 1;
        if (seqs[i].n_out >= n_new) seqs[i].done = 1;
    }
}

// Repetition penalty of a speculative round, in place (src/infer.py:658-667 penalises every
// sample with the ids emitted before it). Row r of `lg` (one block each) belongs to sequence
// i = r / per_seq at block position k = (per_seq > 1 ? r % per_seq : kfix); its seen set is the
// slot's bitmap (prompt and emitted tokens, the pending token toks[i][0] included) plus the
// round's drafts toks[i][1..k] before it. Each seen id's logit is divided by the penalty when
// positive and multiplied otherwise, once per id. Rows of finished sequences are left alone
// (seqs null: every row is live). Dynamic shared memory: V / 8 bytes.
__global__ void __launch_bounds__(1024) k_penalize_rows(float* __restrict__ lg, int V, int per_seq, int kfix, int gamma,
                                                        const int* __restrict__ slots, const uint32_t* __restrict__ seen,
                                                        const int* __restrict__ toks, const LoopOut* lo,
                                                        const SeqDev* seqs) {
    extern __shared__ uint32_t sbits[];
    const int r = blockIdx.x;
    const int i = r / per_seq, k = per_seq > 1 ? r % per_seq : kfix;
    if (seqs && seqs[i].done) return;   // uniform
    const int W = V >> 5;
    const uint32_t* sb = seen + (int64_t)slots[i] * W;
    for (int w = threadIdx.x; w < W; w += blockDim.x) sbits[w] = sb[w];
    __syncthreads();
    if (threadIdx.x == 0)
        for (int j = 1; j <= k; ++j) {
            const int t = toks[i * (gamma + 1) + j];
            sbits[t >> 5] |= 1u << (t & 31);
        }
    __syncthreads();
    const float pen = lo->rep_penalty;
    float* row = lg + (int64_t)r * V;
    for (int w = threadIdx.x; w < W; w += blockDim.x) {
        uint32_t b = sbits[w];
        while (b) {
            const int v = w * 32 + __ffs(b) - 1;
            b &= b - 1;
            const float x = row[v];
            row[v] = x > 0.f ? x / pen : x * pen;
        }
    }
}

// Adds token t[i] to the seen set of slots[i] (the first token of a penalised sampled call).
__global__ void k_seen_add(uint32_t* seen, const int* slots, const int* t, int n, int V) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) atomicOr(&seen[(int64_t)slots[i] * (V / 32) + (t[i] >> 5)], 1u << (t[i] & 31));
}

__global__ void k_commit_greedy(SeqDev* seqs, const int* amax, int n, const LoopOut* lo) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || seqs[i].done) return;
    const int n_new = lo->n_new;
    const int t = amax[i];
    lo->out[(int64_t)i * n_new + seqs[i].n_out] = t;
    seqs[i].n_out += 1;
    seqs[i].pending = t;
    seqs[i].len += 1;
    if (seqs[i].n_out >= n_new) seqs[i].done = 1;
}

// Speculative round, draft step j >= 1: toks[i][j] = the token drafted at step j - 1, row i is
// (slot, len + j, toks[i][j]); at j = gamma also the verify block rows (slot, len + k, toks[i][k]).
__global__ void k_rows_spec(const SeqDev* seqs, const int* slots, int n, int gamma, int j, const int* amax,
                            int* toks, int4* rows, int4* rows_v) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int* tk = toks + i * (gamma + 1);
    tk[j] = amax[i];
    rows[i] = make_int4(slots[i], seqs[i].len + j, tk[j], 0);
    if (j == gamma)
        for (int k = 0; k <= gamma; ++k) rows_v[i * (gamma + 1) + k] = make_int4(slots[i], seqs[i].len + k, tk[k], 0);
}

// Greedy acceptance: accept drafts while the verify argmax of the previous row matches;
// the next pending token is the verify argmax after the last accepted draft. Also writes the
// next round's first row and toks[i][0]. With a repetition penalty (seen given) every emitted
// token joins the slot's seen set.
__global__ void k_accept_greedy(SeqDev* seqs, int* toks, const int* amax_v, int n, int gamma, const LoopOut* lo,
                                long long* stats, const int* slots, int4* rows, uint32_t* seen, int V) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || seqs[i].done) return;
    const int n_new = lo->n_new;
    int* out = lo->out;
    int* tk = toks + i * (gamma + 1);
    const int* am = amax_v + i * (gamma + 1);
    int a = 0;
    while (a < gamma && am[a] == tk[a + 1]) ++a;
    const int nxt = am[a];
    int no = seqs[i].n_out;
    uint32_t* sb = seen ? seen + (int64_t)slots[i] * (V / 32) : nullptr;
    for (int j = 1; j <= a && no < n_new; ++j) {
        out[(int64_t)i * n_new + no++] = tk[j];
        if (sb) sb[tk[j] >> 5] |= 1u << (tk[j] & 31);
    }
    if (no < n_new) {
        out[(int64_t)i * n_new + no++] = nxt;
        if (sb) sb[nxt >> 5] |= 1u << (nxt & 31);
    }
    seqs[i].n_out = no;
    seqs[i].len += a + 1;
    seqs[i].pending = nxt;
    seqs[i].rnd += 1;
    if (no >= n_new) seqs[i].done = 1;
    stats[i * 3 + 0] += 1;
    stats[i * 3 + 1] += gamma;
    stats[i * 3 + 2] += a;
    tk[0] = nxt;
    rows[i] = make_int4(slots[i], seqs[i].len, nxt, 0);
}

// ---- sampled decoding (temperature / top-p, Philox uniforms) ----------------------------------
// Warp statistics of row r of `logits` (row stride ld) and, when tok_out is set, a draw with
// uniform 0 of stream (seq_ids[r], round, slot), round = seqs[r].rnd (0xFFFFFFFF, the first
// token of a sequence, when seqs is null). Dynamic shared memory: V floats.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_warp_sample(const float* __restrict__ logits, int ld, int V,
                                                                const LoopOut* lo, const int* seq_ids,
                                                                const SeqDev* seqs, int slot, int* tok_out,
                                                                WarpStats* stats_out) {
    extern __shared__ float ev[];
    __shared__ float red[32];
    __shared__ double redd[33];
    __shared__ int redi[2];
    const int r = blockIdx.x;
    const float* lg = logits + (int64_t)r * ld;
    const WarpStats st = row_warp_stats(lg, V, lo->temperature, lo->top_p, ev, red);
    if (stats_out && threadIdx.x == 0) stats_out[r] = st;
    if (tok_out) {
        const uint32_t rnd = seqs ? (uint32_t)seqs[r].rnd : 0xFFFFFFFFu;
        const float u = stream_uniform(lo->seed, (uint32_t)seq_ids[r], rnd, (uint32_t)slot, 0);
        const int t = draw_index(V, u, [&](int i) { return warped_prob(lg[i], st); }, redd, redi);
        if (threadIdx.x == 0) tok_out[r] = t;
    }
}

// Sampled acceptance of one round (one block per sequence): for j = 1..gamma accept draft
// toks[j] iff u1 <= min(1, p_{j-1}(d) / q_{j-1}(d)); at the first rejection the next token is
// drawn from norm(max(0, p - q)) with u2 (the target argmax if that is empty); if all are
// accepted it is drawn from p_gamma with u2 of slot gamma. p rows: P[i*(gamma+1) + k];
// q rows: Q[k*n + i]. Then the commit of k_accept_greedy and the next round's first row.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_accept_sampled(SeqDev* seqs, int* toks, const float* __restrict__ P,
                                                                   const float* __restrict__ Q,
                                                                   const WarpStats* __restrict__ ps,
                                                                   const WarpStats* __restrict__ qs, int n, int gamma,
                                                                   int V, const int* seq_ids, const LoopOut* lo,
                                                                   long long* stats, const int* slots, int4* rows,
                                                                   uint32_t* seen) {
    __shared__ float red[32];
    __shared__ int redk[32];
    __shared__ double redd[33];
    __shared__ int redi[2];
    const int i = blockIdx.x;
    if (seqs[i].done) return;
    const uint32_t rnd = (uint32_t)seqs[i].rnd, sq = (uint32_t)seq_ids[i];
    const unsigned long long seed = lo->seed;
    int* tk = toks + i * (gamma + 1);
    int a = 0, nxt = -1;
    for (int j = 1; j <= gamma; ++j) {
        const int d = tk[j];
        const float* prow = P + (int64_t)(i * (gamma + 1) + j - 1) * V;
        const float* qrow = Q + (int64_t)((j - 1) * n + i) * V;
        const WarpStats sp = ps[i * (gamma + 1) + j - 1], sqs = qs[(j - 1) * n + i];
        const float pd = warped_prob(prow[d], sp), qd = warped_prob(qrow[d], sqs);
        const double ratio = (qd <= 0.f) ? 1.0 : fmin(1.0, (double)pd / (double)qd);
        const float u1 = stream_uniform(seed, sq, rnd, (uint32_t)(j - 1), 1);
        if ((double)u1 <= ratio) {
            ++a;
            continue;
        }
        float sres = 0.f;
        for (int k = threadIdx.x; k < V; k += SAMPLE_THREADS)
            sres += fmaxf(warped_prob(prow[k], sp) - warped_prob(qrow[k], sqs), 0.f);
        const float S = sblock_sum(sres, red);
        if (S > 0.f) {
            const float u2 = stream_uniform(seed, sq, rnd, (uint32_t)(j - 1), 2);
            nxt = draw_index(
                V, u2, [&](int k) { return fmaxf(warped_prob(prow[k], sp) - warped_prob(qrow[k], sqs), 0.f) / S; },
                redd, redi);
        } else {   // p <= q everywhere: the target argmax (ties to the lowest index)
            ArgMax b{-INFINITY, 1 << 30};
            for (int k = threadIdx.x; k < V; k += SAMPLE_THREADS) b = argmax_merge(b, ArgMax{prow[k], k});
            b = warp_argmax(b);
            __syncthreads();
            if ((threadIdx.x & 31) == 0) {
                red[threadIdx.x >> 5] = b.v;
                redk[threadIdx.x >> 5] = b.i;
            }
            __syncthreads();
            if (threadIdx.x < 32) {
                ArgMax c2{red[threadIdx.x], redk[threadIdx.x]};
                c2 = warp_argmax(c2);
                if (threadIdx.x == 0) redi[0] = c2.i;
            }
            __syncthreads();
            nxt = redi[0];
        }
        break;
    }
    if (nxt < 0) {
        const float* prow = P + (int64_t)(i * (gamma + 1) + gamma) * V;
        const WarpStats sp = ps[i * (gamma + 1) + gamma];
        const float u2 = stream_uniform(seed, sq, rnd, (uint32_t)gamma, 2);
        nxt = draw_index(V, u2, [&](int k) { return warped_prob(prow[k], sp); }, redd, redi);
    }
    if (threadIdx.x != 0) return;
    const int n_new = lo->n_new;
    int* out = lo->out;
    int no = seqs[i].n_out;
    uint32_t* sb = seen ? seen + (int64_t)slots[i] * (V / 32) : nullptr;   // repetition penalty on
    for (int j = 1; j <= a && no < n_new; ++j) {
        out[(int64_t)i * n_new + no++] = tk[j];
        if (sb) sb[tk[j] >> 5] |= 1u << (tk[j] & 31);
    }
    if (no < n_new) {
        out[(int64_t)i * n_new + no++] = nxt;
        if (sb) sb[nxt >> 5] |= 1u << (nxt & 31);
    }
    seqs[i].n_out = no;
    seqs[i].len += a + 1;
    seqs[i].pending = nxt;
    seqs[i].rnd += 1;
    if (no >= n_new) seqs[i].done = 1;
    stats[i * 3 + 0] += 1;
    stats[i * 3 + 1] += gamma;
    stats[i * 3 + 2] += a;
    tk[0] = nxt;
    rows[i] = make_int4(slots[i], seqs[i].len, nxt, 0);
}

int prefill_capacity(int T) {
    // src/model.py:1339-1342 with top_k 4, 16 experts, factor 1.25, align 32
    const double avg = (double)T * TOPK / E;
    const int raw = (int)std::ceil(avg * 1.25);
    return std::max(32, ((raw + 31) / 32) * 32);
}

}  // namespace

// ====================================================================================
struct pulsar_engine {
    pulsar_engine_config cfg{};
    int V = 0, P = 0;
    bool finalized = false, has_lora = false;
    std::map<std::string, float*> t;            // staged fp32 tensors (device)
    std::map<std::string, int64_t> expect;      // name -> numel
    std::vector<void*> allocs;
    // bf16 arena
    __nv_bfloat16* emb = nullptr;
    __nv_bfloat16 *wqkv[NL] = {}, *wo[NL] = {}, *sh_gu[NL] = {}, *sh_dn[NL] = {}, *r_gu[NL] = {}, *r_dn[NL] = {};
    // repacked bf16 arena tensors written before finalize (pulsar_engine_arena_write): the fp32
    // state_dict tensors they stand for need not be uploaded
    std::vector<std::string> arena_names;
    std::map<std::string, std::vector<std::string>> arena_covers;
    std::map<std::string, bool> arena_written;
    // option "merged_adapter": per-pulse bf16 merged wqkv / wo (the reference's GPU numerics);
    // every pass then runs without the fp32 adapter correction (and on the persistent kernel)
    bool merge_adapter = false;
    __nv_bfloat16 *wqkv_m[NP][NL] = {}, *wo_m[NP][NL] = {};
    float *lb_qkv[NP][NL] = {}, *lb_wo[NP][NL] = {};
    float vres[NP][NL] = {};
    float *cos_l = nullptr, *sin_l = nullptr, *cos_g = nullptr, *sin_g = nullptr;
    int rope_len = 0;
    // KV
    void* kv = nullptr;
    int64_t kv_bytes = 0, arena_bytes = 0, work_bytes = 0;
    KVLayer kvl[NL];
    int nch[NL] = {};
    // bf16 cache: one 2-D tensor map over the whole arena (rows of 64 elements, boxes of 128 rows)
    // for the tensor-core decode attention, and each layer's first row in it
    alignas(64) CUtensorMap kv_map{};
    bool kv_map_ok = false;
    int64_t kv_lrow[NL] = {};
    std::vector<int> len;
    // decode workspace (R <= MAX_ROWS)
    struct {
        float *h, *h_in, *xn, *qkv, *q, *vfirst, *part, *att, *act_sh, *act_r, *hn, *t_qkv, *t_wo, *wts, *pmax;
        int *idx, *pidx;
    } w{};
    // wide decode workspace: pulse passes of more than MAX_ROWS rows (GEMM regime), up to
    // wide_rows rows; MoE rows bucketed per expert with capacity = rows (nothing dropped)
    int wide_rows = 0;
    // rows per block of the split-K decode attention (the verify passes of the speculative loops
    // set gamma + 1 so a block stages each chunk of K/V once for its rows; 1 otherwise)
    int attn_rpb = 1;
    bool force_wide = false;   // option "wide": every pulse pass through the wide path
    bool use_tc = true;        // option "tc_gemm": tensor-core GEMMs (prefill, wide path)
    bool tc_attn = true;       // option "tc_attn": prefill attention on the tensor cores
    bool use_tma = true;       // option "tma_gemm": TMA-fed warp-specialised GEMM where it applies
    bool tc_dec = true;        // option "tc_dec_attn": decode attention on the tensor cores (bf16 cache)
    // bf16 hi / lo split of a GEMM's activations (tensor-core path), split_elems each
    __nv_bfloat16 *split_hi = nullptr, *split_lo = nullptr;
    int64_t split_elems = 0;
    struct {
        float *h, *h_in, *xn, *qkv, *q, *vfirst, *part, *att, *act_sh, *sh, *hn, *t_qkv, *t_wo, *wts, *act_e, *ye,
            *logits;
        int *idx, *lists, *cnt, *slot, *rows_e, *kept;
        // bf16 hi / lo of the GEMM operands their producers split: the normed rows, the attention
        // output and the final norm (xs, [rows][1024]), the shared expert's activation (ss), the
        // routed experts' activations (es, laid out like act_e)
        __nv_bfloat16 *xs_hi, *xs_lo, *ss_hi, *ss_lo, *es_hi, *es_lo;
    } ww{};
    // prefill workspace
    struct {
        int* ids;
        float *h0, *h0n_pre, *h0n, *hp, *h, *h_in, *xn, *qkv, *q, *o, *att, *vfirst, *t, *wts, *act_sh, *sh, *act_e,
            *ye, *hn, *pmax;
        int *idx, *lists, *cnt, *slot, *rows_e, *kept, *pidx;
        int cap;
        // bf16 hi / lo of the GEMM operands their producers split (as in the wide workspace)
        __nv_bfloat16 *xs_hi, *xs_lo, *ss_hi, *ss_lo, *es_hi, *es_lo;
    } pf{};
    // decode-loop state
    SeqDev* seqs = nullptr;
    int *slots_dev = nullptr, *toks = nullptr, *amax = nullptr, *lens_dev = nullptr, *first_dev = nullptr;
    int4 *rows = nullptr, *rows_v = nullptr;
    float *hblk = nullptr, *h0blk = nullptr, *htmp = nullptr, *htmp2 = nullptr, *h0tmp = nullptr, *logits_tmp = nullptr;
    long long* stats = nullptr;
    LoopOut* loop_out = nullptr;   // output buffer / length / sampling parameters of the running generate call
    // adaptive early exit of the sequential greedy loop: threshold (off: ee_on false), step
    // state [2 + max_batch], per-pulse argmax of pulses 0 and 1 [2][max_batch], exit tallies [NP]
    bool ee_on = false;
    float ee_thr = 1.f;
    int *ee = nullptr, *ee_amax = nullptr;
    unsigned long long* ee_counts = nullptr;
    // repetition penalty of the sequential greedy loop (off: rp_on false) and the seen-token
    // bitmap of every slot [max_batch][V / 32] (set by prefill and by every emitted token)
    bool rp_on = false;
    float rp = 1.f;
    uint32_t* seen = nullptr;
    // sampled decoding: draft logits rows [wide_rows][V] (row j*n + i), verify logits rows
    // [wide_rows][V] (row i*(gamma+1) + k), their warp statistics, sequence stream ids
    float *qbuf = nullptr, *pbuf = nullptr;
    WarpStats *qstats = nullptr, *pstats = nullptr;
    int* seq_ids_dev = nullptr;
    struct Graph {
        cudaGraphExec_t ex;
        int64_t kernels, mega;   // kernel nodes per replay, of which persistent pulse kernels
    };
    std::map<std::string, Graph> graphs;
    // launch tallies of the decode loop: kernels started by pulsar_engine_generate_greedy and
    // pulsar_engine_pulse (graph kernel nodes counted per replay), and the persistent kernels among them
    int64_t n_kernels = 0, n_mega = 0;
    // option "time_pulses": CUDA events recorded on the caller's stream around every pulse pass
    // launched outside graph capture; get_option("last_pulse_ns") reads the last interval
    cudaEvent_t tev[2] = {nullptr, nullptr};
    bool time_pulses = false;
    // persistent pulse kernel
    bool use_mega = false;
    int mega_grid = 0, mega_nch = 0;
    float *m_gate = nullptr, *m_part = nullptr, *m_g8 = nullptr, *m_pmax = nullptr, *m_rpart = nullptr;
    int *m_pidx = nullptr, *m_err = nullptr;
    unsigned *m_bar = nullptr, *m_tickets = nullptr;
    unsigned long long mega_wait_ns = WAIT_NS;   // option "wait_ns": bound of every wait in the persistent kernel
    int mega_stall_cta = -1;                     // option "stall_cta": test hook (a CTA whose first grid barrier runs out)
    unsigned long long* m_trace = nullptr;   // phase stamps of the last traced launch (option "trace")
    unsigned long long* m_experts = nullptr; // distinct routed experts streamed by persistent launches

    int dmalloc(void** p, size_t bytes, int64_t* counter) {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
        allocs.push_back(*p);
        if (counter) *counter += (int64_t)bytes;
        return PULSAR_OK;
    }
    template <typename T>
    int wmalloc(T** p, size_t n) { return dmalloc(reinterpret_cast<void**>(p), n * sizeof(T), &work_bytes); }

    const float* T_(const std::string& n) const {
        auto it = t.find(n);
        return it == t.end() ? nullptr : it->second;
    }
    std::string L(int l, const char* s) const { return "core." + std::to_string(l) + "." + s; }
    bool kv32() const { return cfg.kv_fp32 != 0; }
    // positions a row may use: inside every global layer's cache and the RoPE tables
    int max_pos() const { return std::min(kvl[3].cap, rope_len); }
};

namespace {

// wqkv / wo of pulse p (merged per pulse under option "merged_adapter"), and whether the fp32
// adapter correction applies
const __nv_bfloat16* w_qkv(const pulsar_engine* e, int p, int l) { return e->merge_adapter ? e->wqkv_m[p][l] : e->wqkv[l]; }
const __nv_bfloat16* w_o(const pulsar_engine* e, int p, int l) { return e->merge_adapter ? e->wo_m[p][l] : e->wo[l]; }
bool lora_live(const pulsar_engine* e) { return e->has_lora && !e->merge_adapter; }

// The engine's bf16 weight arena, tensor by tensor: name, slot, elements, and the fp32 state_dict
// tensors it is built from. Layouts are the engine's: wqkv [1536][1024], wo [1024][1024],
// shared gate_up [2048][1024] and down [1024][1024], routed gate_up transposed to
// [16][1024 out][1024 in] and down to [16][1024 out][512 in], tok_emb [V][1024] (also the LM head).
struct ArenaRef {
    __nv_bfloat16** ptr;
    int64_t numel;
};
ArenaRef arena_ref(pulsar_engine* e, const std::string& name) {
    if (name == "arena.tok_emb") return {&e->emb, (int64_t)e->V * D};
    for (int l = 0; l < NL; ++l) {
        const std::string p = "arena." + std::to_string(l) + ".";
        if (name == p + "wqkv") return {&e->wqkv[l], (int64_t)QKV * D};
        if (name == p + "wo") return {&e->wo[l], (int64_t)D * D};
        if (name == p + "shared_gate_up") return {&e->sh_gu[l], (int64_t)2 * DS * D};
        if (name == p + "shared_down") return {&e->sh_dn[l], (int64_t)D * DS};
        if (name == p + "routed_gate_up_t") return {&e->r_gu[l], (int64_t)E * 2 * DE * D};
        if (name == p + "routed_down_t") return {&e->r_dn[l], (int64_t)E * D * DE};
    }
    return {nullptr, 0};
}

void build_arena_names(pulsar_engine* e) {
    e->arena_names.push_back("arena.tok_emb");
    e->arena_covers["arena.tok_emb"] = {"tok_emb.weight", "lm_head.weight"};
    const char* parts[][2] = {{"wqkv", "attn.wqkv.weight"},
                              {"wo", "attn.wo.weight"},
                              {"shared_gate_up", "mlp.shared_expert.w_gate_up.weight"},
                              {"shared_down", "mlp.shared_expert.w_down.weight"},
                              {"routed_gate_up_t", "mlp.routed_gate_up"},
                              {"routed_down_t", "mlp.routed_down"}};
    for (int l = 0; l < NL; ++l)
        for (auto& pc : parts) {
            const std::string n = "arena." + std::to_string(l) + "." + pc[0];
            e->arena_names.push_back(n);
            e->arena_covers[n] = {e->L(l, pc[1])};
        }
}

bool arena_covered(const pulsar_engine* e, const std::string& tensor) {
    for (auto& kv : e->arena_written)
        if (kv.second)
            for (auto& c : e->arena_covers.at(kv.first))
                if (c == tensor) return true;
    return false;
}

void build_expect(pulsar_engine* e) {
    const int P = e->P, V = e->V, q = 8;
    auto& x = e->expect;
    x["tok_emb.weight"] = (int64_t)V * D;
    x["lm_head.weight"] = (int64_t)V * D;
    x["pulse_step_emb.weight"] = (int64_t)P * D;
    x["pulse_state_norm.weight"] = D;
    x["anchor_norm.weight"] = D;
    x["final_norm.weight"] = D;
    x["stem_canon_weight"] = (int64_t)D * 4;
    x["reinject_gate_down"] = (int64_t)P * RG * 2 * D;
    x["reinject_gate_up"] = (int64_t)P * D * RG;
    x["reinject_gate_bias"] = (int64_t)P * D;
    x["pulse_res_scale"] = (int64_t)P * D;
    x["rope_local.inv_freq"] = DH / 2;
    x["rope_global.inv_freq"] = DH / 2;
    for (int l = 0; l < NL; ++l) {
        x[e->L(l, "attn_norm.weight")] = (int64_t)P * D;
        x[e->L(l, "attn.q_norm_weight")] = (int64_t)P * H * DH;
        x[e->L(l, "attn.k_norm_weight")] = (int64_t)P * HKV * DH;
        x[e->L(l, "attn.v_resid_lambda")] = P;
        x[e->L(l, "attn.attn_gate")] = (int64_t)P * H * D;
        x[e->L(l, "attn.attn_gate_bias")] = (int64_t)P * H;
        x[e->L(l, "attn.wqkv.weight")] = (int64_t)QKV * D;
        x[e->L(l, "attn.wo.weight")] = (int64_t)D * D;
        x[e->L(l, "attn.wqkv_adapter.lora_A")] = (int64_t)P * q * D;
        x[e->L(l, "attn.wqkv_adapter.lora_B")] = (int64_t)P * QKV * q;
        x[e->L(l, "attn.wqkv_adapter.loop_M")] = (int64_t)P * P;
        x[e->L(l, "attn.wo_adapter.lora_A")] = (int64_t)P * q * D;
        x[e->L(l, "attn.wo_adapter.lora_B")] = (int64_t)P * D * q;
        x[e->L(l, "attn.wo_adapter.loop_M")] = (int64_t)P * P;
        x[e->L(l, "mlp_norm.weight")] = (int64_t)P * D;
        x[e->L(l, "mlp.routed_gate_up")] = (int64_t)E * D * 2 * DE;
        x[e->L(l, "mlp.routed_down")] = (int64_t)E * DE * D;
        x[e->L(l, "mlp.router_weight")] = (int64_t)P * E * D;
        x[e->L(l, "mlp.routed_scale")] = (int64_t)P * D;
        x[e->L(l, "mlp.expert_bias")] = e->cfg.per_pulse_bias ? (int64_t)P * E : E;
        x[e->L(l, "mlp.expert_counts_accum")] = E;
        x[e->L(l, "mlp.expert_pulse_counts")] = (int64_t)P * E;
        x[e->L(l, "mlp.shared_expert.w_gate_up.weight")] = (int64_t)2 * DS * D;
        x[e->L(l, "mlp.shared_expert.w_down.weight")] = (int64_t)D * DS;
    }
}

template <typename T>
T* offs(T* p, int64_t n) { return p ? p + n : nullptr; }

// ------------------------------------------------------------------ pulse pass (R <= MAX_ROWS)
// Flash-decoding attention of an R-row pass, instantiated for the pass's rows per block
// (e->attn_rpb: 1 for one row per sequence, gamma + 1 for verify blocks).
template <typename KVT, int NU>
int launch_attn_flash_nu(pulsar_engine* e, dim3 grid, const int4* rows, int R, const float* q, const KVLayer& L,
                         int local, int nsplit, float* part, cudaStream_t st) {
    constexpr int smem = (int)attn_flash_smem<KVT, NU>();
    PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_attn_flash<KVT, NU>), smem, "k_attn_flash shared memory"));
    k_attn_flash<KVT, NU><<<grid, ATT_FTHREADS, smem, st>>>(rows, R, e->attn_rpb, q, L, local, nsplit, part, e->max_pos(),
                                                            e->cfg.max_batch, e->m_err);
    return launch_status("k_attn_flash");
}

// Tensor-core decode attention (k_attn_dec_tc): a bf16 cache whose tensor map was encoded, unless
// option "tc_dec_attn" is 0.
template <typename KVT>
bool dec_tc(const pulsar_engine* e) {
    return std::is_same<KVT, __nv_bfloat16>::value && e->tc_dec && e->kv_map_ok;
}
// Keys per chunk of the decode attention that dec_tc selects (the split count's unit).
template <typename KVT>
int attn_chunk(const pulsar_engine* e) {
    return dec_tc<KVT>(e) ? DT_CK : ATT_FCK;
}

template <int NU>
int launch_attn_dec_tc_nu(pulsar_engine* e, dim3 grid, const int4* rows, int R, const float* q, const KVLayer& L,
                          int local, int nsplit, float* part, cudaStream_t st) {
    constexpr int smem = (int)dt_smem_bytes<NU>();
    PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_attn_dec_tc<NU>), smem, "k_attn_dec_tc shared memory"));
    const int64_t lrow = (static_cast<const char*>(L.base) - static_cast<const char*>(e->kv)) / (DH * 2);
    k_attn_dec_tc<NU><<<grid, DtLayout<NU>::THREADS, smem, st>>>(e->kv_map, rows, R, e->attn_rpb, q, L, lrow, local, nsplit, part,
                                                       e->max_pos(), e->cfg.max_batch, e->m_err);
    return launch_status("k_attn_dec_tc");
}

template <typename KVT>
int launch_attn_flash(pulsar_engine* e, dim3 grid, const int4* rows, int R, const float* q, const KVLayer& L, int local,
                      int nsplit, float* part, cudaStream_t st) {
    if (dec_tc<KVT>(e)) {
        switch (e->attn_rpb) {
            case 1: return launch_attn_dec_tc_nu<1>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 2: return launch_attn_dec_tc_nu<2>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 3: return launch_attn_dec_tc_nu<3>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 4: return launch_attn_dec_tc_nu<4>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 5: return launch_attn_dec_tc_nu<5>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 6: return launch_attn_dec_tc_nu<6>(e, grid, rows, R, q, L, local, nsplit, part, st);
            case 7: return launch_attn_dec_tc_nu<7>(e, grid, rows, R, q, L, local, nsplit, part, st);
            default: return launch_attn_dec_tc_nu<ATT_RPB_MAX>(e, grid, rows, R, q, L, local, nsplit, part, st);
        }
    }
    switch (e->attn_rpb) {
        case 1: return launch_attn_flash_nu<KVT, 1>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 2: return launch_attn_flash_nu<KVT, 2>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 3: return launch_attn_flash_nu<KVT, 3>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 4: return launch_attn_flash_nu<KVT, 4>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 5: return launch_attn_flash_nu<KVT, 5>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 6: return launch_attn_flash_nu<KVT, 6>(e, grid, rows, R, q, L, local, nsplit, part, st);
        case 7: return launch_attn_flash_nu<KVT, 7>(e, grid, rows, R, q, L, local, nsplit, part, st);
        default: return launch_attn_flash_nu<KVT, ATT_RPB_MAX>(e, grid, rows, R, q, L, local, nsplit, part, st);
    }
}

template <typename KVT>
int enqueue_pulse(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in,
                  float* h_out, float* h0n_out, float* logits, int ld_logits, int* amax, cudaStream_t st, int hs) {
    auto& w = e->w;
    const float eps = e->cfg.rms_eps;
    if (p == 0) {
        k_pulse0_input<<<R, 256, 0, st>>>(rows, e->emb, e->T_("anchor_norm.weight"), e->T_("stem_canon_weight"),
                                          e->T_("pulse_step_emb.weight"), eps, e->cfg.use_canon_conv, w.h, w.h_in,
                                          h0n_out, e->V, hs);
    } else {
        k_reinject<<<R, 256, 0, st>>>(R, h_prev, h0n_in, e->T_("pulse_state_norm.weight"),
                                      e->T_("reinject_gate_down") + (int64_t)p * RG * 2 * D,
                                      e->T_("reinject_gate_up") + (int64_t)p * D * RG,
                                      e->T_("reinject_gate_bias") + (int64_t)p * D,
                                      e->T_("pulse_step_emb.weight") + (int64_t)p * D, eps, w.h, w.h_in, h0n_out, hs);
    }
    PULSAR_LAUNCH_CHECK("pulse input");
    for (int l = 0; l < NL; ++l) {
        const bool lora = lora_live(e);
        k_rmsnorm_lora<<<R, 256, 0, st>>>(w.h, e->T_(e->L(l, "attn_norm.weight")) + (int64_t)p * D, eps, w.xn,
                                          lora ? e->T_(e->L(l, "attn.wqkv_adapter.lora_A")) : nullptr, w.t_qkv);
        k_gemv<1024, EPI_STORE><<<QKV / 8, 128, 0, st>>>(w_qkv(e, p, l), QKV, w.xn, R, w.qkv, QKV,
                                                         lora ? e->lb_qkv[p][l] : nullptr, w.t_qkv);
        const int vres_mode = (p == 0) ? (l == 0 ? 1 : 2) : 0;
        const bool local = is_local_layer(l);
        k_qkv_post<KVT><<<R, (H + HKV) * 32, 0, st>>>(
            rows, w.qkv, e->T_(e->L(l, "attn.q_norm_weight")) + (int64_t)p * H * DH,
            e->T_(e->L(l, "attn.k_norm_weight")) + (int64_t)p * HKV * DH, local ? e->cos_l : e->cos_g,
            local ? e->sin_l : e->sin_g, eps, vres_mode, e->vres[p][l], w.vfirst, e->kvl[l], local ? 0 : 1,
            e->cfg.base_seq_len, w.q, e->max_pos(), e->cfg.max_batch);
        const int groups = (R + e->attn_rpb - 1) / e->attn_rpb;
        const int nsplit = attn_splits(groups, local ? WINDOW + ATT_RPB_MAX : e->max_pos(), e->mega_grid, e->nch[l],
                                       attn_chunk<KVT>(e));
        PULSAR_TRY(launch_attn_flash<KVT>(e, dim3(nsplit, HKV, groups), rows, R, w.q, e->kvl[l], local ? 1 : 0, nsplit,
                                          w.part, st));
        k_attn_combine<<<R, H * 32, 0, st>>>(w.part, nsplit, w.xn,
                                             e->T_(e->L(l, "attn.attn_gate")) + (int64_t)p * H * D,
                                             e->T_(e->L(l, "attn.attn_gate_bias")) + (int64_t)p * H, w.att,
                                             lora ? e->T_(e->L(l, "attn.wo_adapter.lora_A")) : nullptr, w.t_wo);
        k_gemv<1024, EPI_ADD><<<D / 8, 128, 0, st>>>(w_o(e, p, l), D, w.att, R, w.h, D, lora ? e->lb_wo[p][l] : nullptr,
                                                     w.t_wo);
        k_rmsnorm_lora<<<R, 256, 0, st>>>(w.h, e->T_(e->L(l, "mlp_norm.weight")) + (int64_t)p * D, eps, w.xn,
                                          nullptr, nullptr);
        const float* eb = e->T_(e->L(l, "mlp.expert_bias")) + (e->cfg.per_pulse_bias ? (int64_t)p * E : 0);
        k_router<<<R, E * 32, 0, st>>>(w.xn, e->T_(e->L(l, "mlp.router_weight")) + (int64_t)p * E * D, eb, w.idx,
                                       w.wts);
        k_moe_up<<<(DS + R * TOPK * DE) / 4, 128, 0, st>>>(R, w.xn, e->sh_gu[l], e->r_gu[l], w.idx, w.act_sh,
                                                          w.act_r);
        k_moe_down<<<D / 4, 128, 0, st>>>(R, w.act_sh, w.act_r, e->sh_dn[l], e->r_dn[l], w.idx, w.wts,
                                          e->T_(e->L(l, "mlp.routed_scale")) + (int64_t)p * D, w.h);
        PULSAR_LAUNCH_CHECK("pulse layer");
    }
    const bool want = logits != nullptr || amax != nullptr;
    k_pulse_end<<<R, 256, 0, st>>>(w.h, w.h_in, e->T_("pulse_res_scale") + (int64_t)p * D, e->T_("final_norm.weight"),
                                   eps, h_out, want ? w.hn : nullptr, hs);
    PULSAR_LAUNCH_CHECK("k_pulse_end");
    if (want) {
        const int nblk = e->V / LM_ROWS_PER_BLOCK;
        for (int rb = 0; rb < R; rb += 8) {
            const int n = std::min(8, R - rb);
            k_lmhead<<<nblk, 128, 0, st>>>(e->emb, e->V, w.hn + (int64_t)rb * D, n, e->cfg.logit_softcap,
                                           logits ? logits + (int64_t)rb * ld_logits : nullptr, ld_logits,
                                           w.pmax + (int64_t)rb * nblk, w.pidx + (int64_t)rb * nblk);
        }
        PULSAR_LAUNCH_CHECK("k_lmhead");
        if (amax) {
            k_argmax_final<<<R, 32, 0, st>>>(w.pmax, w.pidx, nblk, R, amax);
            PULSAR_LAUNCH_CHECK("k_argmax_final");
        }
    }
    return PULSAR_OK;
}

int pulse_mega(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in,
               float* h_out, float* h0n_out, float* logits, int* amax, cudaStream_t st, int hs, const int* skip) {
    MegaArgs a{};
    a.R = R;
    a.pulse = p;
    a.n_slots = e->cfg.max_batch;
    a.max_pos = e->max_pos();
    a.V = e->V;
    a.use_conv = e->cfg.use_canon_conv;
    a.base_seq_len = e->cfg.base_seq_len;
    a.eps = e->cfg.rms_eps;
    a.softcap = e->cfg.logit_softcap;
    a.rows = rows;
    for (int l = 0; l < NL; ++l) {
        a.wqkv[l] = w_qkv(e, p, l);
        a.wo[l] = w_o(e, p, l);
        a.sh_gu[l] = e->sh_gu[l];
        a.sh_dn[l] = e->sh_dn[l];
        a.r_gu[l] = e->r_gu[l];
        a.r_dn[l] = e->r_dn[l];
        a.attn_norm[l] = e->T_(e->L(l, "attn_norm.weight")) + (int64_t)p * D;
        a.mlp_norm[l] = e->T_(e->L(l, "mlp_norm.weight")) + (int64_t)p * D;
        a.qn[l] = e->T_(e->L(l, "attn.q_norm_weight")) + (int64_t)p * H * DH;
        a.kn[l] = e->T_(e->L(l, "attn.k_norm_weight")) + (int64_t)p * HKV * DH;
        a.gate_w[l] = e->T_(e->L(l, "attn.attn_gate")) + (int64_t)p * H * D;
        a.gate_b[l] = e->T_(e->L(l, "attn.attn_gate_bias")) + (int64_t)p * H;
        a.router[l] = e->T_(e->L(l, "mlp.router_weight")) + (int64_t)p * E * D;
        a.ebias[l] = e->T_(e->L(l, "mlp.expert_bias")) + (e->cfg.per_pulse_bias ? (int64_t)p * E : 0);
        a.rscale[l] = e->T_(e->L(l, "mlp.routed_scale")) + (int64_t)p * D;
        a.vres[l] = e->vres[p][l];
        a.kvl[l] = e->kvl[l];
        if (lora_live(e)) {   // exact fp32 loop adapter: W x + Bs (A x), A = the three pulses' lora_A rows
            a.la_qkv[l] = e->T_(e->L(l, "attn.wqkv_adapter.lora_A"));
            a.lb_qkv[l] = e->lb_qkv[p][l];
            a.la_wo[l] = e->T_(e->L(l, "attn.wo_adapter.lora_A"));
            a.lb_wo[l] = e->lb_wo[p][l];
        }
    }
    a.emb = e->emb;
    a.anchor = e->T_("anchor_norm.weight");
    a.stem = e->T_("stem_canon_weight");
    a.step = e->T_("pulse_step_emb.weight") + (int64_t)p * D;
    a.psn = e->T_("pulse_state_norm.weight");
    a.rg_down = e->T_("reinject_gate_down") + (int64_t)p * RG * 2 * D;
    a.rg_up = e->T_("reinject_gate_up") + (int64_t)p * D * RG;
    a.rg_bias = e->T_("reinject_gate_bias") + (int64_t)p * D;
    a.res_scale = e->T_("pulse_res_scale") + (int64_t)p * D;
    a.fnorm = e->T_("final_norm.weight");
    a.cos_l = e->cos_l;
    a.sin_l = e->sin_l;
    a.cos_g = e->cos_g;
    a.sin_g = e->sin_g;
    a.h_prev = h_prev;
    a.h0n_in = h0n_in;
    a.h_out = h_out;
    a.h0n_out = h0n_out;
    a.hstride = hs;
    a.logits = logits;
    a.amax = amax;
    a.pmax = e->m_pmax;
    a.pidx = e->m_pidx;
    a.nch_max = e->mega_nch;
    auto& w = e->w;
    a.h = w.h;
    a.h_in = w.h_in;
    a.qkv = w.qkv;
    a.gate = e->m_gate;
    a.att = w.att;
    a.act_sh = w.act_sh;
    a.act_r = w.act_r;
    a.part = e->m_part;
    a.vfirst = w.vfirst;
    a.g8 = e->m_g8;
    a.rpart = e->m_rpart;
    a.bar = e->m_bar;
    a.tickets = e->m_tickets;
    a.wait_ns = e->mega_wait_ns;
    a.stall_cta = e->mega_stall_cta;
    a.err = e->m_err;
    a.experts = e->m_experts;
    a.trace = e->m_trace;
    a.skip = skip;
    return launch_mega(a, e->kv32(), e->mega_grid, st);
}

template <typename KVT>
int enqueue_pulse_wide(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in,
                       float* h_out, float* h0n_out, float* logits, int ld_logits, int* amax, cudaStream_t st, int hs);

// skip (optional): a device flag; when it is non-zero at launch the persistent kernel returns
// at once (every row exited early). The per-op and many-row passes run regardless.
int pulse_dispatch(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in,
                   float* h_out, float* h0n_out, float* logits, int ld_logits, int* amax, cudaStream_t st, int hs,
                   const int* skip) {
    if (R > MAX_ROWS || e->force_wide) {
        // rms norm, QKV GEMM, qkv post, attention, combine, Wo GEMM, norm, router, shared GEMMs (2),
        // bucket, slots, expert GEMMs (2), combine per layer; input, end, LM GEMM, argmax
        const bool want = logits != nullptr || amax != nullptr;
        e->n_kernels += 2 + 15 * NL + (want ? 1 : 0) + (amax ? 1 : 0);
        if (e->kv32())
            return enqueue_pulse_wide<float>(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, ld_logits, amax, st, hs);
        return enqueue_pulse_wide<__nv_bfloat16>(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, ld_logits, amax,
                                                 st, hs);
    }
    if (e->use_mega && R <= MEGA_RMAX && (logits == nullptr || ld_logits == e->V)) {
        e->n_kernels += 1;
        e->n_mega += 1;
        return pulse_mega(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, amax, st, hs, skip);
    }
    // per-op pass: input, 10 kernels per layer, end, LM head per 8 rows, argmax
    const bool want = logits != nullptr || amax != nullptr;
    e->n_kernels += 2 + 10 * NL + (want ? (R + 7) / 8 : 0) + (amax ? 1 : 0);
    if (e->kv32())
        return enqueue_pulse<float>(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, ld_logits, amax, st, hs);
    return enqueue_pulse<__nv_bfloat16>(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, ld_logits, amax, st,
                                        hs);
}

// hs: row stride (in rows of D floats) of h_out and h0n_out
int pulse(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in, float* h_out,
          float* h0n_out, float* logits, int ld_logits, int* amax, cudaStream_t st, int hs = 1,
          const int* skip = nullptr) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const bool timed = e->time_pulses && cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone;
    if (timed) PULSAR_TRY(cuda_status(cudaEventRecord(e->tev[0], st), "cudaEventRecord"));
    PULSAR_TRY(pulse_dispatch(e, p, R, rows, h_prev, h0n_in, h_out, h0n_out, logits, ld_logits, amax, st, hs, skip));
    if (timed) PULSAR_TRY(cuda_status(cudaEventRecord(e->tev[1], st), "cudaEventRecord"));
    return PULSAR_OK;
}

// ------------------------------------------------------------------ prefill
// Tiled GEMM launch: the tcgen05 tensor-core kernel when the shape fits its tiles (K a
// multiple of 64, output columns a multiple of 128, or of 64 for SWIGLU; 16-byte aligned rows)
// and the activation split fits the engine's hi/lo buffers, else the SIMT kernel.
// 2-D bf16 tensor map [rows][cols] (row-major, cols contiguous) with a box of 64 columns
// (128 bytes) x box_rows rows and the 128-byte swizzle; false when the driver entry point is
// missing or the operand does not qualify (alignment, sizes).
bool encode_bf16_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static std::mutex mu;
    static Encode fn = nullptr;
    static bool looked = false;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!looked) {
            void* f = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                fn = reinterpret_cast<Encode>(f);
            looked = true;
        }
    }
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || cols % 64 || rows == 0 || box_rows > 256) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Returns PULSAR_OK / an error, or 1 when the weights do not fit a tensor map (the caller falls
// back to k_tc_gemm).
template <int EPI, int BN>
int launch_tma_gemm(pulsar_engine* e, const GemmArgs& g, int batches, const CUtensorMap& ma, const CUtensorMap& mb,
                    int w_rows_per_batch, cudaStream_t st) {
    CUtensorMap mw;
    const uint64_t w_rows = (uint64_t)(batches - 1) * w_rows_per_batch + g.N;
    if (!encode_bf16_map(&mw, g.W, w_rows, g.K, EPI == GEPI_SWIGLU ? BN / 2 : BN)) return 1;   // not applicable
    PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_tma_gemm<EPI, BN>), (int)tma_smem_bytes<BN>(),
                                "k_tma_gemm shared memory"));
    const int ntiles = (EPI == GEPI_SWIGLU) ? (g.N / 2) / (BN / 2) : g.N / BN;
    dim3 grid(ntiles, (g.M + TC_BM - 1) / TC_BM, batches);
    k_tma_gemm<EPI, BN><<<grid, TC_THREADS, tma_smem_bytes<BN>(), st>>>(ma, mb, mw, g, w_rows_per_batch, e->m_err);
    return launch_status("k_tma_gemm");
}

template <int EPI>
int gemm(pulsar_engine* e, const GemmArgs& g, int batches, cudaStream_t st) {
    constexpr int BN = 128;
    const bool fits = g.K % TC_BK == 0 && (EPI == GEPI_SWIGLU ? (g.N / 2) % (BN / 2) == 0 : g.N % BN == 0) &&
                      (reinterpret_cast<uintptr_t>(g.C) & 15) == 0 && g.ldc % 4 == 0 && g.c_stride % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(g.A) & 15) == 0 && g.lda % 4 == 0 && g.a_stride % 4 == 0 &&
                      (int64_t)batches * g.M * g.K <= e->split_elems;
    // an operand its producer already split: [batch * M][K] rows, 16-byte aligned
    const bool presplit = g.a_hi && g.a_lo && !g.a_rows && g.lda == g.K && (batches == 1 || g.a_stride == (int64_t)g.M * g.K) &&
                          (reinterpret_cast<uintptr_t>(g.a_hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.a_lo) & 15) == 0;
    if (e->use_tc && fits) {
        const __nv_bfloat16* ahi = e->split_hi;
        const __nv_bfloat16* alo = e->split_lo;
        if (presplit) {
            ahi = g.a_hi;
            alo = g.a_lo;
        } else {
            const int64_t per_batch = (int64_t)g.M * g.K / 8;
            k_split_hilo<<<dim3((unsigned)((per_batch + 255) / 256), batches), 256, 0, st>>>(g, e->split_hi, e->split_lo);
            PULSAR_TRY(launch_status("k_split_hilo"));
        }
        // TMA-fed kernel: weights of every batch at a whole number of rows from the first
        CUtensorMap ma, mb;
        if (e->use_tma && (batches == 1 || g.w_stride % g.K == 0) &&
            encode_bf16_map(&ma, ahi, (uint64_t)batches * g.M, g.K, TC_BM) &&
            encode_bf16_map(&mb, alo, (uint64_t)batches * g.M, g.K, TC_BM)) {
            const int wpb = batches > 1 ? (int)(g.w_stride / g.K) : 0;
            // narrow grids (under one CTA per SM) take 64-column tiles: twice the CTAs
            const int tiles128 = ((EPI == GEPI_SWIGLU) ? (g.N / 2) / (BN / 2) : g.N / BN) *
                                 ((g.M + TC_BM - 1) / TC_BM) * batches;
            int r = (tiles128 < e->mega_grid) ? launch_tma_gemm<EPI, 64>(e, g, batches, ma, mb, wpb, st)
                                              : launch_tma_gemm<EPI, BN>(e, g, batches, ma, mb, wpb, st);
            if (r != 1) return r;
        }
        PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_tc_gemm<EPI, BN>), (int)tc_smem_bytes<BN>(),
                                    "k_tc_gemm shared memory"));
        const int ntiles = (EPI == GEPI_SWIGLU) ? (g.N / 2) / (BN / 2) : g.N / BN;
        dim3 grid(ntiles, (g.M + TC_BM - 1) / TC_BM, batches);
        k_tc_gemm<EPI, BN><<<grid, TC_THREADS, tc_smem_bytes<BN>(), st>>>(g, ahi, alo, e->m_err);
        return launch_status("k_tc_gemm");
    }
    const int ntiles = (EPI == GEPI_SWIGLU) ? (g.N / 2 + 31) / 32 : (g.N + GB_N - 1) / GB_N;
    dim3 grid(ntiles, (g.M + GB_M - 1) / GB_M, batches);
    k_gemm<EPI><<<grid, 256, 0, st>>>(g);
    PULSAR_TRY(launch_status("k_gemm"));
    if (g.c_hi) {
        // the split the tensor-core epilogue would have written, for a consumer that reads it
        GemmArgs c{};
        c.A = g.C;
        c.lda = g.ldc;
        c.a_stride = g.c_stride;
        c.m_count = g.m_count;
        c.M = g.M;
        c.K = (EPI == GEPI_SWIGLU) ? g.N / 2 : g.N;
        if (g.ldc != c.K || (batches > 1 && g.c_stride != (int64_t)g.M * c.K) || c.K % 8) {
            set_error("gemm: the split output needs C as [batch * M][N] rows");
            return PULSAR_ERR_UNSUPPORTED;
        }
        const int64_t per_batch = (int64_t)c.M * c.K / 8;
        k_split_hilo<<<dim3((unsigned)((per_batch + 255) / 256), batches), 256, 0, st>>>(c, g.c_hi, g.c_lo);
        return launch_status("k_split_hilo");
    }
    return PULSAR_OK;
}

GemmArgs gargs(const float* A, int lda, int M, const __nv_bfloat16* W, int N, int K, float* C, int ldc) {
    GemmArgs g{};
    g.A = A;
    g.lda = lda;
    g.M = M;
    g.W = W;
    g.N = N;
    g.K = K;
    g.C = C;
    g.ldc = ldc;
    return g;
}

template <typename KVT>
// fwd = false: the inference prefill (src/infer.py:353-461). fwd = true: the training-style
// forward of model.generate (src/model.py:1956-2125, T <= the local ring): value residual in every
// pulse, YaRN query scale on global layers, plain causal attention on local layers, softcapped
// last-position logits.
int enqueue_prefill(pulsar_engine* e, int slot, const int* ids, int T, float* logits, cudaStream_t st, bool fwd) {
    auto& f = e->pf;
    const float eps = e->cfg.rms_eps;
    k_embed_rows<<<T, 256, 0, st>>>(ids, e->emb, e->T_("anchor_norm.weight"), eps, f.h0, f.h0n_pre);
    if (e->cfg.use_canon_conv)
        k_conv_seq<<<T, 256, 0, st>>>(f.h0n_pre, e->T_("stem_canon_weight"), T, f.h0n);
    else
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(f.h0n, f.h0n_pre, (size_t)T * D * 4, cudaMemcpyDeviceToDevice, st),
                               "prefill copy"));
    PULSAR_LAUNCH_CHECK("prefill embed");
    const int cap = prefill_capacity(T);
    const int M4 = T * TOPK;
    for (int p = 0; p < NP; ++p) {
        if (p == 0)
            k_pulse0_rows<<<T, 256, 0, st>>>(f.h0n, e->T_("pulse_step_emb.weight"), f.h, f.h_in);
        else
            k_reinject<<<T, 256, 0, st>>>(T, f.hp, f.h0n, e->T_("pulse_state_norm.weight"),
                                          e->T_("reinject_gate_down") + (int64_t)p * RG * 2 * D,
                                          e->T_("reinject_gate_up") + (int64_t)p * D * RG,
                                          e->T_("reinject_gate_bias") + (int64_t)p * D,
                                          e->T_("pulse_step_emb.weight") + (int64_t)p * D, eps, f.h, f.h_in, nullptr, 1);
        PULSAR_LAUNCH_CHECK("prefill pulse input");
        for (int l = 0; l < NL; ++l) {
            const bool lora = lora_live(e);
            const bool local = is_local_layer(l);
            k_rmsnorm_lora<<<T, 256, 0, st>>>(f.h, e->T_(e->L(l, "attn_norm.weight")) + (int64_t)p * D, eps, f.xn,
                                              lora ? e->T_(e->L(l, "attn.wqkv_adapter.lora_A")) : nullptr, f.t,
                                              f.xs_hi, f.xs_lo);
            GemmArgs g = gargs(f.xn, D, T, w_qkv(e, p, l), QKV, D, f.qkv, QKV);
            g.a_hi = f.xs_hi;
            g.a_lo = f.xs_lo;
            if (lora) { g.lora_b = e->lb_qkv[p][l]; g.lora_t = f.t; }
            PULSAR_TRY(gemm<GEPI_STORE>(e, g, 1, st));
            const int vres_mode = fwd ? ((p == 0 && l == 0) ? 1 : 2) : ((p == 0) ? (l == 0 ? 1 : 2) : 0);
            const int yarn_base = (fwd && !local && T > e->cfg.base_seq_len) ? e->cfg.base_seq_len : 0;
            k_qkv_post_prefill<KVT><<<T, (H + HKV) * 32, 0, st>>>(
                slot, T, f.qkv, e->T_(e->L(l, "attn.q_norm_weight")) + (int64_t)p * H * DH,
                e->T_(e->L(l, "attn.k_norm_weight")) + (int64_t)p * HKV * DH, local ? e->cos_l : e->cos_g,
                local ? e->sin_l : e->sin_g, eps, vres_mode, e->vres[p][l], f.vfirst, e->kvl[l], local ? 1 : 0, f.q,
                yarn_base);
            const int attn_local = (local && !fwd) ? 1 : 0;   // forward: plain causal (T <= 4096)
            if (e->tc_attn) {
                PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_attn_prefill_tc<KVT>), (int)pt_smem_bytes<KVT>(),
                                            "k_attn_prefill_tc shared memory"));
                k_attn_prefill_tc<KVT><<<dim3((T + PT_Q - 1) / PT_Q, H), PT_THREADS, pt_smem_bytes<KVT>(), st>>>(
                    slot, T, f.q, e->kvl[l], attn_local, f.o, e->m_err);
            } else {
                k_attn_prefill<KVT><<<dim3((T + PA_Q - 1) / PA_Q, H), 256, 0, st>>>(slot, T, f.q, e->kvl[l],
                                                                                   attn_local, f.o);
            }
            k_gate_rows<<<T, H * 32, 0, st>>>(f.o, f.xn, e->T_(e->L(l, "attn.attn_gate")) + (int64_t)p * H * D,
                                              e->T_(e->L(l, "attn.attn_gate_bias")) + (int64_t)p * H, f.att,
                                              lora ? e->T_(e->L(l, "attn.wo_adapter.lora_A")) : nullptr, f.t,
                                              f.xs_hi, f.xs_lo);
            PULSAR_LAUNCH_CHECK("prefill attention");
            g = gargs(f.att, D, T, w_o(e, p, l), D, D, f.h, D);
            g.a_hi = f.xs_hi;
            g.a_lo = f.xs_lo;
            if (lora) { g.lora_b = e->lb_wo[p][l]; g.lora_t = f.t; }
            PULSAR_TRY(gemm<GEPI_ADD>(e, g, 1, st));
            k_rmsnorm_lora<<<T, 256, 0, st>>>(f.h, e->T_(e->L(l, "mlp_norm.weight")) + (int64_t)p * D, eps, f.xn,
                                              nullptr, nullptr, f.xs_hi, f.xs_lo);
            const float* eb = e->T_(e->L(l, "mlp.expert_bias")) + (e->cfg.per_pulse_bias ? (int64_t)p * E : 0);
            k_router<<<T, E * 32, 0, st>>>(f.xn, e->T_(e->L(l, "mlp.router_weight")) + (int64_t)p * E * D, eb, f.idx,
                                           f.wts);
            PULSAR_LAUNCH_CHECK("prefill router");
            GemmArgs gs = gargs(f.xn, D, T, e->sh_gu[l], 2 * DS, D, f.act_sh, DS);
            gs.a_hi = f.xs_hi;
            gs.a_lo = f.xs_lo;
            gs.c_hi = f.ss_hi;
            gs.c_lo = f.ss_lo;
            PULSAR_TRY(gemm<GEPI_SWIGLU>(e, gs, 1, st));
            gs = gargs(f.act_sh, DS, T, e->sh_dn[l], D, DS, f.sh, D);
            gs.a_hi = f.ss_hi;
            gs.a_lo = f.ss_lo;
            PULSAR_TRY(gemm<GEPI_STORE>(e, gs, 1, st));
            k_moe_bucket<<<E, 1024, 0, st>>>(f.idx, M4, f.lists, M4, f.cnt);
            k_moe_slots<<<dim3((M4 + 255) / 256, E), 256, 0, st>>>(f.lists, M4, f.cnt, f.wts, cap, f.slot, f.rows_e,
                                                                  f.kept);
            PULSAR_LAUNCH_CHECK("prefill slots");
            GemmArgs gu = gargs(f.xn, D, cap, e->r_gu[l], 2 * DE, D, f.act_e, DE);
            gu.a_rows = f.rows_e;
            gu.m_count = f.kept;
            gu.w_stride = (int64_t)2 * DE * D;
            gu.c_stride = (int64_t)cap * DE;
            gu.c_hi = f.es_hi;
            gu.c_lo = f.es_lo;
            PULSAR_TRY(gemm<GEPI_SWIGLU>(e, gu, E, st));
            GemmArgs gd = gargs(f.act_e, DE, cap, e->r_dn[l], D, DE, f.ye, D);
            gd.a_hi = f.es_hi;
            gd.a_lo = f.es_lo;
            gd.a_stride = (int64_t)cap * DE;
            gd.m_count = f.kept;
            gd.w_stride = (int64_t)D * DE;
            gd.c_stride = (int64_t)cap * D;
            PULSAR_TRY(gemm<GEPI_STORE>(e, gd, E, st));
            k_moe_combine_rows<<<T, 256, 0, st>>>(f.sh, f.ye, cap, f.idx, f.wts, f.slot,
                                                  e->T_(e->L(l, "mlp.routed_scale")) + (int64_t)p * D, f.h);
            PULSAR_LAUNCH_CHECK("prefill moe combine");
        }
        k_pulse_end<<<T, 256, 0, st>>>(f.h, f.h_in, e->T_("pulse_res_scale") + (int64_t)p * D,
                                       e->T_("final_norm.weight"), eps, f.hp, nullptr, 1);
        PULSAR_LAUNCH_CHECK("prefill pulse end");
    }
    // last position logits without softcap (src/infer.py:458-461)
    k_rmsnorm_lora<<<1, 256, 0, st>>>(f.hp + (int64_t)(T - 1) * D, e->T_("final_norm.weight"), eps, f.hn, nullptr,
                                      nullptr);
    const int nblk = e->V / LM_ROWS_PER_BLOCK;
    k_lmhead<<<nblk, 128, 0, st>>>(e->emb, e->V, f.hn, 1, fwd ? e->cfg.logit_softcap : 0.f, logits, e->V, f.pmax,
                                   f.pidx);
    PULSAR_LAUNCH_CHECK("prefill lm head");
    return PULSAR_OK;
}

// Pulse pass over R rows in the GEMM regime (R > MAX_ROWS, or option "wide"): the same
// arithmetic as enqueue_pulse with every weight product a tiled GEMM over all rows, the
// routed experts bucketed per expert (capacity R: no row is dropped, unlike prefill), and
// the LM head a GEMM with the softcap epilogue followed by a row argmax.
template <typename KVT>
int enqueue_pulse_wide(pulsar_engine* e, int p, int R, const int4* rows, const float* h_prev, const float* h0n_in,
                       float* h_out, float* h0n_out, float* logits, int ld_logits, int* amax, cudaStream_t st, int hs) {
    if (R > e->wide_rows) {
        set_error("pulse: %d rows exceed the wide workspace (%d rows)", R, e->wide_rows);
        return PULSAR_ERR_CAPACITY;
    }
    auto& w = e->ww;
    const float eps = e->cfg.rms_eps;
    if (p == 0) {
        k_pulse0_input<<<R, 256, 0, st>>>(rows, e->emb, e->T_("anchor_norm.weight"), e->T_("stem_canon_weight"),
                                          e->T_("pulse_step_emb.weight"), eps, e->cfg.use_canon_conv, w.h, w.h_in,
                                          h0n_out, e->V, hs);
    } else {
        k_reinject<<<R, 256, 0, st>>>(R, h_prev, h0n_in, e->T_("pulse_state_norm.weight"),
                                      e->T_("reinject_gate_down") + (int64_t)p * RG * 2 * D,
                                      e->T_("reinject_gate_up") + (int64_t)p * D * RG,
                                      e->T_("reinject_gate_bias") + (int64_t)p * D,
                                      e->T_("pulse_step_emb.weight") + (int64_t)p * D, eps, w.h, w.h_in, h0n_out, hs);
    }
    PULSAR_LAUNCH_CHECK("wide pulse input");
    const int cap = R, M4 = R * TOPK;
    for (int l = 0; l < NL; ++l) {
        const bool lora = lora_live(e);
        const bool local = is_local_layer(l);
        k_rmsnorm_lora<<<R, 256, 0, st>>>(w.h, e->T_(e->L(l, "attn_norm.weight")) + (int64_t)p * D, eps, w.xn,
                                          lora ? e->T_(e->L(l, "attn.wqkv_adapter.lora_A")) : nullptr, w.t_qkv,
                                          w.xs_hi, w.xs_lo);
        GemmArgs g = gargs(w.xn, D, R, w_qkv(e, p, l), QKV, D, w.qkv, QKV);
        g.a_hi = w.xs_hi;
        g.a_lo = w.xs_lo;
        if (lora) { g.lora_b = e->lb_qkv[p][l]; g.lora_t = w.t_qkv; }
        PULSAR_TRY(gemm<GEPI_STORE>(e, g, 1, st));
        const int vres_mode = (p == 0) ? (l == 0 ? 1 : 2) : 0;
        k_qkv_post<KVT><<<R, (H + HKV) * 32, 0, st>>>(
            rows, w.qkv, e->T_(e->L(l, "attn.q_norm_weight")) + (int64_t)p * H * DH,
            e->T_(e->L(l, "attn.k_norm_weight")) + (int64_t)p * HKV * DH, local ? e->cos_l : e->cos_g,
            local ? e->sin_l : e->sin_g, eps, vres_mode, e->vres[p][l], w.vfirst, e->kvl[l], local ? 0 : 1,
            e->cfg.base_seq_len, w.q, e->max_pos(), e->cfg.max_batch);
        const int groups = (R + e->attn_rpb - 1) / e->attn_rpb;
        const int nsplit = attn_splits(groups, local ? WINDOW + ATT_RPB_MAX : e->max_pos(), e->mega_grid, e->nch[l],
                                       attn_chunk<KVT>(e));
        PULSAR_TRY(launch_attn_flash<KVT>(e, dim3(nsplit, HKV, groups), rows, R, w.q, e->kvl[l], local ? 1 : 0, nsplit,
                                          w.part, st));
        k_attn_combine<<<R, H * 32, 0, st>>>(w.part, nsplit, w.xn, e->T_(e->L(l, "attn.attn_gate")) + (int64_t)p * H * D,
                                             e->T_(e->L(l, "attn.attn_gate_bias")) + (int64_t)p * H, w.att,
                                             lora ? e->T_(e->L(l, "attn.wo_adapter.lora_A")) : nullptr, w.t_wo,
                                             w.xs_hi, w.xs_lo);
        PULSAR_LAUNCH_CHECK("wide attention");
        g = gargs(w.att, D, R, w_o(e, p, l), D, D, w.h, D);
        g.a_hi = w.xs_hi;
        g.a_lo = w.xs_lo;
        if (lora) { g.lora_b = e->lb_wo[p][l]; g.lora_t = w.t_wo; }
        PULSAR_TRY(gemm<GEPI_ADD>(e, g, 1, st));
        k_rmsnorm_lora<<<R, 256, 0, st>>>(w.h, e->T_(e->L(l, "mlp_norm.weight")) + (int64_t)p * D, eps, w.xn, nullptr,
                                          nullptr, w.xs_hi, w.xs_lo);
        const float* eb = e->T_(e->L(l, "mlp.expert_bias")) + (e->cfg.per_pulse_bias ? (int64_t)p * E : 0);
        k_router<<<R, E * 32, 0, st>>>(w.xn, e->T_(e->L(l, "mlp.router_weight")) + (int64_t)p * E * D, eb, w.idx, w.wts);
        PULSAR_LAUNCH_CHECK("wide router");
        GemmArgs gs = gargs(w.xn, D, R, e->sh_gu[l], 2 * DS, D, w.act_sh, DS);
        gs.a_hi = w.xs_hi;
        gs.a_lo = w.xs_lo;
        gs.c_hi = w.ss_hi;
        gs.c_lo = w.ss_lo;
        PULSAR_TRY(gemm<GEPI_SWIGLU>(e, gs, 1, st));
        gs = gargs(w.act_sh, DS, R, e->sh_dn[l], D, DS, w.sh, D);
        gs.a_hi = w.ss_hi;
        gs.a_lo = w.ss_lo;
        PULSAR_TRY(gemm<GEPI_STORE>(e, gs, 1, st));
        k_moe_bucket<<<E, 1024, 0, st>>>(w.idx, M4, w.lists, M4, w.cnt);
        k_moe_slots<<<dim3((M4 + 255) / 256, E), 256, 0, st>>>(w.lists, M4, w.cnt, w.wts, cap, w.slot, w.rows_e, w.kept);
        PULSAR_LAUNCH_CHECK("wide slots");
        GemmArgs gu = gargs(w.xn, D, cap, e->r_gu[l], 2 * DE, D, w.act_e, DE);
        gu.a_rows = w.rows_e;
        gu.m_count = w.kept;
        gu.w_stride = (int64_t)2 * DE * D;
        gu.c_stride = (int64_t)cap * DE;
        gu.c_hi = w.es_hi;
        gu.c_lo = w.es_lo;
        PULSAR_TRY(gemm<GEPI_SWIGLU>(e, gu, E, st));
        GemmArgs gd = gargs(w.act_e, DE, cap, e->r_dn[l], D, DE, w.ye, D);
        gd.a_hi = w.es_hi;
        gd.a_lo = w.es_lo;
        gd.a_stride = (int64_t)cap * DE;
        gd.m_count = w.kept;
        gd.w_stride = (int64_t)D * DE;
        gd.c_stride = (int64_t)cap * D;
        PULSAR_TRY(gemm<GEPI_STORE>(e, gd, E, st));
        k_moe_combine_rows<<<R, 256, 0, st>>>(w.sh, w.ye, cap, w.idx, w.wts, w.slot,
                                              e->T_(e->L(l, "mlp.routed_scale")) + (int64_t)p * D, w.h);
        PULSAR_LAUNCH_CHECK("wide moe combine");
    }
    const bool want = logits != nullptr || amax != nullptr;
    k_pulse_end<<<R, 256, 0, st>>>(w.h, w.h_in, e->T_("pulse_res_scale") + (int64_t)p * D, e->T_("final_norm.weight"),
                                   eps, h_out, want ? w.hn : nullptr, hs, w.xs_hi, w.xs_lo);
    PULSAR_LAUNCH_CHECK("wide pulse end");
    if (want) {
        float* lg = logits ? logits : w.logits;
        const int ld = logits ? ld_logits : e->V;
        GemmArgs g = gargs(w.hn, D, R, e->emb, e->V, D, lg, ld);
        g.softcap = e->cfg.logit_softcap;
        g.a_hi = w.xs_hi;
        g.a_lo = w.xs_lo;
        PULSAR_TRY(gemm<GEPI_STORE>(e, g, 1, st));
        if (amax) {
            k_argmax_rows<<<R, 1024, 0, st>>>(lg, e->V, ld, amax);
            PULSAR_LAUNCH_CHECK("wide argmax");
        }
    }
    return PULSAR_OK;
}

// The persistent kernel raises a device flag when a bounded wait runs out; report it once.
int check_kernel_err(pulsar_engine* e) {
    if (!e->m_err) return PULSAR_OK;
    int v = 0;
    PULSAR_TRY(cuda_status(cudaMemcpy(&v, e->m_err, 4, cudaMemcpyDeviceToHost), "read error flag"));
    if (v) {
        cudaMemset(e->m_err, 0, 4);
        cudaMemset(e->m_bar, 0, 4);
        cudaMemset(e->m_tickets, 0, ((size_t)MEGA_RMAX * HKV + 2) * 4);
        set_error("a bounded device wait ran out (persistent pulse kernel grid barrier or weight stream, or a "
                  "tensor-core GEMM's MMA completion); results of the affected launch are invalid");
        return PULSAR_ERR_CUDA;
    }
    return PULSAR_OK;
}

int check_engine(pulsar_engine* e, bool need_final) {
    PULSAR_CHECK_ARG(e != nullptr, "null engine handle");
    if (need_final && !e->finalized) {
        set_error("engine not finalized: call pulsar_engine_finalize after uploading every tensor");
        return PULSAR_ERR_STATE;
    }
    return PULSAR_OK;
}

int run_graph(pulsar_engine* e, const std::string& key, cudaStream_t st, int (*body)(pulsar_engine*, cudaStream_t, void*),
              void* ctx) {
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t g;
        cudaStream_t cs;
        PULSAR_TRY(cuda_status(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate"));
        PULSAR_TRY(cuda_status(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "BeginCapture"));
        const int64_t k0 = e->n_kernels, m0 = e->n_mega;   // the body tallies its launches while capturing
        int st_body = body(e, cs, ctx);
        const int64_t mega = e->n_mega - m0;
        e->n_kernels = k0;
        e->n_mega = m0;
        cudaError_t ce = cudaStreamEndCapture(cs, &g);
        cudaStreamDestroy(cs);
        PULSAR_TRY(st_body);
        PULSAR_TRY(cuda_status(ce, "EndCapture"));
        size_t n_nodes = 0;
        int64_t kernels = 0;
        ce = cudaGraphGetNodes(g, nullptr, &n_nodes);
        if (ce == cudaSuccess && n_nodes) {
            std::vector<cudaGraphNode_t> nodes(n_nodes);
            ce = cudaGraphGetNodes(g, nodes.data(), &n_nodes);
            for (size_t i = 0; ce == cudaSuccess && i < n_nodes; ++i) {
                cudaGraphNodeType t;
                ce = cudaGraphNodeGetType(nodes[i], &t);
                if (ce == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
            }
        }
        if (ce != cudaSuccess) {
            cudaGraphDestroy(g);
            return cuda_status(ce, "count graph nodes");
        }
        cudaGraphExec_t ex;
        ce = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        PULSAR_TRY(cuda_status(ce, "cudaGraphInstantiate"));
        it = e->graphs.emplace(key, pulsar_engine::Graph{ex, kernels, mega}).first;
    }
    e->n_kernels += it->second.kernels;
    e->n_mega += it->second.mega;
    return cuda_status(cudaGraphLaunch(it->second.ex, st), "cudaGraphLaunch");
}

struct LoopCtx {
    int n, gamma;
};

int body_step(pulsar_engine* e, cudaStream_t st, void* vctx) {
    LoopCtx* c = static_cast<LoopCtx*>(vctx);
    const int n = c->n;
    k_rows_step<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->slots_dev, n, e->rows);
    PULSAR_TRY(pulse(e, 0, n, e->rows, nullptr, nullptr, e->htmp, e->h0tmp, nullptr, 0, nullptr, st));
    PULSAR_TRY(pulse(e, 1, n, e->rows, e->htmp, e->h0tmp, e->htmp2, nullptr, nullptr, 0, nullptr, st));
    PULSAR_TRY(pulse(e, 2, n, e->rows, e->htmp2, e->h0tmp, e->htmp, nullptr, nullptr, 0, e->amax, st));
    k_commit_greedy<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->amax, n, e->loop_out);
    return launch_status("k_commit_greedy");
}

// Sequential step with adaptive early exit (src/infer.py:526-549) and / or a repetition
// penalty (src/infer.py:582-589). Early exit: pulses 0 and 1 also write logits (qbuf rows
// [k * n, k * n + n)) and argmax; k_ee_check marks the rows that exit; later pulses keep their
// K/V and a persistent pass whose rows have all exited returns at once. Penalty: the last
// pulse writes logits (pbuf) and the commit takes the penalized argmax of the exiting (or last)
// pulse's row and adds the token to the seen set. Which of the two is on is fixed at capture.
int body_step_x(pulsar_engine* e, cudaStream_t st, void* vctx) {
    LoopCtx* c = static_cast<LoopCtx*>(vctx);
    const int n = c->n, V = e->V, NB = e->cfg.max_batch;
    const bool ee = e->ee_on, rp = e->rp_on;
    float* lg0 = e->qbuf;
    float* lg1 = e->qbuf + (int64_t)n * V;
    if (ee) k_rows_step_ee<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->slots_dev, n, e->rows, e->ee);
    else k_rows_step<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->slots_dev, n, e->rows);
    PULSAR_TRY(pulse(e, 0, n, e->rows, nullptr, nullptr, e->htmp, e->h0tmp, ee ? lg0 : nullptr, V,
                     ee ? e->ee_amax : nullptr, st));
    if (ee) {
        k_ee_check<<<n, SAMPLE_THREADS, 0, st>>>(lg0, V, n, 0, e->loop_out, e->seqs, e->rows, e->ee);
        PULSAR_LAUNCH_CHECK("k_ee_check");
    }
    PULSAR_TRY(pulse(e, 1, n, e->rows, e->htmp, e->h0tmp, e->htmp2, nullptr, ee ? lg1 : nullptr, V,
                     ee ? e->ee_amax + NB : nullptr, st, 1, ee ? e->ee : nullptr));
    if (ee) {
        k_ee_check<<<n, SAMPLE_THREADS, 0, st>>>(lg1, V, n, 1, e->loop_out, e->seqs, e->rows, e->ee);
        PULSAR_LAUNCH_CHECK("k_ee_check");
    }
    PULSAR_TRY(pulse(e, 2, n, e->rows, e->htmp2, e->h0tmp, e->htmp, nullptr, rp ? e->pbuf : nullptr, V,
                     rp ? nullptr : e->amax, st, 1, ee ? e->ee : nullptr));
    if (rp) {
        k_commit_penalized<<<n, 1024, 0, st>>>(e->seqs, lg0, lg1, e->pbuf, ee ? e->ee : nullptr, n, V, e->loop_out,
                                               e->slots_dev, e->seen, e->ee_counts);
        return launch_status("k_commit_penalized");
    }
    k_commit_ee<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->ee_amax, e->ee_amax + NB, e->amax, e->ee, n, e->loop_out,
                                                 e->ee_counts);
    return launch_status("k_commit_ee");
}

// Repetition penalty of the rows of one speculative pass (k_penalize_rows), in place.
int penalize(pulsar_engine* e, float* lg, int nrows, int per_seq, int kfix, int gamma, const SeqDev* seqs,
             cudaStream_t st) {
    k_penalize_rows<<<nrows, 1024, (size_t)e->V / 8, st>>>(lg, e->V, per_seq, kfix, gamma, e->slots_dev, e->seen,
                                                           e->toks, e->loop_out, seqs);
    return launch_status("k_penalize_rows");
}

// One speculative round: gamma + 1 pulse-0 passes (the drafts, then the last draft's own
// pass), whose outputs land directly in the verify block buffers (row stride gamma + 1), then
// the batched pulse-1 and pulse-2 verify passes and the acceptance. Round 0's first row is set
// by k_seq_init, later rounds' by the acceptance kernel. With a repetition penalty (fixed at
// capture) the draft and verify passes write logits, which are penalised with each row's seen
// set (k_penalize_rows) before their argmax, and the acceptance adds the emitted tokens to it.
int body_round(pulsar_engine* e, cudaStream_t st, void* vctx) {
    LoopCtx* c = static_cast<LoopCtx*>(vctx);
    const int n = c->n, g = c->gamma, rows_v = n * (g + 1), V = e->V;
    const bool rp = e->rp_on;
    for (int j = 0; j <= g; ++j) {
        if (j > 0) {
            k_rows_spec<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->slots_dev, n, g, j, e->amax, e->toks, e->rows, e->rows_v);
            PULSAR_LAUNCH_CHECK("k_rows_spec");
        }
        float* qrows = (rp && j < g) ? e->qbuf + (int64_t)j * n * V : nullptr;
        PULSAR_TRY(pulse(e, 0, n, e->rows, nullptr, nullptr, e->hblk + (int64_t)j * D, e->h0blk + (int64_t)j * D,
                         qrows, V, (j < g && !rp) ? e->amax : nullptr, st, g + 1));
        if (qrows) {
            PULSAR_TRY(penalize(e, qrows, n, 1, j, g, e->seqs, st));
            k_argmax_rows<<<n, 1024, 0, st>>>(qrows, V, V, e->amax);
            PULSAR_LAUNCH_CHECK("k_argmax_rows");
        }
    }
    e->attn_rpb = g + 1;   // verify blocks: one pass over each chunk of K/V per block in the attention
    const int v1 = pulse(e, 1, rows_v, e->rows_v, e->hblk, e->h0blk, e->htmp2, nullptr, nullptr, 0, nullptr, st);
    const int v2 = v1 ? v1
                      : pulse(e, 2, rows_v, e->rows_v, e->htmp2, e->h0blk, e->htmp, nullptr, rp ? e->pbuf : nullptr, V,
                              rp ? nullptr : e->amax, st);
    e->attn_rpb = 1;
    PULSAR_TRY(v2);
    if (rp) {
        PULSAR_TRY(penalize(e, e->pbuf, rows_v, g + 1, 0, g, e->seqs, st));
        k_argmax_rows<<<rows_v, 1024, 0, st>>>(e->pbuf, V, V, e->amax);
        PULSAR_LAUNCH_CHECK("k_argmax_rows");
    }
    k_accept_greedy<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->toks, e->amax, n, g, e->loop_out, e->stats, e->slots_dev,
                                                     e->rows, rp ? e->seen : nullptr, V);
    return launch_status("k_accept_greedy");
}

// Sampled round: the drafts' logits are kept (rows j*n + i of qbuf) and each draft token is
// drawn from its warped distribution; the verify pass writes its logits (pbuf), their warp
// statistics are computed per row, and k_accept_sampled runs the ratio test per sequence.
int body_round_sampled(pulsar_engine* e, cudaStream_t st, void* vctx) {
    LoopCtx* c = static_cast<LoopCtx*>(vctx);
    const int n = c->n, g = c->gamma, rows_v = n * (g + 1), V = e->V;
    const bool rp = e->rp_on;   // repetition penalty: draft and verify logits penalised in place
    const size_t smem = (size_t)V * sizeof(float);
    for (int j = 0; j <= g; ++j) {
        if (j > 0) {
            k_rows_spec<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->slots_dev, n, g, j, e->amax, e->toks, e->rows, e->rows_v);
            PULSAR_LAUNCH_CHECK("k_rows_spec");
        }
        float* qrows = j < g ? e->qbuf + (int64_t)j * n * V : nullptr;
        PULSAR_TRY(pulse(e, 0, n, e->rows, nullptr, nullptr, e->hblk + (int64_t)j * D, e->h0blk + (int64_t)j * D,
                         qrows, V, nullptr, st, g + 1));
        if (j < g) {
            if (rp) PULSAR_TRY(penalize(e, qrows, n, 1, j, g, e->seqs, st));
            k_warp_sample<<<n, SAMPLE_THREADS, smem, st>>>(qrows, V, V, e->loop_out, e->seq_ids_dev, e->seqs, j, e->amax,
                                                           e->qstats + (int64_t)j * n);
            PULSAR_LAUNCH_CHECK("k_warp_sample");
        }
    }
    e->attn_rpb = g + 1;   // verify blocks: one pass over each chunk of K/V per block in the attention
    const int v1 = pulse(e, 1, rows_v, e->rows_v, e->hblk, e->h0blk, e->htmp2, nullptr, nullptr, 0, nullptr, st);
    const int v2 = v1 ? v1 : pulse(e, 2, rows_v, e->rows_v, e->htmp2, e->h0blk, e->htmp, nullptr, e->pbuf, V, nullptr, st);
    e->attn_rpb = 1;
    PULSAR_TRY(v2);
    if (rp) PULSAR_TRY(penalize(e, e->pbuf, rows_v, g + 1, 0, g, e->seqs, st));
    k_warp_sample<<<rows_v, SAMPLE_THREADS, smem, st>>>(e->pbuf, V, V, e->loop_out, e->seq_ids_dev, nullptr, 0, nullptr,
                                                        e->pstats);
    PULSAR_LAUNCH_CHECK("k_warp_sample");
    k_accept_sampled<<<n, SAMPLE_THREADS, 0, st>>>(e->seqs, e->toks, e->pbuf, e->qbuf, e->pstats, e->qstats, n, g, V,
                                                  e->seq_ids_dev, e->loop_out, e->stats, e->slots_dev, e->rows,
                                                  rp ? e->seen : nullptr);
    return launch_status("k_accept_sampled");
}

}  // namespace

// ==================================================================================== C ABI
extern "C" int pulsar_engine_create(const pulsar_engine_config* cfg, pulsar_engine** out) {
    PULSAR_CHECK_ARG(cfg && out, "pulsar_engine_create: null argument");
    PULSAR_CHECK_ARG(cfg->vocab_size > 0 && cfg->vocab_size % 256 == 0, "vocab_size must be a positive multiple of 256");
    PULSAR_CHECK_ARG(cfg->max_pulses >= NP, "max_pulses must be >= %d", NP);
    PULSAR_CHECK_ARG(cfg->loop_lora_rank == 0 || cfg->loop_lora_rank == 8, "loop_lora_rank must be 0 or 8");
    PULSAR_CHECK_ARG(cfg->max_batch >= 1 && cfg->max_batch <= MAX_BATCH, "max_batch must be in [1, %d]", MAX_BATCH);
    PULSAR_CHECK_ARG(cfg->max_seq_len >= 16, "max_seq_len too small");
    PULSAR_CHECK_ARG(cfg->max_prefill >= 1 && cfg->max_prefill <= cfg->max_seq_len, "max_prefill must be in [1, max_seq_len]");
    PULSAR_TRY(cuda_status(cudaSetDevice(cfg->device), "cudaSetDevice"));
    auto* e = new pulsar_engine();
    e->cfg = *cfg;
    e->V = cfg->vocab_size;
    e->P = cfg->max_pulses;
    build_expect(e);
    build_arena_names(e);
    auto fail = [&](int st) {
        pulsar_engine_destroy(e);
        return st;
    };
    // KV cache
    const int maxlen = ((cfg->max_seq_len + 63) / 64) * 64;
    const int cap_local = maxlen <= LOCAL_RING ? maxlen : LOCAL_RING;
    const int esz = cfg->kv_fp32 ? 4 : 2;
    int64_t off = 0;
    int64_t layer_off[NL];
    for (int l = 0; l < NL; ++l) {
        const int cap = is_local_layer(l) ? cap_local : maxlen;
        layer_off[l] = off;
        off += (int64_t)2 * HKV * cap * DH;
        e->kvl[l].cap = cap;
        e->kvl[l].mask = (is_local_layer(l) && cap == LOCAL_RING) ? (LOCAL_RING - 1) : -1;
        // local layers: one chunk more than the window, because a run of verify rows spans up to
        // WINDOW + rows - 1 keys from its first row's window start
        e->nch[l] = is_local_layer(l) ? (WINDOW / ATT_CHUNK + 1) : (maxlen + ATT_CHUNK - 1) / ATT_CHUNK;
    }
    const int64_t slot_elems = off;
    int st = e->dmalloc(&e->kv, (size_t)slot_elems * cfg->max_batch * esz, &e->kv_bytes);
    if (st) return fail(st);
    for (int l = 0; l < NL; ++l) {
        e->kvl[l].base = static_cast<char*>(e->kv) + layer_off[l] * esz;
        e->kvl[l].slot_stride = slot_elems;
        e->kv_lrow[l] = layer_off[l] / DH;
    }
    // Zeroed once: attention reads whole 128-key chunks and masks the keys past a row's position,
    // so positions never written must hold finite values.
    if ((st = cuda_status(cudaMemset(e->kv, 0, (size_t)slot_elems * cfg->max_batch * esz), "zero the KV cache")))
        return fail(st);
    {
        const uint64_t kv_rows = (uint64_t)slot_elems * cfg->max_batch / DH;
        e->kv_map_ok = !cfg->kv_fp32 && kv_rows + DT_CK <= (uint64_t)INT32_MAX &&
                       encode_bf16_map(&e->kv_map, e->kv, kv_rows, DH, DT_CK);
    }
    e->len.assign(cfg->max_batch, 0);
    // decode workspace
    const int R = MAX_ROWS;
    int nch_max = 0;
    for (int l = 0; l < NL; ++l) nch_max = std::max(nch_max, e->nch[l]);
    auto& w = e->w;
    const int nblk = e->V / LM_ROWS_PER_BLOCK;
    if ((st = e->wmalloc(&w.h, (size_t)R * D)) || (st = e->wmalloc(&w.h_in, (size_t)R * D)) ||
        (st = e->wmalloc(&w.xn, (size_t)R * D)) || (st = e->wmalloc(&w.qkv, (size_t)R * QKV)) ||
        (st = e->wmalloc(&w.q, (size_t)R * H * DH)) || (st = e->wmalloc(&w.vfirst, (size_t)R * HKV * DH)) ||
        (st = e->wmalloc(&w.part, (size_t)R * H * nch_max * PART)) || (st = e->wmalloc(&w.att, (size_t)R * D)) ||
        (st = e->wmalloc(&w.act_sh, (size_t)R * DS)) || (st = e->wmalloc(&w.act_r, (size_t)R * TOPK * DE)) ||
        (st = e->wmalloc(&w.hn, (size_t)R * D)) || (st = e->wmalloc(&w.t_qkv, (size_t)R * LORA_R)) ||
        (st = e->wmalloc(&w.t_wo, (size_t)R * LORA_R)) || (st = e->wmalloc(&w.wts, (size_t)R * TOPK)) ||
        (st = e->wmalloc(&w.pmax, (size_t)R * nblk)) || (st = e->wmalloc(&w.idx, (size_t)R * TOPK)) ||
        (st = e->wmalloc(&w.pidx, (size_t)R * nblk)))
        return fail(st);
    // wide workspace: every row of a speculative round of max_batch sequences (gamma <= 7)
    const int RW = std::max(MAX_ROWS, cfg->max_batch * (MAX_GAMMA + 1));
    e->wide_rows = RW;
    auto& x = e->ww;
    if ((st = e->wmalloc(&x.h, (size_t)RW * D)) || (st = e->wmalloc(&x.h_in, (size_t)RW * D)) ||
        (st = e->wmalloc(&x.xn, (size_t)RW * D)) || (st = e->wmalloc(&x.qkv, (size_t)RW * QKV)) ||
        (st = e->wmalloc(&x.q, (size_t)RW * H * DH)) || (st = e->wmalloc(&x.vfirst, (size_t)RW * HKV * DH)) ||
        (st = e->wmalloc(&x.part, (size_t)RW * H * nch_max * PART)) || (st = e->wmalloc(&x.att, (size_t)RW * D)) ||
        (st = e->wmalloc(&x.act_sh, (size_t)RW * DS)) || (st = e->wmalloc(&x.sh, (size_t)RW * D)) ||
        (st = e->wmalloc(&x.hn, (size_t)RW * D)) || (st = e->wmalloc(&x.t_qkv, (size_t)RW * LORA_R)) ||
        (st = e->wmalloc(&x.t_wo, (size_t)RW * LORA_R)) || (st = e->wmalloc(&x.wts, (size_t)RW * TOPK)) ||
        (st = e->wmalloc(&x.act_e, (size_t)E * RW * DE)) || (st = e->wmalloc(&x.ye, (size_t)E * RW * D)) ||
        (st = e->wmalloc(&x.logits, (size_t)RW * cfg->vocab_size)) || (st = e->wmalloc(&x.idx, (size_t)RW * TOPK)) ||
        (st = e->wmalloc(&x.lists, (size_t)E * RW * TOPK)) || (st = e->wmalloc(&x.cnt, E)) ||
        (st = e->wmalloc(&x.slot, (size_t)RW * TOPK)) || (st = e->wmalloc(&x.rows_e, (size_t)E * RW)) ||
        (st = e->wmalloc(&x.kept, E)) || (st = e->wmalloc(&x.xs_hi, (size_t)RW * D)) ||
        (st = e->wmalloc(&x.xs_lo, (size_t)RW * D)) || (st = e->wmalloc(&x.ss_hi, (size_t)RW * DS)) ||
        (st = e->wmalloc(&x.ss_lo, (size_t)RW * DS)) || (st = e->wmalloc(&x.es_hi, (size_t)E * RW * DE)) ||
        (st = e->wmalloc(&x.es_lo, (size_t)E * RW * DE)))
        return fail(st);
    {   // activation split for the tensor-core GEMMs: the largest A of prefill or a wide pass
        const int cap_pf = prefill_capacity(cfg->max_prefill);
        e->split_elems = (int64_t)E * std::max(cap_pf, RW) * std::max(D, DS);
        e->split_elems = std::max(e->split_elems, (int64_t)cfg->max_prefill * std::max(D, DS));
        if ((st = e->wmalloc(&e->split_hi, (size_t)e->split_elems)) || (st = e->wmalloc(&e->split_lo, (size_t)e->split_elems)))
            return fail(st);
    }
    // prefill workspace
    auto& f = e->pf;
    const int T = cfg->max_prefill;
    const int cap = prefill_capacity(T);
    f.cap = cap;
    const size_t TD = (size_t)T * D;
    if ((st = e->wmalloc(&f.ids, T)) || (st = e->wmalloc(&f.h0, TD)) || (st = e->wmalloc(&f.h0n_pre, TD)) ||
        (st = e->wmalloc(&f.h0n, TD)) || (st = e->wmalloc(&f.hp, TD)) || (st = e->wmalloc(&f.h, TD)) ||
        (st = e->wmalloc(&f.h_in, TD)) || (st = e->wmalloc(&f.xn, TD)) || (st = e->wmalloc(&f.qkv, (size_t)T * QKV)) ||
        (st = e->wmalloc(&f.q, (size_t)T * H * DH)) || (st = e->wmalloc(&f.o, (size_t)T * H * DH)) ||
        (st = e->wmalloc(&f.att, TD)) || (st = e->wmalloc(&f.vfirst, (size_t)T * HKV * DH)) ||
        (st = e->wmalloc(&f.t, (size_t)T * LORA_R)) || (st = e->wmalloc(&f.wts, (size_t)T * TOPK)) ||
        (st = e->wmalloc(&f.act_sh, (size_t)T * DS)) || (st = e->wmalloc(&f.sh, TD)) ||
        (st = e->wmalloc(&f.act_e, (size_t)E * cap * DE)) || (st = e->wmalloc(&f.ye, (size_t)E * cap * D)) ||
        (st = e->wmalloc(&f.hn, (size_t)D)) || (st = e->wmalloc(&f.pmax, (size_t)nblk)) ||
        (st = e->wmalloc(&f.idx, (size_t)T * TOPK)) || (st = e->wmalloc(&f.lists, (size_t)E * T * TOPK)) ||
        (st = e->wmalloc(&f.cnt, E)) || (st = e->wmalloc(&f.slot, (size_t)T * TOPK)) ||
        (st = e->wmalloc(&f.rows_e, (size_t)E * cap)) || (st = e->wmalloc(&f.kept, E)) ||
        (st = e->wmalloc(&f.pidx, (size_t)nblk)) || (st = e->wmalloc(&f.xs_hi, TD)) ||
        (st = e->wmalloc(&f.xs_lo, TD)) || (st = e->wmalloc(&f.ss_hi, (size_t)T * DS)) ||
        (st = e->wmalloc(&f.ss_lo, (size_t)T * DS)) || (st = e->wmalloc(&f.es_hi, (size_t)E * cap * DE)) ||
        (st = e->wmalloc(&f.es_lo, (size_t)E * cap * DE)))
        return fail(st);
    // decode-loop state
    const int NB = cfg->max_batch;
    if ((st = e->wmalloc(&e->seqs, NB)) || (st = e->wmalloc(&e->slots_dev, NB)) ||
        (st = e->wmalloc(&e->toks, RW)) || (st = e->wmalloc(&e->amax, RW)) ||
        (st = e->wmalloc(&e->loop_out, 1)) || (st = e->wmalloc(&e->qbuf, (size_t)RW * cfg->vocab_size)) ||
        (st = e->wmalloc(&e->pbuf, (size_t)RW * cfg->vocab_size)) || (st = e->wmalloc(&e->qstats, RW)) ||
        (st = e->wmalloc(&e->pstats, RW)) || (st = e->wmalloc(&e->seq_ids_dev, NB)) ||
        (st = e->wmalloc(&e->lens_dev, NB)) || (st = e->wmalloc(&e->first_dev, NB)) ||
        (st = e->wmalloc(&e->rows, RW)) || (st = e->wmalloc(&e->rows_v, RW)) ||
        (st = e->wmalloc(&e->hblk, (size_t)RW * D)) || (st = e->wmalloc(&e->h0blk, (size_t)RW * D)) ||
        (st = e->wmalloc(&e->htmp, (size_t)RW * D)) || (st = e->wmalloc(&e->htmp2, (size_t)RW * D)) ||
        (st = e->wmalloc(&e->h0tmp, (size_t)RW * D)) || (st = e->wmalloc(&e->stats, (size_t)NB * 3)) ||
        (st = e->wmalloc(&e->ee, (size_t)NB + 2)) || (st = e->wmalloc(&e->ee_amax, (size_t)2 * NB)) ||
        (st = e->wmalloc(&e->ee_counts, NP)) || (st = e->wmalloc(&e->seen, (size_t)NB * (cfg->vocab_size / 32))))
        return fail(st);
    if ((st = cuda_status(cudaMemset(e->ee_counts, 0, NP * sizeof(unsigned long long)), "zero exit tallies")))
        return fail(st);
    // persistent pulse kernel: one CTA per SM, co-resident (cooperative launch)
    {
        int sms = 0, per_sm = 0;
        if ((st = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device), "SM count")))
            return fail(st);
        if ((st = mega_occupancy(cfg->kv_fp32 != 0, &per_sm))) return fail(st);
        if ((st = cuda_status(cudaFuncSetAttribute(k_warp_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   SAMPLE_MAX_V * (int)sizeof(float)),
                              "k_warp_sample shared memory")))
            return fail(st);
        // the per-CTA staging sizes assume >= 144 CTAs (ceil(8192 / C) + ceil(1024 / C) <= 64 pairs)
        e->mega_grid = sms;
        e->use_mega = per_sm >= 1 && sms >= 144;
        e->mega_nch = std::max(2400 / 32 + 2, (maxlen + MEGA_CHUNK - 1) / MEGA_CHUNK + 2);   // see attn_chunk()
        if ((st = e->wmalloc(&e->m_gate, (size_t)MEGA_RMAX * H)) ||
            (st = e->wmalloc(&e->m_part, (size_t)MEGA_RMAX * H * e->mega_nch * PART)) ||
            (st = e->wmalloc(&e->m_g8, (size_t)MEGA_RMAX * RG)) ||
            (st = e->wmalloc(&e->m_rpart, (size_t)std::max(sms, 1) * MEGA_RMAX * E)) ||
            (st = e->wmalloc(&e->m_pmax, (size_t)MEGA_RMAX * std::max(sms, 1))) ||
            (st = e->wmalloc(&e->m_pidx, (size_t)MEGA_RMAX * std::max(sms, 1))) || (st = e->wmalloc(&e->m_err, 1)) ||
            (st = e->wmalloc(&e->m_bar, 1)) || (st = e->wmalloc(&e->m_tickets, (size_t)MEGA_RMAX * HKV + 2)) ||
            (st = e->wmalloc(&e->m_experts, 1)))
            return fail(st);
        if ((st = cuda_status(cudaMemset(e->m_tickets, 0, ((size_t)MEGA_RMAX * HKV + 2) * 4), "zero tickets")) ||
            (st = cuda_status(cudaMemset(e->m_bar, 0, 4), "zero grid barrier")) ||
            (st = cuda_status(cudaMemset(e->m_err, 0, 4), "zero err")) ||
            (st = cuda_status(cudaMemset(e->m_experts, 0, 8), "zero expert count")))
            return fail(st);
    }
    *out = e;
    clear_error();
    return PULSAR_OK;
}

extern "C" int pulsar_engine_destroy(pulsar_engine* e) {
    if (!e) return PULSAR_OK;
    cudaSetDevice(e->cfg.device);
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
    for (cudaEvent_t ev : e->tev)
        if (ev) cudaEventDestroy(ev);
    for (auto& kv : e->t) cudaFree(kv.second);
    for (void* p : e->allocs) cudaFree(p);
    delete e;
    return PULSAR_OK;
}

extern "C" int pulsar_engine_set_tensor(pulsar_engine* e, const char* name, const float* data, int64_t numel) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(name && data, "set_tensor: null argument");
    auto it = e->expect.find(name);
    PULSAR_CHECK_ARG(it != e->expect.end(), "set_tensor: unknown tensor name '%s'", name);
    PULSAR_CHECK_ARG(it->second == numel, "set_tensor: '%s' has %lld elements, expected %lld", name, (long long)numel,
                     (long long)it->second);
    if (e->finalized) {
        set_error("set_tensor after finalize is not supported ('%s')", name);
        return PULSAR_ERR_STATE;
    }
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    float*& dst = e->t[name];
    if (!dst) PULSAR_TRY(cuda_status(cudaMalloc(&dst, (size_t)numel * 4), "cudaMalloc(staging)"));
    PULSAR_TRY(cuda_status(cudaMemcpy(dst, data, (size_t)numel * 4, cudaMemcpyHostToDevice), "set_tensor copy"));
    if (strstr(name, "lora_B")) {
        for (int64_t i = 0; i < numel; ++i)
            if (data[i] != 0.f) { e->has_lora = e->cfg.loop_lora_rank > 0; break; }
    }
    return PULSAR_OK;
}

extern "C" int pulsar_engine_finalize(pulsar_engine* e) {
    PULSAR_TRY(check_engine(e, false));
    if (e->finalized) return PULSAR_OK;
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    for (auto& kv : e->expect) {
        if (kv.first == "lm_head.weight" || kv.first.find("expert_counts") != std::string::npos ||
            kv.first.find("expert_pulse_counts") != std::string::npos)
            continue;
        if (!e->cfg.loop_lora_rank && (kv.first.find("_adapter.") != std::string::npos)) continue;
        if (!e->T_(kv.first) && !arena_covered(e, kv.first)) {
            set_error("finalize: tensor '%s' was never uploaded", kv.first.c_str());
            return PULSAR_ERR_STATE;
        }
    }
    cudaStream_t st = 0;
    auto conv = [&](const std::string& n, __nv_bfloat16** dst, int64_t numel) -> int {
        if (*dst) return PULSAR_OK;   // written from a repacked arena
        PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(dst), (size_t)numel * 2, &e->arena_bytes));
        k_f32_to_bf16<<<1024, 256, 0, st>>>(e->T_(n), *dst, numel);
        return launch_status("k_f32_to_bf16");
    };
    PULSAR_TRY(conv("tok_emb.weight", &e->emb, (int64_t)e->V * D));
    for (int l = 0; l < NL; ++l) {
        PULSAR_TRY(conv(e->L(l, "attn.wqkv.weight"), &e->wqkv[l], (int64_t)QKV * D));
        PULSAR_TRY(conv(e->L(l, "attn.wo.weight"), &e->wo[l], (int64_t)D * D));
        PULSAR_TRY(conv(e->L(l, "mlp.shared_expert.w_gate_up.weight"), &e->sh_gu[l], (int64_t)2 * DS * D));
        PULSAR_TRY(conv(e->L(l, "mlp.shared_expert.w_down.weight"), &e->sh_dn[l], (int64_t)D * DS));
        if (!e->r_gu[l]) {
            PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->r_gu[l]), (size_t)E * D * 2 * DE * 2, &e->arena_bytes));
            // routed_gate_up [E][D in][2*DE out] -> [E][2*DE out][D in]
            k_transpose_bf16<<<dim3(2 * DE / 32, D / 32, E), dim3(32, 8), 0, st>>>(
                e->T_(e->L(l, "mlp.routed_gate_up")), e->r_gu[l], D, 2 * DE);
        }
        if (!e->r_dn[l]) {
            PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->r_dn[l]), (size_t)E * DE * D * 2, &e->arena_bytes));
            // routed_down [E][DE in][D out] -> [E][D out][DE in]
            k_transpose_bf16<<<dim3(D / 32, DE / 32, E), dim3(32, 8), 0, st>>>(e->T_(e->L(l, "mlp.routed_down")),
                                                                                e->r_dn[l], DE, D);
        }
        PULSAR_LAUNCH_CHECK("expert transpose");
        std::vector<float> lam(e->P);
        PULSAR_TRY(cuda_status(cudaMemcpy(lam.data(), e->T_(e->L(l, "attn.v_resid_lambda")), e->P * 4,
                                          cudaMemcpyDeviceToHost),
                               "read v_resid_lambda"));
        for (int p = 0; p < NP; ++p) e->vres[p][l] = 1.f / (1.f + std::exp(-lam[p]));
        if (e->has_lora) {
            const float scale = e->cfg.loop_lora_alpha / 8.f;
            for (int p = 0; p < NP; ++p) {
                PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->lb_qkv[p][l]), (size_t)QKV * LORA_R * 4, &e->arena_bytes));
                PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->lb_wo[p][l]), (size_t)D * LORA_R * 4, &e->arena_bytes));
                k_lora_b<<<256, 256, 0, st>>>(e->T_(e->L(l, "attn.wqkv_adapter.lora_B")),
                                              e->T_(e->L(l, "attn.wqkv_adapter.loop_M")), e->P, p, scale, QKV, 8,
                                              e->lb_qkv[p][l]);
                k_lora_b<<<256, 256, 0, st>>>(e->T_(e->L(l, "attn.wo_adapter.lora_B")),
                                              e->T_(e->L(l, "attn.wo_adapter.loop_M")), e->P, p, scale, D, 8,
                                              e->lb_wo[p][l]);
                PULSAR_LAUNCH_CHECK("k_lora_b");
            }
        }
    }
    // RoPE tables covering every position the KV cache can hold
    e->rope_len = ((e->cfg.max_seq_len + 63) / 64) * 64 + 64;
    for (float** p : {&e->cos_l, &e->sin_l, &e->cos_g, &e->sin_g})
        PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(p), (size_t)e->rope_len * 32 * 4, &e->arena_bytes));
    k_rope_table<<<256, 256, 0, st>>>(e->T_("rope_local.inv_freq"), e->rope_len, e->cos_l, e->sin_l);
    k_rope_table<<<256, 256, 0, st>>>(e->T_("rope_global.inv_freq"), e->rope_len, e->cos_g, e->sin_g);
    PULSAR_LAUNCH_CHECK("k_rope_table");
    PULSAR_TRY(cuda_status(cudaDeviceSynchronize(), "finalize"));
    // the big fp32 staging copies are no longer needed
    const char* big[] = {"attn.wqkv.weight", "attn.wo.weight", "mlp.shared_expert.w_gate_up.weight",
                         "mlp.shared_expert.w_down.weight", "mlp.routed_gate_up", "mlp.routed_down"};
    for (int l = 0; l < NL; ++l)
        for (const char* b : big) {
            auto it = e->t.find(e->L(l, b));
            if (it != e->t.end()) { cudaFree(it->second); e->t.erase(it); }
        }
    for (const char* b : {"tok_emb.weight", "lm_head.weight"}) {
        auto it = e->t.find(b);
        if (it != e->t.end()) { cudaFree(it->second); e->t.erase(it); }
    }
    e->finalized = true;
    clear_error();
    return PULSAR_OK;
}

extern "C" int pulsar_engine_arena_count(pulsar_engine* e, int32_t* count) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(count, "arena_count: null argument");
    *count = (int32_t)e->arena_names.size();
    return PULSAR_OK;
}

extern "C" int pulsar_engine_arena_info(pulsar_engine* e, int32_t index, const char** name, int64_t* numel) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(name && numel, "arena_info: null argument");
    PULSAR_CHECK_ARG(index >= 0 && index < (int32_t)e->arena_names.size(), "arena_info: index %d out of range", index);
    *name = e->arena_names[index].c_str();
    *numel = arena_ref(e, e->arena_names[index]).numel;
    return PULSAR_OK;
}

extern "C" int pulsar_engine_arena_read(pulsar_engine* e, const char* name, void* host_dst, int64_t numel) {
    PULSAR_TRY(check_engine(e, true));
    PULSAR_CHECK_ARG(name && host_dst, "arena_read: null argument");
    const ArenaRef r = arena_ref(e, name);
    PULSAR_CHECK_ARG(r.ptr, "arena_read: unknown arena tensor '%s'", name);
    PULSAR_CHECK_ARG(numel == r.numel, "arena_read: '%s' has %lld elements, asked for %lld", name, (long long)r.numel,
                     (long long)numel);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    return cuda_status(cudaMemcpy(host_dst, *r.ptr, (size_t)numel * 2, cudaMemcpyDeviceToHost), "arena_read copy");
}

extern "C" int pulsar_engine_arena_write(pulsar_engine* e, const char* name, const void* host_src, int64_t numel) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(name && host_src, "arena_write: null argument");
    if (e->finalized) {
        set_error("arena_write after finalize is not supported ('%s')", name);
        return PULSAR_ERR_STATE;
    }
    const ArenaRef r = arena_ref(e, name);
    PULSAR_CHECK_ARG(r.ptr, "arena_write: unknown arena tensor '%s'", name);
    PULSAR_CHECK_ARG(numel == r.numel, "arena_write: '%s' has %lld elements, got %lld", name, (long long)r.numel,
                     (long long)numel);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    if (!*r.ptr) PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(r.ptr), (size_t)numel * 2, &e->arena_bytes));
    PULSAR_TRY(cuda_status(cudaMemcpy(*r.ptr, host_src, (size_t)numel * 2, cudaMemcpyHostToDevice), "arena_write copy"));
    e->arena_written[name] = true;
    return PULSAR_OK;
}

extern "C" int pulsar_engine_memory(const pulsar_engine* e, int64_t* a, int64_t* k, int64_t* w) {
    PULSAR_CHECK_ARG(e, "null engine handle");
    if (a) *a = e->arena_bytes;
    if (k) *k = e->kv_bytes;
    if (w) *w = e->work_bytes;
    return PULSAR_OK;
}

extern "C" int pulsar_engine_prefill(pulsar_engine* e, int32_t slot, const int32_t* ids, int32_t T, float* logits,
                                     void* stream) {
    PULSAR_TRY(check_engine(e, true));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch, "prefill: slot %d out of range", slot);
    PULSAR_CHECK_ARG(T >= 1, "prefill: empty prompt");
    if (T > e->cfg.max_prefill) {
        set_error("prefill: prompt of %d tokens exceeds max_prefill %d", T, e->cfg.max_prefill);
        return PULSAR_ERR_CAPACITY;
    }
    PULSAR_CHECK_ARG(ids && logits, "prefill: null pointer");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    {
        std::vector<int32_t> h(T);
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(h.data(), ids, (size_t)T * 4, cudaMemcpyDeviceToHost, st), "copy ids"));
        PULSAR_TRY(cuda_status(cudaStreamSynchronize(st), "copy ids"));
        for (int i = 0; i < T; ++i)
            if (h[i] < 0 || h[i] >= e->V) {
                set_error("prefill: token %d at index %d outside [0, %d)", h[i], i, e->V);
                return PULSAR_ERR_INVALID;
            }
    }
    const int rc = e->kv32() ? enqueue_prefill<float>(e, slot, ids, T, logits, st, false)
                             : enqueue_prefill<__nv_bfloat16>(e, slot, ids, T, logits, st, false);
    if (rc != PULSAR_OK) return rc;
    e->len[slot] = T;
    // the slot's seen-token set for the repetition penalty: the prompt
    k_seen_init<<<1, 1024, 0, st>>>(e->seen + (int64_t)slot * (e->V / 32), ids, T, e->V / 32);
    return launch_status("k_seen_init");
}

extern "C" int pulsar_engine_forward(pulsar_engine* e, int32_t slot, const int32_t* ids, int32_t T, float* logits,
                                     void* stream) {
    PULSAR_TRY(check_engine(e, true));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch, "forward: slot %d out of range", slot);
    PULSAR_CHECK_ARG(T >= 1, "forward: empty sequence");
    PULSAR_CHECK_ARG(ids && logits, "forward: null pointer");
    const int lim = std::min(e->cfg.max_prefill, e->kvl[0].cap);   // every local key in the ring
    if (T > lim) {
        set_error("forward: %d tokens exceed %d (max_prefill, and the local layers' %d-position ring)", T, lim,
                  e->kvl[0].cap);
        return PULSAR_ERR_CAPACITY;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    {
        std::vector<int32_t> h(T);
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(h.data(), ids, (size_t)T * 4, cudaMemcpyDeviceToHost, st), "copy ids"));
        PULSAR_TRY(cuda_status(cudaStreamSynchronize(st), "copy ids"));
        for (int i = 0; i < T; ++i)
            if (h[i] < 0 || h[i] >= e->V) {
                set_error("forward: token %d at index %d outside [0, %d)", h[i], i, e->V);
                return PULSAR_ERR_INVALID;
            }
    }
    const int rc = e->kv32() ? enqueue_prefill<float>(e, slot, ids, T, logits, st, true)
                             : enqueue_prefill<__nv_bfloat16>(e, slot, ids, T, logits, st, true);
    // the slot's cache now holds the forward's keys and values, not a decodable prefix
    e->len[slot] = 0;
    return rc;
}

extern "C" int pulsar_engine_pulse(pulsar_engine* e, int32_t p, int32_t R, const int32_t* rows, const float* h_prev,
                                   const float* h0n, float* h_out, float* h0n_out, float* logits, void* stream) {
    PULSAR_TRY(check_engine(e, true));
    PULSAR_CHECK_ARG(p >= 0 && p < NP, "pulse index %d out of range [0, %d)", p, NP);
    PULSAR_CHECK_ARG(R >= 1 && R <= e->wide_rows, "rows %d out of range [1, %d]", R, e->wide_rows);
    PULSAR_CHECK_ARG(rows && h_out && h0n_out, "pulse: null pointer");
    PULSAR_CHECK_ARG(p == 0 || (h_prev && h0n), "pulse %d needs h_prev and h0n", p);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    {
        // validate the row descriptors before any kernel indexes the cache with them
        std::vector<int4> hr(R);
        cudaStream_t vs = reinterpret_cast<cudaStream_t>(stream);
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(hr.data(), rows, (size_t)R * sizeof(int4), cudaMemcpyDeviceToHost, vs), "copy rows"));
        PULSAR_TRY(cuda_status(cudaStreamSynchronize(vs), "copy rows"));
        PULSAR_TRY(check_kernel_err(e));
        for (int r = 0; r < R; ++r) {
            if (hr[r].x < 0 || hr[r].x >= e->cfg.max_batch) {
                set_error("pulse: row %d has slot %d outside [0, %d)", r, hr[r].x, e->cfg.max_batch);
                return PULSAR_ERR_INVALID;
            }
            if (hr[r].y < 0 || hr[r].y >= e->max_pos()) {
                set_error("pulse: row %d position %d outside [0, %d)", r, hr[r].y, e->max_pos());
                return PULSAR_ERR_CAPACITY;
            }
            if (hr[r].z < 0 || hr[r].z >= e->V) {
                set_error("pulse: row %d token %d outside [0, %d)", r, hr[r].z, e->V);
                return PULSAR_ERR_INVALID;
            }
            // the rows of one sequence form one contiguous run of consecutive positions
            if (r > 0 && hr[r].x == hr[r - 1].x && hr[r].y != hr[r - 1].y + 1) {
                set_error("pulse: rows %d and %d of slot %d do not have consecutive positions", r - 1, r, hr[r].x);
                return PULSAR_ERR_INVALID;
            }
            for (int q = 0; q + 1 < r; ++q)
                if (hr[q].x == hr[r].x && hr[r - 1].x != hr[r].x) {
                    set_error("pulse: rows of slot %d are not contiguous", hr[r].x);
                    return PULSAR_ERR_INVALID;
                }
        }
    }
    return pulse(e, p, R, reinterpret_cast<const int4*>(rows), h_prev, h0n, h_out, h0n_out, logits, e->V, nullptr,
                 reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int pulsar_engine_get_length(pulsar_engine* e, int32_t slot, int32_t* length) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch && length, "get_length: bad slot %d", slot);
    *length = e->len[slot];
    return PULSAR_OK;
}

extern "C" int pulsar_engine_set_length(pulsar_engine* e, int32_t slot, int32_t length) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch, "set_length: bad slot %d", slot);
    if (length < 0 || length > e->cfg.max_seq_len) {
        set_error("set_length: %d outside [0, max_seq_len=%d]", length, e->cfg.max_seq_len);
        return PULSAR_ERR_CAPACITY;
    }
    e->len[slot] = length;
    return PULSAR_OK;
}

namespace {
// out[0][g][i][d] = K, out[1][g][i][d] = V of position pos0 + i, head g, as fp32.
template <typename KVT>
__global__ void k_kv_gather(KVLayer L, int slot, int pos0, int n, float* __restrict__ out) {
    const int64_t per = (int64_t)HKV * n * DH;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < 2 * per; e += (int64_t)gridDim.x * blockDim.x) {
        const int isv = (int)(e / per);
        const int64_t r = e % per;
        const int g = (int)(r / ((int64_t)n * DH)), i = (int)((r / DH) % n), d = (int)(r % DH);
        const KVT* p = isv ? kv_v<KVT>(L, slot, g, pos0 + i) : kv_k<KVT>(L, slot, g, pos0 + i);
        out[e] = kv_load(p + d);
    }
}
}  // namespace

namespace {
template <typename KVT>
int prefill_attention(pulsar_engine* e, int slot, int layer, int T, const float* q, float* out, bool tc,
                      cudaStream_t st) {
    const int local = is_local_layer(layer) ? 1 : 0;
    if (tc) {
        PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k_attn_prefill_tc<KVT>), (int)pt_smem_bytes<KVT>(),
                                    "k_attn_prefill_tc shared memory"));
        k_attn_prefill_tc<KVT><<<dim3((T + PT_Q - 1) / PT_Q, H), PT_THREADS, pt_smem_bytes<KVT>(), st>>>(
            slot, T, q, e->kvl[layer], local, out, e->m_err);
        return launch_status("k_attn_prefill_tc");
    }
    k_attn_prefill<KVT><<<dim3((T + PA_Q - 1) / PA_Q, H), 256, 0, st>>>(slot, T, q, e->kvl[layer], local, out);
    return launch_status("k_attn_prefill");
}
}  // namespace

extern "C" int pulsar_engine_prefill_attention(pulsar_engine* e, int32_t slot, int32_t layer, int32_t T,
                                               const float* q_dev, float* out_dev, int32_t tensor_cores,
                                               void* stream) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch, "prefill_attention: slot %d out of range", slot);
    PULSAR_CHECK_ARG(layer >= 0 && layer < NL, "prefill_attention: layer %d out of range [0, %d)", layer, NL);
    PULSAR_CHECK_ARG(q_dev && out_dev, "prefill_attention: null pointer");
    PULSAR_CHECK_ARG(T >= 1 && T <= e->len[slot], "prefill_attention: T = %d, the slot holds %d positions", T,
                     e->len[slot]);
    PULSAR_CHECK_ARG(!is_local_layer(layer) || std::min(T, WINDOW) <= e->kvl[layer].cap,
                     "prefill_attention: the local ring holds %d positions", e->kvl[layer].cap);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return e->kv32() ? prefill_attention<float>(e, slot, layer, T, q_dev, out_dev, tensor_cores != 0, st)
                     : prefill_attention<__nv_bfloat16>(e, slot, layer, T, q_dev, out_dev, tensor_cores != 0, st);
}

// Merge of the split partials of decode_attention: per (row, head) o / l over the splits (0
// when no key was visible), without the head gate.
__global__ void __launch_bounds__(H * 32) k_attn_merge_plain(const float* __restrict__ part, int nsplit,
                                                             float* __restrict__ out) {
    const int r = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* pp = part + ((int64_t)r * H + h) * nsplit * PART;
    float M = -INFINITY;
    for (int c = 0; c < nsplit; ++c) M = fmaxf(M, pp[c * PART]);
    float l = 0.f, o1 = 0.f, o2 = 0.f;
    for (int c = 0; c < nsplit; ++c) {
        const float m = pp[c * PART];
        if (m == -INFINITY) continue;
        const float w = expf(m - M);
        l += w * pp[c * PART + 1];
        o1 += w * pp[c * PART + 2 + lane];
        o2 += w * pp[c * PART + 2 + lane + 32];
    }
    float* y = out + ((int64_t)r * H + h) * DH;
    y[lane] = l > 0.f ? o1 / l : 0.f;
    y[lane + 32] = l > 0.f ? o2 / l : 0.f;
}

template <typename KVT>
int decode_attention(pulsar_engine* e, int layer, int R, const int4* rows, int rpb, const float* q, float* out,
                     bool tc, cudaStream_t st) {
    const bool local = is_local_layer(layer);
    const int save_rpb = e->attn_rpb;
    const bool save_tc = e->tc_dec;
    e->attn_rpb = rpb;
    e->tc_dec = tc;
    const int groups = (R + rpb - 1) / rpb;
    const int nsplit = attn_splits(groups, local ? WINDOW + ATT_RPB_MAX : e->max_pos(), e->mega_grid, e->nch[layer],
                                   attn_chunk<KVT>(e));
    float* part = nullptr;
    int rc = cuda_status(cudaMalloc(&part, (size_t)R * H * nsplit * PART * sizeof(float)), "decode_attention: partials");
    if (rc == PULSAR_OK)
        rc = launch_attn_flash<KVT>(e, dim3(nsplit, HKV, groups), rows, R, q, e->kvl[layer], local ? 1 : 0, nsplit, part,
                                    st);
    if (rc == PULSAR_OK) {
        k_attn_merge_plain<<<R, H * 32, 0, st>>>(part, nsplit, out);
        rc = launch_status("k_attn_merge_plain");
    }
    if (rc == PULSAR_OK) rc = cuda_status(cudaStreamSynchronize(st), "decode_attention");
    if (rc == PULSAR_OK) rc = check_kernel_err(e);
    if (part) cudaFree(part);
    e->attn_rpb = save_rpb;
    e->tc_dec = save_tc;
    return rc;
}

extern "C" int pulsar_engine_decode_attention(pulsar_engine* e, int32_t layer, int32_t R, const int32_t* rows_dev,
                                              int32_t rows_per_block, const float* q_dev, float* out_dev,
                                              int32_t tensor_cores, void* stream) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(layer >= 0 && layer < NL, "decode_attention: layer %d out of range [0, %d)", layer, NL);
    PULSAR_CHECK_ARG(R >= 1, "decode_attention: R = %d", R);
    PULSAR_CHECK_ARG(rows_per_block >= 1 && rows_per_block <= ATT_RPB_MAX,
                     "decode_attention: rows_per_block %d out of range [1, %d]", rows_per_block, ATT_RPB_MAX);
    PULSAR_CHECK_ARG(rows_dev && q_dev && out_dev, "decode_attention: null pointer");
    PULSAR_CHECK_ARG(((uintptr_t)rows_dev & 15) == 0 && ((uintptr_t)q_dev & 15) == 0,
                     "decode_attention: rows and queries must be 16-byte aligned");
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int4* rows = reinterpret_cast<const int4*>(rows_dev);
    return e->kv32() ? decode_attention<float>(e, layer, R, rows, rows_per_block, q_dev, out_dev, tensor_cores != 0, st)
                     : decode_attention<__nv_bfloat16>(e, layer, R, rows, rows_per_block, q_dev, out_dev,
                                                       tensor_cores != 0, st);
}

extern "C" int pulsar_engine_read_kv(pulsar_engine* e, int32_t slot, int32_t layer, int32_t pos0, int32_t n,
                                     float* k_host, float* v_host) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(slot >= 0 && slot < e->cfg.max_batch, "read_kv: slot %d out of range", slot);
    PULSAR_CHECK_ARG(layer >= 0 && layer < NL, "read_kv: layer %d out of range [0, %d)", layer, NL);
    PULSAR_CHECK_ARG(k_host && v_host, "read_kv: null pointer");
    PULSAR_CHECK_ARG(n >= 0 && pos0 >= 0, "read_kv: negative position or count");
    const KVLayer& L = e->kvl[layer];
    if ((int64_t)pos0 + n > e->max_pos() || n > L.cap) {
        set_error("read_kv: positions [%d, %lld) exceed the layer's %d cached positions (max position %d)", pos0,
                  (long long)pos0 + n, L.cap, e->max_pos());
        return PULSAR_ERR_CAPACITY;
    }
    if (n == 0) return PULSAR_OK;
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    PULSAR_TRY(cuda_status(cudaDeviceSynchronize(), "read_kv: pending work"));
    PULSAR_TRY(check_kernel_err(e));
    const size_t per = (size_t)HKV * n * DH;
    float* tmp = nullptr;
    PULSAR_TRY(cuda_status(cudaMalloc(&tmp, 2 * per * sizeof(float)), "read_kv: staging"));
    if (e->kv32()) k_kv_gather<float><<<256, 256>>>(L, slot, pos0, n, tmp);
    else k_kv_gather<__nv_bfloat16><<<256, 256>>>(L, slot, pos0, n, tmp);
    int st = launch_status("k_kv_gather");
    if (st == PULSAR_OK) st = cuda_status(cudaMemcpy(k_host, tmp, per * sizeof(float), cudaMemcpyDeviceToHost), "read_kv: copy K");
    if (st == PULSAR_OK)
        st = cuda_status(cudaMemcpy(v_host, tmp + per, per * sizeof(float), cudaMemcpyDeviceToHost), "read_kv: copy V");
    cudaFree(tmp);
    return st;
}

namespace {
int generate_impl(pulsar_engine* e, int32_t n, const int32_t* slots_host, const int32_t* seq_ids_host,
                  const float* first_logits, int32_t n_new, int32_t gamma, bool sampled, float temperature, float top_p,
                  uint64_t seed, int32_t* out, int64_t* stats_host, void* stream) {
    PULSAR_TRY(check_engine(e, true));
    PULSAR_CHECK_ARG(n >= 1 && n <= e->cfg.max_batch, "generate: n_seq %d out of range", n);
    PULSAR_CHECK_ARG(gamma >= 0 && gamma <= MAX_GAMMA, "generate: gamma %d outside [0, %d]", gamma, MAX_GAMMA);
    PULSAR_CHECK_ARG(n_new >= 1 && slots_host && first_logits && out, "generate: bad arguments");
    if (sampled) {
        PULSAR_CHECK_ARG(gamma >= 1, "generate_sampled: gamma must be >= 1");
        PULSAR_CHECK_ARG(seq_ids_host != nullptr, "generate_sampled: null seq_ids");
        PULSAR_CHECK_ARG(temperature > 0.f && top_p > 0.f && top_p <= 1.f,
                         "generate_sampled: need temperature > 0 and 0 < top_p <= 1");
        PULSAR_CHECK_ARG(e->V <= SAMPLE_MAX_V, "generate_sampled: vocab_size %d above %d", e->V, SAMPLE_MAX_V);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    std::vector<int> lens(n);
    for (int i = 0; i < n; ++i) {
        const int s = slots_host[i];
        PULSAR_CHECK_ARG(s >= 0 && s < e->cfg.max_batch, "generate: slot %d out of range", s);
        PULSAR_CHECK_ARG(e->len[s] >= 1, "generate: slot %d has no prefilled context", s);
        for (int k = 0; k < i; ++k) PULSAR_CHECK_ARG(slots_host[k] != s, "generate: slot %d listed twice", s);
        lens[i] = e->len[s];
        if (lens[i] + n_new + gamma + 1 > e->cfg.max_seq_len) {
            set_error("generate: slot %d needs %d positions, max_seq_len is %d", s, lens[i] + n_new + gamma + 1,
                      e->cfg.max_seq_len);
            return PULSAR_ERR_CAPACITY;
        }
    }
    const LoopOut lp{out, n_new, (unsigned long long)seed, temperature, top_p, e->ee_thr, e->rp};
    PULSAR_TRY(cuda_status(cudaMemcpyAsync(e->slots_dev, slots_host, n * 4, cudaMemcpyHostToDevice, st), "copy slots"));
    PULSAR_TRY(cuda_status(cudaMemcpyAsync(e->lens_dev, lens.data(), n * 4, cudaMemcpyHostToDevice, st), "copy lens"));
    PULSAR_TRY(cuda_status(cudaMemcpyAsync(e->loop_out, &lp, sizeof(lp), cudaMemcpyHostToDevice, st), "copy params"));
    PULSAR_TRY(cuda_status(cudaMemsetAsync(e->stats, 0, (size_t)n * 3 * 8, st), "zero stats"));
    if (sampled) {
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(e->seq_ids_dev, seq_ids_host, n * 4, cudaMemcpyHostToDevice, st),
                               "copy seq ids"));
        const float* fl = first_logits;
        if (e->rp_on) {   // the first draw sees the penalised prompt ids (a copy: the caller's row stays)
            PULSAR_TRY(cuda_status(cudaMemcpyAsync(e->pbuf, first_logits, (size_t)n * e->V * 4, cudaMemcpyDeviceToDevice, st),
                                   "copy first logits"));
            PULSAR_TRY(penalize(e, e->pbuf, n, 1, 0, 0, nullptr, st));
            fl = e->pbuf;
        }
        k_warp_sample<<<n, SAMPLE_THREADS, (size_t)e->V * 4, st>>>(fl, e->V, e->V, e->loop_out,
                                                                   e->seq_ids_dev, nullptr, 0, e->first_dev, nullptr);
        if (e->rp_on) k_seen_add<<<(n + 127) / 128, 128, 0, st>>>(e->seen, e->slots_dev, e->first_dev, n, e->V);
    } else if (e->rp_on) {
        k_first_penalized<<<n, 1024, 0, st>>>(first_logits, e->V, e->slots_dev, e->seen, e->loop_out, e->first_dev);
    } else {
        k_argmax_rows<<<n, 1024, 0, st>>>(first_logits, e->V, e->V, e->first_dev);
    }
    k_seq_init<<<(n + 127) / 128, 128, 0, st>>>(e->seqs, e->lens_dev, e->first_dev, n, out, n_new, e->slots_dev, gamma, e->toks,
                                 e->rows);
    PULSAR_LAUNCH_CHECK("generate init");
    e->n_kernels += 2;
    LoopCtx ctx{n, gamma};
    // output, length and sampling parameters live on the device: graphs depend on (n, gamma, mode)
    // (gamma = 0 with early exit and / or a repetition penalty: its own body, key suffixes
    // ":e" / ":r")
    const bool ee = gamma == 0 && e->ee_on, rp = e->rp_on;
    const std::string key = std::to_string(n) + ":" + std::to_string(gamma) + (sampled ? ":s" : ":g") +
                            (ee ? ":e" : "") + (rp ? ":r" : "");
    std::vector<SeqDev> hs(n);
    int remaining_steps = n_new - 1;
    while (true) {
        if (gamma == 0) {
            for (int s = 0; s < remaining_steps; ++s)
                PULSAR_TRY(run_graph(e, key, st, (ee || rp) ? body_step_x : body_step, &ctx));
        } else {
            // each round emits between 1 and gamma+1 tokens; launch the minimum, then check
            const int rounds = std::max(1, (remaining_steps + gamma) / (gamma + 1));
            for (int s = 0; s < rounds; ++s)
                PULSAR_TRY(run_graph(e, key, st, sampled ? body_round_sampled : body_round, &ctx));
        }
        PULSAR_TRY(cuda_status(cudaMemcpyAsync(hs.data(), e->seqs, n * sizeof(SeqDev), cudaMemcpyDeviceToHost, st),
                               "read state"));
        PULSAR_TRY(cuda_status(cudaStreamSynchronize(st), "generate sync"));
        int min_out = n_new;
        for (int i = 0; i < n; ++i) min_out = std::min(min_out, hs[i].n_out);
        if (min_out >= n_new) break;
        remaining_steps = n_new - min_out;
    }
    for (int i = 0; i < n; ++i) e->len[slots_host[i]] = hs[i].len;
    PULSAR_TRY(check_kernel_err(e));
    if (stats_host) {
        std::vector<long long> sv((size_t)n * 3);
        PULSAR_TRY(cuda_status(cudaMemcpy(sv.data(), e->stats, sv.size() * 8, cudaMemcpyDeviceToHost), "read stats"));
        stats_host[0] = stats_host[1] = stats_host[2] = 0;
        for (int i = 0; i < n; ++i)
            for (int k = 0; k < 3; ++k) stats_host[k] += sv[(size_t)i * 3 + k];
    }
    return PULSAR_OK;
}
}  // namespace

extern "C" int pulsar_engine_generate_greedy(pulsar_engine* e, int32_t n, const int32_t* slots_host,
                                             const float* first_logits, int32_t n_new, int32_t gamma, int32_t* out,
                                             int64_t* stats_host, void* stream) {
    return generate_impl(e, n, slots_host, nullptr, first_logits, n_new, gamma, false, 0.f, 1.f, 0, out, stats_host,
                         stream);
}

extern "C" int pulsar_engine_generate_sampled(pulsar_engine* e, int32_t n, const int32_t* slots_host,
                                              const int32_t* seq_ids_host, const float* first_logits, int32_t n_new,
                                              int32_t gamma, float temperature, float top_p, uint64_t seed,
                                              int32_t* out, int64_t* stats_host, void* stream) {
    // temperature <= 1e-4 is greedy decoding in the reference (src/infer.py:591, :669)
    if (temperature > 0.f && temperature <= 1e-4f && top_p > 0.f && top_p <= 1.f)
        return generate_impl(e, n, slots_host, nullptr, first_logits, n_new, gamma, false, 0.f, 1.f, 0, out,
                             stats_host, stream);
    return generate_impl(e, n, slots_host, seq_ids_host, first_logits, n_new, gamma, true, temperature, top_p, seed,
                         out, stats_host, stream);
}

extern "C" int pulsar_engine_set_early_exit(pulsar_engine* e, int32_t enabled, float threshold) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(!enabled || std::isfinite(threshold), "set_early_exit: threshold must be finite");
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    e->ee_on = enabled != 0;
    e->ee_thr = enabled ? threshold : 1.f;
    return cuda_status(cudaMemset(e->ee_counts, 0, NP * sizeof(unsigned long long)), "zero exit tallies");
}

extern "C" int pulsar_engine_set_repetition_penalty(pulsar_engine* e, float penalty) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(std::isfinite(penalty) && penalty > 0.f, "set_repetition_penalty: penalty must be finite and > 0");
    PULSAR_CHECK_ARG(penalty == 1.f || e->V <= 393216, "set_repetition_penalty: vocab_size %d above 393216", e->V);
    e->rp = penalty;
    e->rp_on = penalty != 1.f;
    return PULSAR_OK;
}

extern "C" int pulsar_engine_early_exit_counts(pulsar_engine* e, int64_t* counts_host) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(counts_host, "early_exit_counts: null argument");
    PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
    unsigned long long c[NP];
    PULSAR_TRY(cuda_status(cudaMemcpy(c, e->ee_counts, sizeof(c), cudaMemcpyDeviceToHost), "read exit tallies"));
    for (int k = 0; k < NP; ++k) counts_host[k] = (int64_t)c[k];
    return PULSAR_OK;
}

extern "C" int pulsar_engine_set_option(pulsar_engine* e, const char* name, int64_t value) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(name, "set_option: null name");
    if (strcmp(name, "megakernel") == 0) {
        if (value && (e->mega_grid < 144)) {
            set_error("set_option: the persistent pulse kernel needs >= 144 co-resident CTAs (this GPU: %d)", e->mega_grid);
            return PULSAR_ERR_UNSUPPORTED;
        }
        const bool v = value != 0;
        if (v != e->use_mega) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->use_mega = v;
        return PULSAR_OK;
    }
    if (strcmp(name, "merged_adapter") == 0) {
        // weights without a live loop adapter have nothing to merge: the option stays off
        const bool v = value != 0 && e->has_lora;
        if (v && !e->wqkv_m[0][0]) {
            PULSAR_CHECK_ARG(e->finalized, "set_option(merged_adapter): finalize the engine first");
            PULSAR_TRY(cuda_status(cudaSetDevice(e->cfg.device), "cudaSetDevice"));
            const int q = e->cfg.loop_lora_rank;   // rank per pulse (8); LORA_R is 3 x q
            const float scale = e->cfg.loop_lora_alpha / (float)q;
            for (int p = 0; p < NP; ++p)
                for (int l = 0; l < NL; ++l) {
                    PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->wqkv_m[p][l]), (size_t)QKV * D * 2, &e->arena_bytes));
                    PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->wo_m[p][l]), (size_t)D * D * 2, &e->arena_bytes));
                    k_merge_adapter<<<592, 256>>>(e->wqkv[l], e->T_(e->L(l, "attn.wqkv_adapter.lora_A")),
                                                  e->T_(e->L(l, "attn.wqkv_adapter.lora_B")),
                                                  e->T_(e->L(l, "attn.wqkv_adapter.loop_M")), e->P, p, scale, QKV, D,
                                                  q, e->wqkv_m[p][l]);
                    k_merge_adapter<<<592, 256>>>(e->wo[l], e->T_(e->L(l, "attn.wo_adapter.lora_A")),
                                                  e->T_(e->L(l, "attn.wo_adapter.lora_B")),
                                                  e->T_(e->L(l, "attn.wo_adapter.loop_M")), e->P, p, scale, D, D, q,
                                                  e->wo_m[p][l]);
                    PULSAR_LAUNCH_CHECK("k_merge_adapter");
                }
            PULSAR_TRY(cuda_status(cudaDeviceSynchronize(), "merge adapter"));
        }
        if (v != e->merge_adapter) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->merge_adapter = v;
        return PULSAR_OK;
    }
    if (strcmp(name, "tc_gemm") == 0) {
        if ((value != 0) != e->use_tc) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->use_tc = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "tc_attn") == 0) {   // prefill only (never captured in a graph)
        e->tc_attn = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "tc_dec_attn") == 0) {
        if ((value != 0) != e->tc_dec) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->tc_dec = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "tma_gemm") == 0) {
        if ((value != 0) != e->use_tma) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->use_tma = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "wide") == 0) {
        if ((value != 0) != e->force_wide) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->force_wide = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "time_pulses") == 0) {
        for (cudaEvent_t& ev : e->tev)
            if (value && !ev) PULSAR_TRY(cuda_status(cudaEventCreate(&ev), "cudaEventCreate"));
        e->time_pulses = value != 0;
        return PULSAR_OK;
    }
    if (strcmp(name, "trace") == 0) {
        if (value && !e->m_trace) {
            PULSAR_TRY(e->dmalloc(reinterpret_cast<void**>(&e->m_trace), (size_t)e->mega_grid * MEGA_TRACE * 8,
                                  &e->work_bytes));
            PULSAR_TRY(cuda_status(cudaMemset(e->m_trace, 0, (size_t)e->mega_grid * MEGA_TRACE * 8), "zero trace"));
        }
        if (!value) e->m_trace = nullptr;   // the buffer stays allocated until destroy
        for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
        e->graphs.clear();
        return PULSAR_OK;
    }
    if (strcmp(name, "wait_ns") == 0) {   // bound of every wait in the persistent kernel
        PULSAR_CHECK_ARG(value >= 100000 && value <= (int64_t)WAIT_NS, "set_option(wait_ns): %lld outside [1e5, %llu]",
                         (long long)value, (unsigned long long)WAIT_NS);
        if ((unsigned long long)value != e->mega_wait_ns) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->mega_wait_ns = (unsigned long long)value;
        return PULSAR_OK;
    }
    if (strcmp(name, "stall_cta") == 0) {   // test hook: -1 off
        PULSAR_CHECK_ARG(value >= -1 && value < e->mega_grid, "set_option(stall_cta): %lld outside [-1, %d)",
                         (long long)value, e->mega_grid);
        if (value != e->mega_stall_cta) {
            for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second.ex);
            e->graphs.clear();
        }
        e->mega_stall_cta = (int)value;
        return PULSAR_OK;
    }
    set_error("set_option: unknown option '%s'", name);
    return PULSAR_ERR_INVALID;
}

extern "C" int pulsar_engine_read_trace(pulsar_engine* e, uint64_t* host, int64_t n) {
    PULSAR_TRY(check_engine(e, false));
    if (!e->m_trace) {
        set_error("read_trace: tracing is off (set option \"trace\" to 1 first)");
        return PULSAR_ERR_STATE;
    }
    PULSAR_CHECK_ARG(host && n >= (int64_t)e->mega_grid * MEGA_TRACE, "read_trace: need %d entries",
                     e->mega_grid * MEGA_TRACE);
    return cuda_status(cudaMemcpy(host, e->m_trace, (size_t)e->mega_grid * MEGA_TRACE * 8, cudaMemcpyDeviceToHost),
                       "read trace");
}

extern "C" int pulsar_engine_get_option(pulsar_engine* e, const char* name, int64_t* value) {
    PULSAR_TRY(check_engine(e, false));
    PULSAR_CHECK_ARG(name && value, "get_option: null argument");
    if (strcmp(name, "megakernel") == 0) { *value = e->use_mega ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "megakernel_grid") == 0) { *value = e->mega_grid; return PULSAR_OK; }
    if (strcmp(name, "wait_ns") == 0) { *value = (int64_t)e->mega_wait_ns; return PULSAR_OK; }
    if (strcmp(name, "stall_cta") == 0) { *value = e->mega_stall_cta; return PULSAR_OK; }
    if (strcmp(name, "wide") == 0) { *value = e->force_wide ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "tc_gemm") == 0) { *value = e->use_tc ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "tc_attn") == 0) { *value = e->tc_attn ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "tma_gemm") == 0) { *value = e->use_tma ? 1 : 0; return PULSAR_OK; }
    // 1 when the decode attention runs on the tensor cores (bf16 cache, option on)
    if (strcmp(name, "tc_dec_attn") == 0) { *value = (e->tc_dec && e->kv_map_ok) ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "merged_adapter") == 0) { *value = e->merge_adapter ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "wide_rows") == 0) { *value = e->wide_rows; return PULSAR_OK; }
    if (strcmp(name, "loop_adapter") == 0) { *value = e->has_lora ? 1 : 0; return PULSAR_OK; }
    if (strcmp(name, "kernel_launches") == 0) { *value = e->n_kernels; return PULSAR_OK; }
    if (strcmp(name, "mega_launches") == 0) { *value = e->n_mega; return PULSAR_OK; }
    if (strcmp(name, "routed_experts") == 0) {
        unsigned long long v = 0;
        if (e->m_experts)
            PULSAR_TRY(cuda_status(cudaMemcpy(&v, e->m_experts, 8, cudaMemcpyDeviceToHost), "read expert count"));
        *value = (int64_t)v;
        return PULSAR_OK;
    }
    if (strcmp(name, "last_pulse_ns") == 0) {
        if (!e->time_pulses) {
            set_error("get_option: last_pulse_ns needs option \"time_pulses\" = 1");
            return PULSAR_ERR_STATE;
        }
        float ms = 0.f;
        PULSAR_TRY(cuda_status(cudaEventSynchronize(e->tev[1]), "cudaEventSynchronize"));
        PULSAR_TRY(cuda_status(cudaEventElapsedTime(&ms, e->tev[0], e->tev[1]), "cudaEventElapsedTime"));
        *value = (int64_t)llround((double)ms * 1e6);
        return PULSAR_OK;
    }
    set_error("get_option: unknown option '%s'", name);
    return PULSAR_ERR_INVALID;
}
