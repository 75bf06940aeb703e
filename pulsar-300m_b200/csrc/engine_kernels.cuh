// Device kernels of the Pulsar decode engine (small-row "GEMV regime" pulse pass, the
// prefill "GEMM regime" pass, LM head, argmax and the greedy accept step).
//
// Data layout in HBM (all row-major):
//   bf16 weights: wqkv [1536][1024], wo [1024][1024], shared gate_up [2048][1024],
//     shared down [1024][1024], routed gate_up transposed to [E][1024 out][1024 in]
//     (outputs 0..511 gate, 512..1023 up), routed down transposed to [E][1024 out][512 in],
//     embedding / LM head [V][1024].
//   fp32 small tensors stay in the reference layout ([max_pulses][...]).
//   Loop adapter (src/model.py:716-727) is applied unmerged and exact in fp32:
//     y = W x + Bs (A x), A = lora_A[:3] as [24][d_in], Bs[p] = [d_out][24] with the
//     loop_M[p, j] * alpha / q scale folded in.
//   KV cache per sequence slot and layer: K [HKV][cap][64] then V [HKV][cap][64] of
//     type KVT (bf16 or fp32); local layers are a ring of `cap` = 2048 slots addressed
//     by pos & 2047 (or by pos when the whole context fits), global layers by pos.
//   Activations fp32: h (residual stream), h_in, h0n, xn (normed input) [R][1024].
#pragma once

#include "common.cuh"
#include "kv.cuh"
#include "mega_ptx.cuh"

namespace pulsar {

// ------------------------------------------------------------------------------------
// Row descriptors: int4 {slot, pos, token, unused}
// ------------------------------------------------------------------------------------

// Pulse-0 input (src/infer.py:474-482): embed, anchor RMSNorm, single-token stem conv
// (x + w[:,0] * x, the reference's decode quirk), + step embedding.
__global__ void __launch_bounds__(256) k_pulse0_input(const int4* __restrict__ rows, const __nv_bfloat16* __restrict__ emb,
                                                      const float* __restrict__ anchor_w, const float* __restrict__ stem,
                                                      const float* __restrict__ step0, float eps, int use_conv,
                                                      float* __restrict__ h, float* __restrict__ h_in,
                                                      float* __restrict__ h0n, int V, int hs) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int tok = min(max(rows[r].z, 0), V - 1);   // host validates; clamp keeps reads in bounds
    const __nv_bfloat16* e = emb + (int64_t)tok * D;
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[i] = __bfloat162float(e[threadIdx.x + i * 256]);
        ss += x[i] * x[i];
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = threadIdx.x + i * 256;
        float n = anchor_w[d] * (x[i] * inv);
        if (use_conv) n = n + stem[d * 4] * n;
        const float hi = n + step0[d];
        h0n[(int64_t)r * hs * D + d] = n;
        h_in[r * D + d] = hi;
        h[r * D + d] = hi;
    }
}

// Re-injection for pulse p > 0 (src/infer.py:483-501): r = RMSNorm(h_prev);
// g = Wd[:, :D] h0n + Wd[:, D:] r (rank 8); mix = sigmoid(Wu g + b);
// h_in = lerp(r, h0n, mix) + step_emb[p]  (torch.lerp's two-sided formula).
__global__ void __launch_bounds__(256) k_reinject(int R, const float* __restrict__ h_prev, const float* __restrict__ h0n,
                                                  const float* __restrict__ psn_w, const float* __restrict__ wd,
                                                  const float* __restrict__ wu, const float* __restrict__ wb,
                                                  const float* __restrict__ step, float eps, float* __restrict__ h,
                                                  float* __restrict__ h_in, float* __restrict__ h0n_out, int hs) {
    __shared__ float red[32];
    __shared__ float g_s[RG];
    const int r = blockIdx.x;
    const float* hp = h_prev + (int64_t)r * D;
    const float* an = h0n + (int64_t)r * D;
    float x[4], a[4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[i] = hp[threadIdx.x + i * 256];
        a[i] = an[threadIdx.x + i * 256];
        ss += x[i] * x[i];
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)D + eps);
    float rn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rn[i] = psn_w[threadIdx.x + i * 256] * (x[i] * inv);
    for (int j = 0; j < RG; ++j) {
        float pe = 0.f, pr = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = threadIdx.x + i * 256;
            pe += wd[j * 2 * D + d] * a[i];
            pr += wd[j * 2 * D + D + d] * rn[i];
        }
        pe = block_sum(pe, red);
        pr = block_sum(pr, red);
        if (threadIdx.x == 0) g_s[j] = pe + pr;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = threadIdx.x + i * 256;
        float z = wb[d];
#pragma unroll
        for (int j = 0; j < RG; ++j) z += wu[d * RG + j] * g_s[j];
        const float mix = sigmoidf_(z);
        const float diff = a[i] - rn[i];
        const float lerp = (mix < 0.5f) ? rn[i] + mix * diff : a[i] - diff * (1.f - mix);
        const float hi = lerp + step[d];
        h_in[r * D + d] = hi;
        h[r * D + d] = hi;
        if (h0n_out) h0n_out[(int64_t)r * hs * D + d] = a[i];
    }
}

// RMSNorm of the residual rows with a per-pulse weight, plus the loop-adapter projection
// t = A xn (24 values) when `lora_a` is set. One block per row.
__global__ void __launch_bounds__(256) k_rmsnorm_lora(const float* __restrict__ h, const float* __restrict__ w, float eps,
                                                      float* __restrict__ xn, const float* __restrict__ lora_a,
                                                      float* __restrict__ lora_t, __nv_bfloat16* __restrict__ xh = nullptr,
                                                      __nv_bfloat16* __restrict__ xl = nullptr) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        x[i] = h[(int64_t)r * D + threadIdx.x + i * 256];
        ss += x[i] * x[i];
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = threadIdx.x + i * 256;
        x[i] = w[d] * (x[i] * inv);
        xn[(int64_t)r * D + d] = x[i];
        if (xh) split_store(xh, xl, (int64_t)r * D + d, x[i]);
    }
    if (lora_a) {
        for (int j = 0; j < LORA_R; ++j) {
            float p = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) p += lora_a[j * D + threadIdx.x + i * 256] * x[i];
            p = block_sum(p, red);
            if (threadIdx.x == 0) lora_t[r * LORA_R + j] = p;
        }
    }
}

// ------------------------------------------------------------------------------------
// GEMV regime: Y[r][o] = sum_k W[o][k] X[r][k] (+ loop adapter) for R <= 32 rows.
// One warp owns two output rows; every lane keeps its 2 x KD/256 16-byte weight chunks
// in registers and reuses them for all rows, so each weight byte is read once per pass.
// ------------------------------------------------------------------------------------
enum { EPI_STORE = 0, EPI_ADD = 1 };

template <int KD, int EPI>
__global__ void __launch_bounds__(128) k_gemv(const __nv_bfloat16* __restrict__ W, int N, const float* __restrict__ X,
                                              int R, float* __restrict__ Y, int ldy,
                                              const float* __restrict__ lora_b, const float* __restrict__ lora_t) {
    constexpr int CH = KD / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o0 = (blockIdx.x * 4 + warp) * 2;
    if (o0 >= N) return;
    float w0[CH * 8], w1[CH * 8];
    {
        uint4 u0[CH], u1[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            u0[c] = ldg_stream(W + (int64_t)o0 * KD + c * 256 + lane * 8);
            u1[c] = ldg_stream(W + (int64_t)(o0 + 1) * KD + c * 256 + lane * 8);
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            bf16x8_to_f32(u0[c], w0 + c * 8);
            bf16x8_to_f32(u1[c], w1 + c * 8);
        }
    }
    for (int rb = 0; rb < R; rb += 8) {
        float a0[8], a1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) a0[i] = a1[i] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (rb + i < R) {
                const float* xr = X + (int64_t)(rb + i) * KD + lane * 8;
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const float4 xa = __ldg(reinterpret_cast<const float4*>(xr + c * 256));
                    const float4 xb = __ldg(reinterpret_cast<const float4*>(xr + c * 256 + 4));
                    const float* p0 = w0 + c * 8;
                    const float* p1 = w1 + c * 8;
                    a0[i] += p0[0] * xa.x + p0[1] * xa.y + p0[2] * xa.z + p0[3] * xa.w + p0[4] * xb.x + p0[5] * xb.y +
                             p0[6] * xb.z + p0[7] * xb.w;
                    a1[i] += p1[0] * xa.x + p1[1] * xa.y + p1[2] * xa.z + p1[3] * xa.w + p1[4] * xb.x + p1[5] * xb.y +
                             p1[6] * xb.z + p1[7] * xb.w;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            a0[i] = warp_sum(a0[i]);
            a1[i] = warp_sum(a1[i]);
        }
        if (lane < 16) {
            const int i = lane & 7;
            const int o = o0 + (lane >> 3);
            const int r = rb + i;
            if (r < R) {
                float y = 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k == i) y = (lane >> 3) ? a1[k] : a0[k];
                if (lora_b) {
                    const float* bt = lora_b + (int64_t)o * LORA_R;
                    const float* tt = lora_t + r * LORA_R;
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < LORA_R; ++j) d += bt[j] * tt[j];
                    y += d;
                }
                if (EPI == EPI_ADD)
                    Y[(int64_t)r * ldy + o] += y;
                else
                    Y[(int64_t)r * ldy + o] = y;
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// Attention, decode: QK-RMSNorm + RoPE (+ YaRN) + value residual + KV write, then a
// split-K pass over ATT_CHUNK-key chunks and a combine that applies the head gate.
// ------------------------------------------------------------------------------------
template <typename KVT>
__global__ void __launch_bounds__((H + HKV) * 32) k_qkv_post(
    const int4* __restrict__ rows, const float* __restrict__ qkv, const float* __restrict__ qn_w,
    const float* __restrict__ kn_w, const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps,
    int vres_mode, float lv, float* __restrict__ vfirst, KVLayer L, int yarn_global, int base_seq_len,
    float* __restrict__ q_out, int max_pos, int n_slots) {
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int4 row = rows[r];
    const int pos = row.y;
    if (pos < 0 || pos >= max_pos || row.x < 0 || row.x >= n_slots) return;   // rejected row: no access
    const float* src = qkv + (int64_t)r * QKV;
    const float c = cos_t[(int64_t)pos * 32 + lane], s = sin_t[(int64_t)pos * 32 + lane];
    if (warp < H) {
        const float x1 = src[warp * DH + lane], x2 = src[warp * DH + lane + 32];
        const float inv = rsqrtf(warp_sum(x1 * x1 + x2 * x2) / (float)DH + eps);
        const float q1 = qn_w[warp * DH + lane] * (x1 * inv);
        const float q2 = qn_w[warp * DH + lane + 32] * (x2 * inv);
        float y1 = q1 * c - q2 * s, y2 = q2 * c + q1 * s;
        if (yarn_global && pos + 1 > base_seq_len) {
            // src/infer.py:288-291, scale = 1 + 0.1 ln(max(pos+1, base) / base) (fp32 multiply)
            const double b = (double)base_seq_len;
            const float sc = (float)(1.0 + 0.1 * log(fmax((double)(pos + 1), b) / b));
            y1 *= sc;
            y2 *= sc;
        }
        q_out[((int64_t)r * H + warp) * DH + lane] = y1;
        q_out[((int64_t)r * H + warp) * DH + lane + 32] = y2;
    } else {
        const int g = warp - H;
        const float k1 = src[H * DH + g * DH + lane], k2 = src[H * DH + g * DH + lane + 32];
        float v1 = src[H * DH + HKV * DH + g * DH + lane], v2 = src[H * DH + HKV * DH + g * DH + lane + 32];
        if (vres_mode == 1) {          // layer 0, pulse 0: remember v (src/infer.py:263-264)
            vfirst[((int64_t)r * HKV + g) * DH + lane] = v1;
            vfirst[((int64_t)r * HKV + g) * DH + lane + 32] = v2;
        } else if (vres_mode == 2) {   // later layers of pulse 0 (src/infer.py:265-267)
            v1 = (1.f - lv) * v1 + lv * vfirst[((int64_t)r * HKV + g) * DH + lane];
            v2 = (1.f - lv) * v2 + lv * vfirst[((int64_t)r * HKV + g) * DH + lane + 32];
        }
        const float inv = rsqrtf(warp_sum(k1 * k1 + k2 * k2) / (float)DH + eps);
        const float a1 = kn_w[g * DH + lane] * (k1 * inv);
        const float a2 = kn_w[g * DH + lane + 32] * (k2 * inv);
        KVT* kp = kv_k<KVT>(L, row.x, g, pos);
        KVT* vp = kv_v<KVT>(L, row.x, g, pos);
        if (!(rows[r].w & 1)) {   // bit 0: the row keeps its cached K/V (exited early)
            kv_store(kp + lane, a1 * c - a2 * s);
            kv_store(kp + lane + 32, a2 * c + a1 * s);
            kv_store(vp + lane, v1);
            kv_store(vp + lane + 32, v2);
        }
    }
}

// Flash-decoding attention of the per-op and many-row pulse passes. Block (split sp, kv head
// g, group of rpb rows), 256 threads. A group is cut into runs of consecutive rows of one slot
// at consecutive positions (a verify block). For each run the block walks the chunks
// sp, sp + nsplit, ... of ATT_FCK keys (keys lo_first + [c * ATT_FCK, ...), lo_first the run's
// first row's window start) with an online softmax: the chunk's cached K and V rows arrive as
// stored (bf16 or fp32) by 1-D bulk copies into a two-stage shared-memory ring, two chunks ahead
// of the compute; every row scores them under its own mask [lo_r, pos_r]. Per (row, q head)
// the split writes (m, l, o[64]) (o not yet divided by l; m = -inf when no key was visible) at
// partial index sp of a stride of nsplit, which k_attn_combine merges. Rows with an invalid
// slot or position read nothing. A bulk copy that has not landed after a 2 s wait sets *err.
constexpr int ATT_RPB_MAX = 8;
constexpr int ATT_FCK = 64;          // keys per chunk
constexpr int ATT_FTHREADS = 256;
// KT: blocks of two or more rows keep an fp32 K^T copy of the chunk (kt[dim][key]) for their
// scores, so that a warp reads one K^T row (consecutive keys) and broadcasts the queries.
// NQ: query units a block holds (its rows per block x GQA), which sizes the query and score
// arrays (a one-row block needs 4 of the 32 an eight-row block needs, and fits more blocks per SM).
template <typename KVT, bool KT = false, int NQ = ATT_RPB_MAX * GQA>
struct AttnFlashSmem {
    uint64_t full[2];
    alignas(128) KVT k[2][ATT_FCK * DH];
    alignas(128) KVT v[2][ATT_FCK * DH];
    alignas(16) float q[NQ][DH];
    alignas(16) float sc[NQ][ATT_FCK];
    float m[NQ], l[NQ], scale[NQ];
    float kt[KT ? DH : 1][ATT_FCK + 1];
};

// 16 consecutive elements of a K row as fp32 (two 16-byte loads for bf16, four for fp32).
__device__ __forceinline__ void attn_row16(const __nv_bfloat16* p, float* f) {
    bf16x8_to_f32(reinterpret_cast<const uint4*>(p)[0], f);
    bf16x8_to_f32(reinterpret_cast<const uint4*>(p)[1], f + 8);
}
__device__ __forceinline__ void attn_row16(const float* p, float* f) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 v = reinterpret_cast<const float4*>(p)[i];
        f[4 * i] = v.x;
        f[4 * i + 1] = v.y;
        f[4 * i + 2] = v.z;
        f[4 * i + 3] = v.w;
    }
}

// Issue the bulk copies of chunk [k0, k0 + nk) of (slot, head g) into ring stage st (one thread).
template <typename KVT, bool KT, int NQ>
__device__ __forceinline__ void attn_issue(AttnFlashSmem<KVT, KT, NQ>* s, int st, const KVLayer& L, int slot, int g, int k0,
                                           int nk) {
    constexpr uint32_t ROW = DH * sizeof(KVT);
    mbar_arrive_expect_tx(&s->full[st], 2u * nk * ROW);
    const int i0 = k0 & L.mask;
    const int m1 = (L.mask >= 0 && i0 + nk > L.cap) ? L.cap - i0 : nk;   // a run wrapping around the ring
    for (int isv = 0; isv < 2; ++isv) {
        KVT* dst = isv ? s->v[st] : s->k[st];
        const KVT* p0 = isv ? kv_v<KVT>(L, slot, g, k0) : kv_k<KVT>(L, slot, g, k0);
        tma_load_1d(dst, p0, (uint32_t)m1 * ROW, &s->full[st]);
        if (m1 < nk) {
            const KVT* p1 = isv ? kv_v<KVT>(L, slot, g, k0 + m1) : kv_k<KVT>(L, slot, g, k0 + m1);
            tma_load_1d(reinterpret_cast<unsigned char*>(dst) + m1 * ROW, p1, (uint32_t)(nk - m1) * ROW, &s->full[st]);
        }
    }
}

__device__ __forceinline__ float2 attn_pair(const __nv_bfloat16* row, int w) {
    return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row)[w]);
}
__device__ __forceinline__ float2 attn_pair(const float* row, int w) { return reinterpret_cast<const float2*>(row)[w]; }
__device__ __forceinline__ float attn_elem(const __nv_bfloat16* row, int d) { return __bfloat162float(row[d]); }
__device__ __forceinline__ float attn_elem(const float* row, int d) { return row[d]; }

// NU: query units (rows x GQA heads) per thread group of four = the launch's rows per block
// (rpb <= NU <= ATT_RPB_MAX), a compile-time bound so that a one-row pass does not issue the
// instructions of eight.
template <typename KVT, int NU>
__global__ void __launch_bounds__(ATT_FTHREADS) k_attn_flash(const int4* __restrict__ rows, int R, int rpb,
                                                             const float* __restrict__ q, KVLayer L, int is_local,
                                                             int nsplit, float* __restrict__ part, int max_pos,
                                                             int n_slots, int* err) {
    constexpr bool KT = NU >= 2;
    extern __shared__ __align__(128) unsigned char att_raw[];
    auto* s = reinterpret_cast<AttnFlashSmem<KVT, KT, NU * GQA>*>(att_raw);
    const int sp = blockIdx.x, g = blockIdx.y;
    const int rb0 = blockIdx.z * rpb, rb1 = min(R, rb0 + rpb);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int key = tid & (ATT_FCK - 1), grp = tid >> 6;   // scores / P.V: key or dimension, unit group
    auto bad_row = [&](const int4& rw) { return rw.y < 0 || rw.y >= max_pos || rw.x < 0 || rw.x >= n_slots; };
    if (tid == 0) {
        mbar_init(&s->full[0], 1);
        mbar_init(&s->full[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    uint32_t uses[2] = {0u, 0u};   // completed phases of each stage's barrier
    for (int s0 = rb0; s0 < rb1;) {
        const int4 first = rows[s0];
        int s1 = s0 + 1;
        if (!bad_row(first))
            while (s1 < rb1 && s1 - s0 < ATT_RPB_MAX) {
                const int4 nx = rows[s1];
                if (bad_row(nx) || nx.x != first.x || nx.y != rows[s1 - 1].y + 1) break;
                ++s1;
            }
        const int nr = s1 - s0, nq = nr * GQA;
        const int posF = first.y, posL = posF + nr - 1;
        const int lo0 = is_local ? max(0, posF - WINDOW + 1) : 0;
        const int nchunks = bad_row(first) ? 0 : (posL - lo0 + ATT_FCK) / ATT_FCK;
        const int mine = nchunks > sp ? (nchunks - sp + nsplit - 1) / nsplit : 0;   // chunks of this split
        // queries of the run (fp32, already normed and rotated), the online-softmax state
        for (int i = tid; i < nq * DH; i += ATT_FTHREADS)
            s->q[i / DH][i % DH] = q[((int64_t)(s0 + i / (GQA * DH)) * H + g * GQA) * DH + i % (GQA * DH)] * 0.125f;
        if (tid < nq) {
            s->m[tid] = -INFINITY;
            s->l[tid] = 0.f;
        }
        auto chunk_k0 = [&](int i) { return lo0 + (sp + i * nsplit) * ATT_FCK; };
        auto chunk_nk = [&](int i) { return min(chunk_k0(i) + ATT_FCK, posL + 1) - chunk_k0(i); };
        if (tid == 0)
            for (int i = 0; i < 2 && i < mine; ++i) attn_issue<KVT, KT, NU * GQA>(s, i, L, first.x, g, chunk_k0(i), chunk_nk(i));
        // P.V accumulators of dimension `key`: one-row blocks, every unit over key quarter grp;
        // wider blocks, units grp, grp + 4, ... over all keys
        constexpr int NQ = NU * GQA;
        constexpr int NO = NU == 1 ? NQ : NU;
        float o[NO];
#pragma unroll
        for (int j = 0; j < NO; ++j) o[j] = 0.f;
        __syncthreads();
        for (int i = 0; i < mine; ++i) {
            const int st = i & 1;
            const int k0 = chunk_k0(i), nk = chunk_nk(i);
            // a copy that has not landed after the bounded wait ends the block (uniformly), after
            // a second bounded wait for the copies still in flight into either stage
            if (__syncthreads_or(!mbar_wait(&s->full[st], uses[st] & 1))) {
                if (tid == 0) {
                    atomicExch(err, 1);
                    mbar_wait(&s->full[st], uses[st] & 1);
                    if (i + 1 < mine) mbar_wait(&s->full[st ^ 1], uses[st ^ 1] & 1);
                }
                __syncthreads();
                return;
            }
            ++uses[st];
            const KVT* Kt = s->k[st];
            const KVT* Vt = s->v[st];
            // scores: thread (key, unit group). Blocks of one row read the key's row in rotated
            // pair order (pair (j + lane) mod 32 at step j: one bank per lane of the warp); blocks
            // of several rows first transpose the chunk to fp32 K^T (thread: key t / 4, dims
            // 16 (t % 4) ..), then read K^T rows by key and broadcast each unit's query.
            if constexpr (KT) {
                const int tk = tid >> 2, tq = tid & 3;
                if (tk < nk) {
                    float f[16];
                    attn_row16(Kt + tk * DH + 16 * tq, f);
#pragma unroll
                    for (int j = 0; j < 16; ++j) s->kt[16 * tq + j][tk] = f[j];
                }
                __syncthreads();
            }
            {
                const int kk = key, kpos = k0 + kk;
                float acc[NU];
#pragma unroll
                for (int j = 0; j < NU; ++j) acc[j] = 0.f;
                if (KT && kk < nk) {
#pragma unroll 4
                    for (int d = 0; d < DH; d += 4) {
                        const float c0 = s->kt[d][kk], c1 = s->kt[d + 1][kk], c2 = s->kt[d + 2][kk],
                                    c3 = s->kt[d + 3][kk];
#pragma unroll
                        for (int uu = 0; uu < NU; ++uu) {
                            const int u = grp + 4 * uu;
                            if (u < nq) {
                                const float4 qv = *reinterpret_cast<const float4*>(&s->q[u][d]);
                                acc[uu] += qv.x * c0 + qv.y * c1 + qv.z * c2 + qv.w * c3;
                            }
                        }
                    }
                } else if (kk < nk) {
                    const KVT* kr = Kt + kk * DH;
#pragma unroll 4
                    for (int j = 0; j < DH / 2; ++j) {
                        const int w = (j + lane) & (DH / 2 - 1);
                        const float2 kv = attn_pair(kr, w);
#pragma unroll
                        for (int uu = 0; uu < NU; ++uu) {
                            const int u = grp + 4 * uu;
                            if (u < nq) {
                                const float2 qv = reinterpret_cast<const float2*>(s->q[u])[w];
                                acc[uu] += qv.x * kv.x + qv.y * kv.y;
                            }
                        }
                    }
                }
#pragma unroll
                for (int uu = 0; uu < NU; ++uu) {
                    const int u = grp + 4 * uu;
                    if (u < nq) {
                        const int pos = posF + u / GQA;
                        const int lor = is_local ? max(0, pos - WINDOW + 1) : 0;
                        const bool vis = kk < nk && kpos <= pos && kpos >= lor;
                        s->sc[u][kk] = vis ? acc[uu] : -INFINITY;
                    }
                }
            }
            __syncthreads();
            // online softmax: a warp per unit; weights back into sc, the rescale of the old state
            for (int u = warp; u < nq; u += ATT_FTHREADS / 32) {
                const float a0 = s->sc[u][lane], a1 = s->sc[u][lane + 32];
                const float mo = s->m[u];
                const float mn = fmaxf(mo, warp_max(fmaxf(a0, a1)));
                const float e0 = (a0 == -INFINITY) ? 0.f : expf(a0 - mn);
                const float e1 = (a1 == -INFINITY) ? 0.f : expf(a1 - mn);
                const float sum = warp_sum(e0 + e1);
                s->sc[u][lane] = e0;
                s->sc[u][lane + 32] = e1;
                __syncwarp();
                if (lane == 0) {
                    const float scl = (mo == -INFINITY) ? 0.f : expf(mo - mn);
                    s->scale[u] = scl;
                    s->l[u] = s->l[u] * scl + sum;
                    s->m[u] = mn;
                }
            }
            __syncthreads();
            // P.V. One-row blocks: thread (dimension `key`, key quarter grp), every unit of the
            // block for its dimension over keys [16 grp, 16 grp + 16) of the chunk, each V element
            // read once for all units, the weights as float4 broadcasts (a warp shares its quarter).
            // Wider blocks: thread (dimension `key`, unit group grp), keys in order, each V element
            // read once for the group's units, the weights four keys at a time.
            if constexpr (NU == 1) {
#pragma unroll
                for (int u = 0; u < NO; ++u)
                    if (u < nq) o[u] *= s->scale[u];
                const int ke = min(16 * grp + 16, nk);
                int kk = 16 * grp;
                for (; kk + 4 <= ke; kk += 4) {
                    const float v0 = attn_elem(Vt + kk * DH, key), v1 = attn_elem(Vt + (kk + 1) * DH, key);
                    const float v2 = attn_elem(Vt + (kk + 2) * DH, key), v3 = attn_elem(Vt + (kk + 3) * DH, key);
#pragma unroll
                    for (int u = 0; u < NQ; ++u) {
                        if (u < nq) {
                            const float4 pw = *reinterpret_cast<const float4*>(&s->sc[u][kk]);
                            o[u] += pw.x * v0 + pw.y * v1 + pw.z * v2 + pw.w * v3;
                        }
                    }
                }
                for (; kk < ke; ++kk) {
                    const float v = attn_elem(Vt + kk * DH, key);
#pragma unroll
                    for (int u = 0; u < NQ; ++u)
                        if (u < nq) o[u] += s->sc[u][kk] * v;
                }
            } else {
                const int nu = (nq - grp + 3) / 4;   // units of this group
#pragma unroll
                for (int uu = 0; uu < NU; ++uu)
                    if (uu < nu) o[uu] *= s->scale[grp + 4 * uu];
                int kk = 0;
                for (; kk + 4 <= nk; kk += 4) {
                    const float v0 = attn_elem(Vt + kk * DH, key), v1 = attn_elem(Vt + (kk + 1) * DH, key);
                    const float v2 = attn_elem(Vt + (kk + 2) * DH, key), v3 = attn_elem(Vt + (kk + 3) * DH, key);
#pragma unroll
                    for (int uu = 0; uu < NU; ++uu) {
                        if (uu < nu) {
                            const float4 pw = *reinterpret_cast<const float4*>(&s->sc[grp + 4 * uu][kk]);
                            o[uu] += pw.x * v0 + pw.y * v1 + pw.z * v2 + pw.w * v3;
                        }
                    }
                }
                for (; kk < nk; ++kk) {
                    const float v = attn_elem(Vt + kk * DH, key);
#pragma unroll
                    for (int uu = 0; uu < NU; ++uu)
                        if (uu < nu) o[uu] += s->sc[grp + 4 * uu][kk] * v;
                }
            }
            __syncthreads();   // stage st is free again
            if (tid == 0 && i + 2 < mine) attn_issue<KVT, KT, NU * GQA>(s, st, L, first.x, g, chunk_k0(i + 2), chunk_nk(i + 2));
        }
        // one-row blocks: the four key quarters' sums, (q0 + q2) + (q1 + q3), through the query
        // and score arrays (free now: red[2][NQ][64]); then the partial (m, l, o) of every unit
        // at index sp
        if constexpr (NU == 1) {
            float* red = &s->q[0][0];
            if (grp >= 2) {
#pragma unroll
                for (int u = 0; u < NQ; ++u)
                    if (u < nq) red[((grp - 2) * NQ + u) * DH + key] = o[u];
            }
            __syncthreads();
            if (grp < 2) {
#pragma unroll
                for (int u = 0; u < NQ; ++u)
                    if (u < nq) o[u] += red[(grp * NQ + u) * DH + key];
            }
            __syncthreads();
            if (grp == 1) {
#pragma unroll
                for (int u = 0; u < NQ; ++u)
                    if (u < nq) red[u * DH + key] = o[u];
            }
            __syncthreads();
            if (grp == 0) {
#pragma unroll
                for (int u = 0; u < NQ; ++u) {
                    if (u < nq) {
                        float* out = part + (((int64_t)(s0 + u / GQA) * H + g * GQA + u % GQA) * nsplit + sp) * PART;
                        out[2 + key] = o[u] + red[u * DH + key];
                        if (key == 0) {
                            out[0] = s->m[u];
                            out[1] = s->m[u] == -INFINITY ? 0.f : s->l[u];
                        }
                    }
                }
            }
        } else {
#pragma unroll
            for (int uu = 0; uu < NU; ++uu) {
                const int u = grp + 4 * uu;
                if (u < nq) {
                    float* out = part + (((int64_t)(s0 + u / GQA) * H + g * GQA + u % GQA) * nsplit + sp) * PART;
                    out[2 + key] = o[uu];
                    if (key == 0) {
                        out[0] = s->m[u];
                        out[1] = s->m[u] == -INFINITY ? 0.f : s->l[u];
                    }
                }
            }
        }
        __syncthreads();   // shared memory is reused by the next run
        s0 = s1;
    }
}

template <typename KVT, int NU = 1>
constexpr size_t attn_flash_smem() {
    return sizeof(AttnFlashSmem<KVT, (NU >= 2), NU * GQA>) + 128;
}

// Splits of a flash-decoding launch: enough blocks to fill the GPU (about 6 per SM) when a pass
// has few row groups, never more than the chunks (of `chunk` keys, one more for an unaligned
// start) of the longest span nor than `cap` (the partial stride the buffers hold).
inline int attn_splits(int groups, int max_span, int sms, int cap, int chunk = ATT_FCK) {
    const int base = HKV * groups;
    int n = (6 * sms + base - 1) / base;
    const int chunks = (max_span + chunk - 1) / chunk + 1;
    if (n > chunks) n = chunks;
    if (n > cap) n = cap;
    return n < 1 ? 1 : n;
}

// Combine the split partials of each head, apply the head gate sigmoid(xn . Wg[h] + bg[h])
// (src/infer.py:302-306) and, if the loop adapter is on, project t = A_wo . out.
__global__ void __launch_bounds__(H * 32) k_attn_combine(const float* __restrict__ part, int nchunk,
                                                         const float* __restrict__ xn, const float* __restrict__ gw,
                                                         const float* __restrict__ gb, float* __restrict__ att,
                                                         const float* __restrict__ lora_a, float* __restrict__ lora_t,
                                                         __nv_bfloat16* __restrict__ ah = nullptr,
                                                         __nv_bfloat16* __restrict__ al = nullptr) {
    __shared__ float outs[H * DH];
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* pp = part + ((int64_t)r * H + h) * nchunk * PART;
    float M = -INFINITY;
    for (int c = 0; c < nchunk; ++c) M = fmaxf(M, pp[c * PART]);
    float L = 0.f, o1 = 0.f, o2 = 0.f;
    for (int c = 0; c < nchunk; ++c) {
        const float m = pp[c * PART];
        if (m == -INFINITY) continue;
        const float w = expf(m - M);
        L += w * pp[c * PART + 1];
        o1 += w * pp[c * PART + 2 + lane];
        o2 += w * pp[c * PART + 2 + lane + 32];
    }
    // gate logit for head h
    float z = 0.f;
    const float* xr = xn + (int64_t)r * D;
    for (int k = lane; k < D; k += 32) z += gw[h * D + k] * xr[k];
    z = warp_sum(z) + gb[h];
    const float g = sigmoidf_(z);
    const float inv = 1.f / L;
    const float y1 = (o1 * inv) * g, y2 = (o2 * inv) * g;
    att[(int64_t)r * D + h * DH + lane] = y1;
    att[(int64_t)r * D + h * DH + lane + 32] = y2;
    if (ah) {
        split_store(ah, al, (int64_t)r * D + h * DH + lane, y1);
        split_store(ah, al, (int64_t)r * D + h * DH + lane + 32, y2);
    }
    outs[h * DH + lane] = y1;
    outs[h * DH + lane + 32] = y2;
    if (lora_a) {
        __syncthreads();
        for (int j = 0; j < LORA_R; ++j) {
            float p = 0.f;
            for (int k = threadIdx.x; k < D; k += H * 32) p += lora_a[j * D + k] * outs[k];
            p = block_sum(p, red);
            if (threadIdx.x == 0) lora_t[r * LORA_R + j] = p;
        }
    }
}

// ------------------------------------------------------------------------------------
// MoE decode (src/infer.py:316-351)
// ------------------------------------------------------------------------------------

// Router: fp32 logits (16 x 1024), centre, sigmoid, top-4 of s + bias (ties to the lower
// expert), weights s_k / (sum + 1e-6). Slots sorted by descending biased score, which is
// the order torch.topk returns and the order the routed sum is accumulated in.
__global__ void __launch_bounds__(E * 32) k_router(const float* __restrict__ xn, const float* __restrict__ rw,
                                                   const float* __restrict__ bias, int* __restrict__ idx,
                                                   float* __restrict__ wts) {
    __shared__ float lg[E];
    const int r = blockIdx.x;
    const int e = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* xr = xn + (int64_t)r * D;
    float z = 0.f;
    for (int k = lane; k < D; k += 32) z += rw[e * D + k] * xr[k];
    z = warp_sum(z);
    if (lane == 0) lg[e] = z;
    __syncthreads();
    if (e == 0) {
        const float l = (lane < E) ? lg[lane] : 0.f;
        const float mean = warp_sum(l) / (float)E;
        const float s = sigmoidf_(l - mean);
        float b = (lane < E) ? s + bias[lane] : -INFINITY;
        float sum = 0.f;
        float sel_s[TOPK];
        int sel_i[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            ArgMax a{b, lane < E ? lane : 1 << 30};
            a = warp_argmax(a);
            sel_i[k] = a.i;
            sel_s[k] = __shfl_sync(0xffffffffu, s, a.i & 31);
            if (lane == a.i) b = -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < TOPK; ++k) sum += sel_s[k];
        sum += 1e-6f;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < TOPK; ++k) {
                idx[r * TOPK + k] = sel_i[k];
                wts[r * TOPK + k] = sel_s[k] / sum;
            }
        }
    }
}

// Expert up-projections with the SwiGLU epilogue (src/model.py:930-935 in fp32).
// Blocks [0, DS/4): shared expert, one (gate, up) output pair per warp, all R rows.
// Blocks [DS/4, ...): routed, item = (row r, slot k, output j), W = routed_gate_up[e].
__global__ void __launch_bounds__(128) k_moe_up(int R, const float* __restrict__ xn, const __nv_bfloat16* __restrict__ sh_gu,
                                                const __nv_bfloat16* __restrict__ r_gu, const int* __restrict__ idx,
                                                float* __restrict__ act_sh, float* __restrict__ act_r) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + warp;
    const __nv_bfloat16 *wg, *wu;
    int r0, r1, j;
    float* dst;
    int dst_stride;
    if (item < DS) {
        j = item;
        wg = sh_gu + (int64_t)j * D;
        wu = sh_gu + (int64_t)(DS + j) * D;
        r0 = 0;
        r1 = R;
        dst = act_sh + j;
        dst_stride = DS;
    } else {
        const int it = item - DS;
        const int rk = it / DE;
        j = it % DE;
        if (rk >= R * TOPK) return;
        const int e = idx[rk];
        const __nv_bfloat16* we = r_gu + (int64_t)e * (2 * DE) * D;
        wg = we + (int64_t)j * D;
        wu = we + (int64_t)(DE + j) * D;
        r0 = rk / TOPK;
        r1 = r0 + 1;
        dst = act_r + (int64_t)rk * DE + j - (int64_t)r0 * TOPK * DE;  // row stride TOPK*DE below
        dst_stride = TOPK * DE;
    }
    float fg[32], fu[32];
    {
        uint4 ug[4], uu[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            ug[c] = ldg_stream(wg + c * 256 + lane * 8);
            uu[c] = ldg_stream(wu + c * 256 + lane * 8);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            bf16x8_to_f32(ug[c], fg + c * 8);
            bf16x8_to_f32(uu[c], fu + c * 8);
        }
    }
    for (int r = r0; r < r1; ++r) {
        const float* xr = xn + (int64_t)r * D + lane * 8;
        float ag = 0.f, au = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4 xa = __ldg(reinterpret_cast<const float4*>(xr + c * 256));
            const float4 xb = __ldg(reinterpret_cast<const float4*>(xr + c * 256 + 4));
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                ag += fg[c * 8 + i] * xv[i];
                au += fu[c * 8 + i] * xv[i];
            }
        }
        ag = warp_sum(ag);
        au = warp_sum(au);
        if (lane == 0) dst[(int64_t)r * dst_stride] = siluf_(ag) * au;
    }
}

// Expert down-projections + combine + residual (src/infer.py:336-351):
// h[r][o] += sh_dn[o] . act_sh[r] + rscale[o] * sum_k w_rk * (r_dn[e_rk][o] . act_r[r][k]).
__global__ void __launch_bounds__(128) k_moe_down(int R, const float* __restrict__ act_sh, const float* __restrict__ act_r,
                                                  const __nv_bfloat16* __restrict__ sh_dn,
                                                  const __nv_bfloat16* __restrict__ r_dn, const int* __restrict__ idx,
                                                  const float* __restrict__ wts, const float* __restrict__ rscale,
                                                  float* __restrict__ h) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o = blockIdx.x * 4 + warp;
    if (o >= D) return;
    float ws[32];
    {
        uint4 u[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) u[c] = ldg_stream(sh_dn + (int64_t)o * DS + c * 256 + lane * 8);
#pragma unroll
        for (int c = 0; c < 4; ++c) bf16x8_to_f32(u[c], ws + c * 8);
    }
    const float rs = rscale[o];
    for (int r = 0; r < R; ++r) {
        uint4 ur[TOPK][2];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            const int e = idx[r * TOPK + k];
            const __nv_bfloat16* wr = r_dn + ((int64_t)e * D + o) * DE;
            ur[k][0] = ldg_stream(wr + lane * 8);
            ur[k][1] = ldg_stream(wr + 256 + lane * 8);
        }
        const float* xs = act_sh + (int64_t)r * DS + lane * 8;
        float sh = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float4 xa = __ldg(reinterpret_cast<const float4*>(xs + c * 256));
            const float4 xb = __ldg(reinterpret_cast<const float4*>(xs + c * 256 + 4));
            sh += ws[c * 8 + 0] * xa.x + ws[c * 8 + 1] * xa.y + ws[c * 8 + 2] * xa.z + ws[c * 8 + 3] * xa.w +
                  ws[c * 8 + 4] * xb.x + ws[c * 8 + 5] * xb.y + ws[c * 8 + 6] * xb.z + ws[c * 8 + 7] * xb.w;
        }
        float ex[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            const float* xa_p = act_r + ((int64_t)r * TOPK + k) * DE + lane * 8;
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float wf[8];
                bf16x8_to_f32(ur[k][c], wf);
                const float4 xa = __ldg(reinterpret_cast<const float4*>(xa_p + c * 256));
                const float4 xb = __ldg(reinterpret_cast<const float4*>(xa_p + c * 256 + 4));
                acc += wf[0] * xa.x + wf[1] * xa.y + wf[2] * xa.z + wf[3] * xa.w + wf[4] * xb.x + wf[5] * xb.y +
                       wf[6] * xb.z + wf[7] * xb.w;
            }
            ex[k] = acc;
        }
        sh = warp_sum(sh);
        float routed = 0.f;
#pragma unroll
        for (int k = 0; k < TOPK; ++k) routed = routed + warp_sum(ex[k]) * wts[r * TOPK + k];
        if (lane == 0) h[(int64_t)r * D + o] += sh + routed * rs;
    }
}

// End of pulse (src/infer.py:516-519): h_out = h_in + (h - h_in) * res_scale[p];
// hn = final RMSNorm(h_out) for the LM head.
__global__ void __launch_bounds__(256) k_pulse_end(const float* __restrict__ h, const float* __restrict__ h_in,
                                                   const float* __restrict__ res_scale, const float* __restrict__ fnorm,
                                                   float eps, float* __restrict__ h_out, float* __restrict__ hn, int hs,
                                                   __nv_bfloat16* __restrict__ hnh = nullptr,
                                                   __nv_bfloat16* __restrict__ hnl = nullptr) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    float y[4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = threadIdx.x + i * 256;
        const float hi = h_in[(int64_t)r * D + d];
        y[i] = hi + (h[(int64_t)r * D + d] - hi) * res_scale[d];
        h_out[(int64_t)r * hs * D + d] = y[i];
        ss += y[i] * y[i];
    }
    if (!hn) return;
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = threadIdx.x + i * 256;
        hn[(int64_t)r * D + d] = fnorm[d] * (y[i] * inv);
        if (hnh) split_store(hnh, hnl, (int64_t)r * D + d, hn[(int64_t)r * D + d]);
    }
}

// LM head (tied embedding) over R <= 8 rows: logits[r][v] = softcap(emb[v] . hn[r]), and
// per-block argmax partials (ties to the lowest vocabulary index).
constexpr int LM_ROWS_PER_BLOCK = 64;
__global__ void __launch_bounds__(128) k_lmhead(const __nv_bfloat16* __restrict__ emb, int V, const float* __restrict__ hn,
                                                int R, float softcap, float* __restrict__ logits, int ld_logits,
                                                float* __restrict__ pmax, int* __restrict__ pidx) {
    __shared__ float bv[4][8];
    __shared__ int bi[4][8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    ArgMax best[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) best[i] = ArgMax{-INFINITY, 1 << 30};
    for (int it = 0; it < LM_ROWS_PER_BLOCK / 8; ++it) {
        const int v0 = blockIdx.x * LM_ROWS_PER_BLOCK + it * 8 + warp * 2;
        float w0[32], w1[32];
        {
            uint4 u0[4], u1[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                u0[c] = ldg_stream(emb + (int64_t)v0 * D + c * 256 + lane * 8);
                u1[c] = ldg_stream(emb + (int64_t)(v0 + 1) * D + c * 256 + lane * 8);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                bf16x8_to_f32(u0[c], w0 + c * 8);
                bf16x8_to_f32(u1[c], w1 + c * 8);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < R) {
                const float* xr = hn + (int64_t)i * D + lane * 8;
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 xa = __ldg(reinterpret_cast<const float4*>(xr + c * 256));
                    const float4 xb = __ldg(reinterpret_cast<const float4*>(xr + c * 256 + 4));
                    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        a0 += w0[c * 8 + k] * xv[k];
                        a1 += w1[c * 8 + k] * xv[k];
                    }
                }
                a0 = warp_sum(a0);
                a1 = warp_sum(a1);
                if (softcap > 0.f) {
                    a0 = softcap * tanhf(a0 / softcap);
                    a1 = softcap * tanhf(a1 / softcap);
                }
                if (lane == 0 && logits) {
                    logits[(int64_t)i * ld_logits + v0] = a0;
                    logits[(int64_t)i * ld_logits + v0 + 1] = a1;
                }
                best[i] = argmax_merge(best[i], ArgMax{a0, v0});
                best[i] = argmax_merge(best[i], ArgMax{a1, v0 + 1});
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            bv[warp][i] = best[i].v;
            bi[warp][i] = best[i].i;
        }
    }
    __syncthreads();
    if (threadIdx.x < 8 && threadIdx.x < R) {
        const int i = threadIdx.x;
        ArgMax b{bv[0][i], bi[0][i]};
        for (int w = 1; w < 4; ++w) b = argmax_merge(b, ArgMax{bv[w][i], bi[w][i]});
        pmax[(int64_t)i * gridDim.x + blockIdx.x] = b.v;
        pidx[(int64_t)i * gridDim.x + blockIdx.x] = b.i;
    }
}

// Final argmax over the LM-head block partials: one warp per row.
__global__ void k_argmax_final(const float* __restrict__ pmax, const int* __restrict__ pidx, int nblk, int R,
                               int* __restrict__ out) {
    const int r = blockIdx.x;
    const int lane = threadIdx.x;
    ArgMax b{-INFINITY, 1 << 30};
    for (int i = lane; i < nblk; i += 32) b = argmax_merge(b, ArgMax{pmax[(int64_t)r * nblk + i], pidx[(int64_t)r * nblk + i]});
    b = warp_argmax(b);
    if (lane == 0) out[r] = b.i;
}

// Argmax of a dense logits row (prefill logits), ties to the lowest index.
__global__ void k_argmax_rows(const float* __restrict__ logits, int V, int ld, int* __restrict__ out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int r = blockIdx.x;
    ArgMax b{-INFINITY, 1 << 30};
    for (int i = threadIdx.x; i < V; i += blockDim.x) b = argmax_merge(b, ArgMax{logits[(int64_t)r * ld + i], i});
    b = warp_argmax(b);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { bv[w] = b.v; bi[w] = b.i; }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        ArgMax c = threadIdx.x < nw ? ArgMax{bv[threadIdx.x], bi[threadIdx.x]} : ArgMax{-INFINITY, 1 << 30};
        c = warp_argmax(c);
        if (threadIdx.x == 0) out[r] = c.i;
    }
}

}  // namespace pulsar
