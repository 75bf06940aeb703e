// Prefill kernels (src/infer.py:353-461): many rows per pass.
//
// GEMM: C[m][n] = sum_k A[m][k] W[n][k] with fp32 activations and bf16 weights, fp32
// accumulation, 64x64 tiles. Optional row gather (routed experts), per-expert batches
// (blockIdx.z), loop-adapter epilogue, SwiGLU epilogue and residual-add epilogue.
#pragma once

#include "engine_kernels.cuh"

namespace pulsar {

constexpr int GB_M = 64, GB_N = 64, GB_K = 32;

enum { GEPI_STORE = 0, GEPI_ADD = 1, GEPI_SWIGLU = 2 };

struct GemmArgs {
    const float* A;          // [*, K] rows (gathered by a_rows when set)
    int lda;
    int64_t a_stride;        // elements between batches of A (ungathered batched GEMMs)
    const int* a_rows;       // [batch][cap] row indices into A, or null
    const int* m_count;      // [batch] valid rows per batch, or null (use M)
    int M;                   // rows (per batch capacity when batched)
    const __nv_bfloat16* W;  // [N][K] (+ batch * w_stride)
    int64_t w_stride;
    int N, K;                // N = output columns (for SWIGLU: 2*d, output has d)
    float* C;                // [M][ldc] (+ batch * c_stride)
    int ldc;
    int64_t c_stride;
    const float* lora_b;     // [N][24] or null
    const float* lora_t;     // [M][24]
    float softcap;           // STORE epilogue: y = softcap * tanh(y / softcap) when > 0
    // tensor-core GEMMs: A already split into bf16 hi / lo ([batch * M][K] rows, lda == K, no
    // gather), or null (the GEMM splits it)
    const __nv_bfloat16* a_hi;
    const __nv_bfloat16* a_lo;
    // tensor-core SWIGLU epilogue: also the bf16 hi / lo split of its output, laid out like C
    // (the operand of the GEMM that reads C), or null
    __nv_bfloat16* c_hi;
    __nv_bfloat16* c_lo;
};

template <int EPI>
__global__ void __launch_bounds__(256) k_gemm(GemmArgs g) {
    __shared__ float As[GB_K][GB_M + 4];
    __shared__ float Ws[GB_K][GB_N + 4];
    const int b = blockIdx.z;
    const int m_valid = g.m_count ? g.m_count[b] : g.M;
    const int m0 = blockIdx.y * GB_M;
    if (m0 >= m_valid) return;
    const int n_tile = blockIdx.x;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const __nv_bfloat16* W = g.W + (int64_t)b * g.w_stride;
    // weight rows of this tile: plain -> n_tile*64 + c; SWIGLU -> 32 gate + 32 up rows
    const int half = g.N / 2;
    auto wrow = [&](int c) -> int {
        if (EPI == GEPI_SWIGLU) return (c < 32) ? n_tile * 32 + c : half + n_tile * 32 + (c - 32);
        return n_tile * GB_N + c;
    };
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    // loaders: A tile 64 x 32 fp32 (each thread 8 floats), W tile 64 x 32 bf16 (each thread 8)
    const int la_r = tid >> 2, la_k = (tid & 3) * 8;
    const int lw_r = tid >> 2, lw_k = (tid & 3) * 8;
    int arow = -1;
    {
        const int m = m0 + la_r;
        if (m < m_valid) arow = g.a_rows ? g.a_rows[(int64_t)b * g.M + m] : m;
    }
    const float* Ab = g.A + (g.a_rows ? 0 : (int64_t)b * g.a_stride);
    const int wr = wrow(lw_r);
    const bool wr_ok = wr < g.N;
    for (int k0 = 0; k0 < g.K; k0 += GB_K) {
        float av[8];
        if (arow >= 0) {
            const float4 x0 = *reinterpret_cast<const float4*>(Ab + (int64_t)arow * g.lda + k0 + la_k);
            const float4 x1 = *reinterpret_cast<const float4*>(Ab + (int64_t)arow * g.lda + k0 + la_k + 4);
            av[0] = x0.x; av[1] = x0.y; av[2] = x0.z; av[3] = x0.w;
            av[4] = x1.x; av[5] = x1.y; av[6] = x1.z; av[7] = x1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) av[i] = 0.f;
        }
        float wv[8];
        if (wr_ok) {
            const uint4 u = *reinterpret_cast<const uint4*>(W + (int64_t)wr * g.K + k0 + lw_k);
            bf16x8_to_f32(u, wv);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[i] = 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            As[la_k + i][la_r] = av[i];
            Ws[lw_k + i][lw_r] = wv[i];
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < GB_K; ++kk) {
            const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 w4 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
            const float a[4] = {a4.x, a4.y, a4.z, a4.w};
            const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * w[j];
        }
    }
    float* C = g.C + (int64_t)b * g.c_stride;
    if (EPI == GEPI_SWIGLU) {
        __syncthreads();
        float(*Cs)[GB_N + 4] = reinterpret_cast<float(*)[GB_N + 4]>(&As[0][0]);  // reuse: 64 x 68 > 32 x 68
        // As is only 32 x 68 floats; stage in two halves of 32 rows
        for (int hh = 0; hh < 2; ++hh) {
            __syncthreads();
            if ((ty >> 3) == hh) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) Cs[(ty & 7) * 4 + i][tx * 4 + j] = acc[i][j];
            }
            __syncthreads();
            for (int e = tid; e < 32 * 32; e += 256) {
                const int rr = e >> 5, cc = e & 31;
                const int m = m0 + hh * 32 + rr;
                const int n = n_tile * 32 + cc;
                if (m < m_valid && n < half) C[(int64_t)m * g.ldc + n] = siluf_(Cs[rr][cc]) * Cs[rr][cc + 32];
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= m_valid) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n_tile * GB_N + tx * 4 + j;
            if (n >= g.N) continue;
            float y = acc[i][j];
            if (g.lora_b) {
                float d = 0.f;
#pragma unroll
                for (int q = 0; q < LORA_R; ++q) d += g.lora_b[(int64_t)n * LORA_R + q] * g.lora_t[(int64_t)m * LORA_R + q];
                y += d;
            }
            if (EPI == GEPI_ADD) {
                C[(int64_t)m * g.ldc + n] += y;
            } else {
                if (g.softcap > 0.f) y = g.softcap * tanhf(y / g.softcap);
                C[(int64_t)m * g.ldc + n] = y;
            }
        }
    }
}

// Prefill K/V production: per (row t, head) like k_qkv_post but with the prefill rules:
// no YaRN (src/infer.py:422-425), positions 0..T-1, and on local layers only the positions
// that survive in the ring (>= T - cap) are written. q goes to q_out [T][H][64].
template <typename KVT>
__global__ void __launch_bounds__((H + HKV) * 32) k_qkv_post_prefill(
    int slot, int T, const float* __restrict__ qkv, const float* __restrict__ qn_w, const float* __restrict__ kn_w,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps, int vres_mode, float lv,
    float* __restrict__ vfirst, KVLayer L, int is_local, float* __restrict__ q_out, int yarn_base) {
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* src = qkv + (int64_t)t * QKV;
    const float c = cos_t[(int64_t)t * 32 + lane], s = sin_t[(int64_t)t * 32 + lane];
    if (warp < H) {
        const float x1 = src[warp * DH + lane], x2 = src[warp * DH + lane + 32];
        const float inv = rsqrtf(warp_sum(x1 * x1 + x2 * x2) / (float)DH + eps);
        const float q1 = qn_w[warp * DH + lane] * (x1 * inv);
        const float q2 = qn_w[warp * DH + lane + 32] * (x2 * inv);
        // forward mode on global layers (yarn_base > 0): the query of position t scaled by
        // 1 + 0.1 ln(max(t + 1, base) / base) (src/model.py:511-522, 871-879)
        const float ys = yarn_base > 0 ? 1.f + 0.1f * logf(fmaxf((float)(t + 1), (float)yarn_base) / (float)yarn_base)
                                       : 1.f;
        q_out[((int64_t)t * H + warp) * DH + lane] = (q1 * c - q2 * s) * ys;
        q_out[((int64_t)t * H + warp) * DH + lane + 32] = (q2 * c + q1 * s) * ys;
    } else {
        const int g = warp - H;
        const float k1 = src[H * DH + g * DH + lane], k2 = src[H * DH + g * DH + lane + 32];
        float v1 = src[H * DH + HKV * DH + g * DH + lane], v2 = src[H * DH + HKV * DH + g * DH + lane + 32];
        if (vres_mode == 1) {
            vfirst[((int64_t)t * HKV + g) * DH + lane] = v1;
            vfirst[((int64_t)t * HKV + g) * DH + lane + 32] = v2;
        } else if (vres_mode == 2) {
            v1 = (1.f - lv) * v1 + lv * vfirst[((int64_t)t * HKV + g) * DH + lane];
            v2 = (1.f - lv) * v2 + lv * vfirst[((int64_t)t * HKV + g) * DH + lane + 32];
        }
        if (is_local && L.mask != -1 && t < T - L.cap) return;   // evicted from the ring
        const float inv = rsqrtf(warp_sum(k1 * k1 + k2 * k2) / (float)DH + eps);
        const float a1 = kn_w[g * DH + lane] * (k1 * inv);
        const float a2 = kn_w[g * DH + lane + 32] * (k2 * inv);
        KVT* kp = kv_k<KVT>(L, slot, g, t);
        KVT* vp = kv_v<KVT>(L, slot, g, t);
        kv_store(kp + lane, a1 * c - a2 * s);
        kv_store(kp + lane + 32, a2 * c + a1 * s);
        kv_store(vp + lane, v1);
        kv_store(vp + lane + 32, v2);
    }
}

// Causal prefill attention of one head over the prompt, flash style, register tiled.
// Local layers with T > WINDOW see the truncated cache of the last WINDOW positions: relative
// keys kr in [0, S) at position kbase + kr, S = WINDOW and kbase = T - WINDOW (SDPA is_causal
// aligned top-left on the truncated cache); otherwise S = T, kbase = 0 (plain causal). Query
// qi sees relative keys 0 .. min(qi, S - 1). Block = 64 queries x one head, key tiles of 64;
// thread (ty, tx) = (tid / 16, tid % 16) owns queries 4ty..4ty+3 and, per tile, the scores of
// keys 4tx..4tx+3 and the outputs of dims 4tx..4tx+3 (float4 shared-memory operands); online
// softmax in fp32 with row statistics reduced over the 16 threads of a row group.
constexpr int PA_Q = 64, PA_K = 64;
template <typename KVT>
__global__ void __launch_bounds__(256) k_attn_prefill(int slot, int T, const float* __restrict__ q, KVLayer L,
                                                      int is_local, float* __restrict__ out) {
    __shared__ __align__(16) float Qt[DH * PA_Q];    // [d][query], pre-scaled by 1/8
    __shared__ __align__(16) float KtP[DH * PA_K];   // [d][key] for the scores, then P [query][key]
    __shared__ __align__(16) float Vs[PA_K * DH];    // [key][d]
    const int h = blockIdx.y, g = h / GQA;
    const int q0 = blockIdx.x * PA_Q;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const bool trunc = is_local && T > WINDOW;
    const int S = trunc ? WINDOW : T;
    const int kbase = trunc ? T - WINDOW : 0;
    // Q tile, transposed: thread -> (query tid & 63, dims 16 * (tid >> 6) .. +15)
    {
        const int ql = tid & 63, d0 = (tid >> 6) * 16, qi = q0 + ql;
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (qi < T) v = *reinterpret_cast<const float4*>(q + ((int64_t)qi * H + h) * DH + d0 + j);
            Qt[(d0 + j) * PA_Q + ql] = v.x * 0.125f;
            Qt[(d0 + j + 1) * PA_Q + ql] = v.y * 0.125f;
            Qt[(d0 + j + 2) * PA_Q + ql] = v.z * 0.125f;
            Qt[(d0 + j + 3) * PA_Q + ql] = v.w * 0.125f;
        }
    }
    float m[4], l[4], o[4][4];
    int qlast[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
        const int qi = q0 + ty * 4 + i;
        qlast[i] = (qi < T) ? min(qi, S - 1) : -1;   // last relative key of this query
    }
    const int qmax = min(q0 + PA_Q - 1, T - 1);
    const int rel_end = min(qmax, S - 1);             // last relative key any query needs
    for (int kt = 0; kt <= rel_end; kt += PA_K) {
        __syncthreads();   // previous tile's P and V consumed
        {   // K (transposed) and V of relative keys kt .. kt+63: thread -> (key tid & 63, 16 dims)
            const int kl = tid & 63, d0 = (tid >> 6) * 16, kr = kt + kl;
            float kv[16], vv[16];
            if (kr <= rel_end) {
                const KVT* kp = kv_k<KVT>(L, slot, g, kbase + kr) + d0;
                const KVT* vp = kv_v<KVT>(L, slot, g, kbase + kr) + d0;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    kv[j] = kv_load(kp + j);
                    vv[j] = kv_load(vp + j);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) kv[j] = vv[j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) KtP[(d0 + j) * PA_K + kl] = kv[j];
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(Vs + kl * DH + d0 + j) = make_float4(vv[j], vv[j + 1], vv[j + 2], vv[j + 3]);
        }
        __syncthreads();
        // scores of queries 4ty.. x keys 4tx..
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 8
        for (int d = 0; d < DH; ++d) {
            const float4 qa = *reinterpret_cast<const float4*>(Qt + d * PA_Q + ty * 4);
            const float4 ka = *reinterpret_cast<const float4*>(KtP + d * PA_K + tx * 4);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kvv[4] = {ka.x, ka.y, ka.z, ka.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] += qv[i] * kvv[j];
        }
        // online softmax per query row (16 threads per row group share a row)
        float p[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (kt + tx * 4 + j > qlast[i]) sc[i][j] = -INFINITY;
                mt = fmaxf(mt, sc[i][j]);
            }
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o2));
            const float mn = fmaxf(m[i], mt);
            const float corr = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                p[i][j] = (sc[i][j] == -INFINITY) ? 0.f : expf(sc[i][j] - mn);
                ps += p[i][j];
            }
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
            l[i] = l[i] * corr + ps;
            m[i] = mn;
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] *= corr;
        }
        __syncthreads();   // K^T consumed: the buffer becomes P [query][key]
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4*>(KtP + (ty * 4 + i) * PA_K + tx * 4) = make_float4(p[i][0], p[i][1], p[i][2], p[i][3]);
        __syncthreads();
        // O[4 queries][dims 4tx..] += P[queries][keys] V[keys][dims]
#pragma unroll 4
        for (int k = 0; k < PA_K; k += 4) {
            float4 pr[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pr[i] = *reinterpret_cast<const float4*>(KtP + (ty * 4 + i) * PA_K + k);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 v = *reinterpret_cast<const float4*>(Vs + (k + kk) * DH + tx * 4);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float pk = kk == 0 ? pr[i].x : kk == 1 ? pr[i].y : kk == 2 ? pr[i].z : pr[i].w;
                    o[i][0] += pk * v.x;
                    o[i][1] += pk * v.y;
                    o[i][2] += pk * v.z;
                    o[i][3] += pk * v.w;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int qi = q0 + ty * 4 + i;
        if (qi >= T) continue;
        const float inv = 1.f / l[i];
        *reinterpret_cast<float4*>(out + ((int64_t)qi * H + h) * DH + tx * 4) =
            make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
    }
}

// Head gate for prefill rows: att[t][h*64+d] = o[t][h][d] * sigmoid(xn[t] . Wg[h] + bg[h]),
// plus the Wo loop-adapter projection t = A_wo . att when enabled. One block per row.
__global__ void __launch_bounds__(H * 32) k_gate_rows(const float* __restrict__ o, const float* __restrict__ xn,
                                                      const float* __restrict__ gw, const float* __restrict__ gb,
                                                      float* __restrict__ att, const float* __restrict__ lora_a,
                                                      float* __restrict__ lora_t, __nv_bfloat16* __restrict__ ah = nullptr,
                                                      __nv_bfloat16* __restrict__ al = nullptr) {
    __shared__ float outs[H * DH];
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float z = 0.f;
    const float* xr = xn + (int64_t)r * D;
    for (int k = lane; k < D; k += 32) z += gw[h * D + k] * xr[k];
    z = warp_sum(z) + gb[h];
    const float gt = sigmoidf_(z);
    const float y1 = o[((int64_t)r * H + h) * DH + lane] * gt;
    const float y2 = o[((int64_t)r * H + h) * DH + lane + 32] * gt;
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

// ---- capacity-limited MoE slotting (src/model.py:996-1054, 1339-1342) ----
// Per expert, the assignments in flat (t*K + k) order; counts in `cnt`.
__global__ void k_moe_bucket(const int* __restrict__ idx, int M, int* __restrict__ lists, int list_cap,
                             int* __restrict__ cnt) {
    // one block per expert; deterministic stable compaction over the flat order
    __shared__ int base;
    __shared__ int wsum[32];
    const int e = blockIdx.x;
    if (threadIdx.x == 0) base = 0;
    __syncthreads();
    for (int a0 = 0; a0 < M; a0 += blockDim.x) {
        const int a = a0 + threadIdx.x;
        const bool hit = a < M && idx[a] == e;
        const unsigned bal = __ballot_sync(0xffffffffu, hit);
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        if (lane == 0) wsum[w] = __popc(bal);
        __syncthreads();
        int off = 0;
        for (int i = 0; i < w; ++i) off += wsum[i];
        int tot = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += wsum[i];
        const int pos = base + off + __popc(bal & ((1u << lane) - 1u));
        if (hit && pos < list_cap) lists[(int64_t)e * list_cap + pos] = a;
        __syncthreads();
        if (threadIdx.x == 0) base += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) cnt[e] = base;
}

// Slot of each assignment: the rank of key = e - 0.5 * w / (1 + w) (fp32) among the
// expert's assignments, ties broken by flat index (torch.argsort(stable=True)); dropped
// (-1) when rank >= capacity. When an expert is within capacity every assignment is kept
// and the rank is its position in the flat-order list (a different but equivalent slot
// numbering: which assignments survive is what the outputs depend on).
__global__ void k_moe_slots(const int* __restrict__ lists, int list_cap, const int* __restrict__ cnt,
                            const float* __restrict__ w, int capacity, int* __restrict__ slot,
                            int* __restrict__ rows_e, int* __restrict__ kept) {
    const int e = blockIdx.y;
    const int n = cnt[e];
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0 && threadIdx.x == 0) kept[e] = min(n, capacity);
    if (i >= n) return;
    const int a = lists[(int64_t)e * list_cap + i];
    int rank = i;
    if (n > capacity) {
        const float wa = fmaxf(w[a], 0.f);
        const float ka = (float)e - (wa / (1.f + wa)) * 0.5f;
        rank = 0;
        for (int j = 0; j < n; ++j) {
            const int b = lists[(int64_t)e * list_cap + j];
            const float wb = fmaxf(w[b], 0.f);
            const float kb = (float)e - (wb / (1.f + wb)) * 0.5f;
            if (kb < ka || (kb == ka && b < a)) ++rank;
        }
    }
    if (rank < capacity) {
        slot[a] = rank;
        rows_e[(int64_t)e * capacity + rank] = a / TOPK;   // token row feeding this slot
    } else {
        slot[a] = -1;
    }
}

// Router for many rows (same arithmetic as k_router) writing idx and fp32 weights.
// (k_router is reused directly: one block per row.)

// Combine for prefill rows: h[t] += sh[t] + sum_k [slot >= 0] w_tk * y_e[e][slot] * rscale.
__global__ void __launch_bounds__(256) k_moe_combine_rows(const float* __restrict__ sh, const float* __restrict__ ye,
                                                          int capacity, const int* __restrict__ idx,
                                                          const float* __restrict__ w, const int* __restrict__ slot,
                                                          const float* __restrict__ rscale, float* __restrict__ h) {
    const int t = blockIdx.x;
    for (int d = threadIdx.x; d < D; d += 256) {
        float routed = 0.f;
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            const int a = t * TOPK + k;
            const int s = slot[a];
            if (s >= 0) routed = routed + w[a] * (ye[((int64_t)idx[a] * capacity + s) * D + d] * rscale[d]);
        }
        h[(int64_t)t * D + d] += sh[(int64_t)t * D + d] + routed;
    }
}

// Stem conv over the prompt (src/model.py:592-602 on the anchor-normed rows).
__global__ void k_conv_seq(const float* __restrict__ x, const float* __restrict__ w, int T, float* __restrict__ y) {
    const int t = blockIdx.x;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = x[(int64_t)t * D + d];
        float conv = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (t >= k) conv += w[d * 4 + k] * x[(int64_t)(t - k) * D + d];
        y[(int64_t)t * D + d] = acc + conv;
    }
}

// Prefill embedding + anchor norm (before the conv): h0 = emb[id], h0n = anchor(h0).
__global__ void __launch_bounds__(256) k_embed_rows(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ emb,
                                                    const float* __restrict__ anchor_w, float eps,
                                                    float* __restrict__ h0, float* __restrict__ h0n) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    const __nv_bfloat16* e = emb + (int64_t)ids[t] * D;
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
        h0[(int64_t)t * D + d] = x[i];
        h0n[(int64_t)t * D + d] = anchor_w[d] * (x[i] * inv);
    }
}

// h_in = h0n + step_emb[0]; h = h_in (prefill pulse 0).
__global__ void k_pulse0_rows(const float* __restrict__ h0n, const float* __restrict__ step0, float* __restrict__ h,
                              float* __restrict__ h_in) {
    const int t = blockIdx.x;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float v = h0n[(int64_t)t * D + d] + step0[d];
        h[(int64_t)t * D + d] = v;
        h_in[(int64_t)t * D + d] = v;
    }
}

}  // namespace pulsar
