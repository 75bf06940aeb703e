// The pulsar_cuda forward ops behind the C ABI (include/pulsar_b200.h, pulsar_op_*).
//
// Each op keeps the reference binding's argument meaning (csrc/pulsar_cuda.cpp:199-279)
// but is written for sm_100a: 128-bit vector loads where the layout allows, fp32
// arithmetic, launches on the caller's stream with every launch checked, and
// deterministic reductions (no float atomics) for the router's z-loss / probs_mean.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "capi_util.h"
#include "common.cuh"

using namespace pulsar;

namespace {

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline int grid_cap(int64_t n, int64_t per) {
    int64_t g = (n + per - 1) / per;
    if (g > 65535 * 16) g = 65535 * 16;
    return (int)(g < 1 ? 1 : g);
}
// 16-byte vector accesses need every base pointer 16-byte aligned (null counts as aligned).
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- rmsnorm
__global__ void k_rmsnorm_rows(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, int64_t rows,
                               int D, float eps, __nv_bfloat16* __restrict__ y, float* __restrict__ rs) {
    __shared__ float red[32];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const __nv_bfloat16* xr = x + r * D;
        float ss = 0.f;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = __bfloat162float(xr[i]);
            ss += v * v;
        }
        ss = block_sum(ss, red);
        const float inv = rsqrtf(ss / (float)D + eps);
        if (threadIdx.x == 0 && rs) rs[r] = inv;
        for (int i = threadIdx.x; i < D; i += blockDim.x)
            y[r * D + i] = __float2bfloat16(w[i] * (__bfloat162float(xr[i]) * inv));
    }
}

// Warp per row, 16-byte accesses (D % 256 == 0, D <= 2048, x / y / w 16-byte aligned): lane
// holds chunks lane, lane + 32, ... of 8 elements; warp-only reduction.
__global__ void k_rmsnorm_warp(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, int64_t rows, int D,
                               float eps, __nv_bfloat16* __restrict__ y, float* __restrict__ rs) {
    const int lane = threadIdx.x & 31;
    const int nc = D >> 8;   // 8-element chunks per lane (<= 8)
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + r * D);
        float v[8][8];
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if (c < nc) {
                bf16x8_to_f32(__ldg(xr + lane + 32 * c), v[c]);
#pragma unroll
                for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
            }
        }
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / (float)D + eps);
        if (lane == 0 && rs) rs[r] = inv;
        uint4* yr = reinterpret_cast<uint4*>(y + r * D);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            if (c < nc) {
                const float4* w4 = reinterpret_cast<const float4*>(w + (lane + 32 * c) * 8);
                const float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
                const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                float o[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = wv[j] * (v[c][j] * inv);
                yr[lane + 32 * c] = f32_to_bf16x8(o);
            }
        }
    }
}

// ---------------------------------------------------------------- rope
__global__ void k_rope(const __nv_bfloat16* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
                       int64_t rows, int64_t T, int half, __nv_bfloat16* __restrict__ y) {
    const int64_t n = rows * half;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / half;
        const int j = (int)(i % half);
        const int64_t t = r % T;
        const float c = cs[t * half + j], s = sn[t * half + j];
        const float x1 = __bfloat162float(x[r * 2 * half + j]);
        const float x2 = __bfloat162float(x[r * 2 * half + j + half]);
        // explicit FMAs (the 16-byte form uses the same ones, so both round identically)
        y[r * 2 * half + j] = __float2bfloat16(__fmaf_rn(x1, c, -(x2 * s)));
        y[r * 2 * half + j + half] = __float2bfloat16(__fmaf_rn(x2, c, x1 * s));
    }
}

// 16-byte form (half % 8 == 0, x / y / cs / sn 16-byte aligned): a thread per 8 rotation
// pairs of one row; IT is the index type (32-bit when the element count allows).
template <typename IT>
__global__ void k_rope_v8(const __nv_bfloat16* __restrict__ x, const float* __restrict__ cs,
                          const float* __restrict__ sn, IT rows, IT T, int half, __nv_bfloat16* __restrict__ y) {
    const int h8 = half >> 3;
    const IT n = rows * h8;
    for (IT i = blockIdx.x * (IT)blockDim.x + threadIdx.x; i < n; i += (IT)gridDim.x * blockDim.x) {
        const IT r = i / h8;
        const int j = (int)(i - r * h8) * 8;
        const IT t = r % T;
        const float4* c4 = reinterpret_cast<const float4*>(cs + t * half + j);
        const float4* s4 = reinterpret_cast<const float4*>(sn + t * half + j);
        const float4 ca = __ldg(c4), cb = __ldg(c4 + 1), sa = __ldg(s4), sb = __ldg(s4 + 1);
        const float c[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
        const float s[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
        float x1[8], x2[8], y1[8], y2[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + r * 2 * half + j)), x1);
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + r * 2 * half + half + j)), x2);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            y1[k] = __fmaf_rn(x1[k], c[k], -(x2[k] * s[k]));
            y2[k] = __fmaf_rn(x2[k], c[k], x1[k] * s[k]);
        }
        *reinterpret_cast<uint4*>(y + r * 2 * half + j) = f32_to_bf16x8(y1);
        *reinterpret_cast<uint4*>(y + r * 2 * half + half + j) = f32_to_bf16x8(y2);
    }
}

// ---------------------------------------------------------------- swiglu
__global__ void k_swiglu(const __nv_bfloat16* __restrict__ gu, int64_t rows, int64_t d, __nv_bfloat16* __restrict__ out) {
    const int64_t n = rows * d;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / d, j = i % d;
        const float g = __bfloat162float(gu[r * 2 * d + j]);
        const float u = __bfloat162float(gu[r * 2 * d + d + j]);
        out[i] = __float2bfloat16(siluf_(g) * u);
    }
}

// 16-byte form (d % 8 == 0, gu / out 16-byte aligned): a thread per 8 outputs.
// sh >= 0: d / 8 is 2^sh, so the row and column come from a shift and a mask.
template <typename IT>
__global__ void k_swiglu_v8(const __nv_bfloat16* __restrict__ gu, IT rows, IT d, int sh,
                            __nv_bfloat16* __restrict__ out) {
    const IT d8 = d >> 3, n = rows * d8;
    for (IT i = blockIdx.x * (IT)blockDim.x + threadIdx.x; i < n; i += (IT)gridDim.x * blockDim.x) {
        const IT r = sh >= 0 ? (i >> sh) : i / d8;
        const IT j = (i - r * d8) * 8;
        float g[8], u[8], o[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(gu + r * 2 * d + j)), g);
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(gu + r * 2 * d + d + j)), u);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = siluf_(g[k]) * u[k];
        *reinterpret_cast<uint4*>(out + r * d + j) = f32_to_bf16x8(o);
    }
}

// ---------------------------------------------------------------- router top-k
// One warp per token; lane e holds expert e. Top-K by K rounds of a warp argmax with ties
// to the lowest expert index (the order the reference's insertion sort with strict '>'
// produces). Per-token lse^2 and sigmoid scores go to `ws` for a deterministic mean.
template <bool BF16>
__global__ void k_router_topk(const void* __restrict__ logits_v, const float* __restrict__ bias, int64_t N, int E,
                              int K, int64_t* __restrict__ idx_out, __nv_bfloat16* __restrict__ w_out,
                              float* __restrict__ ws) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); t < N; t += warps) {
        float l = 0.f;
        if (lane < E) {
            if (BF16)
                l = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(logits_v)[t * E + lane]);
            else
                l = reinterpret_cast<const float*>(logits_v)[t * E + lane];
        }
        const float mean = warp_sum(l) / (float)E;
        const float c = l - mean;
        const float s = sigmoidf_(c);
        float b = (lane < E) ? s + bias[lane] : -INFINITY;
        float sel_s[8];
        int sel_i[8];
        for (int k = 0; k < K; ++k) {
            ArgMax a{b, lane < E ? lane : 1 << 30};
            a = warp_argmax(a);
            sel_i[k] = a.i;
            sel_s[k] = __shfl_sync(0xffffffffu, s, a.i & 31);
            if (lane == a.i) b = -INFINITY;
        }
        float sum = 0.f;
        for (int k = 0; k < K; ++k) sum += sel_s[k];
        sum += 1e-6f;
        if (lane < K) {
            float my_s = 0.f;
            int my_i = 0;
            for (int k = 0; k < K; ++k)
                if (k == lane) { my_s = sel_s[k]; my_i = sel_i[k]; }
            idx_out[t * K + lane] = my_i;
            w_out[t * K + lane] = __float2bfloat16(my_s / sum);
        }
        // centred-logit logsumexp for the z-loss, sigmoid scores for probs_mean
        const float mx = warp_max(lane < E ? c : -INFINITY);
        const float se = warp_sum(lane < E ? expf(c - mx) : 0.f);
        if (lane == 0) {
            const float lse = mx + logf(fmaxf(se, 1e-20f));
            ws[t] = lse * lse;
        }
        if (lane < E) ws[N + t * E + lane] = s;
    }
}

// Deterministic column means over the per-token workspace (fixed summation order): block c
// reduces column c - 1 (-1: the lse^2 column), each thread a fixed stride of tokens.
__global__ void k_router_means(const float* __restrict__ ws, int64_t N, int E, float zw, float* __restrict__ z_loss,
                               float* __restrict__ probs_mean) {
    __shared__ float red[32];
    {
        const int col = (int)blockIdx.x - 1;
        float acc = 0.f;
        for (int64_t t = threadIdx.x; t < N; t += blockDim.x) acc += (col < 0) ? ws[t] : ws[N + t * E + col];
        acc = block_sum(acc, red);
        if (threadIdx.x == 0) {
            if (col < 0) {
                if (z_loss) z_loss[0] = (zw > 0.f && N > 0) ? zw * acc / (float)N : 0.f;
            } else if (probs_mean) {
                probs_mean[col] = N > 0 ? acc / (float)N : 0.f;
            }
        }
    }
}

// ---------------------------------------------------------------- qk rmsnorm + rope
__global__ void k_qk_rmsnorm_rope(const __nv_bfloat16* __restrict__ x, int64_t sB, int64_t sH, int64_t sT,
                                  int64_t n_vec, int n_heads, int64_t T, const float* __restrict__ w,
                                  const float* __restrict__ cs, const float* __restrict__ sn, float eps,
                                  __nv_bfloat16* __restrict__ y, float* __restrict__ rs) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t v = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); v < n_vec; v += warps) {
        const int64_t t = v % T;
        const int h = (int)((v / T) % n_heads);
        const int64_t b = v / (T * n_heads);
        const __nv_bfloat16* xv = x + b * sB + (int64_t)h * sH + t * sT;
        const float x1 = __bfloat162float(xv[lane]);
        const float x2 = __bfloat162float(xv[lane + 32]);
        const float inv = rsqrtf(warp_sum(x1 * x1 + x2 * x2) / 64.f + eps);
        if (lane == 0 && rs) rs[v] = inv;
        const float q1 = w[h * 64 + lane] * (x1 * inv);
        const float q2 = w[h * 64 + lane + 32] * (x2 * inv);
        const float c = cs[t * 32 + lane], s = sn[t * 32 + lane];
        y[v * 64 + lane] = __float2bfloat16(q1 * c - q2 * s);
        y[v * 64 + lane + 32] = __float2bfloat16(q2 * c + q1 * s);
    }
}

// Half-warp per vector form (every vector's base 8-byte aligned): lane j of the half holds
// elements 4j..4j+3 (one 8-byte load); the rotation partner of element d (d +- 32) sits on lane
// j ^ 8, one shuffle away. Each warp takes two vectors per step (the loop stays warp-uniform).
template <typename IT>
__global__ void k_qk_rmsnorm_rope_h(const __nv_bfloat16* __restrict__ x, IT sB, IT sH, IT sT, IT n_vec, int n_heads,
                                    IT T, const float* __restrict__ w, const float* __restrict__ cs,
                                    const float* __restrict__ sn, float eps, __nv_bfloat16* __restrict__ y,
                                    float* __restrict__ rs) {
    const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
    const IT warps = (IT)gridDim.x * (blockDim.x >> 5);
    for (IT vp = blockIdx.x * (IT)(blockDim.x >> 5) + (threadIdx.x >> 5); 2 * vp < n_vec; vp += warps) {
        const IT v = 2 * vp + half;
        const bool ok = v < n_vec;
        const IT vv = ok ? v : 2 * vp;
        const IT t = vv % T;
        const IT ht = vv / T;
        const int h = (int)(ht % n_heads);
        const IT b = ht / n_heads;
        const __nv_bfloat16* xv = x + b * sB + (IT)h * sH + t * sT + 4 * hl;
        const uint2 u = *reinterpret_cast<const uint2*>(xv);
        const float2 p0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 p1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        const float f[4] = {p0.x, p0.y, p1.x, p1.y};
        float ss = f[0] * f[0] + f[1] * f[1] + f[2] * f[2] + f[3] * f[3];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss / 64.f + eps);
        if (ok && hl == 0 && rs) rs[v] = inv;
        const float4 wv = *reinterpret_cast<const float4*>(w + h * 64 + 4 * hl);
        const float q[4] = {wv.x * (f[0] * inv), wv.y * (f[1] * inv), wv.z * (f[2] * inv), wv.w * (f[3] * inv)};
        float pq[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pq[i] = __shfl_xor_sync(0xffffffffu, q[i], 8);
        const float4 c4 = *reinterpret_cast<const float4*>(cs + t * 32 + 4 * (hl & 7));
        const float4 s4 = *reinterpret_cast<const float4*>(sn + t * 32 + 4 * (hl & 7));
        const float c[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = hl < 8 ? q[i] * c[i] - pq[i] * sv[i] : q[i] * c[i] + pq[i] * sv[i];
        if (ok) {
            const __nv_bfloat162 a0 = __floats2bfloat162_rn(o[0], o[1]), a1 = __floats2bfloat162_rn(o[2], o[3]);
            uint2 st;
            st.x = *reinterpret_cast<const uint32_t*>(&a0);
            st.y = *reinterpret_cast<const uint32_t*>(&a1);
            *reinterpret_cast<uint2*>(y + v * 64 + 4 * hl) = st;
        }
    }
}

// ---------------------------------------------------------------- attention gate
// IT: index type (32-bit when the element count allows: cheaper divisions).
template <typename IT>
__global__ void k_attn_gate(const __nv_bfloat16* __restrict__ attn, const float* __restrict__ gl, IT B, int H, IT T,
                            __nv_bfloat16* __restrict__ out) {
    const IT n = B * T * H * 8;   // 8 chunks of 8 elements per head vector
    for (IT i = blockIdx.x * (IT)blockDim.x + threadIdx.x; i < n; i += (IT)gridDim.x * blockDim.x) {
        const int c = (int)(i & 7);
        const IT bth = i >> 3;            // (b, t, h)
        const IT bt = bth / H;
        const int h = (int)(bth - bt * H);
        const IT b = bt / T, t = bt - b * T;
        const float g = sigmoidf_(gl[bt * H + h]);
        const uint4 v = *reinterpret_cast<const uint4*>(attn + (((b * H + h) * T + t) * 64 + c * 8));
        float f[8];
        bf16x8_to_f32(v, f);
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] *= g;
        *reinterpret_cast<uint4*>(out + (bt * H + h) * 64 + c * 8) = f32_to_bf16x8(f);
    }
}

// ---------------------------------------------------------------- causal conv k4
__global__ void k_conv1d_k4(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, int64_t B, int64_t T,
                            int64_t D, __nv_bfloat16* __restrict__ y) {
    const int64_t n = B * T * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = i % D;
        const int64_t t = (i / D) % T;
        float acc = __bfloat162float(x[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (t >= k) acc += w[d * 4 + k] * __bfloat162float(x[i - k * D]);
        y[i] = __float2bfloat16(acc);
    }
}

// 16-byte form (D % 8 == 0, x / y / w 16-byte aligned): a thread per 8 channels of one (b, t);
// the four taps' rows are 16-byte loads, the 8 channels' weights two float4 each. Same
// summation order per channel as k_conv1d_k4, so the results are identical.
template <typename IT>
__global__ void k_conv1d_k4_v8(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, IT B, IT T, IT D,
                               __nv_bfloat16* __restrict__ y) {
    const IT D8 = D >> 3, n = B * T * D8;
    for (IT i = blockIdx.x * (IT)blockDim.x + threadIdx.x; i < n; i += (IT)gridDim.x * blockDim.x) {
        const IT bt = i / D8, d0 = (i - bt * D8) * 8;
        const IT t = bt % T;
        const IT at = bt * D + d0;
        float xs[4][8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (t >= k) bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + at - k * D)), xs[k]);
        }
        const float4* w4 = reinterpret_cast<const float4*>(w + d0 * 4);   // w[d][0..3] per channel
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 wj = __ldg(w4 + j);
            float a = xs[0][j];
            a += wj.x * xs[0][j];
            if (t >= 1) a += wj.y * xs[1][j];
            if (t >= 2) a += wj.z * xs[2][j];
            if (t >= 3) a += wj.w * xs[3][j];
            acc[j] = a;
        }
        *reinterpret_cast<uint4*>(y + at) = f32_to_bf16x8(acc);
    }
}

// ---------------------------------------------------------------- moe combine / dispatch
__global__ void k_moe_combine(const __nv_bfloat16* __restrict__ eo, const int64_t* __restrict__ idx,
                              const __nv_bfloat16* __restrict__ tw, const int32_t* __restrict__ slot,
                              const __nv_bfloat16* __restrict__ sh, int64_t N, int K, int64_t E, int64_t C, int64_t D,
                              __nv_bfloat16* __restrict__ out) {
    for (int64_t t = blockIdx.x; t < N; t += gridDim.x) {
        for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
            float acc = sh ? __bfloat162float(sh[t * D + d]) : 0.f;
            for (int k = 0; k < K; ++k) {
                const int64_t e = idx[t * K + k];
                const int s = slot[t * K + k];
                if (s >= 0 && s < C && e >= 0 && e < E)
                    acc += __bfloat162float(tw[t * K + k]) * __bfloat162float(eo[(e * C + s) * D + d]);
            }
            out[t * D + d] = __float2bfloat16(acc);
        }
    }
}

// 16-byte form of k_moe_combine (D % 8 == 0, every bf16 tensor 16-byte aligned): a thread per
// 8 channels of one token, same summation order (shared output, then the routes in k order).
// KC > 0: the route count K known at compile time (the model's top-4), the routes unrolled.
template <int KC>
__global__ void k_moe_combine_v8(const __nv_bfloat16* __restrict__ eo, const int64_t* __restrict__ idx,
                                 const __nv_bfloat16* __restrict__ tw, const int32_t* __restrict__ slot,
                                 const __nv_bfloat16* __restrict__ sh, int N, int Kr, int E, int C, int D,
                                 __nv_bfloat16* __restrict__ out) {
    const int K = KC > 0 ? KC : Kr;
    const int D8 = D >> 3;
    for (int t = blockIdx.x; t < N; t += gridDim.x) {
        for (int c = threadIdx.x; c < D8; c += blockDim.x) {
            float acc[8];
            if (sh) {
                bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(sh + (int64_t)t * D) + c), acc);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = 0.f;
            }
            // routes in groups of G: every route's 16-byte load in flight before the accumulation
            // (in k order)
            constexpr int G = KC > 0 ? KC : 8;
            for (int k0 = 0; k0 < K; k0 += G) {
                uint4 rv[G];
                float wt[G];
                bool ok[G];
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    const int k = k0 + u;
                    ok[u] = false;
                    if (k < K) {
                        const int64_t e = __ldg(idx + (int64_t)t * K + k);
                        const int s = __ldg(slot + (int64_t)t * K + k);
                        ok[u] = s >= 0 && s < C && e >= 0 && e < E;
                        wt[u] = __bfloat162float(tw[(int64_t)t * K + k]);
                        if (ok[u]) rv[u] = __ldg(reinterpret_cast<const uint4*>(eo + (e * C + s) * (int64_t)D) + c);
                    }
                }
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    if (ok[u]) {
                        float v[8];
                        bf16x8_to_f32(rv[u], v);
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc[j] += wt[u] * v[j];
                    }
                }
            }
            reinterpret_cast<uint4*>(out + (int64_t)t * D)[c] = f32_to_bf16x8(acc);
        }
    }
}

__device__ __forceinline__ bool aligned16_dev(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__global__ void k_moe_tail_zero(__nv_bfloat16* __restrict__ buf, const int64_t* __restrict__ counts, int64_t E,
                                int64_t C, int64_t D) {
    for (int64_t e = blockIdx.y; e < E; e += gridDim.y) {
        int64_t c = counts[e];
        const int64_t start = c < 0 ? 0 : (c > C ? C : c);
        const int64_t n = (C - start) * D;
        __nv_bfloat16* p = buf + (e * C + start) * D;
        if ((D & 7) == 0 && aligned16_dev(buf)) {   // 16-byte stores (D % 8 == 0 keeps rows aligned)
            uint4* p4 = reinterpret_cast<uint4*>(p);
            for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n / 8;
                 i += (int64_t)gridDim.x * blockDim.x)
                p4[i] = make_uint4(0u, 0u, 0u, 0u);
        } else {
            for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
                 i += (int64_t)gridDim.x * blockDim.x)
                p[i] = __float2bfloat16(0.f);
        }
    }
}

__global__ void k_moe_dispatch(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ idx,
                               const int32_t* __restrict__ slot, int64_t N, int K, int64_t E, int64_t C, int64_t D,
                               __nv_bfloat16* __restrict__ ei) {
    for (int64_t t = blockIdx.x; t < N; t += gridDim.x) {
        for (int k = 0; k < K; ++k) {
            const int64_t e = idx[t * K + k];
            const int s = slot[t * K + k];
            if (s < 0 || s >= C || e < 0 || e >= E) continue;
            for (int64_t d = threadIdx.x; d < D; d += blockDim.x) ei[(e * C + s) * D + d] = x[t * D + d];
        }
    }
}

// 16-byte form of k_moe_dispatch (x / ei 16-byte aligned; D % 8 == 0 is required anyway): the
// token's row is read once into registers (up to 8 chunks a thread) and stored to each route.
__global__ void k_moe_dispatch_v8(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ idx,
                                  const int32_t* __restrict__ slot, int64_t N, int K, int64_t E, int64_t C, int64_t D,
                                  __nv_bfloat16* __restrict__ ei) {
    const int64_t D8 = D >> 3;
    for (int64_t t = blockIdx.x; t < N; t += gridDim.x) {
        const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
        for (int64_t c0 = 0; c0 < D8; c0 += 8 * (int64_t)blockDim.x) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int64_t c = c0 + threadIdx.x + (int64_t)u * blockDim.x;
                if (c < D8) v[u] = __ldg(src + c);
            }
            for (int k = 0; k < K; ++k) {
                const int64_t e = __ldg(idx + t * K + k);
                const int s = __ldg(slot + t * K + k);
                if (s < 0 || s >= C || e < 0 || e >= E) continue;
                uint4* dst = reinterpret_cast<uint4*>(ei + (e * C + s) * D);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int64_t c = c0 + threadIdx.x + (int64_t)u * blockDim.x;
                    if (c < D8) dst[c] = v[u];
                }
            }
        }
    }
}

}  // namespace

// ==================================================================================== C ABI

extern "C" int pulsar_op_rmsnorm(const void* x, const float* w, int64_t rows, int64_t D, float eps, void* y,
                                 float* rsqrt_out, void* stream) {
    PULSAR_CHECK_ARG(rows >= 0 && D > 0, "rmsnorm: invalid shape rows=%lld D=%lld", (long long)rows, (long long)D);
    if (rows == 0) return PULSAR_OK;
    PULSAR_CHECK_ARG(x && w && y, "rmsnorm: null pointer");
    if (D % 256 == 0 && D <= 2048 && aligned16(x) && aligned16(w) && aligned16(y)) {
        k_rmsnorm_warp<<<grid_cap(rows, 8), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, w, rows, (int)D, eps,
                                                                  (__nv_bfloat16*)y, rsqrt_out);
        PULSAR_LAUNCH_CHECK("k_rmsnorm_warp");
        return PULSAR_OK;
    }
    k_rmsnorm_rows<<<grid_cap(rows, 1), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, w, rows, (int)D, eps,
                                                              (__nv_bfloat16*)y, rsqrt_out);
    PULSAR_LAUNCH_CHECK("k_rmsnorm_rows");
    return PULSAR_OK;
}

extern "C" int pulsar_op_rope(const void* qk, const float* cs, const float* sn, int64_t rows, int64_t T, int64_t Dh,
                              void* y, void* stream) {
    PULSAR_CHECK_ARG(rows >= 0 && Dh > 0 && Dh % 2 == 0, "rope: head dim must be even, got %lld", (long long)Dh);
    if (rows == 0) return PULSAR_OK;
    PULSAR_CHECK_ARG(T > 0 && qk && cs && sn && y, "rope: invalid arguments (T=%lld)", (long long)T);
    const int64_t n = rows * (Dh / 2);
    if ((Dh / 2) % 8 == 0 && aligned16(qk) && aligned16(cs) && aligned16(sn) && aligned16(y)) {
        if (rows * Dh < (int64_t)1 << 31)
            k_rope_v8<int><<<grid_cap(n / 8, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)qk, cs, sn, (int)rows,
                                                                         (int)T, (int)(Dh / 2), (__nv_bfloat16*)y);
        else
            k_rope_v8<int64_t><<<grid_cap(n / 8, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)qk, cs, sn, rows, T,
                                                                             (int)(Dh / 2), (__nv_bfloat16*)y);
        PULSAR_LAUNCH_CHECK("k_rope_v8");
        return PULSAR_OK;
    }
    k_rope<<<grid_cap(n, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)qk, cs, sn, rows, T, (int)(Dh / 2),
                                                    (__nv_bfloat16*)y);
    PULSAR_LAUNCH_CHECK("k_rope");
    return PULSAR_OK;
}

extern "C" int pulsar_op_swiglu(const void* gu, int64_t rows, int64_t d_ff, void* out, void* stream) {
    PULSAR_CHECK_ARG(rows >= 0 && d_ff > 0, "swiglu: invalid shape");
    if (rows == 0) return PULSAR_OK;
    if (d_ff % 8 == 0 && aligned16(gu) && aligned16(out)) {
        const int64_t d8 = d_ff / 8;
        const int sh = (d8 & (d8 - 1)) == 0 ? __builtin_ctzll((unsigned long long)d8) : -1;
        if (rows * d_ff * 2 < (int64_t)1 << 31)
            k_swiglu_v8<int><<<grid_cap(rows * d_ff / 8, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)gu, (int)rows,
                                                                                     (int)d_ff, sh, (__nv_bfloat16*)out);
        else
            k_swiglu_v8<int64_t><<<grid_cap(rows * d_ff / 8, 256), 256, 0, S(stream)>>>(
                (const __nv_bfloat16*)gu, rows, d_ff, sh, (__nv_bfloat16*)out);
        PULSAR_LAUNCH_CHECK("k_swiglu_v8");
        return PULSAR_OK;
    }
    k_swiglu<<<grid_cap(rows * d_ff, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)gu, rows, d_ff,
                                                                (__nv_bfloat16*)out);
    PULSAR_LAUNCH_CHECK("k_swiglu");
    return PULSAR_OK;
}

extern "C" int pulsar_op_moe_router_topk(const void* logits, int logits_bf16, const float* bias, int64_t N, int64_t E,
                                         int64_t K, float zw, int64_t* idx, void* w, float* z_loss,
                                         float* probs_mean, float* ws, void* stream) {
    PULSAR_CHECK_ARG(E >= 1 && E <= 32, "moe_router_topk_forward_cuda supports E <= 32, got %lld", (long long)E);
    PULSAR_CHECK_ARG(K > 0 && K <= 8 && K <= E, "top_k must be in [1, min(8, E)], got %lld", (long long)K);
    PULSAR_CHECK_ARG(N >= 0, "moe_router_topk: N must be >= 0");
    if (N > 0) {
        PULSAR_CHECK_ARG(logits && bias && idx && w && ws, "moe_router_topk: null pointer");
        const int threads = 256;
        const int grid = grid_cap(N, threads / 32);
        if (logits_bf16)
            k_router_topk<true><<<grid, threads, 0, S(stream)>>>(logits, bias, N, (int)E, (int)K, idx,
                                                                 (__nv_bfloat16*)w, ws);
        else
            k_router_topk<false><<<grid, threads, 0, S(stream)>>>(logits, bias, N, (int)E, (int)K, idx,
                                                                  (__nv_bfloat16*)w, ws);
        PULSAR_LAUNCH_CHECK("k_router_topk");
    }
    if (z_loss || probs_mean) {
        k_router_means<<<(int)E + 1, 256, 0, S(stream)>>>(ws, N, (int)E, zw, z_loss, probs_mean);
        PULSAR_LAUNCH_CHECK("k_router_means");
    }
    return PULSAR_OK;
}

extern "C" int pulsar_op_qk_rmsnorm_rope(const void* x, int64_t sB, int64_t sH, int64_t sT, int64_t n_vec,
                                         int64_t n_heads, int64_t T, const float* w, const float* cs, const float* sn,
                                         float eps, void* y, float* rs, void* stream) {
    PULSAR_CHECK_ARG(n_vec >= 0 && n_heads > 0, "qk_rmsnorm_rope: invalid shape");
    if (n_vec == 0) return PULSAR_OK;
    PULSAR_CHECK_ARG(T > 0 && x && w && cs && sn && y, "qk_rmsnorm_rope: invalid arguments");
    const bool a8 = (reinterpret_cast<uintptr_t>(x) & 7) == 0 && sB % 4 == 0 && sH % 4 == 0 && sT % 4 == 0 &&
                    aligned16(w) && aligned16(cs) && aligned16(sn) && (reinterpret_cast<uintptr_t>(y) & 7) == 0;
    if (a8) {
        // largest element offset read: (B - 1) sB + (heads - 1) sH + (T - 1) sT + 63
        const int64_t nb = n_vec / (T * n_heads);
        const int64_t span = (nb > 0 ? nb - 1 : 0) * sB + (n_heads - 1) * sH + (T - 1) * sT + 64;
        if (n_vec * 64 < (int64_t)1 << 31 && span < (int64_t)1 << 31 && sB >= 0 && sH >= 0 && sT >= 0)
            k_qk_rmsnorm_rope_h<int><<<grid_cap(n_vec, 16), 256, 0, S(stream)>>>(
                (const __nv_bfloat16*)x, (int)sB, (int)sH, (int)sT, (int)n_vec, (int)n_heads, (int)T, w, cs, sn, eps,
                (__nv_bfloat16*)y, rs);
        else
            k_qk_rmsnorm_rope_h<int64_t><<<grid_cap(n_vec, 16), 256, 0, S(stream)>>>(
                (const __nv_bfloat16*)x, sB, sH, sT, n_vec, (int)n_heads, T, w, cs, sn, eps, (__nv_bfloat16*)y, rs);
        PULSAR_LAUNCH_CHECK("k_qk_rmsnorm_rope_h");
        return PULSAR_OK;
    }
    k_qk_rmsnorm_rope<<<grid_cap(n_vec, 8), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, sB, sH, sT, n_vec,
                                                                  (int)n_heads, T, w, cs, sn, eps,
                                                                  (__nv_bfloat16*)y, rs);
    PULSAR_LAUNCH_CHECK("k_qk_rmsnorm_rope");
    return PULSAR_OK;
}

extern "C" int pulsar_op_attn_gate(const void* attn, const float* gl, int64_t B, int64_t H, int64_t T, void* out,
                                   void* stream) {
    PULSAR_CHECK_ARG(B >= 0 && H >= 0 && T >= 0, "fused_attn_gate: invalid shape");
    const int64_t n = B * T * H * 8;
    if (n == 0) return PULSAR_OK;
    if (n < (int64_t)1 << 31)
        k_attn_gate<int><<<grid_cap(n, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)attn, gl, (int)B, (int)H,
                                                                   (int)T, (__nv_bfloat16*)out);
    else
        k_attn_gate<int64_t><<<grid_cap(n, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)attn, gl, B, (int)H, T,
                                                                       (__nv_bfloat16*)out);
    PULSAR_LAUNCH_CHECK("k_attn_gate");
    return PULSAR_OK;
}

extern "C" int pulsar_op_conv1d_k4(const void* x, const float* w, int64_t B, int64_t T, int64_t D, void* y,
                                   void* stream) {
    PULSAR_CHECK_ARG(B >= 0 && T >= 0 && D > 0, "causal_depthwise_conv1d_k4: invalid shape");
    const int64_t n = B * T * D;
    if (n == 0) return PULSAR_OK;
    if (D % 8 == 0 && aligned16(x) && aligned16(w) && aligned16(y)) {
        if (n < (int64_t)1 << 31)
            k_conv1d_k4_v8<int><<<grid_cap(n / 8, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, w, (int)B, (int)T,
                                                                               (int)D, (__nv_bfloat16*)y);
        else
            k_conv1d_k4_v8<int64_t><<<grid_cap(n / 8, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, w, B, T, D,
                                                                                   (__nv_bfloat16*)y);
        PULSAR_LAUNCH_CHECK("k_conv1d_k4_v8");
        return PULSAR_OK;
    }
    k_conv1d_k4<<<grid_cap(n, 256), 256, 0, S(stream)>>>((const __nv_bfloat16*)x, w, B, T, D, (__nv_bfloat16*)y);
    PULSAR_LAUNCH_CHECK("k_conv1d_k4");
    return PULSAR_OK;
}

extern "C" int pulsar_op_moe_combine(const void* eo, const int64_t* idx, const void* tw, const int32_t* slot,
                                     const void* sh, int64_t N, int64_t K, int64_t E, int64_t C, int64_t D, void* out,
                                     void* stream) {
    PULSAR_CHECK_ARG(N >= 0 && K >= 0 && E > 0 && C >= 0 && D > 0, "moe_combine: invalid shape");
    if (N == 0) return PULSAR_OK;
    const bool fits32 = N < ((int64_t)1 << 31) && E * C < ((int64_t)1 << 31) && D < ((int64_t)1 << 31);
    if (D % 8 == 0 && fits32 && aligned16(eo) && aligned16(sh) && aligned16(out)) {
        const int threads = D / 8 >= 128 ? 128 : (int)((D / 8 + 31) / 32 * 32);
        if (K == 4)
            k_moe_combine_v8<4><<<grid_cap(N, 1), threads, 0, S(stream)>>>(
                (const __nv_bfloat16*)eo, idx, (const __nv_bfloat16*)tw, slot, (const __nv_bfloat16*)sh, (int)N, 4,
                (int)E, (int)C, (int)D, (__nv_bfloat16*)out);
        else
            k_moe_combine_v8<0><<<grid_cap(N, 1), threads, 0, S(stream)>>>(
                (const __nv_bfloat16*)eo, idx, (const __nv_bfloat16*)tw, slot, (const __nv_bfloat16*)sh, (int)N, (int)K,
                (int)E, (int)C, (int)D, (__nv_bfloat16*)out);
        PULSAR_LAUNCH_CHECK("k_moe_combine_v8");
        return PULSAR_OK;
    }
    k_moe_combine<<<grid_cap(N, 1), 128, 0, S(stream)>>>((const __nv_bfloat16*)eo, idx, (const __nv_bfloat16*)tw,
                                                          slot, (const __nv_bfloat16*)sh, N, (int)K, E, C, D,
                                                          (__nv_bfloat16*)out);
    PULSAR_LAUNCH_CHECK("k_moe_combine");
    return PULSAR_OK;
}

extern "C" int pulsar_op_moe_dispatch(const void* x, const int64_t* idx, const int32_t* slot, const int64_t* counts,
                                      int64_t N, int64_t K, int64_t E, int64_t C, int64_t D, void* ei, void* stream) {
    PULSAR_CHECK_ARG(N >= 0 && K >= 0 && E > 0 && C >= 0 && D > 0, "moe_dispatch: invalid shape");
    PULSAR_CHECK_ARG(D % 8 == 0, "D must be a multiple of 8 for vectorised dispatch, got %lld", (long long)D);
    if (E * C * D > 0) {
        if (counts) {
            dim3 grid(64, (unsigned)(E < 65535 ? E : 65535));
            k_moe_tail_zero<<<grid, 256, 0, S(stream)>>>((__nv_bfloat16*)ei, counts, E, C, D);
            PULSAR_LAUNCH_CHECK("k_moe_tail_zero");
        } else {
            PULSAR_TRY(cuda_status(cudaMemsetAsync(ei, 0, (size_t)(E * C * D) * 2, S(stream)), "moe_dispatch memset"));
        }
    }
    if (N > 0 && K > 0 && aligned16(x) && aligned16(ei)) {
        const int threads = D / 8 >= 128 ? 128 : (int)((D / 8 + 31) / 32 * 32);
        k_moe_dispatch_v8<<<grid_cap(N, 1), threads, 0, S(stream)>>>((const __nv_bfloat16*)x, idx, slot, N, (int)K, E,
                                                                      C, D, (__nv_bfloat16*)ei);
        PULSAR_LAUNCH_CHECK("k_moe_dispatch_v8");
    } else if (N > 0 && K > 0) {
        k_moe_dispatch<<<grid_cap(N, 1), 128, 0, S(stream)>>>((const __nv_bfloat16*)x, idx, slot, N, (int)K, E, C, D,
                                                               (__nv_bfloat16*)ei);
        PULSAR_LAUNCH_CHECK("k_moe_dispatch");
    }
    return PULSAR_OK;
}

// ==================================================================================== no-allocation router
// The router top-k below needs N * (E + 1) floats of scratch for its deterministic means. The
// regular entry point takes that scratch from the caller. This variant serves callers that
// cannot allocate device memory at all - a host whose memory manager owns every device byte
// and rejects outside allocations, or a foreign-language caller with no device allocator of
// its own - by using a fixed array compiled into the library instead. Every GPU that loads
// the library holds this 4 MiB array until the process exits.
static constexpr int64_t kRouterScratchFloats = int64_t(1) << 20;   // N * (E + 1) <= 1,048,576
static __device__ __align__(256) float g_router_scratch[kRouterScratchFloats];

namespace {
constexpr int kMaxDevices = 64;
struct ScratchAddr {
    unsigned long long ctx_id;   // unique id of the context the address belongs to (0: none yet)
    float* ptr;
};
ScratchAddr g_router_scratch_addr[kMaxDevices] = {};
std::mutex g_router_scratch_mu;

// Unique id of the calling thread's current context (0 when none is current or the driver does
// not export the calls). The driver functions are reached through the runtime, so the library
// does not link the driver library itself.
unsigned long long current_context_id() {
    using CtxGetCurrent = int (*)(void**);
    using CtxGetId = int (*)(void*, unsigned long long*);
    static CtxGetCurrent get_current = nullptr;
    static CtxGetId get_id = nullptr;
    static bool resolved = false;
    if (!resolved) {   // under g_router_scratch_mu
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrent>(f);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetId>(f);
        resolved = true;
    }
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return id;
}

// Device address of g_router_scratch in the current context. Host code cannot use the
// symbol's name as a device pointer, so the address is looked up with the device current and
// cached per device together with the id of the context it was looked up in; a different
// context (after cudaDeviceReset, say, the module is loaded again and the array may move) looks
// it up again. Without context ids the address is looked up on every call.
int router_scratch(float** out) {
    int dev = 0;
    PULSAR_TRY(cuda_status(cudaGetDevice(&dev), "cudaGetDevice"));
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("moe_router_topk_noalloc: device ordinal %d outside [0, %d)", dev, kMaxDevices);
        return PULSAR_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_router_scratch_mu);
    ScratchAddr& c = g_router_scratch_addr[dev];
    const unsigned long long id = current_context_id();
    if (id == 0 || c.ctx_id != id || !c.ptr) {
        void* p = nullptr;
        PULSAR_TRY(cuda_status(cudaGetSymbolAddress(&p, g_router_scratch), "cudaGetSymbolAddress(router scratch)"));
        c.ptr = static_cast<float*>(p);
        c.ctx_id = current_context_id();   // the lookup makes the device's primary context current
    }
    *out = c.ptr;
    return PULSAR_OK;
}
}  // namespace

extern "C" int pulsar_op_moe_router_topk_noalloc(const void* logits, int logits_bf16, const float* bias, int64_t N,
                                                 int64_t E, int64_t K, float zw, int64_t* idx, void* w,
                                                 float* z_loss, float* probs_mean, void* stream) {
    PULSAR_CHECK_ARG(E >= 1 && E <= 32, "moe_router_topk_forward_cuda supports E <= 32, got %lld", (long long)E);
    PULSAR_CHECK_ARG(K > 0 && K <= 8 && K <= E, "top_k must be in [1, min(8, E)], got %lld", (long long)K);
    PULSAR_CHECK_ARG(N >= 0, "moe_router_topk: N must be >= 0");
    if (N * (E + 1) > kRouterScratchFloats) {
        set_error("moe_router_topk_noalloc: N * (E + 1) = %lld exceeds the built-in scratch of %lld floats "
                  "(use pulsar_op_moe_router_topk with a caller workspace)",
                  (long long)(N * (E + 1)), (long long)kRouterScratchFloats);
        return PULSAR_ERR_CAPACITY;
    }
    float* ws = nullptr;
    PULSAR_TRY(router_scratch(&ws));
    if (N > 0) {
        PULSAR_CHECK_ARG(logits && bias && idx && w, "moe_router_topk: null pointer");
        const int threads = 256;
        const int grid = grid_cap(N, threads / 32);
        if (logits_bf16)
            k_router_topk<true><<<grid, threads, 0, S(stream)>>>(logits, bias, N, (int)E, (int)K, idx,
                                                                 (__nv_bfloat16*)w, ws);
        else
            k_router_topk<false><<<grid, threads, 0, S(stream)>>>(logits, bias, N, (int)E, (int)K, idx,
                                                                  (__nv_bfloat16*)w, ws);
        PULSAR_LAUNCH_CHECK("k_router_topk");
    }
    if (z_loss || probs_mean) {
        k_router_means<<<(int)E + 1, 256, 0, S(stream)>>>(ws, N, (int)E, zw, z_loss, probs_mean);
        PULSAR_LAUNCH_CHECK("k_router_means");
    }
    return PULSAR_OK;
}
