// Sampled speculative acceptance on the device: Philox4x32-10 uniforms, the warped
// (temperature, top-p) distribution of a logits row, inverse-CDF draws in vocabulary order,
// and the pieces of the per-sequence ratio test with residual resampling. No host sync.
//
// Semantics (block_spec_generate_ids of the oracle; the warping is src/infer.py:594-608):
//   scaled = logits / max(T, 1e-5); e_i = exp(scaled_i - max); top-p keeps token i iff the
//   mass of tokens with a strictly larger weight is <= top_p (the top token always kept);
//   p_i = e_i / sum_kept e. A draw with uniform u returns the first index whose inclusive
//   prefix sum (fp64, vocabulary order) exceeds u * total, stepped back to the nearest
//   index with p > 0. Uniforms of stream (seq, round, slot): Philox4x32-10 with counter
//   (seq, round, slot, 0) and key (seed lo, seed hi), u_k = (x_k >> 8) * 2^-24.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace pulsar {

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_MAX_V = 49152;   // logits row held in shared memory (192 KB)

// ---- Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) -------------------------------------
__host__ __device__ inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)M0 * c[0], p1 = (uint64_t)M1 * c[2];
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0;
        c[1] = lo1;
        c[2] = n2;
        c[3] = lo0;
        k0 += W0;
        k1 += W1;
    }
}

// Uniform k (0..3) of stream (seq, round, slot).
__host__ __device__ inline float stream_uniform(uint64_t seed, uint32_t seq, uint32_t rnd, uint32_t slot, int k) {
    uint32_t c[4] = {seq, rnd, slot, 0u};
    philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    return (float)(c[k] >> 8) * (1.0f / 16777216.0f);
}

// Warped-distribution statistics of one logits row.
struct WarpStats {
    float mx;     // max of scaled logits
    float tc;     // max(T, 1e-5)
    uint32_t x0;  // token kept iff the bit pattern of its weight e_i is >= x0
    float zk;     // sum of kept e_i
};

__device__ __forceinline__ float warp_weight(float logit, const WarpStats& s) { return expf(logit / s.tc - s.mx); }

__device__ __forceinline__ float warped_prob(float logit, const WarpStats& s) {
    const float e = warp_weight(logit, s);
    return (__float_as_uint(e) >= s.x0) ? e / s.zk : 0.f;
}

// ---- block reductions over SAMPLE_THREADS threads ------------------------------------------
__device__ __forceinline__ float sblock_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    const float t = lane < (SAMPLE_THREADS >> 5) ? red[lane] : 0.f;
    return warp_sum(t);
}

__device__ __forceinline__ float sblock_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    const float t = lane < (SAMPLE_THREADS >> 5) ? red[lane] : -INFINITY;
    return warp_max(t);
}

// Warp statistics of row `lg` (V entries); ev: V floats of shared scratch. Every thread
// returns the same statistics.
__device__ WarpStats row_warp_stats(const float* __restrict__ lg, int V, float T, float top_p, float* ev,
                                    float* red) {
    WarpStats s;
    s.tc = fmaxf(T, 1e-5f);
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) {
        const float x = lg[i] / s.tc;
        ev[i] = x;
        mx = fmaxf(mx, x);
    }
    s.mx = sblock_max(mx, red);
    float z = 0.f;
    for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) {
        const float e = expf(ev[i] - s.mx);   // the same value as warp_weight(lg[i], s)
        ev[i] = e;
        z += e;
    }
    const float Z = sblock_sum(z, red);
    s.x0 = 0u;
    s.zk = Z;
    if (top_p < 1.f) {
        // bisection for the smallest pattern x with mass(e > x) <= top_p * Z; the pattern of
        // 1.0 qualifies (no weight exceeds 1)
        const float tp = top_p * Z;
        uint32_t lo = 0u, hi = 0x3F800000u;
        while (lo < hi) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            float m = 0.f;
            for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) {
                const float e = ev[i];
                if (__float_as_uint(e) > mid) m += e;
            }
            if (sblock_sum(m, red) <= tp) hi = mid;
            else lo = mid + 1;
        }
        s.x0 = lo;
        float k = 0.f;
        for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) {
            const float e = ev[i];
            if (__float_as_uint(e) >= lo) k += e;
        }
        s.zk = sblock_sum(k, red);
    }
    return s;
}

// Inverse-CDF draw over V probabilities prob(i) (fp32 values accumulated in fp64 in
// vocabulary order). Thread t owns the contiguous chunk [t*ch, (t+1)*ch). Every thread
// returns the index. redd: 33 doubles, redi: 2 ints of shared memory.
template <typename F>
__device__ int draw_index(int V, float u, F&& prob, double* redd, int* redi) {
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int ch = (V + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
    const int i0 = min(V, t * ch), i1 = min(V, i0 + ch);
    double loc = 0.0;
    for (int i = i0; i < i1; ++i) loc += (double)prob(i);
    double incl = loc;   // inclusive scan of the thread sums within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) redd[w] = incl;
    __syncthreads();
    if (w == 0) {
        const double x = lane < (SAMPLE_THREADS >> 5) ? redd[lane] : 0.0;
        double y = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += z;
        }
        redd[lane] = y - x;             // exclusive prefix of the warp totals
        if (lane == 31) redd[32] = y;   // grand total
    }
    __syncthreads();
    const double base = redd[w] + (incl - loc);
    const double target = (double)u * redd[32];
    if (t == 0) redi[0] = V - 1;        // u * total at or past the total: the last index
    __syncthreads();
    if (i0 < i1 && base <= target && target < base + loc) {
        double c = base;
        int found = i1 - 1;
        for (int i = i0; i < i1; ++i) {
            c += (double)prob(i);
            if (c > target) {
                found = i;
                break;
            }
        }
        redi[0] = found;
    }
    __syncthreads();
    int idx = redi[0];
    if (t == 0) redi[1] = 0;
    __syncthreads();
    // never a zero-probability token: the largest index <= idx with p > 0 (else 0)
    int best = -1;
    for (int i = i0; i < i1 && i <= idx; ++i)
        if (prob(i) > 0.f) best = i;
    if (best >= 0) atomicMax(&redi[1], best);
    __syncthreads();
    if (!(prob(idx) > 0.f)) idx = redi[1];
    __syncthreads();
    return idx;
}

}  // namespace pulsar
