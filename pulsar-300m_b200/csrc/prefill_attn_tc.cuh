// Causal prefill attention on the tensor cores (tcgen05 MMAs, TMEM accumulators), with the
// masks of the SIMT k_attn_prefill: local layers with T > WINDOW attend over the truncated
// cache of the last WINDOW positions with the causal mask aligned top-left on it (src/infer.py
// 422-435: SDPA is_causal on the truncated keys, no YaRN); otherwise plain causal.
//
// CTA = 128 queries of one head (thread t owns query row t, which is TMEM lane t), 4 warps.
// Key tiles of 64 keys, each tile in two steps:
//   S = Q K^T     tcgen05.mma M=128, N=64, K=64 into TMEM columns [0, 64)
//   O_t = P V     tcgen05.mma M=128, N=64 (dims), K=64 (keys) into TMEM columns [64, 128)
// and in between the online softmax of the thread's own row in registers (tcgen05.ld of its
// lane: no shuffles), with O accumulated in registers as O = O * corr + O_t.
//
// Exactness: the tensor cores take bf16 operands. Q (fp32) and P (fp32) are split into
// bf16 hi + lo halves (|x - hi - lo| <= 2^-16 |x|) and both halves are multiplied into the
// same fp32 accumulator. K and V of a bf16 cache are exact bf16. With an fp32 cache (the parity
// mode) K and V are split as well, and the hi.lo cross terms are added (three MMAs per step;
// the lo.lo term, below 2^-32 relative, is dropped).
//
// Operands live in shared memory in the K-major no-swizzle canonical layout of tc_gemm.cuh
// (tc_off): Q and P as [128 rows][64], K as [64 keys][64 dims], and V transposed to
// [64 dims][64 keys] while it is staged (V is stored key-major in the cache). One thread issues
// the MMAs and commits them to an mbarrier; every wait is bounded (mbar_wait) and a wait that
// runs out raises the error flag, waits again for the MMAs it issued and returns.
#pragma once

#include <stdint.h>

#include "kv.cuh"
#include "mega_ptx.cuh"
#include "tc_gemm.cuh"

namespace pulsar {

constexpr int PT_Q = 128, PT_K = 64, PT_THREADS = 128;

// Byte layout of the shared memory (1024-aligned base).
template <typename KVT>
struct PtLayout {
    static constexpr bool F32 = sizeof(KVT) == 4;
    static constexpr uint32_t TQ = PT_Q * DH * 2;   // 16 KB: a [128][64] bf16 tile
    static constexpr uint32_t TK = PT_K * DH * 2;   // 8 KB: a [64][64] bf16 tile
    static constexpr uint32_t Q_HI = 0, Q_LO = Q_HI + TQ, P_HI = Q_LO + TQ, P_LO = P_HI + TQ;
    static constexpr uint32_t K_HI = P_LO + TQ, V_HI = K_HI + TK;
    static constexpr uint32_t K_LO = V_HI + TK, V_LO = K_LO + (F32 ? TK : 0);
    static constexpr uint32_t BARS = V_LO + (F32 ? TK : 0);
    static constexpr uint32_t BYTES = BARS + 64;
};

template <typename KVT>
constexpr size_t pt_smem_bytes() {
    return PtLayout<KVT>::BYTES + 1024;
}

__device__ __forceinline__ void pt_split8(const float* x, uint4& hi, uint4& lo) {
    __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        h[j] = __float2bfloat16(x[j]);
        l[j] = __float2bfloat16(x[j] - __bfloat162float(h[j]));
    }
    hi = *reinterpret_cast<const uint4*>(h);
    lo = *reinterpret_cast<const uint4*>(l);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_shared_b16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// Eight bf16 values of one K/V row (dims 8c .. 8c+7) as hi (and lo for an fp32 cache).
template <typename KVT>
__device__ __forceinline__ void pt_load_row8(const KVT* p, int c, bool valid, uint4& hi, uint4& lo);

template <>
__device__ __forceinline__ void pt_load_row8<__nv_bfloat16>(const __nv_bfloat16* p, int c, bool valid, uint4& hi,
                                                            uint4& lo) {
    hi = valid ? __ldg(reinterpret_cast<const uint4*>(p) + c) : make_uint4(0u, 0u, 0u, 0u);
    lo = make_uint4(0u, 0u, 0u, 0u);
}

template <>
__device__ __forceinline__ void pt_load_row8<float>(const float* p, int c, bool valid, uint4& hi, uint4& lo) {
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (valid) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p) + 2 * c);
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 2 * c + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    pt_split8(x, hi, lo);
}

// Scatter the 8 bf16 of `v` (dims 8c .. 8c+7 of key `key`) into the transposed V tile.
__device__ __forceinline__ void pt_store_vt(uint32_t base, int key, int c, uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
        st_shared_b16(base + tc_off(8 * c + j, key), (uint16_t)((w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu));
}

template <typename KVT>
__global__ void __launch_bounds__(PT_THREADS) k_attn_prefill_tc(int slot, int T, const float* __restrict__ q,
                                                                KVLayer L, int is_local, float* __restrict__ out,
                                                                int* err_flag) {
    using Lay = PtLayout<KVT>;
    extern __shared__ __align__(1024) unsigned char pt_raw[];
    unsigned char* sm = pt_raw + ((1024 - (smem_u32(pt_raw) & 1023)) & 1023);
    const uint32_t sb = smem_u32(sm);
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + Lay::BARS);
    uint64_t* bar_o = bar_s + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
    const int ntile = (T + PT_Q - 1) / PT_Q;
    const int q0 = (ntile - 1 - (int)blockIdx.x) * PT_Q;   // the longest (latest) query tiles first
    const int h = blockIdx.y, g = h / GQA;
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool trunc = is_local && T > WINDOW;
    const int S = trunc ? WINDOW : T;
    const int kbase = trunc ? T - WINDOW : 0;

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(128)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // this thread's query row, pre-scaled by 1/8 (exact), split into hi / lo
    const int qi = q0 + tid;
    {
        const float* src = q + ((int64_t)qi * H + h) * DH;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (qi < T) {
                const float4 a = *reinterpret_cast<const float4*>(src + 8 * c);
                const float4 b = *reinterpret_cast<const float4*>(src + 8 * c + 4);
                x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
#pragma unroll
                for (int j = 0; j < 8; ++j) x[j] *= 0.125f;
            }
            uint4 hi, lo;
            pt_split8(x, hi, lo);
            st_shared_v4(sb + Lay::Q_HI + tc_off(tid, 8 * c), hi);
            st_shared_v4(sb + Lay::Q_LO + tc_off(tid, 8 * c), lo);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    constexpr uint32_t idesc = tc_idesc<64>();
    const int qlast = qi < T ? min(qi, S - 1) : -1;   // last relative key of this query
    const int rel_end = min(min(q0 + PT_Q - 1, T - 1), S - 1);
    float o[DH];
#pragma unroll
    for (int d = 0; d < DH; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool err = false;
    uint32_t phase = 0;
    int issued = 0;   // 1: MMAs committed to bar_s, 2: to bar_o, whose completion was not seen yet
    for (int kt = 0; kt <= rel_end; kt += PT_K) {
        // 1) K tile [key][dim] and V tile transposed [dim][key]: 512 pieces of 8 dims, 4 a thread
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = tid + PT_THREADS * r;
            const int key = i >> 3, c = i & 7;
            const int kr = kt + key;
            const bool valid = kr <= rel_end;
            const int pos = kbase + (valid ? kr : 0);
            uint4 khi, klo, vhi, vlo;
            pt_load_row8<KVT>(kv_k<KVT>(L, slot, g, pos), c, valid, khi, klo);
            pt_load_row8<KVT>(kv_v<KVT>(L, slot, g, pos), c, valid, vhi, vlo);
            st_shared_v4(sb + Lay::K_HI + tc_off(key, 8 * c), khi);
            pt_store_vt(sb + Lay::V_HI, key, c, vhi);
            if (Lay::F32) {
                st_shared_v4(sb + Lay::K_LO + tc_off(key, 8 * c), klo);
                pt_store_vt(sb + Lay::V_LO, key, c, vlo);
            }
        }
        tc_fence_proxy_async();   // generic-proxy stores -> visible to the tensor core
        tc_fence_before();
        if (__syncthreads_or(err)) break;
        // 2) S = Q K^T
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < DH / 16; ++ks) {
                const uint64_t bk = tc_desc(sb + Lay::K_HI + ks * 256);
                tc_mma(tmem, tc_desc(sb + Lay::Q_HI + ks * 256), bk, idesc, ks > 0 ? 1u : 0u);
                tc_mma(tmem, tc_desc(sb + Lay::Q_LO + ks * 256), bk, idesc, 1u);
                if (Lay::F32) tc_mma(tmem, tc_desc(sb + Lay::Q_HI + ks * 256), tc_desc(sb + Lay::K_LO + ks * 256), idesc, 1u);
            }
            tc_commit(bar_s);
        }
        issued = 1;
        if (!mbar_wait(bar_s, phase)) err = true;
        if (__syncthreads_or(err)) break;
        issued = 0;
        tc_fence_after();
        // 3) online softmax of this thread's row; P (fp32) split into hi / lo tiles
        float s[PT_K];
#pragma unroll
        for (int c = 0; c < PT_K; c += 16) tc_ld16(lane_addr + c, s + c);
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < PT_K; ++j) {
            if (kt + j > qlast) s[j] = -INFINITY;
            mt = fmaxf(mt, s[j]);
        }
        const float mn = fmaxf(m, mt);
        const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
        float ps = 0.f;
#pragma unroll
        for (int j = 0; j < PT_K; ++j) {
            s[j] = (s[j] == -INFINITY) ? 0.f : expf(s[j] - mn);
            ps += s[j];
        }
        l = l * corr + ps;
        m = mn;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            uint4 hi, lo;
            pt_split8(s + 8 * c, hi, lo);
            st_shared_v4(sb + Lay::P_HI + tc_off(tid, 8 * c), hi);
            st_shared_v4(sb + Lay::P_LO + tc_off(tid, 8 * c), lo);
        }
        tc_fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        // 4) O_t = P V
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < PT_K / 16; ++ks) {
                const uint64_t bv = tc_desc(sb + Lay::V_HI + ks * 256);
                tc_mma(tmem + 64, tc_desc(sb + Lay::P_HI + ks * 256), bv, idesc, ks > 0 ? 1u : 0u);
                tc_mma(tmem + 64, tc_desc(sb + Lay::P_LO + ks * 256), bv, idesc, 1u);
                if (Lay::F32)
                    tc_mma(tmem + 64, tc_desc(sb + Lay::P_HI + ks * 256), tc_desc(sb + Lay::V_LO + ks * 256), idesc, 1u);
            }
            tc_commit(bar_o);
        }
        issued = 2;
        if (!mbar_wait(bar_o, phase)) err = true;
        if (__syncthreads_or(err)) break;
        issued = 0;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < DH; c += 16) tc_ld16(lane_addr + 64 + c, s + c);
#pragma unroll
        for (int d = 0; d < DH; ++d) o[d] = o[d] * corr + s[d];
        phase ^= 1u;
        tc_fence_before();   // this thread's TMEM reads precede the next tile's MMAs (barrier in step 1)
    }
    if (err) {
        // a wait ran out: wait once more (bounded) for the MMAs in flight before the tensor
        // memory is released, and report the failure
        if (issued == 1) mbar_wait(bar_s, phase);
        if (issued == 2) mbar_wait(bar_o, phase);
        if (tid == 0) atomicExch(err_flag, 1);
    } else if (qi < T) {
        const float inv = 1.f / l;
        float* dst = out + ((int64_t)qi * H + h) * DH;
#pragma unroll
        for (int d = 0; d < DH; d += 4)
            *reinterpret_cast<float4*>(dst + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128) : "memory");
}

}  // namespace pulsar
