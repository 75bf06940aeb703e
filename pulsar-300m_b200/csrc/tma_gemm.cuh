// TMA-fed, warp-specialised tensor-core GEMM for sm_100a: C[m][n] (+)= sum_k A[m][k] W[n][k],
// the same contract, operand split and epilogues as k_tc_gemm (tc_gemm.cuh), which stays as the
// fallback for operands a tensor map cannot describe.
//
// Roles (128 threads): warp 0 lane 0 is the producer. Per 64-wide K chunk it issues three
// (SWIGLU: four) 2-D tensor-map loads (cp.async.bulk.tensor into this CTA only, SWIZZLE_128B)
// into a STAGES-deep ring: A hi, A lo [128 rows x 64] and W [BN rows x 64], completion counted
// in bytes on the stage's `full` mbarrier. Warp 1 lane 0 waits on `full`, issues the tcgen05
// MMAs (M = 128, N = BN, K = 16 per instruction, A hi and A lo into the same TMEM accumulator)
// and commits them to the stage's `empty` mbarrier, which the producer waits on before it
// refills the stage. After the last chunk the MMA thread commits to `acc`; all four warps
// wait on it and read the accumulator with tcgen05.ld for the shared epilogue (tc_epilogue).
//
// Shared-memory operand layout: the canonical K-major SWIZZLE_128B layout that the tensor map
// writes (rows of 128 B, 16-byte chunks permuted within each 8-row, 1024-byte atom); its
// descriptor has SBO = 1024 B and layout type 2, and the K steps of 16 elements advance the
// start address by 32 B inside the atom. Every wait is bounded; a wait that runs out stops
// the issuing, drains the copies and MMAs in flight (bounded again) and raises the error flag.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "mega_ptx.cuh"
#include "tc_gemm.cuh"

namespace pulsar {

template <int BN>
struct TmaSmem {
    static constexpr int S = BN == 128 ? 4 : 5;   // stages: 48 KB (BN 128) or 40 KB (BN 64) each
    alignas(1024) __nv_bfloat16 a_hi[S][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 a_lo[S][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 w[S][BN * TC_BK];
    uint64_t full[S], empty[S], acc;
    uint32_t tmem_base;
    int err, issued, consumed;
};

template <int BN>
constexpr size_t tma_smem_bytes() {
    return sizeof(TmaSmem<BN>) + 1024;
}

// K-major SWIZZLE_128B shared-memory descriptor (sm_100): start >> 4, LBO 16 B (unused for
// swizzled K-major), SBO 1024 B (8-row atoms), version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

template <int EPI, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tma_gemm(const __grid_constant__ CUtensorMap ta_hi,
                                                            const __grid_constant__ CUtensorMap ta_lo,
                                                            const __grid_constant__ CUtensorMap tw, GemmArgs g,
                                                            int w_rows_per_batch, int* err_flag) {
    using Sm = TmaSmem<BN>;
    constexpr int S = Sm::S;
    extern __shared__ __align__(1024) unsigned char tm_raw[];
    Sm* s = reinterpret_cast<Sm*>(tm_raw + ((1024 - (smem_u32(tm_raw) & 1023)) & 1023));
    const int b = blockIdx.z;
    const int m_valid = g.m_count ? g.m_count[b] : g.M;
    const int m0 = blockIdx.y * TC_BM;
    if (m0 >= m_valid) return;   // uniform over the CTA, before any TMEM allocation
    const int n_tile = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = g.K / TC_BK;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&s->full[i], 1);
            mbar_init(&s->empty[i], 1);
        }
        mbar_init(&s->acc, 1);
        s->err = 0;
        s->issued = 0;
        s->consumed = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s->tmem_base)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s->tmem_base;
    if (warp == 0 && lane == 0) {
        // producer
        constexpr uint32_t stage_bytes = (uint32_t)(2 * TC_BM * TC_BK + BN * TC_BK) * 2;
        const int arow = b * g.M + m0;
        const int wrow = b * w_rows_per_batch;
        int kc = 0;
        for (; kc < nk; ++kc) {
            const int st = kc % S, use = kc / S;
            if (use > 0 && !mbar_wait(&s->empty[st], (use - 1) & 1)) {
                s->err = 1;
                break;
            }
            mbar_arrive_expect_tx(&s->full[st], stage_bytes);
            const int k0 = kc * TC_BK;
            tma_load_2d(s->a_hi[st], &ta_hi, k0, arow, &s->full[st]);
            tma_load_2d(s->a_lo[st], &ta_lo, k0, arow, &s->full[st]);
            if (EPI == GEPI_SWIGLU) {
                const int half = g.N / 2, n0 = n_tile * (BN / 2);
                tma_load_2d(s->w[st], &tw, k0, wrow + n0, &s->full[st]);
                tma_load_2d(s->w[st] + (BN / 2) * TC_BK, &tw, k0, wrow + half + n0, &s->full[st]);
            } else {
                tma_load_2d(s->w[st], &tw, k0, wrow + n_tile * BN, &s->full[st]);
            }
        }
        s->issued = kc;
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = tc_idesc<BN>();
        int kc = 0;
        for (; kc < nk; ++kc) {
            const int st = kc % S;
            if (!mbar_wait(&s->full[st], (kc / S) & 1)) {
                s->err = 1;
                break;
            }
            tc_fence_after();
            const uint32_t ah = smem_u32(s->a_hi[st]), al = smem_u32(s->a_lo[st]), wb = smem_u32(s->w[st]);
#pragma unroll
            for (int ks = 0; ks < TC_BK / 16; ++ks) {
                const uint64_t bd = tc_desc_sw128(wb + ks * 32);
                tc_mma(tmem, tc_desc_sw128(ah + ks * 32), bd, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                tc_mma(tmem, tc_desc_sw128(al + ks * 32), bd, idesc, 1u);
            }
            tc_commit(&s->empty[st]);   // the stage is free once these MMAs have read it
        }
        s->consumed = kc;
        tc_commit(&s->acc);   // arrives when every MMA issued above has completed
    }
    __syncwarp();
    bool err = !mbar_wait(&s->acc, 0);
    tc_fence_after();
    if (__syncthreads_or(err || s->err)) {
        if (threadIdx.x == 0) {
            // drain: the copies issued but not consumed (each stage's latest use), then the MMAs
            for (int kc = max(s->consumed, s->issued - S); kc < s->issued; ++kc) mbar_wait(&s->full[kc % S], (kc / S) & 1);
            mbar_wait(&s->acc, 0);
            atomicExch(err_flag, 1);
        }
    } else {
        tc_epilogue<EPI, BN>(g, b, m0, m_valid, n_tile, tmem);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
}

}  // namespace pulsar
