// Tensor-core GEMM for sm_100a (tcgen05 + TMEM): C[m][n] (+)= sum_k A[m][k] W[n][k] with
// fp32 activations A and bf16 weights W, fp32 accumulation in tensor memory.
//
// Exactness: the tensor cores take bf16 operands, so every fp32 activation is split into
// a_hi = bf16(a) and a_lo = bf16(a - a_hi) and both halves are multiplied by the (exact bf16)
// weights into the same accumulator: |a - a_hi - a_lo| <= 2^-16 |a|, close to fp32 products.
//
// Tile: 128 rows x BN columns per CTA (one M=128, N=BN instruction shape), K in chunks of 64.
// Operands are staged in shared memory in the K-major, no-swizzle canonical layout: core
// matrices of 8 rows x 16 bytes stored contiguously (128 B), the 8 K-chunks of a 64-wide
// chunk at 128 B strides (LBO), 8-row groups at 1 KB strides (SBO). The activations are split
// into bf16 hi / lo once per GEMM (k_split_hilo, gathered rows compacted per batch); then every
// operand chunk (A hi, A lo, W) is copied with cp.async into a 4-stage ring, three chunks ahead
// of the tensor core. One thread issues the MMAs and commits them to an mbarrier per stage.
// The accumulator is read back with tcgen05.ld (each warp its 32 lanes = rows) for the
// epilogue (vectorised stores).
#pragma once

#include <stdint.h>

#include "mega_ptx.cuh"
#include "prefill_kernels.cuh"

namespace pulsar {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_THREADS = 128;

constexpr int TC_STAGES = 4;

template <int BN>
struct TcSmem {
    // per stage: A hi, A lo [128 x 64] bf16, W [BN x 64] bf16 (canonical layout)
    alignas(1024) __nv_bfloat16 a_hi[TC_STAGES][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 a_lo[TC_STAGES][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 w[TC_STAGES][BN * TC_BK];
    uint64_t mma_done[TC_STAGES];
    uint32_t tmem_base;
};

// Byte offset of element (row, k) (k < 64) inside a canonical K-major no-swizzle tile.
__device__ __forceinline__ uint32_t tc_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint64_t tc_desc(uint32_t smem_addr) {
    // start >> 4 | LBO 128 B >> 4 | SBO 1024 B >> 4 | version 1 (sm_100) | layout SWIZZLE_NONE
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46);
}

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, M = 128.
template <int BN>
__host__ __device__ constexpr uint32_t tc_idesc() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Rows of this CTA's 128-row tile: global row of tile row r (or -1 past the valid rows).
__device__ __forceinline__ const float* tc_arow(const GemmArgs& g, int b, int m, int m_valid) {
    if (m >= m_valid) return nullptr;
    if (g.a_rows) return g.A + (int64_t)g.a_rows[(int64_t)b * g.M + m] * g.lda;
    return g.A + (int64_t)b * g.a_stride + (int64_t)m * g.lda;
}

// Output column n of tile column j: for SWIGLU the tile holds 64 gate and 64 up columns of
// the same output range ([n0, n0+64) and [half + n0, half + n0 + 64)).
template <int EPI, int BN>
__device__ __forceinline__ int tc_wrow(const GemmArgs& g, int n_tile, int j) {
    if (EPI == GEPI_SWIGLU) {
        const int half = g.N / 2, n0 = n_tile * (BN / 2);
        return (j < BN / 2) ? n0 + j : half + n0 + (j - BN / 2);
    }
    return n_tile * BN + j;
}

// Split of the activation rows: hi/lo [batch][M][K] bf16 (row m of batch b = the GEMM's
// A row of tile row m, gathered rows compacted); rows past the batch's valid count are not
// written (the GEMM zero-fills them). Thread: 8 consecutive k.
__global__ void __launch_bounds__(256) k_split_hilo(GemmArgs g, __nv_bfloat16* __restrict__ hi,
                                                    __nv_bfloat16* __restrict__ lo) {
    const int b = blockIdx.y;
    const int m_valid = g.m_count ? g.m_count[b] : g.M;
    const int per_row = g.K / 8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int m = (int)(i / per_row), k = (int)(i % per_row) * 8;
    if (m >= m_valid) return;
    const float* src = tc_arow(g, b, m, m_valid) + k;
    const float4 v0 = *reinterpret_cast<const float4*>(src), v1 = *reinterpret_cast<const float4*>(src + 4);
    const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        h[j] = __float2bfloat16(x[j]);
        l[j] = __float2bfloat16(x[j] - __bfloat162float(h[j]));
    }
    const int64_t o = ((int64_t)b * g.M + m) * g.K + k;
    *reinterpret_cast<uint4*>(hi + o) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + o) = *reinterpret_cast<const uint4*>(l);
}

__device__ __forceinline__ void tc_cp16(uint32_t dst, const void* src, bool valid) {
    // zero-fill when !valid (source size 0)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

// Issue chunk kc (64 columns of K) of A hi, A lo and W into stage st (one cp.async group).
template <int EPI, int BN>
__device__ __forceinline__ void tc_issue_chunk(const GemmArgs& g, const __nv_bfloat16* ahi,
                                               const __nv_bfloat16* alo, TcSmem<BN>* s, int st, int b, int m0,
                                               int m_valid, int n_tile, int kc) {
    const int t = threadIdx.x, k0 = kc * TC_BK;
    const uint32_t sh = smem_u32(s->a_hi[st]), sl = smem_u32(s->a_lo[st]), sw = smem_u32(s->w[st]);
    // A: 128 rows x 8 pieces of 16 B, for hi and lo
#pragma unroll
    for (int q = 0; q < TC_BM * 8 / TC_THREADS; ++q) {
        const int i = t + TC_THREADS * q;
        const int r = i >> 3, c = i & 7;
        const bool ok = m0 + r < m_valid;
        const int64_t off = ((int64_t)b * g.M + (ok ? m0 + r : 0)) * g.K + k0 + c * 8;
        tc_cp16(sh + tc_off(r, c * 8), ahi + off, ok);
        tc_cp16(sl + tc_off(r, c * 8), alo + off, ok);
    }
    const __nv_bfloat16* W = g.W + (int64_t)b * g.w_stride;
#pragma unroll
    for (int q = 0; q < BN * 8 / TC_THREADS; ++q) {
        const int i = t + TC_THREADS * q;
        const int j = i >> 3, c = i & 7;
        const int n = tc_wrow<EPI, BN>(g, n_tile, j);
        tc_cp16(sw + tc_off(j, c * 8), W + (int64_t)n * g.K + k0 + c * 8, true);
    }
}

// Epilogue of a 128 x BN tile whose fp32 accumulator sits in TMEM columns [tmem, tmem + BN):
// warp w holds rows 32w..32w+31 (its lanes), 16 columns per tcgen05.ld; STORE (optional
// loop-adapter correction and softcap), ADD or SWIGLU into C. Every thread of the CTA calls it.
template <int EPI, int BN>
__device__ __forceinline__ void tc_epilogue(const GemmArgs& g, int b, int m0, int m_valid, int n_tile, uint32_t tmem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = m0 + warp * 32 + lane;
    const bool row_ok = m < m_valid;
    float* C = g.C + (int64_t)b * g.c_stride + (int64_t)m * g.ldc;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    if (EPI == GEPI_SWIGLU) {
        const int n0 = n_tile * (BN / 2);
        for (int c = 0; c < BN / 2; c += 16) {
            float gt[16], up[16];
            tc_ld16(lane_addr + c, gt);
            tc_ld16(lane_addr + BN / 2 + c, up);
            if (row_ok) {
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<float4*>(C + n0 + c + i) =
                        make_float4(siluf_(gt[i]) * up[i], siluf_(gt[i + 1]) * up[i + 1],
                                    siluf_(gt[i + 2]) * up[i + 2], siluf_(gt[i + 3]) * up[i + 3]);
                if (g.c_hi) {   // the split operand of the GEMM that reads C: 16 bf16 hi and lo
                    const int64_t o = (int64_t)b * g.c_stride + (int64_t)m * g.ldc + n0 + c;
                    __nv_bfloat16 h[16], l[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float y = siluf_(gt[i]) * up[i];
                        h[i] = __float2bfloat16(y);
                        l[i] = __float2bfloat16(y - __bfloat162float(h[i]));
                    }
                    reinterpret_cast<uint4*>(g.c_hi + o)[0] = reinterpret_cast<const uint4*>(h)[0];
                    reinterpret_cast<uint4*>(g.c_hi + o)[1] = reinterpret_cast<const uint4*>(h)[1];
                    reinterpret_cast<uint4*>(g.c_lo + o)[0] = reinterpret_cast<const uint4*>(l)[0];
                    reinterpret_cast<uint4*>(g.c_lo + o)[1] = reinterpret_cast<const uint4*>(l)[1];
                }
            }
        }
    } else {
        for (int c = 0; c < BN; c += 16) {
            float v[16];
            tc_ld16(lane_addr + c, v);
            if (!row_ok) continue;
            const int nb = n_tile * BN + c;
            if (g.lora_b) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float d = 0.f;
#pragma unroll
                    for (int q = 0; q < LORA_R; ++q)
                        d += g.lora_b[(int64_t)(nb + i) * LORA_R + q] * g.lora_t[(int64_t)m * LORA_R + q];
                    v[i] += d;
                }
            }
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float4* dst = reinterpret_cast<float4*>(C + nb + i);
                if (EPI == GEPI_ADD) {
                    const float4 o = *dst;
                    *dst = make_float4(o.x + v[i], o.y + v[i + 1], o.z + v[i + 2], o.w + v[i + 3]);
                } else {
                    float4 y = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    if (g.softcap > 0.f) {
                        const float sc = g.softcap;
                        y = make_float4(sc * tanhf(y.x / sc), sc * tanhf(y.y / sc), sc * tanhf(y.z / sc),
                                        sc * tanhf(y.w / sc));
                    }
                    *dst = y;
                }
            }
        }
    }
}

__device__ __forceinline__ void tc_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tc_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int EPI, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc_gemm(GemmArgs g, const __nv_bfloat16* __restrict__ ahi,
                                                           const __nv_bfloat16* __restrict__ alo, int* err_flag) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    TcSmem<BN>* s = reinterpret_cast<TcSmem<BN>*>(tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023));
    const int b = blockIdx.z;
    const int m_valid = g.m_count ? g.m_count[b] : g.M;
    const int m0 = blockIdx.y * TC_BM;
    if (m0 >= m_valid) return;   // uniform over the CTA, before any TMEM allocation
    const int n_tile = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < TC_STAGES; ++i) mbar_init(&s->mma_done[i], 1);
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
    constexpr uint32_t idesc = tc_idesc<BN>();
    const int nk = g.K / TC_BK;
    // prologue: chunks 0 .. STAGES-2 (one cp.async group each, empty groups past the end)
#pragma unroll
    for (int c = 0; c < TC_STAGES - 1; ++c) {
        if (c < nk) tc_issue_chunk<EPI, BN>(g, ahi, alo, s, c, b, m0, m_valid, n_tile, c);
        tc_commit_group();
    }
    // A bounded wait that runs out ends the K loop for the whole CTA (the OR at the next
    // barrier): no further copies or MMAs are issued. The results of such a launch are invalid;
    // its tensor memory is read and released only after the last committed MMA group has been
    // waited for (or that wait has run out too).
    bool err = false;
    int last = -1;   // last chunk whose MMAs were committed
    for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % TC_STAGES;
        tc_wait_group<TC_STAGES - 2>();   // chunk kc landed (this thread's copies)
        tc_fence_proxy_async();           // -> visible to the tensor core (async proxy)
        if (__syncthreads_or(err)) break;
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t ah = smem_u32(s->a_hi[st]), al = smem_u32(s->a_lo[st]), wb = smem_u32(s->w[st]);
#pragma unroll
            for (int ks = 0; ks < TC_BK / 16; ++ks) {
                const uint64_t bd = tc_desc(wb + ks * 256);
                tc_mma(tmem, tc_desc(ah + ks * 256), bd, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                tc_mma(tmem, tc_desc(al + ks * 256), bd, idesc, 1u);
            }
            tc_commit(&s->mma_done[st]);
        }
        last = kc;
        // refill the stage of chunk kc-1 with chunk kc+STAGES-1 once that chunk's MMAs are done
        const int nc = kc + TC_STAGES - 1;
        if (nc < nk) {
            if (kc >= 1) {
                const int ps = (kc - 1) % TC_STAGES;
                if (!mbar_wait(&s->mma_done[ps], ((kc - 1) / TC_STAGES) & 1)) err = true;
            }
            if (!err) tc_issue_chunk<EPI, BN>(g, ahi, alo, s, nc % TC_STAGES, b, m0, m_valid, n_tile, nc);
        }
        tc_commit_group();
    }
    tc_wait_group<0>();   // this thread's copies have landed (none is left in flight at exit)
    if (last >= 0 && !mbar_wait(&s->mma_done[last % TC_STAGES], (last / TC_STAGES) & 1)) err = true;
    if (last != nk - 1) err = true;
    tc_fence_after();
    if (__syncthreads_or(err)) {
        if (threadIdx.x == 0) atomicExch(err_flag, 1);
    } else {
        tc_epilogue<EPI, BN>(g, b, m0, m_valid, n_tile, tmem);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
}

template <int BN>
constexpr size_t tc_smem_bytes() {
    return sizeof(TcSmem<BN>) + 1024;
}

}  // namespace pulsar
