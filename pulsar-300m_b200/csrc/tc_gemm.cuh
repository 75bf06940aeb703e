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
// chunk at 128 B strides (LBO), 8-row groups at 1 KB strides (SBO). Two stages: while the
// tensor core runs chunk i, the 128 threads hold chunk i+1's A in registers (all loads issued
// at once) and copy its W with cp.async; one thread issues the MMAs and commits them to an
// mbarrier per stage. The accumulator is read back with
// tcgen05.ld (each warp its 32 lanes = rows) for the epilogue.
#pragma once

#include <stdint.h>

#include "mega_ptx.cuh"
#include "prefill_kernels.cuh"

namespace pulsar {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_THREADS = 128;

template <int BN>
struct TcSmem {
    // per stage: A hi, A lo [128 x 64] bf16, W [BN x 64] bf16 (canonical layout)
    alignas(1024) __nv_bfloat16 a_hi[2][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 a_lo[2][TC_BM * TC_BK];
    alignas(1024) __nv_bfloat16 w[2][BN * TC_BK];
    uint64_t mma_done[2];
    uint32_t tmem_base;
    int err;
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

// A chunk of 128 rows x 64 fp32 is 2048 float4: thread t holds float4 i = t + 128 * q, q < 16
// (row i / 16, columns 4 * (i % 16)); all 16 loads are issued together.
struct TcARegs {
    float4 v[16];
};

__device__ __forceinline__ void tc_load_a(const GemmArgs& g, int b, int m0, int m_valid, int kc, TcARegs& r) {
    const int t = threadIdx.x, k0 = kc * TC_BK;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        const int i = t + TC_THREADS * q;
        const float* src = tc_arow(g, b, m0 + (i >> 4), m_valid);
        r.v[q] = src ? *reinterpret_cast<const float4*>(src + k0 + (i & 15) * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Split the held A chunk into bf16 hi / lo and store both in the canonical layout.
template <int BN>
__device__ __forceinline__ void tc_store_a(TcSmem<BN>* s, int st, const TcARegs& r) {
    const int t = threadIdx.x;
    unsigned char* ahi = reinterpret_cast<unsigned char*>(s->a_hi[st]);
    unsigned char* alo = reinterpret_cast<unsigned char*>(s->a_lo[st]);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        const int i = t + TC_THREADS * q;
        const float4 v = r.v[q];
        const __nv_bfloat16 h0 = __float2bfloat16(v.x), h1 = __float2bfloat16(v.y), h2 = __float2bfloat16(v.z),
                            h3 = __float2bfloat16(v.w);
        const __nv_bfloat16 l0 = __float2bfloat16(v.x - __bfloat162float(h0)),
                            l1 = __float2bfloat16(v.y - __bfloat162float(h1)),
                            l2 = __float2bfloat16(v.z - __bfloat162float(h2)),
                            l3 = __float2bfloat16(v.w - __bfloat162float(h3));
        const uint32_t off = tc_off(i >> 4, (i & 15) * 4);   // 4 consecutive k stay in one 16-byte chunk
        __nv_bfloat162 hp[2] = {__halves2bfloat162(h0, h1), __halves2bfloat162(h2, h3)};
        __nv_bfloat162 lp[2] = {__halves2bfloat162(l0, l1), __halves2bfloat162(l2, l3)};
        *reinterpret_cast<uint2*>(ahi + off) = *reinterpret_cast<uint2*>(hp);
        *reinterpret_cast<uint2*>(alo + off) = *reinterpret_cast<uint2*>(lp);
    }
}

// W chunk: BN rows x 64 bf16 = BN * 8 pieces of 16 B, copied straight into the canonical
// layout with cp.async (completion: cp.async.wait_all of the issuing thread).
template <int EPI, int BN>
__device__ __forceinline__ void tc_issue_w(const GemmArgs& g, TcSmem<BN>* s, int st, int b, int n_tile, int kc) {
    const int t = threadIdx.x, k0 = kc * TC_BK;
    const uint32_t ws = smem_u32(s->w[st]);
    const __nv_bfloat16* W = g.W + (int64_t)b * g.w_stride;
#pragma unroll
    for (int q = 0; q < BN * 8 / TC_THREADS; ++q) {
        const int i = t + TC_THREADS * q;
        const int j = i >> 3, c = i & 7;
        const int n = tc_wrow<EPI, BN>(g, n_tile, j);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ws + tc_off(j, c * 8)),
                     "l"(W + (int64_t)n * g.K + k0 + c * 8)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tc_wait_w() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int EPI, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc_gemm(GemmArgs g, int* err_flag) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    TcSmem<BN>* s = reinterpret_cast<TcSmem<BN>*>(tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023));
    const int b = blockIdx.z;
    const int m_valid = g.m_count ? g.m_count[b] : g.M;
    const int m0 = blockIdx.y * TC_BM;
    if (m0 >= m_valid) return;   // uniform over the CTA, before any TMEM allocation
    const int n_tile = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&s->mma_done[0], 1);
        mbar_init(&s->mma_done[1], 1);
        s->err = 0;
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
    uint32_t phase[2] = {0u, 0u};
    TcARegs ar;
    tc_issue_w<EPI, BN>(g, s, 0, b, n_tile, 0);
    tc_load_a(g, b, m0, m_valid, 0, ar);
    tc_store_a(s, 0, ar);
    for (int kc = 0; kc < nk; ++kc) {
        const int st = kc & 1;
        if (kc + 1 < nk) tc_load_a(g, b, m0, m_valid, kc + 1, ar);   // in flight during this chunk's MMAs
        tc_wait_w();
        tc_fence_proxy_async();   // this thread's smem writes (stores, cp.async) -> tensor-core reads
        __syncthreads();
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
        if (kc + 1 < nk) {
            // the other stage is free once the MMAs of chunk kc-1 completed
            if (kc >= 1) {
                if (!mbar_wait(&s->mma_done[st ^ 1], phase[st ^ 1])) s->err = 1;
                phase[st ^ 1] ^= 1u;
            }
            tc_issue_w<EPI, BN>(g, s, st ^ 1, b, n_tile, kc + 1);
            tc_store_a(s, st ^ 1, ar);
        }
    }
    // the last commit covers every MMA issued before it
    const int last = (nk - 1) & 1;
    if (!mbar_wait(&s->mma_done[last], phase[last])) s->err = 1;
    tc_fence_after();
    __syncthreads();
    if (s->err) {
        if (threadIdx.x == 0) atomicExch(err_flag, 1);
    } else {
        // epilogue: warp w holds rows 32w..32w+31 (lanes), 16 columns per load
        const int m = m0 + warp * 32 + lane;
        const bool row_ok = m < m_valid;
        float* C = g.C + (int64_t)b * g.c_stride;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        if (EPI == GEPI_SWIGLU) {
            const int n0 = n_tile * (BN / 2);
            for (int c = 0; c < BN / 2; c += 16) {
                float gt[16], up[16];
                tc_ld16(lane_addr + c, gt);
                tc_ld16(lane_addr + BN / 2 + c, up);
                if (row_ok)
#pragma unroll
                    for (int i = 0; i < 16; ++i) C[(int64_t)m * g.ldc + n0 + c + i] = siluf_(gt[i]) * up[i];
            }
        } else {
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tc_ld16(lane_addr + c, v);
                if (!row_ok) continue;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = n_tile * BN + c + i;
                    float y = v[i];
                    if (g.lora_b) {
                        float d = 0.f;
#pragma unroll
                        for (int q = 0; q < LORA_R; ++q)
                            d += g.lora_b[(int64_t)n * LORA_R + q] * g.lora_t[(int64_t)m * LORA_R + q];
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
