// Flash-decoding attention on the tensor cores for a bf16 KV cache: the same blocks, masks and
// split partials as the SIMT k_attn_flash (engine_kernels.cuh), for the per-op and many-row
// pulse passes (src/infer.py:290-306 per row: softmax(q k^T / 8) v over the row's visible keys).
//
// Block (split sp, kv head g, group of rpb rows). A group is cut into runs of consecutive rows
// of one slot at consecutive positions (a verify block); a run holds nq = rows x GQA query units
// (<= 32). Its keys are walked in chunks of 128 aligned to absolute multiples of 128 (a chunk
// never wraps a local layer's ring): chunks sp, sp + nsplit, ... Per chunk:
//   S^T = K Q^T   tcgen05.mma M = 128 (keys), N = 2 NQP (the units' Q hi rows, then their lo rows;
//                 NQP = 16 or 32), K = 64 (dims): A = the chunk's K rows as the cache stores them
//                 (K-major), B = the queries; a unit's score is the sum of its two columns
//   softmax       thread = (key, group of units): TMEM lane = key, the group's columns = units
//   O += P V      tcgen05.mma M = 128 (rows: P hi of the units, then P lo of the units at row
//                 8 RG + u; rows past them unused), N = 64 (dims), K = 128 (keys): A = P written
//                 by the softmax threads, B = the chunk's V rows (MN-major: the cache stores V
//                 key-major, dims contiguous); O stays in TMEM over the run, unit u's output is
//                 the sum of its rows u and 8 RG + u
//
// Roles. Warp 4G (one lane) is the producer: it issues the 2-D tensor-map loads of K and V
// (cp.async.bulk.tensor, box 64 x 128 rows, SWIZZLE_128B, this CTA only) into two 3-stage rings
// (a K stage is refilled once the score MMA that read it has completed, a V stage once its P.V
// has), and every MMA, each committed to an mbarrier. Warps 0 .. 4G-1 are G softmax groups of
// four warps (one per TMEM lane quadrant); group gi owns units [gi * UPG, gi * UPG + UPG).
//
// Softmax in base 2 with a lazy running maximum: the queries are pre-scaled by log2(e) / 8, and
// the weights of a chunk are p = 2^(s - m) for the unit's running maximum m. m is exchanged
// among a group's four warps only on a run's first chunk, or when a score exceeds m by more than
// 2^32 (then O, in TMEM, is rescaled in place by warps 0 and 1, which own TMEM lanes 0-63: the
// units' hi and lo rows);
// otherwise a chunk costs the softmax warps one barrier. The weights are exact for any m (they
// are relative to the same m in l and O); the partial's m goes out in natural-log units.
// Each thread keeps partial sums l; the block reduces them once per run.
//
// Keys past a row's position or before its window read whatever the cache holds there (the
// arena is zeroed when it is allocated, so the values are finite) and get weight exactly 0.
//
// Exactness: Q and P (fp32) enter the MMAs as bf16 hi + lo halves (|x - hi - lo| <= 2^-16 |x|)
// multiplied into the same fp32 accumulator; K and V are exact bf16.
//
// Shared-memory operands use the canonical K-major / MN-major SWIZZLE_128B layouts (rows of
// 128 B, 16-byte chunks permuted within each 8-row, 1024-byte atom). The P operand holds only
// the row groups of real units; the MMA's rows past them read other shared memory of the block
// and produce accumulator rows that nobody reads. Every wait is bounded; a wait that runs out
// raises a block-wide abort flag that ends every other wait, the block drains the copies and
// MMAs in flight (bounded again), raises the error flag and returns.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "kv.cuh"
#include "mega_ptx.cuh"
#include "tc_gemm.cuh"
#include "tma_gemm.cuh"

namespace pulsar {

constexpr int DT_CK = 128;      // keys per chunk (the score MMA's M)
constexpr int DT_STAGES = 3;    // stages of the K ring and of the V ring
constexpr float DT_TH = 32.f;   // lazy maximum: rescale when a score exceeds m by more than this (base 2)

template <int NU>
struct DtLayout {
    static constexpr int NQ = NU * GQA;              // query units of a full run
    static constexpr int NQP = NQ <= 16 ? 16 : 32;   // Q rows per half (the score MMA's N is 2 NQP)
    static constexpr int G = (NQ + 7) / 8;           // softmax groups
    static constexpr int UPG = (NQ + G - 1) / G;     // units per group (<= 8)
    static constexpr int THREADS = 128 * G + 32;     // softmax warps + the producer warp
    static constexpr int RG = (NQ + 7) / 8;          // 8-row groups of P that hold units
    static constexpr int LO = 8 * RG;                // P's (and O's) row of unit u's lo half: LO + u
    static constexpr uint32_t PKB = 2 * RG * 1024;   // one 64-key block of P: hi rows, then lo rows
    static constexpr uint32_t PBUF = 2 * PKB;        // two 64-key blocks
    static constexpr uint32_t P0 = 0;                // two P buffers (and, at a run's end, O's rows)
    static constexpr uint32_t Q_HI = 2 * PBUF, Q_LO = Q_HI + NQP * 128;
    static constexpr uint32_t KR = ((Q_LO + NQP * 128 + 1023) / 1024) * 1024;
    static constexpr uint32_t TILE = DT_CK * DH * 2;   // 128 rows of K or V: 16 KB
    static constexpr uint32_t VR = KR + DT_STAGES * TILE;
    static constexpr uint32_t BARS = VR + DT_STAGES * TILE;   // kfull[3] vfull[3] sdone[2] pready[2] odone[2] drain
    static constexpr uint32_t RED = BARS + 128;               // [unit][quadrant] floats
    static constexpr uint32_t SCL = RED + NQP * 4 * 4;        // per-unit rescale of O
    static constexpr uint32_t MISC = SCL + NQP * 4;           // abort flag, TMEM base
    static constexpr uint32_t BYTES = MISC + 16;
    // the P operand's MMA rows reach 16 KB past each 64-key block's start
    static_assert(P0 + PBUF + PKB + 16 * 1024 <= BYTES, "P operand rows must stay inside the block's shared memory");
    static_assert(UPG <= 8 && (G - 1) * UPG + 8 <= NQP, "a group's 8-column TMEM load stays inside the scores");
    static_assert(2 * LO * (DH + 1) * 4 <= 2 * PBUF, "O's rows fit the P buffers at a run's end");
    static_assert(8 * 13 <= RED - BARS && RED % 16 == 0 && KR % 1024 == 0 && VR % 1024 == 0 && Q_HI % 1024 == 0,
                  "the 13 mbarriers fit; float4 reads of red, tensor-map and swizzled destinations are aligned");
    // TMEM columns: S^T double buffer (hi products, then lo products: 2 NQP columns each), O
    static constexpr uint32_t TM_S = 0, TM_SB = 2 * NQP, TM_O = 4 * NQP;
    static constexpr uint32_t TM_COLS = NQP == 16 ? 128 : 256;
};

template <int NU>
constexpr size_t dt_smem_bytes() {
    return DtLayout<NU>::BYTES + 1024;
}

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, M = 128, N = n; B MN-major
// when b_mn (bit 16).
__host__ __device__ constexpr uint32_t dt_idesc(int n, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// Byte offset of element (row, k) (k < 64) in a K-major SWIZZLE_128B tile of 8-row atoms.
__device__ __forceinline__ uint32_t dt_sw_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) << 4) | ((k & 7) << 1)));
}

// 8 and 16 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void dt_ld8(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void dt_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void dt_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void dt_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void dt_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Row of the KV tensor map (rows of 64 elements over the whole arena) where (slot, head g,
// K or V) of this layer holds position k0 (k0 a multiple of 128: the chunk does not wrap).
__device__ __forceinline__ int dt_row(const KVLayer& L, int64_t lrow, int slot, int g, int isv, int k0) {
    return (int)(lrow + (int64_t)slot * (L.slot_stride / DH) + (int64_t)(isv * HKV + g) * L.cap + (k0 & L.mask));
}

// Eight bf16 of x[0..7] as hi and lo halves (|x - hi - lo| <= 2^-16 |x|).
__device__ __forceinline__ void dt_split8(const float* x, uint4& hi, uint4& lo) {
    __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        h[j] = __float2bfloat16(x[j]);
        l[j] = __float2bfloat16(x[j] - __bfloat162float(h[j]));
    }
    hi = *reinterpret_cast<const uint4*>(h);
    lo = *reinterpret_cast<const uint4*>(l);
}

__device__ __forceinline__ void dt_st128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void dt_sts16(uint32_t addr, __nv_bfloat16 v) {
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(__bfloat16_as_ushort(v)) : "memory");
}

// bar.red.or over named barrier 1 of the N softmax threads: true in every participant when v is
// true in any. (Barrier ids are immediates, so the kernel reserves only the ids it names.)
template <int N>
__device__ __forceinline__ bool dt_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(N)
        : "memory");
    return r != 0;
}
template <int N>
__device__ __forceinline__ void dt_bar_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}
// Barrier of softmax group gi's 128 threads (ids 2 .. 5).
__device__ __forceinline__ void dt_group_sync(int gi) {
    switch (gi) {
        case 0: asm volatile("bar.sync 2, 128;" ::: "memory"); break;
        case 1: asm volatile("bar.sync 3, 128;" ::: "memory"); break;
        case 2: asm volatile("bar.sync 4, 128;" ::: "memory"); break;
        default: asm volatile("bar.sync 5, 128;" ::: "memory"); break;
    }
}

// Bounded wait that also gives up once the block's abort flag is raised; a wait that runs out
// raises it.
__device__ __forceinline__ bool dt_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try(bar, parity)) {
        if (*abort) return false;
        if (globaltimer() - t0 > WAIT_NS) {
            *abort = 1;
            return false;
        }
    }
    return true;
}

template <int NU>
__global__ void __launch_bounds__(DtLayout<NU>::THREADS) k_attn_dec_tc(
    const __grid_constant__ CUtensorMap kvmap, const int4* __restrict__ rows, int R, int rpb, const float* __restrict__ q,
    KVLayer L, int64_t lrow, int is_local, int nsplit, float* __restrict__ part, int max_pos, int n_slots, int* err) {
    using Lay = DtLayout<NU>;
    constexpr int NQP = Lay::NQP, G = Lay::G, UPG = Lay::UPG, NSM = 128 * G;   // NSM: softmax threads
    constexpr uint32_t idS = dt_idesc(2 * NQP, false), idO = dt_idesc(DH, true);
    extern __shared__ __align__(1024) unsigned char dt_raw[];
    unsigned char* sm = dt_raw + ((1024 - (smem_u32(dt_raw) & 1023)) & 1023);
    const uint32_t sb = smem_u32(sm);
    uint64_t* kfull = reinterpret_cast<uint64_t*>(sm + Lay::BARS);
    uint64_t* vfull = kfull + DT_STAGES;
    uint64_t* sdone = vfull + DT_STAGES;
    uint64_t* pready = sdone + 2;
    uint64_t* odone = pready + 2;
    uint64_t* drain = odone + 2;
    float* red = reinterpret_cast<float*>(sm + Lay::RED);   // [unit][quadrant]
    float* scl = reinterpret_cast<float*>(sm + Lay::SCL);   // per unit: O's rescale, then the run's maximum
    volatile int* abort = reinterpret_cast<volatile int*>(sm + Lay::MISC);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + Lay::MISC + 4);
    const int sp = blockIdx.x, g = blockIdx.y;
    const int rb0 = blockIdx.z * rpb, rb1 = min(R, rb0 + rpb);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool producer = warp == 4 * G;
    const int gi = warp >> 2, qd = warp & 3;   // softmax group, TMEM lane quadrant
    const int key = qd * 32 + lane;           // a softmax thread's key within a chunk (its TMEM lane)
    const int u0 = gi * UPG;                  // the group's first unit
    auto bad_row = [&](const int4& rw) { return rw.y < 0 || rw.y >= max_pos || rw.x < 0 || rw.x >= n_slots; };
    if (tid == 0) {
        for (int i = 0; i < DT_STAGES; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&vfull[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sdone[i], 1);
            mbar_init(&pready[i], 4 * G);
            mbar_init(&odone[i], 1);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (producer && lane == 0)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kvmap)) : "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(Lay::TM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // the producer's copies issued and waited for, counted over the block's runs (drained on abort)
    int kiss = 0, kwt = 0, viss = 0, vwt = 0;
    int gbase = 0;   // chunks of the block's earlier runs
    bool stop = false;
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
        const int posF = first.y;
        const int c0 = is_local ? (max(0, posF - WINDOW + 1) & ~(DT_CK - 1)) : 0;
        const int nchunks = bad_row(first) ? 0 : (posF + nr - 1 - c0) / DT_CK + 1;
        const int mine = nchunks > sp ? (nchunks - sp + nsplit - 1) / nsplit : 0;
        auto chunk_k0 = [&](int j) { return c0 + (sp + j * nsplit) * DT_CK; };
        if (producer) {
            if (lane == 0)
                for (int j = 0; j < min(DT_STAGES, mine); ++j) {
                    const int st = (gbase + j) % DT_STAGES, k0 = chunk_k0(j);
                    mbar_arrive_expect_tx(&kfull[st], Lay::TILE);
                    tma_load_2d(sm + Lay::KR + st * Lay::TILE, &kvmap, 0, dt_row(L, lrow, first.x, g, 0, k0), &kfull[st]);
                    mbar_arrive_expect_tx(&vfull[st], Lay::TILE);
                    tma_load_2d(sm + Lay::VR + st * Lay::TILE, &kvmap, 0, dt_row(L, lrow, first.x, g, 1, k0), &vfull[st]);
                    ++kiss;
                    ++viss;
                }
        } else {
            // the run's queries: unit u = row u / GQA, head g * GQA + u % GQA, scaled by log2(e) / 8
            for (int i = tid; i < NQP * 8; i += NSM) {
                const int u = i >> 3, c = i & 7;
                float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (u < nq) {
                    const float4* src = reinterpret_cast<const float4*>(
                        q + ((int64_t)(s0 + u / GQA) * H + g * GQA + u % GQA) * DH + 8 * c);
                    const float4 a = src[0], b = src[1];
                    constexpr float QS = 0.18033688f;   // log2(e) / 8
                    x[0] = a.x * QS; x[1] = a.y * QS; x[2] = a.z * QS; x[3] = a.w * QS;
                    x[4] = b.x * QS; x[5] = b.y * QS; x[6] = b.z * QS; x[7] = b.w * QS;
                }
                uint4 hi, lo;
                dt_split8(x, hi, lo);
                dt_st128(sb + Lay::Q_HI + dt_sw_off(u, 8 * c), hi);
                dt_st128(sb + Lay::Q_LO + dt_sw_off(u, 8 * c), lo);
            }
            tc_fence_proxy_async();   // the queries are read by the tensor cores
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (producer) {
            if (lane == 0 && mine > 0) {
                auto mma_s = [&](int c) {   // S^T of chunk c (its K has landed)
                    const uint32_t kt = sb + Lay::KR + (uint32_t)(c % DT_STAGES) * Lay::TILE;
#pragma unroll
                    for (int ks = 0; ks < DH / 16; ++ks)   // B: the Q hi rows, then (contiguous) the lo rows
                        tc_mma(tmem + Lay::TM_S + Lay::TM_SB * (c & 1), tc_desc_sw128(kt + ks * 32),
                               tc_desc_sw128(sb + Lay::Q_HI + ks * 32), idS, ks > 0 ? 1u : 0u);
                    tc_commit(&sdone[c & 1]);
                };
                bool ok = dt_wait(&kfull[gbase % DT_STAGES], (gbase / DT_STAGES) & 1, abort);
                if (ok) {
                    ++kwt;
                    mma_s(gbase);
                }
                for (int j = 0; ok && j < mine; ++j) {
                    const int c = gbase + j;
                    // the next chunk's scores (its S buffer was read by the softmax of chunk c - 1,
                    // whose P is ready)
                    if (j + 1 < mine) {
                        if (!(ok = dt_wait(&kfull[(c + 1) % DT_STAGES], ((c + 1) / DT_STAGES) & 1, abort))) break;
                        ++kwt;
                        mma_s(c + 1);
                    }
                    // this chunk's P.V into O once its P is written
                    if (!(ok = dt_wait(&pready[c & 1], (c >> 1) & 1, abort))) break;
                    tc_fence_after();
                    if (!(ok = dt_wait(&vfull[c % DT_STAGES], (c / DT_STAGES) & 1, abort))) break;
                    ++vwt;
                    const uint32_t pa = sb + Lay::P0 + (uint32_t)(c & 1) * Lay::PBUF;
                    const uint32_t vt = sb + Lay::VR + (uint32_t)(c % DT_STAGES) * Lay::TILE;
#pragma unroll
                    for (int ks = 0; ks < DT_CK / 16; ++ks)
                        tc_mma(tmem + Lay::TM_O, tc_desc_sw128(pa + (uint32_t)(ks >> 2) * Lay::PKB + (ks & 3) * 32),
                               tc_desc_sw128(vt + ks * 2048), idO, (j > 0 || ks > 0) ? 1u : 0u);
                    tc_commit(&odone[c & 1]);
                    // refills: chunk c's K stage (its scores were read before P was ready) takes
                    // chunk c + 3; chunk c - 1's V stage, once its P.V has completed, chunk c + 2
                    if (j + DT_STAGES < mine) {
                        const int st = c % DT_STAGES;
                        mbar_arrive_expect_tx(&kfull[st], Lay::TILE);
                        tma_load_2d(sm + Lay::KR + st * Lay::TILE, &kvmap, 0,
                                    dt_row(L, lrow, first.x, g, 0, chunk_k0(j + DT_STAGES)), &kfull[st]);
                        ++kiss;
                    }
                    if (j >= 1 && j + DT_STAGES - 1 < mine) {
                        if (!(ok = dt_wait(&odone[(c - 1) & 1], ((c - 1) >> 1) & 1, abort))) break;
                        const int st = (c - 1) % DT_STAGES;
                        mbar_arrive_expect_tx(&vfull[st], Lay::TILE);
                        tma_load_2d(sm + Lay::VR + st * Lay::TILE, &kvmap, 0,
                                    dt_row(L, lrow, first.x, g, 1, chunk_k0(j + DT_STAGES - 1)), &vfull[st]);
                        ++viss;
                    }
                }
                // every MMA of the run has completed before the run ends
                if (ok) dt_wait(&odone[(gbase + mine - 1) & 1], ((gbase + mine - 1) >> 1) & 1, abort);
            }
            __syncwarp();
        } else {
            float m_est[UPG], l_t[UPG];
#pragma unroll
            for (int k = 0; k < UPG; ++k) {
                m_est[k] = -INFINITY;
                l_t[k] = 0.f;
            }
            bool aborted = false;
            for (int j = 0; j < mine; ++j) {
                const int c = gbase + j, b = c & 1;
                bool bad = !dt_wait(&sdone[b], (c >> 1) & 1, abort);
                __syncwarp();   // tcgen05.ld is warp-collective
                tc_fence_after();
                uint32_t sr[8], srl[8];
                const uint32_t scol = tmem + ((uint32_t)(qd * 32) << 16) + Lay::TM_S + Lay::TM_SB * b + u0;
                dt_ld8(scol, sr);
                dt_ld8(scol + NQP, srl);
                dt_ld_wait();
                const int kpos = chunk_k0(j) + key;
                float s[UPG];
                bool need = bad;
#pragma unroll
                for (int k = 0; k < UPG; ++k) {
                    const int u = u0 + k;
                    s[k] = -INFINITY;
                    if (u < nq) {
                        const int pos = posF + u / GQA;
                        const int lor = is_local ? max(0, pos - WINDOW + 1) : 0;
                        if (kpos <= pos && kpos >= lor) {
                            s[k] = __uint_as_float(sr[k]) + __uint_as_float(srl[k]);
                            need |= m_est[k] == -INFINITY || s[k] - m_est[k] > DT_TH;
                        }
                    }
                }
                tc_fence_before();   // S is read before the producer's next MMA into its buffer
                if (dt_bar_or<NSM>(need || *abort)) {
                    // the group's maxima over the chunk's 128 keys; l and O rescaled to them
#pragma unroll
                    for (int k = 0; k < UPG; ++k) {
                        const float wm = warp_max(s[k]);
                        if (lane == 0 && u0 + k < NQP) red[(u0 + k) * 4 + qd] = wm;
                    }
                    dt_group_sync(gi);
#pragma unroll
                    for (int k = 0; k < UPG; ++k) {
                        const int u = u0 + k;
                        float sc = 1.f;
                        if (u < nq) {
                            const float4 r4 = *reinterpret_cast<const float4*>(&red[u * 4]);
                            const float mn = fmaxf(m_est[k], fmaxf(fmaxf(r4.x, r4.y), fmaxf(r4.z, r4.w)));
                            sc = (m_est[k] == -INFINITY) ? 0.f : exp2f(m_est[k] - mn);
                            l_t[k] *= sc;
                            m_est[k] = mn;
                        }
                        if (qd == 0 && lane == k && u < NQP) scl[u] = sc;
                    }
                    if (dt_bar_or<NSM>(bad || *abort)) {   // also publishes scl to warp 0
                        aborted = true;
                        break;
                    }
                    if (warp < (2 * Lay::LO + 31) / 32 && j > 0) {
                        // O's rows (TMEM lanes: unit u's hi half at u, lo half at LO + u) after the
                        // previous chunk's P.V, times the unit's rescale; warps 0 and 1 own lanes 0-63
                        const bool ok = __all_sync(0xffffffffu, dt_wait(&odone[(c - 1) & 1], ((c - 1) >> 1) & 1, abort));
                        tc_fence_after();
                        if (ok) {
                            const int row = warp * 32 + lane, u = row < Lay::LO ? row : row - Lay::LO;
                            const float f = (row < 2 * Lay::LO && u < nq) ? scl[u] : 1.f;
                            const uint32_t orow = tmem + ((uint32_t)(warp * 32) << 16) + Lay::TM_O;
#pragma unroll
                            for (int cc = 0; cc < DH / 16; ++cc) {
                                uint32_t r[16];
                                dt_ld16(orow + 16 * cc, r);
                                dt_ld_wait();
#pragma unroll
                                for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
                                dt_st16(orow + 16 * cc, r);
                            }
                            dt_st_wait();
                        }
                    }
                }
                // the weights into P (buffer b: its last reader, the P.V of chunk c - 2, has completed)
                if (j >= 2) bad |= !dt_wait(&odone[b], ((c - 2) >> 1) & 1, abort);
                const uint32_t pb = sb + Lay::P0 + (uint32_t)b * Lay::PBUF + (uint32_t)(key >> 6) * Lay::PKB;
#pragma unroll
                for (int k = 0; k < UPG; ++k) {
                    const int u = u0 + k;
                    if (u < nq) {
                        const float p = (s[k] == -INFINITY) ? 0.f : exp2f(s[k] - m_est[k]);
                        l_t[k] += p;
                        const __nv_bfloat16 ph = __float2bfloat16(p);
                        const __nv_bfloat16 pl = __float2bfloat16(p - __bfloat162float(ph));
                        dt_sts16(pb + dt_sw_off(u, key & 63), ph);
                        dt_sts16(pb + dt_sw_off(Lay::LO + u, key & 63), pl);
                    }
                }
                tc_fence_proxy_async();   // P is read by the tensor cores
                tc_fence_before();        // and the rescale of O is ordered before the next P.V
                __syncwarp();
                if (lane == 0) mbar_arrive(&pready[b]);
            }
            // the run's partials: l summed over the group's four warps; O's rows (TMEM lanes
            // 0 .. 2 LO - 1, owned by warps 0 and 1) staged as [row][65] floats in the P buffers
            // (free once every P.V has completed); (m, l, o) of unit u by lane u of warp 0
#pragma unroll
            for (int k = 0; k < UPG; ++k) {
                const int u = u0 + k;
                if (u < nq) {
                    const float v = warp_sum(l_t[k]);
                    if (lane == 0) red[u * 4 + qd] = v;
                    if (qd == 0 && lane == 0) scl[u] = m_est[k];
                }
            }
            float* ost = reinterpret_cast<float*>(sm + Lay::P0);
            if (warp < (2 * Lay::LO + 31) / 32) {
                const bool ok = __all_sync(0xffffffffu, mine > 0 && !aborted &&
                                                            dt_wait(&odone[(gbase + mine - 1) & 1],
                                                                    ((gbase + mine - 1) >> 1) & 1, abort));
                tc_fence_after();
                const int row = warp * 32 + lane;
                const uint32_t orow = tmem + ((uint32_t)(warp * 32) << 16) + Lay::TM_O;
#pragma unroll
                for (int cc = 0; cc < DH / 16; ++cc) {
                    uint32_t r[16];
                    if (ok) {
                        dt_ld16(orow + 16 * cc, r);
                        dt_ld_wait();
                    }
                    if (row < 2 * Lay::LO)
#pragma unroll
                        for (int i = 0; i < 16; ++i) ost[row * (DH + 1) + 16 * cc + i] = ok ? __uint_as_float(r[i]) : 0.f;
                }
            }
            dt_bar_sync<NSM>();
            if (warp == 0 && lane < nq) {
                float* out = part + (((int64_t)(s0 + lane / GQA) * H + g * GQA + lane % GQA) * nsplit + sp) * PART;
                const float m = mine > 0 ? scl[lane] : -INFINITY;
                const float4 r4 = *reinterpret_cast<const float4*>(&red[lane * 4]);
                out[0] = m == -INFINITY ? -INFINITY : m * 0.69314718f;   // base 2 -> natural log
                out[1] = m == -INFINITY ? 0.f : (r4.x + r4.y) + (r4.z + r4.w);
                const float* oh = ost + lane * (DH + 1);
                const float* ol = ost + (Lay::LO + lane) * (DH + 1);
                float2* o2 = reinterpret_cast<float2*>(out + 2);
#pragma unroll 8
                for (int d = 0; d < DH / 2; ++d) o2[d] = make_float2(oh[2 * d] + ol[2 * d], oh[2 * d + 1] + ol[2 * d + 1]);
            }
        }
        // end of the run: every MMA of it has completed; red, scl and the queries are free
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (*abort) {
            stop = true;
            break;
        }
        gbase += mine;
        s0 = s1;
    }
    if (stop && producer && lane == 0) {
        // drain: the copies issued but not yet seen, then every MMA issued
        for (int c = kwt; c < kiss; ++c) mbar_wait(&kfull[c % DT_STAGES], (c / DT_STAGES) & 1);
        for (int c = vwt; c < viss; ++c) mbar_wait(&vfull[c % DT_STAGES], (c / DT_STAGES) & 1);
        tc_commit(drain);
        mbar_wait(drain, 0);
        atomicExch(err, 1);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Lay::TM_COLS) : "memory");
}

}  // namespace pulsar
