// Persistent per-pulse decode kernel (one CTA per SM, cooperative launch).
//
// One launch runs a whole pulse pass (src/infer.py:463-524) for R <= MEGA_RMAX rows: the
// pulse input, 8 layers x 6 phases separated by grid barriers, the end-of-pulse residual,
// the final norm and, when logits or argmax are requested, the LM head with argmax.
//
// Warp 0 is the producer: one lane streams every weight tile this CTA will consume, in
// consumption order, through a ring of NS 8 KB shared-memory slots with 1-D TMA bulk copies
// (cp.async.bulk + mbarrier complete_tx). Weights do not depend on activations, so the
// producer runs ahead across grid barriers (only the routed-expert tiles wait for this
// layer's router, computed from a flag in shared memory). Warps 1..15 are consumers: tile t
// of the CTA's stream lives in slot t % NS and is consumed by warp t % 15.
//
// Phases per layer (work split evenly over the CTAs, outputs owned by one CTA each; h rows
// [own0, own1) of every sequence row are owned by one CTA, kept in its shared memory):
//   A  xn = RMSNorm(h); QKV GEMV rows (with a live loop adapter every CTA first computes
//      t = A xn from the 24 fp32 A rows streamed through the ring, and the QKV rows add Bs t;
//      phase C does the same for Wo on the attention output)
//   B  gate logits xn.Wg + b on the last 8 CTAs (which usually have no attention item);
//      attention items (sequence block, kv head, key chunk): q of the 4 heads via
//      QK-RMSNorm + RoPE (+YaRN); block rows' K/V produced (norm, RoPE, value residual)
//      and written to the cache by the item that owns their chunk; the cached keys of the
//      chunk arrive through the weight ring for passes of <= 2 rows (issued during phase A);
//      split-K partials (m, l, o[64]) per query head and chunk
//   B2 one CTA per (row, query head) merges its chunk partials in a fixed order and applies
//      the gate sigmoid
//   C  Wo GEMV, h += (owned rows); partial router logits of the owned rows
//      z[r][e] = sum_o router[e][o] * mlp_norm[o] * h[r][o]
//   D  m = RMSNorm(h); router logits = (sum of the CTAs' z in CTA order) / rms(h) (every
//      CTA, identical result); top-4; shared + routed (distinct experts) gate/up GEMVs with
//      the SwiGLU epilogue
//   E  shared + routed down GEMVs for owned output rows, combine in top-k order, h +=
// Then: h_out = h_in + (h - h_in) * res_scale, final RMSNorm, LM head rows, argmax.
#pragma once

#include "kv.cuh"
#include "mega_ptx.cuh"

namespace pulsar {

constexpr int MEGA_THREADS = 512;
constexpr int MEGA_NCW = 15;              // consumer warps
constexpr int MEGA_NCT = MEGA_NCW * 32;   // consumer threads
constexpr int MEGA_NS = 18;               // ring slots
constexpr int MEGA_SLOT = 8192;           // bytes per slot
constexpr int MEGA_RMAX = 5;              // rows per pass
constexpr int MEGA_XS = MEGA_RMAX * 3072; // floats: act_sh [R][1024] + act_r [R][4][512]
constexpr int MEGA_STAGE = 2048;          // floats
constexpr int MEGA_CHUNK = 64;            // keys per attention item
constexpr int MEGA_MAXPAIRS = 64;         // phase-D output pairs per CTA (>= ceil((1024+16*512)/C))
constexpr int MEGA_MAXOROWS = 8;          // phase-E output rows per CTA (>= ceil(1024/C))

struct MegaArgs {
    int R, pulse, n_slots, max_pos, V, use_conv, base_seq_len;
    float eps, softcap;
    const int4* rows;
    const __nv_bfloat16 *wqkv[NL], *wo[NL], *sh_gu[NL], *sh_dn[NL], *r_gu[NL], *r_dn[NL];
    const float *attn_norm[NL], *mlp_norm[NL], *qn[NL], *kn[NL], *gate_w[NL], *gate_b[NL], *router[NL], *ebias[NL],
        *rscale[NL];
    // loop adapter (null: none): A [LORA_R][D] and Bs [d_out][LORA_R] of wqkv and wo for this pulse
    const float *la_qkv[NL], *lb_qkv[NL], *la_wo[NL], *lb_wo[NL];
    float vres[NL];
    KVLayer kvl[NL];
    const __nv_bfloat16* emb;
    const float *anchor, *stem, *step, *psn, *rg_down, *rg_up, *rg_bias, *res_scale, *fnorm;
    const float *cos_l, *sin_l, *cos_g, *sin_g;
    const float* h_prev;
    const float* h0n_in;
    float *h_out, *h0n_out, *logits;
    int hstride;          // row stride (rows of D floats) of h_out and h0n_out
    int* amax;
    // global workspace
    float *h, *h_in, *qkv, *gate, *att, *act_sh, *act_r, *part, *vfirst, *g8, *pmax;
    float* rpart;         // router partial sums [grid][R][E] of the owned h rows (phase C)
    int* pidx;
    int nch_max;          // chunks per (row, head) in `part`
    unsigned* bar;        // grid barrier counter (zeroed before launch)
    unsigned* tickets;    // [MEGA_RMAX * HKV + 2]: [.. + 0] argmax ticket, [.. + 1] exit count (both self-resetting)
    int* err;             // error flag (non-zero: a bounded wait ran out)
    unsigned long long wait_ns;   // bound of every wait
    int stall_cta;        // test hook: this CTA (>= 0) waits at its first grid barrier for a count never reached
    unsigned long long* experts;   // running count of distinct routed experts streamed (per layer)
    const int* skip;      // optional: non-zero -> the whole pass is skipped (every row exited early)
    unsigned long long* trace;   // optional [gridDim][MEGA_TRACE] %globaltimer stamps (null: off)
};

constexpr int MEGA_TRACE = 256;   // stamps per CTA: [0] start, [1 + 16*l + j] phase points of layer l, [255] end

struct MegaSmem {
    uint64_t full[MEGA_NS];
    uint64_t empty[MEGA_NS];
    float logits[MEGA_RMAX][E];   // router: score + bias per (row, expert)
    float rsg[MEGA_RMAX][E];      // router: sigmoid score per (row, expert)
    float wts[MEGA_RMAX][TOPK];
    int idx[MEGA_RMAX][TOPK];
    int elist[E];
    unsigned rmask[MEGA_RMAX];   // experts chosen by each row (bit mask)
    int n_e;
    volatile int moe_ready;
    int ticket;
    int abort;
    alignas(128) unsigned char ring[MEGA_NS][MEGA_SLOT];
    alignas(16) float xs[MEGA_XS];
    alignas(16) float stage[MEGA_STAGE];
    float wout[MEGA_NCW][4 * MEGA_RMAX];   // per-warp reduced tile sums
    int xoff[MEGA_RMAX];                   // X row offsets (elements into xs) of the current phase
    int xoff_e[E][MEGA_RMAX];              // phase E: per routed expert, act_r row of each row or -1
    int eslot[MEGA_RMAX][TOPK];            // phase E: position of expert idx[r][k] in the expert list
    int blk_r0[MEGA_RMAX + 1];             // sequence blocks of the rows: start row
    int blk_nch[MEGA_RMAX];                // attention chunks per (block, head group)
    int blk_chunk[MEGA_RMAX];
    int n_blk;
    int4 rows[MEGA_RMAX];                  // the row descriptors (read everywhere; L1 holds little here)
    float rwn[NL][E][MEGA_MAXOROWS];       // router weight x mlp-norm weight of the owned h rows
    float hown[MEGA_MAXOROWS * MEGA_RMAX]; // owned h rows [row - o0][R] (this CTA is their only writer)
    float rinv[MEGA_RMAX];                 // 1 / rms of h per row (phase D)
    float nred[D / 128];                   // norm_rows (one row): sums of squares of the 128-element slices
    float rsc[NL][MEGA_MAXOROWS];          // routed_scale of the owned h rows
    float ebias[NL][E];                    // expert bias of every layer (router top-k)
    float rope[2][MEGA_RMAX][DH];          // [local, global][row]: cos (32) then sin (32) at the row's position
    alignas(16) float lt[MEGA_RMAX * LORA_R];   // loop-adapter factor t = A x of the current GEMV
};

__device__ __forceinline__ void stamp(const MegaArgs& a, int l, int j) {
    if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 1 + 16 * l + j] = globaltimer();
}

// router-phase sub-steps of layer l (entries 206 + 5*l + k, k < 5)
__device__ __forceinline__ void rstamp(const MegaArgs& a, int l, int k) {
    if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 206 + 5 * l + k] = globaltimer();
}

// attention-item sub-steps of the first item a CTA runs in layer l (entries 130 + 8*l + k)
__device__ __forceinline__ void astamp(const MegaArgs& a, int l, int k, bool first) {
    if (first && a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 130 + 8 * l + k] = globaltimer();
}

__device__ __forceinline__ void rows_split(int N, int c, int C, int& r0, int& r1) {
    r0 = (int)(((long long)N * c) / C);
    r1 = (int)(((long long)N * (c + 1)) / C);
}

// ------------------------------------------------------------------ tile stream
// The producer and the consumers walk the same sequence of tiles; `Ring` keeps the counter.
struct Ring {
    MegaSmem* s;
    uint32_t t;     // tiles so far
    int warp;       // consumer warp index (0..14), or -1 for the producer
    bool ok;
    unsigned long long wait_ns;   // bound of each wait
};

// Bounded mbarrier wait that also gives up once the CTA has aborted. try_wait suspends the
// waiting thread until the phase completes or a hardware time limit passes, so waiting warps do
// not take issue slots from the warps that compute.
__device__ __forceinline__ bool ring_wait(const Ring& g, uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try(bar, parity))
        if (g.s->abort || globaltimer() - t0 > g.wait_ns) return false;
    return true;
}

// Producer side: issue tiles covering rows [r0, r1) of a row-major matrix with row_bytes
// bytes per row, rows_per_tile rows per tile.
__device__ __forceinline__ void produce_rows(Ring& g, const void* base, int row_bytes, int r0, int r1,
                                             int rows_per_tile) {
    for (int r = r0; r < r1 && g.ok; r += rows_per_tile) {
        const int n = min(rows_per_tile, r1 - r);
        const uint32_t slot = g.t % MEGA_NS;
        const uint32_t use = g.t / MEGA_NS;
        if (use > 0 && !ring_wait(g, &g.s->empty[slot], (use - 1) & 1)) { g.ok = false; break; }
        const uint32_t bytes = (uint32_t)n * row_bytes;
        mbar_arrive_expect_tx(&g.s->full[slot], bytes);
        tma_load_1d(g.s->ring[slot], static_cast<const char*>(base) + (int64_t)r * row_bytes, bytes, &g.s->full[slot]);
        ++g.t;
    }
}

// Consumer side: for each tile of the same range, if this warp owns it, wait for it and call
// fn(tile_smem, first_row, n_rows); then release the slot.
template <typename F>
__device__ __forceinline__ void consume_rows(Ring& g, int r0, int r1, int rows_per_tile, F&& fn) {
    const int lane = threadIdx.x & 31;
    for (int r = r0; r < r1; r += rows_per_tile) {
        const int n = min(rows_per_tile, r1 - r);
        const uint32_t slot = g.t % MEGA_NS;
        const uint32_t use = g.t / MEGA_NS;
        if ((int)(g.t % MEGA_NCW) == g.warp && g.ok) {
            if (!ring_wait(g, &g.s->full[slot], use & 1)) {
                g.ok = false;
            } else {
                fn(g.s->ring[slot], r, n);
                __syncwarp();
                if (lane == 0) mbar_arrive(&g.s->empty[slot]);
            }
        }
        ++g.t;
    }
}

// ------------------------------------------------------------------ warp GEMV on a tile
// out[i*R + r] = sum_k W[i][k] X_r[k] for tile rows i < nr (nr <= 4) with bf16 weights and
// fp32 X rows in shared memory (X_r = xbase + xoff[r]; xoff[r] < 0: a zero row). Lane l
// covers the elements seg*256 + j*128 + 4l + q (j < 2, q < 4): conflict-free 8-byte /
// 16-byte shared loads. Not inlined: one copy per (R, KD) keeps the persistent kernel's
// code inside the instruction cache.
template <int R, int KD>
__device__ __noinline__ void tile_gemv(const __nv_bfloat16* w, int nr, const float* xbase, const int* xoff, float* out) {
    const int lane = threadIdx.x & 31;
    float acc[4][R];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[i][r] = 0.f;
    int xo[R];
#pragma unroll
    for (int r = 0; r < R; ++r) xo[r] = xoff[r];
#pragma unroll 1
    for (int seg = 0; seg < KD / 256; ++seg) {
        float x[R][8];
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (xo[r] >= 0) v = *reinterpret_cast<const float4*>(xbase + xo[r] + seg * 256 + j * 128 + lane * 4);
                x[r][j * 4 + 0] = v.x; x[r][j * 4 + 1] = v.y; x[r][j * 4 + 2] = v.z; x[r][j * 4 + 3] = v.w;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (i < nr) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint2 u = *reinterpret_cast<const uint2*>(w + (int64_t)i * KD + seg * 256 + j * 128 + lane * 4);
                    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
                    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[i][r] += a.x * x[r][j * 4] + a.y * x[r][j * 4 + 1] + b.x * x[r][j * 4 + 2] + b.y * x[r][j * 4 + 3];
                }
            }
        }
    }
    // reduce-scatter of the 4R sums over the warp (P = 4R rounded up to a power of two):
    // P - 1 + 5 - log2(P) shuffles instead of 5 per sum; lane L ends with sum L >> (5 - log2 P)
    constexpr int P = (4 * R <= 4) ? 4 : (4 * R <= 8) ? 8 : (4 * R <= 16) ? 16 : 32;
    constexpr int LP = (P == 4) ? 2 : (P == 8) ? 3 : (P == 16) ? 4 : 5;
    float x[P];
#pragma unroll
    for (int v = 0; v < P; ++v) x[v] = (v < 4 * R) ? acc[v / R][v % R] : 0.f;
#pragma unroll
    for (int st = 0; st < LP; ++st) {
        const int o = 16 >> st, half = P >> (st + 1);
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < half; ++j) {
            const float send = upper ? x[j] : x[j + half];
            const float keep = upper ? x[j + half] : x[j];
            x[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
#pragma unroll
    for (int o = 16 >> LP; o >= 1; o >>= 1) x[0] += __shfl_xor_sync(0xffffffffu, x[0], o);
    const int v = lane >> (5 - LP);
    if ((lane & ((1 << (5 - LP)) - 1)) == 0 && v < 4 * R) out[v] = x[0];
    __syncwarp();
}

// fp32 rows (router), two rows per tile; same element mapping, float4 weight loads.
template <int R>
__device__ __noinline__ void tile_gemv_f32(const float* w, int nr, const float* xbase, const int* xoff, float* out) {
    const int lane = threadIdx.x & 31;
    float acc[2][R];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[i][r] = 0.f;
#pragma unroll 1
    for (int seg = 0; seg < 4; ++seg) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int k = seg * 256 + j * 128 + lane * 4;
            float4 xv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) xv[r] = *reinterpret_cast<const float4*>(xbase + xoff[r] + k);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (i < nr) {
                    const float4 wv = *reinterpret_cast<const float4*>(w + i * D + k);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        acc[i][r] += wv.x * xv[r].x + wv.y * xv[r].y + wv.z * xv[r].z + wv.w * xv[r].w;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float v = warp_sum(acc[i][r]);
            if (lane == i * R + r) out[lane] = v;
        }
    __syncwarp();
}

// ------------------------------------------------------------------ loop adapter
// t[r][j] = A[j] . X_r for the 24 fp32 adapter rows streamed through the ring (two per tile) and
// the current GEMV input rows of xs, into s->lt; every CTA computes it (no exchange).
template <int R>
__device__ __forceinline__ void adapter_t(Ring& g, MegaSmem* s, float* wo_) {
    const int lane = threadIdx.x & 31;
    consume_rows(g, 0, LORA_R, 2, [&](const unsigned char* tile, int row0, int n) {
        tile_gemv_f32<R>(reinterpret_cast<const float*>(tile), n, s->xs, s->xoff, wo_);
        if (lane < n * R) s->lt[(lane % R) * LORA_R + row0 + lane / R] = wo_[lane];
    });
    named_bar_sync(1, MEGA_NCT);
}

// The adapter's correction Bs[o] . t of output row o (terms in order, as the per-op GEMV adds them).
__device__ __forceinline__ float adapter_corr(const float* bs, int o, const float* t) {
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < LORA_R; ++j) d += __ldg(bs + (int64_t)o * LORA_R + j) * t[j];
    return d;
}

// ------------------------------------------------------------------ grid barrier (consumers)
__device__ __forceinline__ bool grid_sync(const MegaArgs& a, MegaSmem* s, unsigned& epoch) {
    named_bar_sync(1, MEGA_NCT);
    if (threadIdx.x == 32) {
        epoch += 1;
        // release (cumulative over the CTA's writes ordered before it by the bar.sync above)
        red_release_gpu_add(a.bar, 1u);
        // test hook: the stalled CTA waits at its first barrier for a count the grid never reaches
        // (the others stop at the next barrier, one arrival short), so its bounded wait runs out
        const unsigned target = ((int)blockIdx.x == a.stall_cta && epoch == 1) ? ~0u : epoch * gridDim.x;
        bool ok = true;
        // one acquire poll at a time; the global error flag costs an L2 round trip of its own,
        // so it is read every 64th poll only (more polls in flight measured slower: they
        // contend with the arrivals at the counter's L2 slice)
        if (ld_acquire_gpu(a.bar) < target) {
            const unsigned long long t0 = globaltimer();
            for (unsigned it = 1; ld_acquire_gpu(a.bar) < target; ++it) {
                __nanosleep(20);
                if (globaltimer() - t0 > a.wait_ns || ((it & 63) == 0 && *(volatile int*)a.err)) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) {
            atomicExch(a.err, 1);
            s->abort = 1;
        }
    }
    named_bar_sync(1, MEGA_NCT);
    return s->abort == 0;
}

// RMSNorm of R rows (global, [R][1024]) into dst with weight w; 1/rms of row r goes to rinv[r]
// when rinv is given. One row: every consumer thread loads float4 pieces (all loads in flight
// at once), warps reduce their 128-element slices, the eight slice sums are added in order
// from shared memory (red: 8 floats). More rows (register pressure): one warp per row.
template <int R>
__device__ __forceinline__ void norm_rows(const float* src, const float* w, float eps, float* dst, float* red,
                                          float* rinv = nullptr) {
    const int lane = threadIdx.x & 31;
    if constexpr (R == 1) {
        const int tid = threadIdx.x - 32;
        constexpr int N4 = D / 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f), wv = v;
        if (tid < N4) {
            v = __ldcg(reinterpret_cast<const float4*>(src) + tid);   // written by other CTAs: bypass L1
            wv = __ldg(reinterpret_cast<const float4*>(w) + tid);
            const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);   // warp-uniform branch
            if (lane == 0) red[tid / 32] = ss;
        }
        named_bar_sync(1, MEGA_NCT);
        if (tid < N4) {
            float t = 0.f;
#pragma unroll
            for (int j = 0; j < D / 128; ++j) t += red[j];
            const float inv = rsqrtf(t / (float)D + eps);
            if (rinv && tid == 0) rinv[0] = inv;
            reinterpret_cast<float4*>(dst)[tid] =
                make_float4(wv.x * (v.x * inv), wv.y * (v.y * inv), wv.z * (v.z * inv), wv.w * (v.w * inv));
        }
    } else {
        const int cw = (threadIdx.x >> 5) - 1;
        for (int r = cw; r < R; r += MEGA_NCW) {
            float v[32], wv[32];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = __ldcg(src + (int64_t)r * D + i * 32 + lane);   // written by other CTAs: bypass L1
                wv[i] = __ldg(w + i * 32 + lane);                      // in flight with the rows
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
            ss = warp_sum(ss);
            const float inv = rsqrtf(ss / (float)D + eps);
            if (rinv && lane == 0) rinv[r] = inv;
#pragma unroll
            for (int i = 0; i < 32; ++i) dst[r * D + i * 32 + lane] = wv[i] * (v[i] * inv);
        }
    }
}

// ------------------------------------------------------------------ attention item
// Chunk of keys per attention item: 32 keys when the span is short (more items than CTAs
// would otherwise sit idle), 64 keys for longer spans.
__device__ __forceinline__ int attn_chunk(int span) { return span <= 32 * 37 ? 32 : 64; }

// Copy n floats global -> shared with 16-byte loads, all issued before the stores.
__device__ __forceinline__ void copy_g2s(float* __restrict__ dst, const float* __restrict__ src, int n) {
    const int tid = threadIdx.x - 32;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    const int n4 = n >> 2;
    int i = tid;
    for (; i + 3 * MEGA_NCT < n4; i += 4 * MEGA_NCT) {
        const float4 a0 = __ldcg(s4 + i), a1 = __ldcg(s4 + i + MEGA_NCT), a2 = __ldcg(s4 + i + 2 * MEGA_NCT),
                     a3 = __ldcg(s4 + i + 3 * MEGA_NCT);
        d4[i] = a0;
        d4[i + MEGA_NCT] = a1;
        d4[i + 2 * MEGA_NCT] = a2;
        d4[i + 3 * MEGA_NCT] = a3;
    }
    for (; i < n4; i += MEGA_NCT) d4[i] = __ldcg(s4 + i);
}

template <typename KVT>
__device__ __forceinline__ void load_kv_row16(const KVT* p, int part, float* dst);   // 16 bytes of a K/V row

template <>
__device__ __forceinline__ void load_kv_row16<__nv_bfloat16>(const __nv_bfloat16* p, int part, float* dst) {
    // part 0..7: 8 bf16
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p) + part);
    float f[8];
    bf16x8_to_f32(u, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[part * 8 + i] = f[i];
}

template <>
__device__ __forceinline__ void load_kv_row16<float>(const float* p, int part, float* dst) {
    // part 0..15: 4 floats
    const float4 u = __ldcg(reinterpret_cast<const float4*>(p) + part);
    dst[part * 4 + 0] = u.x;
    dst[part * 4 + 1] = u.y;
    dst[part * 4 + 2] = u.z;
    dst[part * 4 + 3] = u.w;
}

// ------------------------------------------------------------------ attention item geometry
// Items of a layer: for each sequence block b (consecutive rows of one slot), HKV x nch_b
// items (kv head, key chunk). Producer and consumers derive the same geometry from the rows.
struct AttnGeo {
    int r0, nr, g, c, nch, chunk, slot, pos0, k0, nk, nold;
};

__device__ __forceinline__ void attn_block_chunks(const int4* rows, int r0, int r1, bool local, int& chunk, int& nch) {
    const int pos0 = rows[r0].y, posL = rows[r1 - 1].y;
    const int lo = local ? max(0, pos0 - WINDOW + 1) : 0;
    chunk = attn_chunk(posL - lo + 1);
    nch = (posL - lo + chunk) / chunk;
}

// Geometry of item `item` given the block starts blk_r0[0..n_blk] (blk_r0[n_blk] = R);
// false past the last item.
__device__ __forceinline__ bool attn_geo(const int4* rows, const int* blk_r0, int n_blk, bool local, int item,
                                         AttnGeo& o) {
    for (int b = 0; b < n_blk; ++b) {
        int chunk, nch;
        attn_block_chunks(rows, blk_r0[b], blk_r0[b + 1], local, chunk, nch);
        if (item < HKV * nch) {
            o.r0 = blk_r0[b];
            o.nr = blk_r0[b + 1] - blk_r0[b];
            o.g = item / nch;
            o.c = item % nch;
            o.nch = nch;
            o.chunk = chunk;
            o.slot = rows[o.r0].x;
            o.pos0 = rows[o.r0].y;
            const int posL = rows[o.r0 + o.nr - 1].y;
            const int lo = local ? max(0, o.pos0 - WINDOW + 1) : 0;
            o.k0 = lo + o.c * chunk;
            const int k1 = min(o.k0 + chunk, posL + 1);
            o.nk = k1 - o.k0;
            o.nold = max(0, min(k1, o.pos0) - o.k0);   // keys < pos0 come from the cache
            return true;
        }
        item -= HKV * nch;
    }
    return false;
}

// Passes of at most this many rows stream each attention item's cached K/V chunk through the
// weight ring (issued during phase A); larger passes load it directly in phase B, because
// their ring already carries many more routed-expert tiles per layer.
constexpr int MEGA_RING_KV_MAX_R = 2;

// Keys per ring slot of cached K (or V) rows.
template <typename KVT>
constexpr int kv_keys_per_tile() { return MEGA_SLOT / (DH * (int)sizeof(KVT)); }

// Producer: cached K (isv = 0) or V rows of keys [k0, k0 + n) of (slot, head g), in tiles of
// kv_keys_per_tile keys; a run that wraps around a local layer's ring takes two copies.
template <typename KVT>
__device__ __forceinline__ void produce_kv(Ring& g, const KVLayer& L, int slot, int head, int k0, int n, bool isv) {
    constexpr int KPT = kv_keys_per_tile<KVT>();
    constexpr uint32_t ROW = DH * sizeof(KVT);
    for (int k = k0; k < k0 + n && g.ok; k += KPT) {
        const int m = min(KPT, k0 + n - k);
        const uint32_t slot_i = g.t % MEGA_NS;
        const uint32_t use = g.t / MEGA_NS;
        if (use > 0 && !ring_wait(g, &g.s->empty[slot_i], (use - 1) & 1)) { g.ok = false; break; }
        mbar_arrive_expect_tx(&g.s->full[slot_i], (uint32_t)m * ROW);
        const KVT* p0 = isv ? kv_v<KVT>(L, slot, head, k) : kv_k<KVT>(L, slot, head, k);
        const int i0 = k & L.mask;
        const int m1 = (L.mask >= 0 && i0 + m > L.cap) ? L.cap - i0 : m;
        tma_load_1d(g.s->ring[slot_i], p0, (uint32_t)m1 * ROW, &g.s->full[slot_i]);
        if (m1 < m) {
            const KVT* p1 = isv ? kv_v<KVT>(L, slot, head, k + m1) : kv_k<KVT>(L, slot, head, k + m1);
            tma_load_1d(g.s->ring[slot_i] + m1 * ROW, p1, (uint32_t)(m - m1) * ROW, &g.s->full[slot_i]);
        }
        ++g.t;
    }
}

// Consumers (all 15 warps): take the same tiles, widen them to fp32 rows of `dst` (stride
// DH + 1), release each slot after every warp is done with it.
template <typename KVT>
__device__ __forceinline__ void consume_kv(Ring& g, int n, float* dst) {
    constexpr int KPT = kv_keys_per_tile<KVT>();
    constexpr int PARTS = DH * (int)sizeof(KVT) / 16;   // 16-byte pieces per row
    const int tid = threadIdx.x - 32;
    for (int k = 0; k < n; k += KPT) {
        const int m = min(KPT, n - k);
        const uint32_t slot_i = g.t % MEGA_NS;
        const uint32_t use = g.t / MEGA_NS;
        if (g.ok && !ring_wait(g, &g.s->full[slot_i], use & 1)) g.ok = false;
        if (g.ok) {
            const unsigned char* tile = g.s->ring[slot_i];
            for (int e = tid; e < m * PARTS; e += MEGA_NCT) {
                const int kk = e / PARTS, part = e % PARTS;
                const uint4 u = *reinterpret_cast<const uint4*>(tile + kk * DH * sizeof(KVT) + part * 16);
                float* d = dst + (k + kk) * (DH + 1);
                if constexpr (sizeof(KVT) == 2) {
                    float f[8];
                    bf16x8_to_f32(u, f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) d[part * 8 + i] = f[i];
                } else {
                    d[part * 4 + 0] = __uint_as_float(u.x);
                    d[part * 4 + 1] = __uint_as_float(u.y);
                    d[part * 4 + 2] = __uint_as_float(u.z);
                    d[part * 4 + 3] = __uint_as_float(u.w);
                }
            }
        }
        named_bar_sync(1, MEGA_NCT);
        if (threadIdx.x == 32 && g.ok) mbar_arrive(&g.s->empty[slot_i]);
        ++g.t;
    }
}

template <int R, typename KVT>
__device__ __noinline__ void attn_item(const MegaArgs& a, MegaSmem* s, Ring& ring, int l, int r0, int nr, int g,
                                       int c, int chunk, bool first) {
    const int tid = threadIdx.x - 32;   // consumer thread 0..479
    const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
    const bool local = is_local_layer(l);
    const KVLayer& L = a.kvl[l];
    const int4* rows = s->rows;
    const int slot = rows[r0].x;
    const int pos0 = rows[r0].y, posL = rows[r0 + nr - 1].y;
    const int lo = local ? max(0, pos0 - WINDOW + 1) : 0;
    const int k0 = lo + c * chunk;
    const int k1 = min(k0 + chunk, posL + 1);
    const int nk = k1 - k0;
    const int nold = max(0, min(k1, pos0) - k0);          // keys < pos0 come from the cache
    float* qs = s->xs;                                   // [nr*4][64]
    float* Ks = qs + MEGA_RMAX * GQA * DH;               // [64][65]
    float* Vs = Ks + MEGA_CHUNK * (DH + 1);              // [64][65]
    float* Ps = Vs + MEGA_CHUNK * (DH + 1);              // [nr*4][64]
    const int nq = nr * GQA;
    astamp(a, l, 0, first);
    // queries of heads 4g..4g+3 (warps), and the block rows' own keys/values (produced here);
    // they land in rows [nold, nk) of Ks / Vs, disjoint from the cached rows
    auto queries_and_new_keys = [&]() {
        const int vres_mode = (a.pulse == 0) ? (l == 0 ? 1 : 2) : 0;
        const int nnew = max(0, k1 - max(k0, pos0));
        for (int it = cw; it < nq + nnew; it += MEGA_NCW) {
            if (it < nq) {
                const int rr = it / GQA, h = g * GQA + it % GQA;
                const int pos = rows[r0 + rr].y;
                const float* src = a.qkv + (int64_t)(r0 + rr) * QKV + h * DH;
                const float x1 = __ldcg(src + lane), x2 = __ldcg(src + lane + 32);
                const float* qw = a.qn[l] + h * DH;
                const float w1 = __ldg(qw + lane), w2 = __ldg(qw + lane + 32);
                const float* rp = s->rope[local ? 0 : 1][r0 + rr];
                const float cs = rp[lane], sn = rp[32 + lane];
                const float inv = rsqrtf(warp_sum(x1 * x1 + x2 * x2) / (float)DH + a.eps);
                const float q1 = w1 * (x1 * inv), q2 = w2 * (x2 * inv);
                float y1 = q1 * cs - q2 * sn, y2 = q2 * cs + q1 * sn;
                if (!local && pos + 1 > a.base_seq_len) {
                    const double b = (double)a.base_seq_len;
                    const float sc = (float)(1.0 + 0.1 * log(fmax((double)(pos + 1), b) / b));
                    y1 *= sc;
                    y2 *= sc;
                }
                qs[it * DH + lane] = y1 * 0.125f;
                qs[it * DH + lane + 32] = y2 * 0.125f;
            } else {
                const int key = max(k0, pos0) + (it - nq);
                const int kk = key - k0;
                const int rr = r0 + (key - pos0);
                const float* src = a.qkv + (int64_t)rr * QKV;
                const float e1 = __ldcg(src + H * DH + g * DH + lane), e2 = __ldcg(src + H * DH + g * DH + lane + 32);
                float v1 = __ldcg(src + H * DH + HKV * DH + g * DH + lane);
                float v2 = __ldcg(src + H * DH + HKV * DH + g * DH + lane + 32);
                float* vf = a.vfirst + ((int64_t)rr * HKV + g) * DH;
                // the first layer's values (value residual) in flight with the rest
                const float f1 = vres_mode == 2 ? __ldcg(vf + lane) : 0.f;
                const float f2 = vres_mode == 2 ? __ldcg(vf + lane + 32) : 0.f;
                const float* kw = a.kn[l] + g * DH;
                const float w1 = __ldg(kw + lane), w2 = __ldg(kw + lane + 32);
                const float* rp = s->rope[local ? 0 : 1][rr];   // row rr sits at position key
                const float cs = rp[lane], sn = rp[32 + lane];
                if (vres_mode == 1) {
                    vf[lane] = v1;
                    vf[lane + 32] = v2;
                } else if (vres_mode == 2) {
                    const float lv = a.vres[l];
                    v1 = (1.f - lv) * v1 + lv * f1;
                    v2 = (1.f - lv) * v2 + lv * f2;
                }
                const float inv = rsqrtf(warp_sum(e1 * e1 + e2 * e2) / (float)DH + a.eps);
                const float b1 = w1 * (e1 * inv), b2 = w2 * (e2 * inv);
                const float y1 = b1 * cs - b2 * sn, y2 = b2 * cs + b1 * sn;
                if (!(rows[rr].w & 1)) {   // bit 0: the row keeps its cached K/V (exited early)
                    KVT* kp = kv_k<KVT>(L, slot, g, key);
                    KVT* vp = kv_v<KVT>(L, slot, g, key);
                    kv_store(kp + lane, y1);
                    kv_store(kp + lane + 32, y2);
                    kv_store(vp + lane, v1);
                    kv_store(vp + lane + 32, v2);
                }
                // the stored (rounded) values, so every reader sees identical keys
                Ks[kk * (DH + 1) + lane] = kv_round<KVT>(y1);
                Ks[kk * (DH + 1) + lane + 32] = kv_round<KVT>(y2);
                Vs[kk * (DH + 1) + lane] = kv_round<KVT>(v1);
                Vs[kk * (DH + 1) + lane + 32] = kv_round<KVT>(v2);
            }
        }
    };
    // 1) cached keys/values of the chunk. One- and two-row passes: the producer streamed them
    //    through the ring during phase A, so the queries' L2 reads go first and the tiles land
    //    meanwhile. Larger passes load them here, every thread's 16-byte loads issued first.
    if constexpr (R <= MEGA_RING_KV_MAX_R) {
        queries_and_new_keys();
        astamp(a, l, 1, first);
        consume_kv<KVT>(ring, nold, Ks);
        consume_kv<KVT>(ring, nold, Vs);
    } else {
        constexpr int PARTS = (sizeof(KVT) == 2) ? 8 : 16;   // 16-byte pieces per 64-element row
        for (int e = tid; e < 2 * nold * PARTS; e += MEGA_NCT) {
            const int isv = e >= nold * PARTS;
            const int ee = isv ? e - nold * PARTS : e;
            const int kk = ee / PARTS, part = ee % PARTS;
            const KVT* row = isv ? kv_v<KVT>(L, slot, g, k0 + kk) : kv_k<KVT>(L, slot, g, k0 + kk);
            load_kv_row16<KVT>(row, part, (isv ? Vs : Ks) + kk * (DH + 1));
        }
        astamp(a, l, 1, first);
        queries_and_new_keys();
    }
    // rows past the end of a partial chunk: zeros (probabilities are 0 there; 0 * stale
    // shared memory could be NaN)
    for (int e = tid; e < (MEGA_CHUNK - nk) * DH; e += MEGA_NCT) {
        const int kk = nk + e / DH, d = e % DH;
        Ks[kk * (DH + 1) + d] = 0.f;
        Vs[kk * (DH + 1) + d] = 0.f;
    }
    named_bar_sync(1, MEGA_NCT);
    astamp(a, l, 2, first);
    // 3) scores with per-row masks [lo_r, pos_r]. Several rows: a thread per (key, row) covers
    //    the row's four heads (float4 query loads shared by the key's element); one row: a
    //    thread per (key, head)
    if (nq >= 2 * GQA) {
        for (int e = tid; e < nr * MEGA_CHUNK; e += MEGA_NCT) {
            const int rq = e / MEGA_CHUNK, kk = e % MEGA_CHUNK;
            const int key = k0 + kk;
            const int pos = rows[r0 + rq].y;
            const int lor = local ? max(0, pos - WINDOW + 1) : 0;
            const bool vis = kk < nk && key <= pos && key >= lor;
            float acc[GQA] = {0.f, 0.f, 0.f, 0.f};
            if (vis) {
                const float* kv = Ks + kk * (DH + 1);
#pragma unroll 4
                for (int d = 0; d < DH; d += 4) {
                    const float c0 = kv[d], c1 = kv[d + 1], c2 = kv[d + 2], c3 = kv[d + 3];
#pragma unroll
                    for (int i = 0; i < GQA; ++i) {
                        const float4 q = *reinterpret_cast<const float4*>(qs + (rq * GQA + i) * DH + d);
                        acc[i] += q.x * c0 + q.y * c1 + q.z * c2 + q.w * c3;
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < GQA; ++i) Ps[(rq * GQA + i) * MEGA_CHUNK + kk] = vis ? acc[i] : -INFINITY;
        }
    } else
    for (int e = tid; e < nq * MEGA_CHUNK; e += MEGA_NCT) {
        const int qi = e / MEGA_CHUNK, kk = e % MEGA_CHUNK;
        const int key = k0 + kk;
        const int pos = rows[r0 + qi / GQA].y;
        const int lor = local ? max(0, pos - WINDOW + 1) : 0;
        float sc = -INFINITY;
        if (kk < nk && key <= pos && key >= lor) {
            sc = 0.f;
            const float* qv = qs + qi * DH;
            const float* kv = Ks + kk * (DH + 1);
#pragma unroll 16
            for (int d = 0; d < DH; ++d) sc += qv[d] * kv[d];
        }
        Ps[qi * MEGA_CHUNK + kk] = sc;
    }
    named_bar_sync(1, MEGA_NCT);
    astamp(a, l, 3, first);
    // 4) partial softmax per query (warps): max m, weights e = exp(s - m) back into Ps, sum
    for (int qi = cw; qi < nq; qi += MEGA_NCW) {
        const int rr = qi / GQA, h = g * GQA + qi % GQA;
        const float p0 = Ps[qi * MEGA_CHUNK + lane], p1 = Ps[qi * MEGA_CHUNK + lane + 32];
        const float m = warp_max(fmaxf(p0, p1));
        const float e0 = (p0 == -INFINITY) ? 0.f : expf(p0 - m);
        const float e1 = (p1 == -INFINITY) ? 0.f : expf(p1 - m);
        const float lsum = warp_sum(e0 + e1);
        Ps[qi * MEGA_CHUNK + lane] = e0;
        Ps[qi * MEGA_CHUNK + lane + 32] = e1;
        float* out = a.part + (((int64_t)(r0 + rr) * H + h) * a.nch_max + c) * PART;
        if (lane == 0) {
            out[0] = m;   // -inf: no key of the chunk is visible to this row (weights all 0)
            out[1] = m == -INFINITY ? 0.f : lsum;
        }
    }
    named_bar_sync(1, MEGA_NCT);
    astamp(a, l, 4, first);
    // 5) P.V. Several rows: a thread per (dimension, row) covers the row's four heads (float4
    //    weight loads); one row: a thread per (query, dimension), keys in order
    if (nq >= 2 * GQA) {
        for (int e = tid; e < nr * DH; e += MEGA_NCT) {
            const int rq = e / DH, d = e % DH;
            float o[GQA] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int kk = 0; kk < MEGA_CHUNK; kk += 4) {
                const float v0 = Vs[kk * (DH + 1) + d], v1 = Vs[(kk + 1) * (DH + 1) + d];
                const float v2 = Vs[(kk + 2) * (DH + 1) + d], v3 = Vs[(kk + 3) * (DH + 1) + d];
#pragma unroll
                for (int i = 0; i < GQA; ++i) {
                    const float4 pw = *reinterpret_cast<const float4*>(Ps + (rq * GQA + i) * MEGA_CHUNK + kk);
                    o[i] += pw.x * v0 + pw.y * v1 + pw.z * v2 + pw.w * v3;
                }
            }
#pragma unroll
            for (int i = 0; i < GQA; ++i)
                a.part[(((int64_t)(r0 + rq) * H + g * GQA + i) * a.nch_max + c) * PART + 2 + d] = o[i];
        }
    } else
    for (int e = tid; e < nq * DH; e += MEGA_NCT) {
        const int qi = e / DH, d = e % DH;
        const int rr = qi / GQA, h = g * GQA + qi % GQA;
        const float* pr = Ps + qi * MEGA_CHUNK;
        float o = 0.f;
#pragma unroll 16
        for (int kk = 0; kk < MEGA_CHUNK; ++kk) o += pr[kk] * Vs[kk * (DH + 1) + d];
        a.part[(((int64_t)(r0 + rr) * H + h) * a.nch_max + c) * PART + 2 + d] = o;
    }
    named_bar_sync(1, MEGA_NCT);
    astamp(a, l, 5, first);
}

// Merge the chunk partials (m, l, o[64]) of query head h of row r, apply the gate, write
// att[r][h*64 ..]: consumer warps take chunks cw, cw + 15, ... (online softmax merge, loads of
// four chunks in flight), then warp 0 merges the 15 warp states in warp order.
static __device__ __noinline__ void attn_merge(const MegaArgs& a, MegaSmem* s, int r, int h, int nch) {
    const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
    const float* pp = a.part + ((int64_t)r * H + h) * a.nch_max * PART;
    const float graw = (cw == 0) ? __ldcg(a.gate + r * H + h) : 0.f;   // in flight with the partials
    float M = -INFINITY, Ls = 0.f, o1 = 0.f, o2 = 0.f;
    for (int c0 = cw; c0 < nch; c0 += 4 * MEGA_NCW) {
        float mc[4], lc[4], a1[4], a2[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * MEGA_NCW;
            mc[u] = -INFINITY;
            lc[u] = a1[u] = a2[u] = 0.f;
            if (c < nch) {
                const float* q = pp + (int64_t)c * PART;
                mc[u] = __ldcg(q);
                lc[u] = __ldcg(q + 1);
                a1[u] = __ldcg(q + 2 + lane);
                a2[u] = __ldcg(q + 2 + 32 + lane);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (mc[u] == -INFINITY) continue;
            const float Mn = fmaxf(M, mc[u]);
            const float so = expf(M - Mn), sn = expf(mc[u] - Mn);
            Ls = Ls * so + lc[u] * sn;
            o1 = o1 * so + a1[u] * sn;
            o2 = o2 * so + a2[u] * sn;
            M = Mn;
        }
    }
    float* st = s->stage + cw * PART;   // [15][66]
    if (lane == 0) {
        st[0] = M;
        st[1] = Ls;
    }
    st[2 + lane] = o1;
    st[2 + 32 + lane] = o2;
    named_bar_sync(1, MEGA_NCT);
    if (cw == 0) {
        // lane w < 15 holds warp w's (m, l); the weights exp(m_w - max) are computed in
        // parallel and broadcast, so the fold below is FMAs only
        const float mw = lane < MEGA_NCW ? s->stage[lane * PART] : -INFINITY;
        const float lw = lane < MEGA_NCW ? s->stage[lane * PART + 1] : 0.f;
        const float Mx = warp_max(mw);
        const float ww = (mw == -INFINITY) ? 0.f : expf(mw - Mx);
        const float L = warp_sum(ww * lw);
        float p1 = 0.f, p2 = 0.f;
#pragma unroll
        for (int w = 0; w < MEGA_NCW; ++w) {
            const float wt = __shfl_sync(0xffffffffu, ww, w);
            const float* q = s->stage + w * PART;
            p1 += wt * q[2 + lane];
            p2 += wt * q[2 + 32 + lane];
        }
        const float gt = sigmoidf_(graw);
        const float inv = 1.f / L;
        a.att[(int64_t)r * D + h * DH + lane] = (p1 * inv) * gt;
        a.att[(int64_t)r * D + h * DH + 32 + lane] = (p2 * inv) * gt;
    }
    named_bar_sync(1, MEGA_NCT);
}

// Consumer exit of every CTA: the last CTA out (every CTA is past its last grid barrier)
// re-arms the barrier counter for the next launch on this stream.
__device__ __forceinline__ void mega_leave(const MegaArgs& a) {
    if (threadIdx.x == 32) {
        if (a.trace) a.trace[blockIdx.x * MEGA_TRACE + MEGA_TRACE - 2] = globaltimer();
        const unsigned t = atomicAdd(&a.tickets[MEGA_RMAX * HKV + 1], 1u);
        if (t == gridDim.x - 1) {
            a.tickets[MEGA_RMAX * HKV + 1] = 0;
            atomicExch(a.bar, 0u);
        }
    }
}

// ------------------------------------------------------------------ the pulse
template <int R, typename KVT>
__global__ void __launch_bounds__(MEGA_THREADS, 1) k_mega_pulse(const __grid_constant__ MegaArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    MegaSmem* s = reinterpret_cast<MegaSmem*>(smem_raw);
    const int C = gridDim.x, cta = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool want_lm = a.logits != nullptr || a.amax != nullptr;
    const bool lora = a.la_qkv[0] != nullptr;   // live loop adapter (exact fp32 correction)
    if (a.skip && __ldcg(a.skip) != 0) {   // every row exited early (flag written by an earlier kernel)
        mega_leave(a);
        return;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < MEGA_NS; ++i) {
            mbar_init(&s->full[i], 1);
            mbar_init(&s->empty[i], 1);
        }
        s->moe_ready = 0;
        s->abort = 0;
        fence_mbar_init();
    }
    if (threadIdx.x >= 32 && threadIdx.x < 32 + R) s->rows[threadIdx.x - 32] = a.rows[threadIdx.x - 32];
    __syncthreads();

    // ================================================================ producer
    if (warp == 0) {
        if (lane != 0) return;
        Ring g{s, 0u, -1, true, a.wait_ns};
        int pblk[MEGA_RMAX + 1], pnb = 0;   // sequence blocks of the rows (as the consumers build them)
        for (int r0 = 0; r0 < R;) {
            int nr = 1;
            while (r0 + nr < R && s->rows[r0 + nr].x == s->rows[r0].x) ++nr;
            pblk[pnb++] = r0;
            r0 += nr;
        }
        pblk[pnb] = R;
#pragma unroll 1
        for (int l = 0; l < NL && g.ok; ++l) {
            int r0, r1;
            if (a.la_qkv[0]) produce_rows(g, a.la_qkv[l], D * 4, 0, LORA_R, 2);   // adapter A rows (fp32)
            rows_split(QKV, cta, C, r0, r1);
            produce_rows(g, a.wqkv[l], D * 2, r0, r1, 4);
            // gate rows: the last H/2 CTAs, consumed in phase B (usually CTAs without attention items)
            if (cta >= C - H / 2) {
                const int gr = 2 * (cta - (C - H / 2));
                produce_rows(g, a.gate_w[l], D * 4, gr, gr + 2, 2);
            }
            if (R <= MEGA_RING_KV_MAX_R) {   // cached K/V chunks of this CTA's attention items (phase B)
                const bool local = is_local_layer(l);
                AttnGeo geo;
                for (int item = cta; g.ok && attn_geo(s->rows, pblk, pnb, local, item, geo); item += C) {
                    if (geo.nold <= 0) continue;
                    produce_kv<KVT>(g, a.kvl[l], geo.slot, geo.g, geo.k0, geo.nold, false);
                    produce_kv<KVT>(g, a.kvl[l], geo.slot, geo.g, geo.k0, geo.nold, true);
                }
            }
            if (a.la_qkv[0]) produce_rows(g, a.la_wo[l], D * 4, 0, LORA_R, 2);
            rows_split(D, cta, C, r0, r1);
            produce_rows(g, a.wo[l], D * 2, r0, r1, 4);
            {   // shared-expert pairs: a static split, prefetched before the router runs
                int j0, j1;
                rows_split(DS, cta, C, j0, j1);
                produce_rows(g, a.sh_gu[l], D * 2, j0, j1, 4);
                produce_rows(g, a.sh_gu[l], D * 2, DS + j0, DS + j1, 4);
            }
            // routed pairs depend on this layer's router. Short sleeps between polls (a tight
            // spin on shared memory starves the consumers' loads); the global error flag costs
            // an L2 round trip, so it is read every 256th poll only
            const unsigned long long t0 = globaltimer();
            for (unsigned it = 1; s->moe_ready != l + 1; ++it) {
                __nanosleep(32);
                if (globaltimer() - t0 > a.wait_ns || s->abort || ((it & 255) == 0 && *(volatile int*)a.err)) {
                    g.ok = false;
                    break;
                }
            }
            if (!g.ok) break;
            __threadfence_block();   // the expert list was written before the flag
            if (a.trace) a.trace[blockIdx.x * MEGA_TRACE + 194 + l] = globaltimer();
            const int n_e = s->n_e;
            int q0, q1;
            rows_split(DE * n_e, cta, C, q0, q1);
            for (int ei = 0; ei < n_e; ++ei) {
                const int b0 = ei * DE;
                const int j0 = max(q0, b0) - b0, j1 = min(q1, b0 + DE) - b0;
                if (j1 <= j0) continue;
                const __nv_bfloat16* we = a.r_gu[l] + (int64_t)s->elist[ei] * 2 * DE * D;
                produce_rows(g, we, D * 2, j0, j1, 4);
                produce_rows(g, we, D * 2, DE + j0, DE + j1, 4);
            }
            rows_split(D, cta, C, r0, r1);
            produce_rows(g, a.sh_dn[l], DS * 2, r0, r1, 4);
            for (int ei = 0; ei < n_e; ++ei)
                produce_rows(g, a.r_dn[l] + (int64_t)s->elist[ei] * D * DE, DE * 2, r0, r1, 8);
        }
        if (g.ok && want_lm) {
            int v0, v1;
            rows_split(a.V, cta, C, v0, v1);
            produce_rows(g, a.emb, D * 2, v0, v1, 4);
            if (a.trace) a.trace[blockIdx.x * MEGA_TRACE + 205] = globaltimer();
        }
        if (!g.ok) atomicExch(a.err, 1);
        // drain: wait for every copy this thread issued to land before the CTA can exit
        for (uint32_t t = (g.t > MEGA_NS ? g.t - MEGA_NS : 0); t < g.t; ++t)
            if (!mbar_wait(&s->full[t % MEGA_NS], (t / MEGA_NS) & 1)) break;
        return;
    }

    // ================================================================ consumers
    const int cw = warp - 1;
    if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE] = globaltimer();
    Ring g{s, 0u, cw, true, a.wait_ns};
    unsigned epoch = 0;
    float* xs = s->xs;
    float* wo_ = s->wout[cw];   // this warp's reduced tile sums
    const float eps = a.eps;
    const int p = a.pulse;
    // h rows [own0, own1) are this CTA's outputs in phases C and E; their router weights
    // (times the mlp-norm weight) for every layer go to shared memory now
    int own0, own1;
    rows_split(D, cta, C, own0, own1);
    const int nown = own1 - own0;
    for (int t = threadIdx.x - 32; t < NL * E * MEGA_MAXOROWS; t += MEGA_NCT) {
        const int ll = t / (E * MEGA_MAXOROWS), e = (t / MEGA_MAXOROWS) % E, oi = t % MEGA_MAXOROWS;
        s->rwn[ll][e][oi] = oi < nown ? a.router[ll][e * D + own0 + oi] * a.mlp_norm[ll][own0 + oi] : 0.f;
    }
    for (int t = threadIdx.x - 32; t < NL * MEGA_MAXOROWS; t += MEGA_NCT) {
        const int ll = t / MEGA_MAXOROWS, oi = t % MEGA_MAXOROWS;
        s->rsc[ll][oi] = oi < nown ? a.rscale[ll][own0 + oi] : 0.f;
    }
    for (int t = threadIdx.x - 32; t < NL * E; t += MEGA_NCT) s->ebias[t / E][t % E] = a.ebias[t / E][t % E];
    for (int t = threadIdx.x - 32; t < 2 * R * DH; t += MEGA_NCT) {
        const int tab = t / (R * DH), r = (t / DH) % R, j = t % DH;
        const float* T = (j < 32) ? (tab ? a.cos_g : a.cos_l) : (tab ? a.sin_g : a.sin_l);
        s->rope[tab][r][j] = T[(int64_t)s->rows[r].y * 32 + (j & 31)];
    }
    // ---- pulse input: every CTA builds h_in for all rows in xs[0 .. R*D) ----
    if (p == 0) {
        for (int r = cw; r < R; r += MEGA_NCW) {
            const int tok = min(max(s->rows[r].z, 0), a.V - 1);
            const __nv_bfloat16* e = a.emb + (int64_t)tok * D;
            float v[32];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = __bfloat162float(__ldg(e + i * 32 + lane));
                ss += v[i] * v[i];
            }
            const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
            // read-only inputs through the non-coherent path (free to move ahead of the
            // stores); global stores only after the loop
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int d = i * 32 + lane;
                float n = __ldg(a.anchor + d) * (v[i] * inv);
                if (a.use_conv) n = n + __ldg(a.stem + d * 4) * n;
                xs[r * D + d] = n + __ldg(a.step + d);
                v[i] = n;
            }
            if (cta == 0)
#pragma unroll
                for (int i = 0; i < 32; ++i) a.h0n_out[(int64_t)r * a.hstride * D + i * 32 + lane] = v[i];
        }
    } else {
        // g8[r][j] = Wd[j][:D] . h0n[r] + Wd[j][D:] . RMSNorm(h_prev[r])   (CTAs < 8)
        if (cta < RG) {
            const int j = cta;
            for (int r = cw; r < R; r += MEGA_NCW) {
                float ss = 0.f;
                for (int i = lane; i < D; i += 32) ss += a.h_prev[r * D + i] * a.h_prev[r * D + i];
                const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
                float pe = 0.f, pr = 0.f;
                for (int i = lane; i < D; i += 32) {
                    pe += a.rg_down[j * 2 * D + i] * a.h0n_in[r * D + i];
                    pr += a.rg_down[j * 2 * D + D + i] * (a.psn[i] * (a.h_prev[r * D + i] * inv));
                }
                pe = warp_sum(pe);
                pr = warp_sum(pr);
                if (lane == 0) a.g8[r * RG + j] = pe + pr;
            }
        }
        if (!grid_sync(a, s, epoch)) goto done;
        // h_prev and h0n_in are inputs this kernel never writes (h0n_out may alias h0n_in and is
        // then not written): read-only loads, global stores after the loops
        for (int r = cw; r < R; r += MEGA_NCW) {
            float ss = 0.f;
#pragma unroll 8
            for (int i = 0; i < 32; ++i) {
                const float x = __ldg(a.h_prev + r * D + i * 32 + lane);
                ss += x * x;
            }
            const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
            float gg[RG];
#pragma unroll
            for (int j = 0; j < RG; ++j) gg[j] = __ldcg(a.g8 + r * RG + j);
#pragma unroll 4
            for (int i = 0; i < 32; ++i) {
                const int d = i * 32 + lane;
                const float4 u0 = __ldg(reinterpret_cast<const float4*>(a.rg_up + d * RG));
                const float4 u1 = __ldg(reinterpret_cast<const float4*>(a.rg_up + d * RG + 4));
                const float z = __ldg(a.rg_bias + d) + u0.x * gg[0] + u0.y * gg[1] + u0.z * gg[2] + u0.w * gg[3] +
                                u1.x * gg[4] + u1.y * gg[5] + u1.z * gg[6] + u1.w * gg[7];
                const float mix = sigmoidf_(z);
                const float rn = __ldg(a.psn + d) * (__ldg(a.h_prev + r * D + d) * inv);
                const float an = __ldg(a.h0n_in + r * D + d);
                const float diff = an - rn;
                const float lerp = (mix < 0.5f) ? rn + mix * diff : an - diff * (1.f - mix);
                xs[r * D + d] = lerp + __ldg(a.step + d);
            }
        }
        if (cta == 0 && a.h0n_out && a.h0n_out != a.h0n_in) {   // caller buffers: scalar accesses, no alignment assumed
#pragma unroll 4
            for (int i = threadIdx.x - 32; i < R * D; i += MEGA_NCT)
                a.h0n_out[(int64_t)(i / D) * a.hstride * D + i % D] = __ldg(a.h0n_in + i);
        }
    }
    named_bar_sync(1, MEGA_NCT);
    if (cta == 0)
        for (int i = threadIdx.x - 32; i < R * D; i += MEGA_NCT) {
            a.h_in[i] = xs[i];
            a.h[i] = xs[i];
        }
    for (int t = threadIdx.x - 32; t < nown * R; t += MEGA_NCT) s->hown[t] = xs[(t % R) * D + own0 + t / R];
    named_bar_sync(1, MEGA_NCT);
    // sequence blocks of the rows (consecutive rows of one slot), for the attention items
    if (threadIdx.x == 32) {
        int nb = 0, r0 = 0;
        while (r0 < R) {
            int nr = 1;
            while (r0 + nr < R && s->rows[r0 + nr].x == s->rows[r0].x) ++nr;
            s->blk_r0[nb++] = r0;
            r0 += nr;
        }
        s->blk_r0[nb] = R;
        s->n_blk = nb;
    }
    // xs holds h_in; layer 0's attention norm reads it from xs, later layers from a.h
    // one copy of the layer body (not unrolled), so it can stay in the instruction caches
#pragma unroll 1
    for (int l = 0; l < NL; ++l) {
        const bool local = is_local_layer(l);
        // ---------------- phase A: xn, QKV, gate logits
        {
            if (l == 0) {
                // normalise in place (each warp owns its rows)
                for (int r = cw; r < R; r += MEGA_NCW) {
                    float v[32], wv[32];
                    float ss = 0.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        v[i] = xs[r * D + i * 32 + lane];
                        wv[i] = __ldg(a.attn_norm[l] + i * 32 + lane);
                        ss += v[i] * v[i];
                    }
                    const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
                    for (int i = 0; i < 32; ++i) xs[r * D + i * 32 + lane] = wv[i] * (v[i] * inv);
                }
            } else {
                norm_rows<R>(a.h, a.attn_norm[l], eps, xs, s->nred);
            }
            if (threadIdx.x - 32 < R) s->xoff[threadIdx.x - 32] = (threadIdx.x - 32) * D;
            // attention chunking of each block (used in phase B)
            if (threadIdx.x == 33) {
                for (int b = 0; b < s->n_blk; ++b) {
                    const int pos0 = s->rows[s->blk_r0[b]].y, posL = s->rows[s->blk_r0[b + 1] - 1].y;
                    const int lo = local ? max(0, pos0 - WINDOW + 1) : 0;
                    const int chunk = attn_chunk(posL - lo + 1);
                    s->blk_chunk[b] = chunk;
                    s->blk_nch[b] = (posL - lo + chunk) / chunk;
                }
            }
            named_bar_sync(1, MEGA_NCT);
            stamp(a, l, 0);
            if (lora) adapter_t<R>(g, s, wo_);
            int r0, r1;
            rows_split(QKV, cta, C, r0, r1);
            consume_rows(g, r0, r1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) {
                    const int r = lane % R, o = row0 + lane / R;
                    float v = wo_[lane];
                    if (lora) v += adapter_corr(a.lb_qkv[l], o, s->lt + r * LORA_R);
                    a.qkv[(int64_t)r * QKV + o] = v;
                }
            });
            stamp(a, l, 1);
            stamp(a, l, 2);
            if (!g.ok) atomicExch(a.err, 1);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 3);
        }
        // ---------------- phase B: attention (items owned by this CTA: cta, cta + C, ...)
        {
            // gate logits xn . Wg + b of two heads on each of the last H/2 CTAs, first (xs
            // still holds xn; the attention items reuse it)
            if (cta >= C - H / 2) {
                const int gr = 2 * (cta - (C - H / 2));
                consume_rows(g, gr, gr + 2, 2, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv_f32<R>(reinterpret_cast<const float*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) {
                        const int h = row0 + lane / R;
                        a.gate[(lane % R) * H + h] = wo_[lane] + a.gate_b[l][h];
                    }
                });
                named_bar_sync(1, MEGA_NCT);   // xs is scratch for the items below
            }
            int total = 0;
            for (int b = 0; b < s->n_blk; ++b) total += HKV * s->blk_nch[b];
            bool first = true;
            for (int item = cta; item < total; item += C) {
                int b = 0, rem = item;
                while (rem >= HKV * s->blk_nch[b]) { rem -= HKV * s->blk_nch[b]; ++b; }
                const int nch = s->blk_nch[b];
                const int r0 = s->blk_r0[b], nr = s->blk_r0[b + 1] - r0;
                attn_item<R, KVT>(a, s, g, l, r0, nr, rem / nch, rem % nch, s->blk_chunk[b], first);
                first = false;
            }
            stamp(a, l, 4);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 5);
        }
        // ---------------- phase B2: merge the chunk partials of each (row, head) and gate
        {
            for (int u = cta; u < R * H; u += C) {
                const int r = u / H;
                int b = 0;
                while (s->blk_r0[b + 1] <= r) ++b;
                attn_merge(a, s, r, u % H, s->blk_nch[b]);
            }
            stamp(a, l, 6);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 7);
        }
        // ---------------- phase C: Wo, h += (owned rows), router partial sums of the owned rows
        {
            copy_g2s(xs, a.att, R * D);
            named_bar_sync(1, MEGA_NCT);
            if (lora) adapter_t<R>(g, s, wo_);
            consume_rows(g, own0, own1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) {
                    const int r = lane % R, o = row0 + lane / R;
                    float y = wo_[lane];
                    if (lora) y += adapter_corr(a.lb_wo[l], o, s->lt + r * LORA_R);
                    const float v = s->hown[(o - own0) * R + r] + y;
                    s->hown[(o - own0) * R + r] = v;
                    a.h[(int64_t)r * D + o] = v;
                }
            });
            named_bar_sync(1, MEGA_NCT);
            // z[r][e] = sum over owned o of router[e][o] * mlp_norm[o] * h[r][o]  (logit = z / rms)
            for (int t = threadIdx.x - 32; t < R * E; t += MEGA_NCT) {
                const int r = t / E, e = t % E;
                float z = 0.f;
                for (int oi = 0; oi < nown; ++oi) z += s->rwn[l][e][oi] * s->hown[oi * R + r];
                a.rpart[((int64_t)cta * R + r) * E + e] = z;
            }
            stamp(a, l, 8);
            if (!g.ok) atomicExch(a.err, 1);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 9);
        }
        // ---------------- phase D: router (sum of the CTAs' partials), shared + routed up-projections
        {
            float ebias_lane;
            {
                // router logits = fixed-order sum over CTAs of the partials / rms: thread t adds
                // float4 column t % (R*E/4) of CTAs t / (R*E/4), + G, ... (its loads issued
                // before the norm's), then a warp per row adds the G group sums
                constexpr int NC4 = R * E / 4;
                constexpr int G = MEGA_NCT / NC4;
                constexpr int MAXL = (148 + G - 1) / G;   // loads per thread kept in flight
                const int t = threadIdx.x - 32;
                const int col = t % NC4, cg = t / NC4;
                const bool active = t < G * NC4;
                const float4* src = reinterpret_cast<const float4*>(a.rpart) + col;
                float4 pv[MAXL];
                ebias_lane = (lane < E) ? s->ebias[l][lane] : 0.f;   // for the top-k below
#pragma unroll
                for (int k = 0; k < MAXL; ++k) {
                    const int c = cg + k * G;
                    pv[k] = (active && c < C) ? __ldcg(src + (int64_t)c * NC4) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                norm_rows<R>(a.h, a.mlp_norm[l], eps, xs, s->nred, s->rinv);
                rstamp(a, l, 0);
                if (active) {
                    float4 z = pv[0];
#pragma unroll
                    for (int k = 1; k < MAXL; ++k) {
                        z.x += pv[k].x;
                        z.y += pv[k].y;
                        z.z += pv[k].z;
                        z.w += pv[k].w;
                    }
                    for (int c = cg + MAXL * G; c < C; c += G) {   // grids above 148 CTAs
                        const float4 v = __ldcg(src + (int64_t)c * NC4);
                        z.x += v.x;
                        z.y += v.y;
                        z.z += v.z;
                        z.w += v.w;
                    }
                    reinterpret_cast<float4*>(s->stage)[cg * NC4 + col] = z;
                }
                rstamp(a, l, 1);
            }
            named_bar_sync(1, MEGA_NCT);
            rstamp(a, l, 2);
            // a warp per row: logit of expert e = lanes e and e + 16 adding the even / odd
            // groups of the staged sums; centre, sigmoid; top-4 of s + bias by rank (expert e
            // is chosen iff fewer than 4 experts beat it, ties to the lower expert), weights
            for (int r = cw; r < R; r += MEGA_NCW) {
                constexpr int G = MEGA_NCT / (R * E / 4);
                const int e = lane & (E - 1), hf = lane >> 4;
                float z0 = 0.f, z1 = 0.f;
#pragma unroll 8
                for (int k = hf; k < G; k += 4) {
                    z0 += s->stage[k * R * E + r * E + e];
                    if (k + 2 < G) z1 += s->stage[(k + 2) * R * E + r * E + e];
                }
                float z = z0 + z1;
                z += __shfl_xor_sync(0xffffffffu, z, 16);
                const float lg = lane < E ? z * s->rinv[r] : 0.f;
                const float mean = warp_sum(lg) / (float)E;
                const float sg = sigmoidf_(lg - mean);
                const float b = sg + ebias_lane;
                if (lane < E) {
                    s->logits[r][lane] = b;
                    s->rsg[r][lane] = sg;
                }
                __syncwarp();
                int rank = 0;
#pragma unroll
                for (int j = 0; j < E; ++j) {
                    const float bj = s->logits[r][j];
                    rank += (bj > b || (bj == b && j < lane)) ? 1 : 0;
                }
                const bool chosen = lane < E && rank < TOPK;
                if (chosen) s->idx[r][rank] = lane;
                const unsigned used = __ballot_sync(0xffffffffu, chosen);
                __syncwarp();
                // weights: the chosen scores summed in rank order (as the reference's top-k order)
                const float sk = lane < TOPK ? s->rsg[r][s->idx[r][lane]] : 0.f;
                float sum = 0.f;
#pragma unroll
                for (int k = 0; k < TOPK; ++k) sum += __shfl_sync(0xffffffffu, sk, k);
                sum += 1e-6f;
                if (lane < TOPK) s->wts[r][lane] = sk / sum;
                if (lane == 0) s->rmask[r] = used;
            }
            if constexpr (R > 1) named_bar_sync(1, MEGA_NCT);   // every row's expert mask
            rstamp(a, l, 3);
            if (cw == 0) {
                unsigned used = 0;
                __syncwarp();
#pragma unroll
                for (int r = 0; r < R; ++r) used |= s->rmask[r];
                // distinct experts in increasing order (the producer's routed stream), then the flag
                if (lane < E && (used & (1u << lane))) s->elist[__popc(used & ((1u << lane) - 1u))] = lane;
                if (lane == 0) s->n_e = __popc(used);
                __syncwarp();
                if (lane == 0) {
                    __threadfence_block();
                    s->moe_ready = l + 1;
                }
            }
            named_bar_sync(1, MEGA_NCT);
            stamp(a, l, 10);
            if (cta == 0 && threadIdx.x == 32) atomicAdd(a.experts, (unsigned long long)s->n_e);
            // phase E: X row of each row for every routed expert (act_r row, or -1)
            for (int t = threadIdx.x - 32; t < s->n_e * R; t += MEGA_NCT) {
                const int ei = t / R, r = t % R;
                int off = -1;
#pragma unroll
                for (int k = 0; k < TOPK; ++k)
                    if (s->idx[r][k] == s->elist[ei]) off = R * DS + (r * TOPK + k) * DE;
                s->xoff_e[ei][r] = off;
            }
            for (int t = threadIdx.x - 32; t < R * TOPK; t += MEGA_NCT) {
                const int r = t / TOPK, k = t % TOPK;
                const int ex = s->idx[r][k];
                int ei = 0;
                for (int q = 0; q < s->n_e; ++q)
                    if (s->elist[q] == ex) ei = q;
                s->eslot[r][k] = ei;
            }
            const int n_e = s->n_e;
            int s0, s1, q0, q1;
            rows_split(DS, cta, C, s0, s1);          // shared pairs [s0, s1)
            rows_split(DE * n_e, cta, C, q0, q1);    // routed pairs [q0, q1) over the expert list
            const int nsh = s1 - s0;
            float* st_g = s->stage;                         // [pair][R] gate: shared pairs, then routed
            float* st_u = s->stage + MEGA_MAXPAIRS * R;     // [pair][R] up
            consume_rows(g, s0, s1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) st_g[(row0 - s0 + lane / R) * R + lane % R] = wo_[lane];
            });
            consume_rows(g, DS + s0, DS + s1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) st_u[(row0 - DS - s0 + lane / R) * R + lane % R] = wo_[lane];
            });
            for (int ei = 0; ei < n_e; ++ei) {
                const int b0 = ei * DE;
                const int j0 = max(q0, b0) - b0, j1 = min(q1, b0 + DE) - b0;
                if (j1 <= j0) continue;
                const int base = nsh + b0 - q0;   // stage index = base + j
                consume_rows(g, j0, j1, 4, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) st_g[(base + row0 + lane / R) * R + lane % R] = wo_[lane];
                });
                consume_rows(g, DE + j0, DE + j1, 4, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) st_u[(base + row0 - DE + lane / R) * R + lane % R] = wo_[lane];
                });
            }
            stamp(a, l, 11);
            named_bar_sync(1, MEGA_NCT);
            // SwiGLU epilogue -> act_sh [R][1024], act_r [R][4][512]
            for (int e = threadIdx.x - 32; e < (nsh + q1 - q0) * R; e += MEGA_NCT) {
                const int pi = e / R, r = e % R;
                const float v = siluf_(st_g[pi * R + r]) * st_u[pi * R + r];
                if (pi < nsh) {
                    a.act_sh[(int64_t)r * DS + s0 + pi] = v;
                } else {
                    const int q = q0 + pi - nsh;
                    const int ei = q / DE, j = q % DE;
                    const int ex = s->elist[ei];
#pragma unroll
                    for (int k = 0; k < TOPK; ++k)
                        if (s->idx[r][k] == ex) a.act_r[((int64_t)r * TOPK + k) * DE + j] = v;
                }
            }
            stamp(a, l, 12);
            if (!g.ok) atomicExch(a.err, 1);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 13);
        }
        // ---------------- phase E: down projections + combine, h += (owned rows)
        {
            copy_g2s(xs, a.act_sh, R * DS);
            copy_g2s(xs + R * DS, a.act_r, R * TOPK * DE);
            named_bar_sync(1, MEGA_NCT);
            stamp(a, l, 14);
            const int n_e = s->n_e;
            int o0, o1;
            rows_split(D, cta, C, o0, o1);
            float* dsh = s->stage;                                   // [orow][R]
            float* dex = s->stage + MEGA_MAXOROWS * R;               // [orow][ei][R]
            consume_rows(g, o0, o1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, DS>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) dsh[(row0 - o0 + lane / R) * R + lane % R] = wo_[lane];
            });
            for (int ei = 0; ei < n_e; ++ei) {
                consume_rows(g, o0, o1, 8, [&](const unsigned char* tile, int row0, int n) {
                    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(tile);
                    for (int half = 0; half < 2; ++half) {
                        const int nn = min(4, n - half * 4);
                        if (nn <= 0) break;
                        tile_gemv<R, DE>(w + half * 4 * DE, nn, xs, s->xoff_e[ei], wo_);
                        if (lane < nn * R)
                            dex[((row0 + half * 4 - o0 + lane / R) * E + ei) * R + lane % R] = wo_[lane];
                        __syncwarp();
                    }
                });
            }
            named_bar_sync(1, MEGA_NCT);
            if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 130 + 8 * l + 6] = globaltimer();
            for (int e = threadIdx.x - 32; e < (o1 - o0) * R; e += MEGA_NCT) {
                const int oi = e / R, r = e % R;
                const int o = o0 + oi;
                float routed = 0.f;
#pragma unroll
                for (int k = 0; k < TOPK; ++k) routed = routed + dex[(oi * E + s->eslot[r][k]) * R + r] * s->wts[r][k];
                const float v = s->hown[oi * R + r] + (dsh[oi * R + r] + routed * s->rsc[l][oi]);
                s->hown[oi * R + r] = v;
                a.h[(int64_t)r * D + o] = v;
            }
            if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 130 + 8 * l + 7] = globaltimer();
            if (!g.ok) atomicExch(a.err, 1);
            if (!grid_sync(a, s, epoch)) goto done;
            stamp(a, l, 15);
        }
    }
    // ---------------- end of pulse + LM head
    {
        for (int r = cw; r < R; r += MEGA_NCW) {
            float v[32];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {   // loads only: all of them in flight
                const int d = i * 32 + lane;
                const float hi = __ldcg(a.h_in + r * D + d);
                v[i] = hi + (__ldcg(a.h + r * D + d) - hi) * __ldg(a.res_scale + d);
                ss += v[i] * v[i];
            }
            const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
            if (cta == 0)
#pragma unroll
                for (int i = 0; i < 32; ++i) a.h_out[(int64_t)r * a.hstride * D + i * 32 + lane] = v[i];
#pragma unroll
            for (int i = 0; i < 32; ++i) xs[r * D + i * 32 + lane] = __ldg(a.fnorm + i * 32 + lane) * (v[i] * inv);
        }
        if (!want_lm) goto done;
        named_bar_sync(1, MEGA_NCT);
        if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 202] = globaltimer();
        ArgMax best[R];
#pragma unroll
        for (int r = 0; r < R; ++r) best[r] = ArgMax{-INFINITY, 1 << 30};
        int v0, v1;
        rows_split(a.V, cta, C, v0, v1);
        consume_rows(g, v0, v1, 4, [&](const unsigned char* tile, int row0, int n) {
            tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
            // lane i*R + r holds row i of the tile for output row r
            float y = -INFINITY;
            if (lane < n * R) {
                y = wo_[lane];
                if (a.softcap > 0.f) y = a.softcap * tanhf(y / a.softcap);
                if (a.logits) a.logits[(int64_t)(lane % R) * a.V + row0 + lane / R] = y;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float yi = __shfl_sync(0xffffffffu, y, (i * R + r) & 31);
                    if (i < n) best[r] = argmax_merge(best[r], ArgMax{yi, row0 + i});
                }
            }
        });
        if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 203] = globaltimer();
        // per-CTA argmax -> pmax/pidx; the last CTA reduces
        float* bv = s->stage;
        int* bi = reinterpret_cast<int*>(s->stage + MEGA_NCW * R);
        if (lane == 0)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                bv[cw * R + r] = best[r].v;
                bi[cw * R + r] = best[r].i;
            }
        named_bar_sync(1, MEGA_NCT);
        if (threadIdx.x - 32 < R) {
            const int r = threadIdx.x - 32;
            ArgMax b{bv[r], bi[r]};
            for (int w = 1; w < MEGA_NCW; ++w) b = argmax_merge(b, ArgMax{bv[w * R + r], bi[w * R + r]});
            a.pmax[r * C + cta] = b.v;
            a.pidx[r * C + cta] = b.i;
        }
        __threadfence();
        named_bar_sync(1, MEGA_NCT);
        if (threadIdx.x == 32) {
            const unsigned t = atomicAdd(&a.tickets[MEGA_RMAX * HKV], 1u);
            s->ticket = (t == (unsigned)(C - 1));
            if (s->ticket) a.tickets[MEGA_RMAX * HKV] = 0;
            __threadfence();
        }
        named_bar_sync(1, MEGA_NCT);
        if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 204] = globaltimer();
        if (s->ticket && a.amax) {
            for (int r = cw; r < R; r += MEGA_NCW) {
                // the first 192 partials with all loads in flight, then any remainder
                float pv[6];
                int pi[6];
#pragma unroll
                for (int j = 0; j < 6; ++j) {
                    const int i = lane + 32 * j;
                    pv[j] = i < C ? __ldcg(a.pmax + r * C + i) : -INFINITY;
                    pi[j] = i < C ? __ldcg(a.pidx + r * C + i) : 1 << 30;
                }
                ArgMax b{-INFINITY, 1 << 30};
#pragma unroll
                for (int j = 0; j < 6; ++j) b = argmax_merge(b, ArgMax{pv[j], pi[j]});
                for (int i = lane + 192; i < C; i += 32)
                    b = argmax_merge(b, ArgMax{__ldcg(a.pmax + r * C + i), __ldcg(a.pidx + r * C + i)});
                b = warp_argmax(b);
                if (lane == 0) a.amax[r] = b.i;
            }
        }
        if (!g.ok) atomicExch(a.err, 1);
    }
done:
    mega_leave(a);
}

}  // namespace pulsar
