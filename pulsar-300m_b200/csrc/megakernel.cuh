// Persistent per-pulse decode kernel (one CTA per SM, cooperative launch).
//
// One launch runs a whole pulse pass (src/infer.py:463-524) for R <= MEGA_RMAX rows: the
// pulse input, 8 layers x 6 phases, the end-of-pulse residual, the final norm and, when
// logits or argmax are requested, the LM head with argmax.
//
// Warp 0 is the producer: one lane streams every weight tile this CTA will consume, in
// consumption order, through a ring of NS 8 KB shared-memory slots with 1-D TMA bulk copies
// (cp.async.bulk + mbarrier complete_tx). Weights do not depend on activations, so the
// producer runs ahead across phases (only the routed-expert tiles wait for this layer's
// router, signalled through shared memory). Warps 1..15 are consumers: tile t of the CTA's
// stream lives in slot t % NS and is consumed by warp t % 15.
//
// CTAs hand data to each other through exchange buffers of 8-byte units {value, flag}
// (mega_ptx.cuh, ll_st / ll_ld): the flag is this launch's epoch, so a consumer polls the
// data it needs until every unit carries the epoch. There is no grid-wide barrier: each phase
// waits only for the values it reads, one L2 round trip after the producer stored them.
// Every buffer region is written once per launch (per-layer regions; the attention partials
// alternate between two regions, which the data dependencies of the layers in between keep
// apart: a layer-l+2 item needs layer-l+2 QKV rows from CTAs that have consumed layer l+1's
// h, which every merging CTA publishes only after its layer-l merges).
//
// Phases per layer (outputs split evenly over the CTAs; h rows [own0, own1) of every row are
// owned by one CTA, which keeps them in shared memory):
//   A  xn = RMSNorm(h) (h polled from the previous layer's E, or the pulse input); QKV GEMV
//      rows -> qkv units; gate logits xn.Wg + b on the last 8 CTAs -> gate units. With a live
//      loop adapter, CTAs < MEGA_TDES first compute two rows each of t = A xn and publish
//      them; the QKV rows add Bs t once t is complete.
//   B  attention items (sequence block, kv head, key chunk): q of the 4 heads via
//      QK-RMSNorm + RoPE (+YaRN); the block rows' own K/V (norm, RoPE, value residual) written
//      to the cache by the item that owns their chunk; cached keys of the chunk through the
//      weight ring for passes of <= 2 rows; split-K partials (m, l, o[64]) per head and chunk
//   B2 one CTA per (row, query head) merges its chunk partials in a fixed order and applies
//      the gate sigmoid -> att units
//   C  att polled; Wo GEMV (+ adapter), h += (owned rows) -> h units
//   D  h polled; m = RMSNorm(h); router logits from the fp32 router rows (streamed through
//      the ring; the same arithmetic in every CTA, so every CTA picks the same experts);
//      top-4; shared + routed (distinct experts) gate/up GEMVs, SwiGLU -> act units
//   E  act polled; shared + routed down GEMVs of the owned rows, combine in top-k order,
//      h += -> h units (the last layer publishes the pulse output h_in + (h - h_in) * res_scale)
// Then: the pulse output polled, final RMSNorm, LM head rows, argmax.
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
constexpr int MEGA_ACT = DS + TOPK * DE;  // activations per row entering the down projections
constexpr int MEGA_XS = MEGA_RMAX * MEGA_ACT;   // floats of the per-CTA activation staging
constexpr int MEGA_STAGE = 2048;          // floats
constexpr int MEGA_CHUNK = 64;            // keys per attention item
constexpr int MEGA_MAXPAIRS = 64;         // phase-D output pairs per CTA (>= ceil((1024+16*512)/C))
constexpr int MEGA_MAXOROWS = 8;          // phase-E output rows per CTA (>= ceil(1024/C))
constexpr int MEGA_TDES = LORA_R / 2;     // CTAs computing the loop-adapter factor t (2 rows each)

// Exchange buffers: units of {float, epoch} (zeroed at engine creation, so no unit carries a
// valid epoch before its first store).
struct MegaX {
    uint2* h;       // [NL][2][RMAX][D]: after phase C (0) and phase E (1)
    uint2* qkv;     // [NL][RMAX][QKV]
    uint2* gate;    // [NL][RMAX][H]
    uint2* part;    // [2][RMAX][H][nch_max][PART]
    uint2* att;     // [NL][RMAX][D]
    uint2* act;     // [NL][RMAX][MEGA_ACT]: shared SwiGLU (DS), then routed (TOPK x DE)
    uint2* vfirst;  // [RMAX][HKV][DH]
    uint2* lt;      // [NL][2][RMAX][LORA_R]: loop-adapter t of wqkv (0) and wo (1)
};

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
    MegaX x;
    int nch_max;          // chunks per (row, head) in x.part
    float* pmax;          // LM head: per-CTA argmax partials [R][grid]
    int* pidx;
    unsigned* epoch;      // launch counter: this launch's flag is *epoch + 1; the last CTA out increments it
    unsigned* tickets;    // [0] argmax ticket, [1] leave ticket (both self-resetting)
    int* err;             // error flag (non-zero: a bounded wait ran out)
    unsigned long long wait_ns;   // bound of every wait
    int stall_cta;        // test hook: this CTA (>= 0) waits in layer 0 for units nobody stores
    unsigned long long* experts;  // running count of distinct routed experts streamed (per layer)
    const int* skip;      // optional: non-zero -> the whole pass is skipped (every row exited early)
    unsigned long long* trace;    // optional [gridDim][MEGA_TRACE] %globaltimer stamps (null: off)
};

constexpr int MEGA_TRACE = 256;   // stamps per CTA: [0] start, [1 + 16*l + j] phase points of layer l, [255] end

struct MegaSmem {
    uint64_t full[MEGA_NS];
    uint64_t empty[MEGA_NS];
    float rlog[MEGA_RMAX][E];     // router logits (raw) per (row, expert)
    float logits[MEGA_RMAX][E];   // router: score + bias per (row, expert)
    float rsg[MEGA_RMAX][E];      // router: sigmoid score per (row, expert)
    float wts[MEGA_RMAX][TOPK];
    int idx[MEGA_RMAX][TOPK];
    int elist[E];
    unsigned rmask[MEGA_RMAX];   // experts chosen by each row (bit mask)
    int n_e;
    volatile int moe_ready;
    int ticket;
    volatile int abort;
    alignas(128) unsigned char ring[MEGA_NS][MEGA_SLOT];
    alignas(16) float xs[MEGA_XS];
    alignas(16) float stage[MEGA_STAGE];
    float wout[MEGA_NCW][4 * MEGA_RMAX];   // per-warp reduced tile sums
    int xoff[MEGA_RMAX];                   // X row offsets (elements into xs) of the current phase
    int xoff_e[E][MEGA_RMAX];              // phase E: per routed expert, act row of each row or -1
    int eslot[MEGA_RMAX][TOPK];            // phase E: position of expert idx[r][k] in the expert list
    int blk_r0[MEGA_RMAX + 1];             // sequence blocks of the rows: start row
    int blk_nch[MEGA_RMAX];                // attention chunks per (block, head group)
    int blk_chunk[MEGA_RMAX];
    int n_blk;
    int4 rows[MEGA_RMAX];                  // the row descriptors
    float hown[MEGA_MAXOROWS * MEGA_RMAX]; // owned h rows [row - o0][R] (this CTA is their only writer)
    float hin[MEGA_MAXOROWS * MEGA_RMAX];  // the pulse input of the owned rows
    float g8[MEGA_RMAX][RG];               // re-injection gate (pulses > 0)
    alignas(16) float lt[MEGA_RMAX * LORA_R];   // loop-adapter t of the current GEMV
    float nred[D / 128];                   // norm (one row): sums of squares of the 128-element slices
    float rsc[NL][MEGA_MAXOROWS];          // routed_scale of the owned h rows
    float ebias[NL][E];                    // expert bias of every layer (router top-k)
    float rope[2][MEGA_RMAX][DH];          // [local, global][row]: cos (32) then sin (32) at the row's position
};

__device__ __forceinline__ void stamp(const MegaArgs& a, int l, int j) {
    if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 1 + 16 * l + j] = globaltimer();
}

// attention-item sub-steps of the first item a CTA runs in layer l (entries 130 + 8*l + k)
__device__ __forceinline__ void astamp(const MegaArgs& a, int l, int k, bool first) {
    if (first && a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE + 130 + 8 * l + k] = globaltimer();
}

__device__ __forceinline__ void rows_split(int N, int c, int C, int& r0, int& r1) {
    r0 = (int)(((long long)N * c) / C);
    r1 = (int)(((long long)N * (c + 1)) / C);
}

// ------------------------------------------------------------------ exchange addressing
__device__ __forceinline__ uint2* xh(const MegaArgs& a, int l, int which, int r) {
    return a.x.h + (((int64_t)l * 2 + which) * MEGA_RMAX + r) * D;
}
__device__ __forceinline__ uint2* xqkv(const MegaArgs& a, int l, int r) { return a.x.qkv + ((int64_t)l * MEGA_RMAX + r) * QKV; }
__device__ __forceinline__ uint2* xgate(const MegaArgs& a, int l, int r) { return a.x.gate + ((int64_t)l * MEGA_RMAX + r) * H; }
__device__ __forceinline__ uint2* xpart(const MegaArgs& a, int l, int r, int h, int c) {
    return a.x.part + ((((int64_t)(l & 1) * MEGA_RMAX + r) * H + h) * a.nch_max + c) * PART;
}
// Flag of the attention-partial units of layer l. Layers l and l + 2 share a region within one
// launch, so these units carry the layer as well as the launch (a reader must not take a
// layer-l unit for a layer-(l + 2) one).
__device__ __forceinline__ unsigned part_flag(unsigned f, int l) { return (f << 3) | (unsigned)l; }
__device__ __forceinline__ uint2* xatt(const MegaArgs& a, int l, int r) { return a.x.att + ((int64_t)l * MEGA_RMAX + r) * D; }
__device__ __forceinline__ uint2* xact(const MegaArgs& a, int l, int r) {
    return a.x.act + ((int64_t)l * MEGA_RMAX + r) * MEGA_ACT;
}
__device__ __forceinline__ uint2* xvfirst(const MegaArgs& a, int r, int g) { return a.x.vfirst + ((int64_t)r * HKV + g) * DH; }
__device__ __forceinline__ uint2* xlt(const MegaArgs& a, int l, int which, int r) {
    return a.x.lt + (((int64_t)l * 2 + which) * MEGA_RMAX + r) * LORA_R;
}

// ------------------------------------------------------------------ bounded polling
// A failed wait raises the kernel's error flag and this CTA's abort flag; every later poll of
// the CTA gives up at once, and the phase ends with a uniform branch to the exit.
__device__ __forceinline__ void raise_abort(const MegaArgs& a, MegaSmem* s) {
    if (!s->abort) {
        s->abort = 1;
        atomicExch(a.err, 1);
    }
}

struct Poll {
    unsigned long long t0 = 0;
    unsigned it = 0;
};

// May this thread poll once more? No when the CTA aborted, another CTA raised the error flag
// (read every 128th poll: an L2 round trip of its own) or the wait ran past a.wait_ns.
__device__ __forceinline__ bool poll_more(const MegaArgs& a, MegaSmem* s, Poll& w) {
    if (w.it++ == 0) {
        w.t0 = globaltimer();
        return true;
    }
    if ((w.it & 7) == 0) {
        if (s->abort) return false;
        if (globaltimer() - w.t0 > a.wait_ns) return false;
        if ((w.it & 127) == 0 && *(volatile int*)a.err) return false;
    }
    return true;
}

// One unit's value once it carries flag f (ok cleared on a failed wait).
__device__ __forceinline__ float ll_get(const MegaArgs& a, MegaSmem* s, const uint2* p, unsigned f, bool& ok) {
    uint2 v = ll_ld(p);
    if (v.y != f) {
        Poll w;
        do {
            if (!ok || !poll_more(a, s, w)) {
                ok = false;
                raise_abort(a, s);
                break;
            }
            v = ll_ld(p);
        } while (v.y != f);
    }
    return __uint_as_float(v.x);
}

// Two units, both loads in flight before either is checked.
__device__ __forceinline__ void ll_get2(const MegaArgs& a, MegaSmem* s, const uint2* p0, const uint2* p1, unsigned f,
                                        bool& ok, float& v0, float& v1) {
    uint2 u0 = ll_ld(p0), u1 = ll_ld(p1);
    if (u0.y != f) {
        Poll w;
        do {
            if (!ok || !poll_more(a, s, w)) { ok = false; raise_abort(a, s); break; }
            u0 = ll_ld(p0);
        } while (u0.y != f);
    }
    if (u1.y != f) {
        Poll w;
        do {
            if (!ok || !poll_more(a, s, w)) { ok = false; raise_abort(a, s); break; }
            u1 = ll_ld(p1);
        } while (u1.y != f);
    }
    v0 = __uint_as_float(u0.x);
    v1 = __uint_as_float(u1.x);
}

// Every consumer thread: poll 2 * nl units from src (16-byte aligned) until all carry flag f;
// values to dst[0 .. 2 nl). Eight 16-byte loads per thread in flight before any is checked.
// Not inlined: its registers do not add to the callers' (the phase bodies around it).
static __device__ __noinline__ void ll_fetch(const MegaArgs& a, MegaSmem* s, const uint2* src, int nl, unsigned f,
                                      float* dst, bool& ok) {
    const int tid = threadIdx.x - 32;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    for (int i0 = tid; i0 < nl; i0 += 8 * MEGA_NCT) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = i0 + k * MEGA_NCT;
            if (i < nl) v[k] = ll_ld2(s4 + i);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = i0 + k * MEGA_NCT;
            if (i < nl) {
                if (v[k].y != f || v[k].w != f) {
                    Poll w;
                    do {
                        if (!ok || !poll_more(a, s, w)) { ok = false; raise_abort(a, s); break; }
                        v[k] = ll_ld2(s4 + i);
                    } while (v[k].y != f || v[k].w != f);
                }
                reinterpret_cast<float2*>(dst)[i] = make_float2(__uint_as_float(v[k].x), __uint_as_float(v[k].z));
            }
        }
    }
}

// Bounded mbarrier wait that also gives up when the CTA aborted.
__device__ __forceinline__ bool mbar_wait_ab(const MegaArgs& a, MegaSmem* s, uint64_t* bar, uint32_t parity) {
    if (mbar_test(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (unsigned it = 1; !mbar_test(bar, parity); ++it) {
        if ((it & 15) == 0 && (s->abort || globaltimer() - t0 > a.wait_ns)) return false;
    }
    return true;
}

// ------------------------------------------------------------------ tile stream
// The producer and the consumers walk the same sequence of tiles; `Ring` keeps the counter.
struct Ring {
    MegaSmem* s;
    const MegaArgs* a;
    uint32_t t;     // tiles so far
    int warp;       // consumer warp index (0..14), or -1 for the producer
    bool ok;
};

// Producer side: issue tiles covering rows [r0, r1) of a row-major matrix with row_bytes
// bytes per row, rows_per_tile rows per tile.
__device__ __forceinline__ void produce_rows(Ring& g, const void* base, int row_bytes, int r0, int r1,
                                             int rows_per_tile) {
    for (int r = r0; r < r1 && g.ok; r += rows_per_tile) {
        const int n = min(rows_per_tile, r1 - r);
        const uint32_t slot = g.t % MEGA_NS;
        const uint32_t use = g.t / MEGA_NS;
        if (use > 0 && !mbar_wait_ab(*g.a, g.s, &g.s->empty[slot], (use - 1) & 1)) { g.ok = false; break; }
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
            if (!mbar_wait_ab(*g.a, g.s, &g.s->full[slot], use & 1)) {
                g.ok = false;
                raise_abort(*g.a, g.s);
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

// fp32 rows of D elements (router, gate, loop-adapter A), two rows per tile; same element
// mapping, float4 weight loads. Lane i*R + r of out gets row i for X row r.
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

// RMSNorm of R rows of xs in place with weight w. One row: every consumer thread takes a
// float4, warps reduce their 128-element slices, the eight slice sums are added in order from
// shared memory (red: 8 floats). More rows: one warp per row.
template <int R>
__device__ __forceinline__ void norm_inplace(float* xs, const float* w, float eps, float* red) {
    const int lane = threadIdx.x & 31;
    if constexpr (R == 1) {
        const int tid = threadIdx.x - 32;
        constexpr int N4 = D / 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f), wv = v;
        if (tid < N4) {
            v = reinterpret_cast<const float4*>(xs)[tid];
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
            reinterpret_cast<float4*>(xs)[tid] =
                make_float4(wv.x * (v.x * inv), wv.y * (v.y * inv), wv.z * (v.z * inv), wv.w * (v.w * inv));
        }
    } else {
        const int cw = (threadIdx.x >> 5) - 1;
        for (int r = cw; r < R; r += MEGA_NCW) {
            float v[32], wv[32];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = xs[r * D + i * 32 + lane];
                wv[i] = __ldg(w + i * 32 + lane);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
            ss = warp_sum(ss);
            const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
            for (int i = 0; i < 32; ++i) xs[r * D + i * 32 + lane] = wv[i] * (v[i] * inv);
        }
    }
}

// ------------------------------------------------------------------ attention item
// Chunk of keys per attention item: 32 keys when the span is short (more items than CTAs
// would otherwise sit idle), 64 keys for longer spans.
__device__ __forceinline__ int attn_chunk(int span) { return span <= 32 * 37 ? 32 : 64; }

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
        if (use > 0 && !mbar_wait_ab(*g.a, g.s, &g.s->empty[slot_i], (use - 1) & 1)) { g.ok = false; break; }
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

// Pair w (elements 2w, 2w + 1) of a 64-element K/V row stored as KVT.
__device__ __forceinline__ float2 kv_pair(const __nv_bfloat16* row, int w) {
    return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row)[w]);
}
__device__ __forceinline__ float2 kv_pair(const float* row, int w) { return reinterpret_cast<const float2*>(row)[w]; }

// One attention item: queries of heads 4g..4g+3 of rows r0..r0+nr-1 against the chunk's keys
// [k0, k1). Cached keys (< pos0) come from the ring tiles (R <= 2) or are loaded into shared
// memory (R > 2); the block rows' own keys are produced here. Then a warp per query: scores with
// the chunk's keys on the lanes, softmax with warp shuffles, P.V with dimension pairs on the lanes;
// split-K partials (m, l, o[64]) published as units of the layer's partial flag.
template <int R, typename KVT>
__device__ __noinline__ void attn_item(const MegaArgs& a, MegaSmem* s, Ring& ring, int l, int r0, int nr, int g,
                                       int c, int chunk, unsigned f, bool first, bool& ok) {
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
    const unsigned pf = part_flag(f, l);
    float* qs = s->xs;                                   // [nr*4][64]
    float* Ks = qs + MEGA_RMAX * GQA * DH;               // [64][65] fp32 keys (new ones; R > 2: all)
    float* Vs = Ks + MEGA_CHUNK * (DH + 1);              // [64][65]
    const int nq = nr * GQA;
    astamp(a, l, 0, first);
    // queries (warps) and the block rows' own keys/values, produced here into rows [nold, nk)
    {
        const int vres_mode = (a.pulse == 0) ? (l == 0 ? 1 : 2) : 0;
        const int nnew = max(0, k1 - max(k0, pos0));
        for (int it = cw; it < nq + nnew; it += MEGA_NCW) {
            if (it < nq) {
                const int rr = it / GQA, h = g * GQA + it % GQA;
                const int pos = rows[r0 + rr].y;
                const uint2* src = xqkv(a, l, r0 + rr) + h * DH;
                const float* qw = a.qn[l] + h * DH;
                const float w1 = __ldg(qw + lane), w2 = __ldg(qw + lane + 32);
                const float* rp = s->rope[local ? 0 : 1][r0 + rr];
                const float cs = rp[lane], sn = rp[32 + lane];
                float x1, x2;
                ll_get2(a, s, src + lane, src + lane + 32, f, ok, x1, x2);
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
                const uint2* src = xqkv(a, l, rr);
                const float* kw = a.kn[l] + g * DH;
                const float w1 = __ldg(kw + lane), w2 = __ldg(kw + lane + 32);
                const float* rp = s->rope[local ? 0 : 1][rr];   // row rr sits at position key
                const float cs = rp[lane], sn = rp[32 + lane];
                float e1, e2, v1, v2;
                ll_get2(a, s, src + H * DH + g * DH + lane, src + H * DH + g * DH + lane + 32, f, ok, e1, e2);
                ll_get2(a, s, src + H * DH + HKV * DH + g * DH + lane, src + H * DH + HKV * DH + g * DH + lane + 32, f,
                        ok, v1, v2);
                uint2* vf = xvfirst(a, rr, g);
                if (vres_mode == 1) {
                    ll_st(vf + lane, v1, f);
                    ll_st(vf + lane + 32, v2, f);
                } else if (vres_mode == 2) {
                    float f1, f2;   // the first layer's values (value residual)
                    ll_get2(a, s, vf + lane, vf + lane + 32, f, ok, f1, f2);
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
    }
    astamp(a, l, 1, first);
    // cached keys/values: R <= 2 the ring tiles the producer streamed during phase A (ntk tiles of
    // K, then ntk of V, waited for here and released after the compute); larger passes load them
    // here into Ks / Vs, every thread's 16-byte loads issued first
    constexpr int KPT = kv_keys_per_tile<KVT>();
    constexpr int ROW = DH;   // elements per cached row
    const KVT* kt[MEGA_CHUNK / KPT + 1];
    const KVT* vt[MEGA_CHUNK / KPT + 1];
    int ntk = 0;
    if constexpr (R <= MEGA_RING_KV_MAX_R) {
        ntk = (nold + KPT - 1) / KPT;
        for (int i = 0; i < 2 * ntk; ++i) {
            const uint32_t t = ring.t + i;
            if (ring.ok && !mbar_wait_ab(a, s, &s->full[t % MEGA_NS], (t / MEGA_NS) & 1)) {
                ring.ok = false;
                raise_abort(a, s);
            }
            const KVT* tile = reinterpret_cast<const KVT*>(s->ring[t % MEGA_NS]);
            if (i < ntk) kt[i] = tile; else vt[i - ntk] = tile;
        }
    } else {
        constexpr int PARTS = (sizeof(KVT) == 2) ? 8 : 16;   // 16-byte pieces per 64-element row
        for (int e = tid; e < 2 * nold * PARTS; e += MEGA_NCT) {
            const int isv = e >= nold * PARTS;
            const int ee = isv ? e - nold * PARTS : e;
            const int kk = ee / PARTS, part = ee % PARTS;
            const KVT* row = isv ? kv_v<KVT>(L, slot, g, k0 + kk) : kv_k<KVT>(L, slot, g, k0 + kk);
            load_kv_row16<KVT>(row, part, (isv ? Vs : Ks) + kk * (DH + 1));
        }
    }
    named_bar_sync(1, MEGA_NCT);   // queries, produced keys (and loaded keys) visible
    astamp(a, l, 2, first);
    constexpr bool TILES = R <= MEGA_RING_KV_MAX_R;
    for (int qi = cw; qi < nq; qi += MEGA_NCW) {
        const int rr = qi / GQA, h = g * GQA + qi % GQA;
        const int pos = rows[r0 + rr].y;
        const int lor = local ? max(0, pos - WINDOW + 1) : 0;
        const float* q = qs + qi * DH;
        // scores: lane holds keys lane and lane + 32 of the chunk. A cached row in a ring tile is
        // read in rotated pair order (pair (j + lane) mod 32 at step j: one bank per lane)
        float sc[2];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int kk = lane + 32 * half;
            const int key = k0 + kk;
            float v = -INFINITY;
            if (kk < nk && key <= pos && key >= lor) {
                float acc = 0.f;
                if (TILES && kk < nold) {
                    const KVT* row = kt[kk / KPT] + (kk % KPT) * ROW;
#pragma unroll 8
                    for (int j = 0; j < DH / 2; ++j) {
                        const int w = (j + lane) & (DH / 2 - 1);
                        const float2 kv2 = kv_pair(row, w);
                        const float2 q2 = reinterpret_cast<const float2*>(q)[w];
                        acc += q2.x * kv2.x + q2.y * kv2.y;
                    }
                } else {
                    const float* row = Ks + kk * (DH + 1);
#pragma unroll 16
                    for (int d = 0; d < DH; ++d) acc += q[d] * row[d];
                }
                v = acc;
            }
            sc[half] = v;
        }
        const float m = warp_max(fmaxf(sc[0], sc[1]));   // -inf: no key of the chunk is visible to this row
        const float e0 = (sc[0] == -INFINITY) ? 0.f : expf(sc[0] - m);
        const float e1 = (sc[1] == -INFINITY) ? 0.f : expf(sc[1] - m);
        const float lsum = warp_sum(e0 + e1);
        // P.V: lane holds dimensions 2 lane, 2 lane + 1; keys in order
        float o0 = 0.f, o1 = 0.f;
        for (int kk = 0; kk < nk; ++kk) {
            const float pw = __shfl_sync(0xffffffffu, kk < 32 ? e0 : e1, kk & 31);
            if (pw == 0.f) continue;   // warp-uniform: masked key
            float2 v2;
            if (TILES && kk < nold) {
                v2 = kv_pair(vt[kk / KPT] + (kk % KPT) * ROW, lane);
            } else {
                const float* row = Vs + kk * (DH + 1);
                v2 = make_float2(row[2 * lane], row[2 * lane + 1]);
            }
            o0 += pw * v2.x;
            o1 += pw * v2.y;
        }
        uint2* out = xpart(a, l, r0 + rr, h, c);
        if (lane == 0) {
            ll_st(out, m, pf);
            ll_st(out + 1, m == -INFINITY ? 0.f : lsum, pf);
        }
        ll_st(out + 2 + 2 * lane, o0, pf);
        ll_st(out + 3 + 2 * lane, o1, pf);
    }
    named_bar_sync(1, MEGA_NCT);   // every warp is done with the tiles and with Ks / Vs
    if constexpr (TILES) {
        if (threadIdx.x == 32 && ring.ok)
            for (int i = 0; i < 2 * ntk; ++i) mbar_arrive(&s->empty[(ring.t + i) % MEGA_NS]);
        ring.t += 2 * ntk;
    }
    astamp(a, l, 3, first);
}

// Merge the chunk partials (m, l, o[64]) of query head h of row r, apply the gate, publish
// att[r][h*64 ..]: every consumer thread takes part of the partials in one batched poll into
// shared memory; warp 0 then forms the softmax weights of the chunks and the weighted sums.
static __device__ __noinline__ void attn_merge(const MegaArgs& a, MegaSmem* s, int l, int r, int h, int nch,
                                               unsigned f, bool& ok) {
    const int cw = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
    float* P = s->xs;   // [nch][PART]; xs is free between the attention items and phase C
    ll_fetch(a, s, xpart(a, l, r, h, 0), nch * PART / 2, part_flag(f, l), P, ok);
    named_bar_sync(1, MEGA_NCT);
    if (cw == 0) {
        const float graw = ll_get(a, s, xgate(a, l, r) + h, f, ok);
        float mx = -INFINITY;
        for (int c = lane; c < nch; c += 32) mx = fmaxf(mx, P[c * PART]);
        const float M = warp_max(mx);
        float lsum = 0.f;
        for (int c = lane; c < nch; c += 32) {
            const float m = P[c * PART];
            const float w = (m == -INFINITY) ? 0.f : expf(m - M);
            s->stage[c] = w;
            lsum += w * P[c * PART + 1];
        }
        const float Ls = warp_sum(lsum);
        __syncwarp();
        float p1 = 0.f, p2 = 0.f;
        for (int c = 0; c < nch; ++c) {
            const float w = s->stage[c];
            p1 += w * P[c * PART + 2 + lane];
            p2 += w * P[c * PART + 2 + 32 + lane];
        }
        const float gt = sigmoidf_(graw);
        const float inv = 1.f / Ls;
        uint2* out = xatt(a, l, r) + h * DH;
        ll_st(out + lane, (p1 * inv) * gt, f);
        ll_st(out + 32 + lane, (p2 * inv) * gt, f);
    }
    named_bar_sync(1, MEGA_NCT);
}

// Consumer exit of every CTA: the last CTA out advances the launch counter (the next launch's
// flag) and re-arms the leave ticket.
__device__ __forceinline__ void mega_leave(const MegaArgs& a) {
    if (threadIdx.x == 32) {
        if (a.trace) a.trace[blockIdx.x * MEGA_TRACE + MEGA_TRACE - 2] = globaltimer();
        __threadfence();
        const unsigned t = atomicAdd(&a.tickets[1], 1u);
        if (t == gridDim.x - 1) {
            a.tickets[1] = 0;
            atomicAdd(a.epoch, 1u);
        }
    }
}

// Loop-adapter factor rows of this CTA (CTAs < MEGA_TDES): t[r][2 cta + i] = A[2 cta + i] . X_r,
// published for every CTA of the phase.
template <int R>
__device__ __forceinline__ void adapter_t(Ring& g, MegaSmem* s, const MegaArgs& a, int l, int which, unsigned f) {
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    float* wo = s->wout[(threadIdx.x >> 5) - 1];
    consume_rows(g, 2 * cta, 2 * cta + 2, 2, [&](const unsigned char* tile, int row0, int n) {
        tile_gemv_f32<R>(reinterpret_cast<const float*>(tile), n, s->xs, s->xoff, wo);
        if (lane < n * R) ll_st(xlt(a, l, which, lane % R) + row0 + lane / R, wo[lane], f);
    });
}

// ------------------------------------------------------------------ the pulse
template <int R, typename KVT>
__global__ void __launch_bounds__(MEGA_THREADS, 1) k_mega_pulse(const __grid_constant__ MegaArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    MegaSmem* s = reinterpret_cast<MegaSmem*>(smem_raw);
    const int C = gridDim.x, cta = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool want_lm = a.logits != nullptr || a.amax != nullptr;
    const bool adapter = a.la_qkv[0] != nullptr;
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
        Ring g{s, &a, 0u, -1, true};
        int pblk[MEGA_RMAX + 1], pnb = 0;   // sequence blocks of the rows (as the consumers build them)
        for (int r0 = 0; r0 < R;) {
            int nr = 1;
            while (r0 + nr < R && s->rows[r0 + nr].x == s->rows[r0].x) ++nr;
            pblk[pnb++] = r0;
            r0 += nr;
        }
        pblk[pnb] = R;
        if (a.pulse > 0) produce_rows(g, a.rg_down, 2 * D * 4, 0, RG, 1);   // re-injection gate rows
#pragma unroll 1
        for (int l = 0; l < NL && g.ok; ++l) {
            int r0, r1;
            if (adapter && cta < MEGA_TDES) produce_rows(g, a.la_qkv[l], D * 4, 2 * cta, 2 * cta + 2, 2);
            rows_split(QKV, cta, C, r0, r1);
            produce_rows(g, a.wqkv[l], D * 2, r0, r1, 4);
            // gate rows: the last H/2 CTAs
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
            if (adapter && cta < MEGA_TDES) produce_rows(g, a.la_wo[l], D * 4, 2 * cta, 2 * cta + 2, 2);
            rows_split(D, cta, C, r0, r1);
            produce_rows(g, a.wo[l], D * 2, r0, r1, 4);
            produce_rows(g, a.router[l], D * 4, 0, E, 2);   // fp32 router rows (every CTA)
            {   // shared-expert pairs: a static split, prefetched before the router runs
                int j0, j1;
                rows_split(DS, cta, C, j0, j1);
                produce_rows(g, a.sh_gu[l], D * 2, j0, j1, 4);
                produce_rows(g, a.sh_gu[l], D * 2, DS + j0, DS + j1, 4);
            }
            // routed pairs depend on this layer's router. Short sleeps between polls (a tight
            // spin on shared memory starves the consumers' loads)
            const unsigned long long t0 = globaltimer();
            for (unsigned it = 1; s->moe_ready != l + 1; ++it) {
                __nanosleep(32);
                if ((it & 15) == 0 && (s->abort || globaltimer() - t0 > a.wait_ns)) {
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
        if (!g.ok) raise_abort(a, s);
        // drain: wait for every copy this thread issued to land before the CTA can exit
        for (uint32_t t = (g.t > MEGA_NS ? g.t - MEGA_NS : 0); t < g.t; ++t)
            if (!mbar_wait(&s->full[t % MEGA_NS], (t / MEGA_NS) & 1)) break;
        return;
    }

    // ================================================================ consumers
    const int cw = warp - 1;
    const int tid = threadIdx.x - 32;
    if (a.trace && threadIdx.x == 32) a.trace[blockIdx.x * MEGA_TRACE] = globaltimer();
    const unsigned f = ld_acquire_gpu(a.epoch) + 1u;   // this launch's flag (same in every CTA)
    Ring g{s, &a, 0u, cw, true};
    bool ok = true;   // this thread's waits all succeeded
    float* xs = s->xs;
    float* wo_ = s->wout[cw];   // this warp's reduced tile sums
    const float eps = a.eps;
    const int p = a.pulse;
    // h rows [own0, own1) are this CTA's outputs in phases C and E
    int own0, own1;
    rows_split(D, cta, C, own0, own1);
    const int nown = own1 - own0;
    for (int t = tid; t < NL * MEGA_MAXOROWS; t += MEGA_NCT) {
        const int ll = t / MEGA_MAXOROWS, oi = t % MEGA_MAXOROWS;
        s->rsc[ll][oi] = oi < nown ? a.rscale[ll][own0 + oi] : 0.f;
    }
    for (int t = tid; t < NL * E; t += MEGA_NCT) s->ebias[t / E][t % E] = a.ebias[t / E][t % E];
    for (int t = tid; t < 2 * R * DH; t += MEGA_NCT) {
        const int tab = t / (R * DH), r = (t / DH) % R, j = t % DH;
        const float* T = (j < 32) ? (tab ? a.cos_g : a.cos_l) : (tab ? a.sin_g : a.sin_l);
        s->rope[tab][r][j] = T[(int64_t)s->rows[r].y * 32 + (j & 31)];
    }
    if (tid < R) s->xoff[tid] = tid * D;
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
        // xs[r*D ..] = h0n_in[r], xs[R*D + r*D ..] = RMSNorm(h_prev[r]) (pulse-state norm);
        // g8[r][j] = Wd[j][:D] . h0n[r] + Wd[j][D:] . RMSNorm(h_prev[r]) from the ring's gate rows
        float* rn = xs + R * D;
        for (int r = cw; r < R; r += MEGA_NCW) {
            float v[32];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = __ldg(a.h_prev + r * D + i * 32 + lane);
                ss += v[i] * v[i];
            }
            const float inv = rsqrtf(warp_sum(ss) / (float)D + eps);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int d = i * 32 + lane;
                rn[r * D + d] = __ldg(a.psn + d) * (v[i] * inv);
                xs[r * D + d] = __ldg(a.h0n_in + r * D + d);
            }
        }
        named_bar_sync(1, MEGA_NCT);
        consume_rows(g, 0, RG, 1, [&](const unsigned char* tile, int j, int) {
            const float* wd = reinterpret_cast<const float*>(tile);
            for (int r = 0; r < R; ++r) {
                float pe = 0.f, pr = 0.f;
                for (int i = lane * 4; i < D; i += 128) {
                    const float4 w0 = *reinterpret_cast<const float4*>(wd + i);
                    const float4 w1 = *reinterpret_cast<const float4*>(wd + D + i);
                    const float4 x0 = *reinterpret_cast<const float4*>(xs + r * D + i);
                    const float4 x1 = *reinterpret_cast<const float4*>(rn + r * D + i);
                    pe += w0.x * x0.x + w0.y * x0.y + w0.z * x0.z + w0.w * x0.w;
                    pr += w1.x * x1.x + w1.y * x1.y + w1.z * x1.z + w1.w * x1.w;
                }
                pe = warp_sum(pe);
                pr = warp_sum(pr);
                if (lane == 0) s->g8[r][j] = pe + pr;
            }
        });
        named_bar_sync(1, MEGA_NCT);
        for (int e = tid; e < R * D; e += MEGA_NCT) {
            const int r = e / D, d = e % D;
            const float4 u0 = __ldg(reinterpret_cast<const float4*>(a.rg_up + d * RG));
            const float4 u1 = __ldg(reinterpret_cast<const float4*>(a.rg_up + d * RG + 4));
            const float* gg = s->g8[r];
            const float z = __ldg(a.rg_bias + d) + u0.x * gg[0] + u0.y * gg[1] + u0.z * gg[2] + u0.w * gg[3] +
                            u1.x * gg[4] + u1.y * gg[5] + u1.z * gg[6] + u1.w * gg[7];
            const float mix = sigmoidf_(z);
            const float rv = rn[e], an = xs[e];
            const float diff = an - rv;
            const float lerp = (mix < 0.5f) ? rv + mix * diff : an - diff * (1.f - mix);
            xs[e] = lerp + __ldg(a.step + d);
        }
        if (cta == 0 && a.h0n_out && a.h0n_out != a.h0n_in) {   // caller buffers: scalar accesses, no alignment assumed
#pragma unroll 4
            for (int i = tid; i < R * D; i += MEGA_NCT)
                a.h0n_out[(int64_t)(i / D) * a.hstride * D + i % D] = __ldg(a.h0n_in + i);
        }
    }
    named_bar_sync(1, MEGA_NCT);
    for (int t = tid; t < nown * R; t += MEGA_NCT) {
        const float v = xs[(t % R) * D + own0 + t / R];
        s->hown[t] = v;
        s->hin[t] = v;
    }
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
    named_bar_sync(1, MEGA_NCT);
    // one copy of the layer body (not unrolled), so it can stay in the instruction caches
#pragma unroll 1
    for (int l = 0; l < NL; ++l) {
        const bool local = is_local_layer(l);
        // ---------------- phase A: xn, QKV, gate logits
        {
            if (l > 0) {
                ll_fetch(a, s, xh(a, l - 1, 1, 0), R * D / 2, f, xs, ok);
                if (named_bar_or(1, MEGA_NCT, !ok)) goto done;
            }
            norm_inplace<R>(xs, a.attn_norm[l], eps, s->nred);
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
            if (adapter && cta < MEGA_TDES) adapter_t<R>(g, s, a, l, 0, f);
            int r0, r1;
            rows_split(QKV, cta, C, r0, r1);
            if (!adapter) {
                consume_rows(g, r0, r1, 4, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) ll_st(xqkv(a, l, lane % R) + row0 + lane / R, wo_[lane], f);
                });
            } else {
                float* st = s->stage;   // [row - r0][R]
                consume_rows(g, r0, r1, 4, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) st[(row0 - r0 + lane / R) * R + lane % R] = wo_[lane];
                });
                ll_fetch(a, s, xlt(a, l, 0, 0), R * LORA_R / 2, f, s->lt, ok);
                named_bar_sync(1, MEGA_NCT);
                for (int e = tid; e < (r1 - r0) * R; e += MEGA_NCT) {
                    const int o = r0 + e / R, r = e % R;
                    const float* bt = a.lb_qkv[l] + (int64_t)o * LORA_R;
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < LORA_R; ++j) d += __ldg(bt + j) * s->lt[r * LORA_R + j];
                    ll_st(xqkv(a, l, r) + o, st[e] + d, f);
                }
            }
            stamp(a, l, 1);
            // gate logits xn . Wg + b of two heads on each of the last H/2 CTAs
            if (cta >= C - H / 2) {
                const int gr = 2 * (cta - (C - H / 2));
                consume_rows(g, gr, gr + 2, 2, [&](const unsigned char* tile, int row0, int n) {
                    tile_gemv_f32<R>(reinterpret_cast<const float*>(tile), n, xs, s->xoff, wo_);
                    if (lane < n * R) {
                        const int h = row0 + lane / R;
                        ll_st(xgate(a, l, lane % R) + h, wo_[lane] + a.gate_b[l][h], f);
                    }
                });
            }
            stamp(a, l, 2);
            // xs is scratch for the attention items below
            if (named_bar_or(1, MEGA_NCT, !ok || !g.ok)) goto done;
            stamp(a, l, 3);
        }
        // ---------------- phase B: attention (items owned by this CTA: cta, cta + C, ...)
        {
            int total = 0;
            for (int b = 0; b < s->n_blk; ++b) total += HKV * s->blk_nch[b];
            bool first = true;
            for (int item = cta; item < total; item += C) {
                int b = 0, rem = item;
                while (rem >= HKV * s->blk_nch[b]) { rem -= HKV * s->blk_nch[b]; ++b; }
                const int nch = s->blk_nch[b];
                const int r0 = s->blk_r0[b], nr = s->blk_r0[b + 1] - r0;
                attn_item<R, KVT>(a, s, g, l, r0, nr, rem / nch, rem % nch, s->blk_chunk[b], f, first, ok);
                first = false;
            }
            stamp(a, l, 4);
            stamp(a, l, 5);
        }
        // ---------------- phase B2: merge the chunk partials of each (row, head) and gate
        // (units on the last CTAs, which have the fewest attention items)
        {
            for (int u = C - 1 - cta; u < R * H; u += C) {
                const int r = u / H;
                int b = 0;
                while (s->blk_r0[b + 1] <= r) ++b;
                attn_merge(a, s, l, r, u % H, s->blk_nch[b], f, ok);
            }
            stamp(a, l, 6);
            if (named_bar_or(1, MEGA_NCT, !ok || !g.ok)) goto done;
        }
        // ---------------- phase C: Wo, h += (owned rows)
        {
            // test hook: one CTA waits for units of a flag no launch stores (bounded wait)
            ll_fetch(a, s, xatt(a, l, 0), R * D / 2, (cta == a.stall_cta && l == 0) ? (f ^ 0x80000000u) : f, xs, ok);
            if (named_bar_or(1, MEGA_NCT, !ok)) goto done;
            stamp(a, l, 7);
            if (adapter && cta < MEGA_TDES) adapter_t<R>(g, s, a, l, 1, f);
            float* st = s->stage;   // [row - own0][R]
            consume_rows(g, own0, own1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, D>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) st[(row0 - own0 + lane / R) * R + lane % R] = wo_[lane];
            });
            if (adapter) ll_fetch(a, s, xlt(a, l, 1, 0), R * LORA_R / 2, f, s->lt, ok);
            named_bar_sync(1, MEGA_NCT);
            for (int e = tid; e < nown * R; e += MEGA_NCT) {
                const int o = own0 + e / R, r = e % R;
                float y = st[e];
                if (adapter) {
                    const float* bt = a.lb_wo[l] + (int64_t)o * LORA_R;
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < LORA_R; ++j) d += __ldg(bt + j) * s->lt[r * LORA_R + j];
                    y += d;
                }
                const float v = s->hown[e] + y;
                s->hown[e] = v;
                ll_st(xh(a, l, 0, r) + o, v, f);
            }
            stamp(a, l, 8);
            if (named_bar_or(1, MEGA_NCT, !ok || !g.ok)) goto done;
        }
        // ---------------- phase D: router, shared + routed up-projections
        {
            ll_fetch(a, s, xh(a, l, 0, 0), R * D / 2, f, xs, ok);
            if (named_bar_or(1, MEGA_NCT, !ok)) goto done;
            stamp(a, l, 9);
            norm_inplace<R>(xs, a.mlp_norm[l], eps, s->nred);
            named_bar_sync(1, MEGA_NCT);
            // router logits of every row from the fp32 router rows (two per tile)
            consume_rows(g, 0, E, 2, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv_f32<R>(reinterpret_cast<const float*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) s->rlog[lane % R][row0 + lane / R] = wo_[lane];
            });
            named_bar_sync(1, MEGA_NCT);
            // a warp per row: centre, sigmoid; top-4 of s + bias by rank (expert e is chosen
            // iff fewer than 4 experts beat it, ties to the lower expert), weights
            const float ebias_lane = (lane < E) ? s->ebias[l][lane] : 0.f;
            for (int r = cw; r < R; r += MEGA_NCW) {
                const float lg = lane < E ? s->rlog[r][lane] : 0.f;
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
            // phase E: act row of each row for every routed expert (or -1)
            for (int t = tid; t < s->n_e * R; t += MEGA_NCT) {
                const int ei = t / R, r = t % R;
                int off = -1;
#pragma unroll
                for (int k = 0; k < TOPK; ++k)
                    if (s->idx[r][k] == s->elist[ei]) off = r * MEGA_ACT + DS + k * DE;
                s->xoff_e[ei][r] = off;
            }
            for (int t = tid; t < R * TOPK; t += MEGA_NCT) {
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
            // SwiGLU epilogue -> act units: shared [r][0 .. DS), routed [r][DS + k*DE + j]
            for (int e = tid; e < (nsh + q1 - q0) * R; e += MEGA_NCT) {
                const int pi = e / R, r = e % R;
                const float v = siluf_(st_g[pi * R + r]) * st_u[pi * R + r];
                if (pi < nsh) {
                    ll_st(xact(a, l, r) + s0 + pi, v, f);
                } else {
                    const int q = q0 + pi - nsh;
                    const int ei = q / DE, j = q % DE;
                    const int ex = s->elist[ei];
#pragma unroll
                    for (int k = 0; k < TOPK; ++k)
                        if (s->idx[r][k] == ex) ll_st(xact(a, l, r) + DS + k * DE + j, v, f);
                }
            }
            stamp(a, l, 12);
            if (named_bar_or(1, MEGA_NCT, !ok || !g.ok)) goto done;
        }
        // ---------------- phase E: down projections + combine, h += (owned rows)
        {
            ll_fetch(a, s, xact(a, l, 0), R * MEGA_ACT / 2, f, xs, ok);
            if (tid < R) s->xoff[tid] = tid * MEGA_ACT;   // shared act rows
            if (named_bar_or(1, MEGA_NCT, !ok)) goto done;
            stamp(a, l, 13);
            const int n_e = s->n_e;
            float* dsh = s->stage;                                   // [orow][R]
            float* dex = s->stage + MEGA_MAXOROWS * R;               // [orow][ei][R]
            consume_rows(g, own0, own1, 4, [&](const unsigned char* tile, int row0, int n) {
                tile_gemv<R, DS>(reinterpret_cast<const __nv_bfloat16*>(tile), n, xs, s->xoff, wo_);
                if (lane < n * R) dsh[(row0 - own0 + lane / R) * R + lane % R] = wo_[lane];
            });
            for (int ei = 0; ei < n_e; ++ei) {
                consume_rows(g, own0, own1, 8, [&](const unsigned char* tile, int row0, int n) {
                    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(tile);
                    for (int half = 0; half < 2; ++half) {
                        const int nn = min(4, n - half * 4);
                        if (nn <= 0) break;
                        tile_gemv<R, DE>(w + half * 4 * DE, nn, xs, s->xoff_e[ei], wo_);
                        if (lane < nn * R)
                            dex[((row0 + half * 4 - own0 + lane / R) * E + ei) * R + lane % R] = wo_[lane];
                        __syncwarp();
                    }
                });
            }
            named_bar_sync(1, MEGA_NCT);
            stamp(a, l, 14);
            if (tid < R) s->xoff[tid] = tid * D;   // back to [R][D] activation rows
            const bool last = l == NL - 1;
            for (int e = tid; e < nown * R; e += MEGA_NCT) {
                const int oi = e / R, r = e % R;
                const int o = own0 + oi;
                float routed = 0.f;
#pragma unroll
                for (int k = 0; k < TOPK; ++k) routed = routed + dex[(oi * E + s->eslot[r][k]) * R + r] * s->wts[r][k];
                const float v = s->hown[e] + (dsh[e] + routed * s->rsc[l][oi]);
                s->hown[e] = v;
                if (!last) {
                    ll_st(xh(a, l, 1, r) + o, v, f);
                } else {   // the pulse output h_in + (h - h_in) * res_scale
                    const float hi = s->hin[e];
                    const float out = hi + (v - hi) * __ldg(a.res_scale + o);
                    a.h_out[(int64_t)r * a.hstride * D + o] = out;
                    ll_st(xh(a, l, 1, r) + o, out, f);
                }
            }
            stamp(a, l, 15);
            if (named_bar_or(1, MEGA_NCT, !ok || !g.ok)) goto done;
        }
    }
    // ---------------- final norm + LM head
    if (want_lm) {
        ll_fetch(a, s, xh(a, NL - 1, 1, 0), R * D / 2, f, xs, ok);
        if (named_bar_or(1, MEGA_NCT, !ok)) goto done;
        norm_inplace<R>(xs, a.fnorm, eps, s->nred);
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
        if (tid < R) {
            const int r = tid;
            ArgMax b{bv[r], bi[r]};
            for (int w = 1; w < MEGA_NCW; ++w) b = argmax_merge(b, ArgMax{bv[w * R + r], bi[w * R + r]});
            a.pmax[r * C + cta] = b.v;
            a.pidx[r * C + cta] = b.i;
        }
        __threadfence();
        named_bar_sync(1, MEGA_NCT);
        if (threadIdx.x == 32) {
            const unsigned t = atomicAdd(&a.tickets[0], 1u);
            s->ticket = (t == (unsigned)(C - 1));
            if (s->ticket) a.tickets[0] = 0;
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
        if (!g.ok) raise_abort(a, s);
    }
done:
    mega_leave(a);
}

}  // namespace pulsar
