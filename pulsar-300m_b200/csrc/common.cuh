// Shared device helpers and the compiled model shape of the Pulsar-283M decode engine.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pulsar {

// ---- compiled shape (src/model.py:13-72 defaults; every BASELINE config uses them) ----
constexpr int D = 1024;          // d_model
constexpr int H = 16;            // query heads
constexpr int HKV = 4;           // kv heads
constexpr int DH = 64;           // head dim
constexpr int GQA = H / HKV;     // query heads per kv head
constexpr int QKV = H * DH + 2 * HKV * DH;   // 1536
constexpr int E = 16;            // routed experts
constexpr int TOPK = 4;
constexpr int DE = 512;          // routed expert hidden
constexpr int DS = 1024;         // shared expert hidden
constexpr int NL = 8;            // physical layers
constexpr int NP = 3;            // pulses (default_pulses)
constexpr int RG = 8;            // re-injection gate rank
constexpr int WINDOW = 1024;     // sliding window of local layers
constexpr int LOCAL_RING = 2048; // ring slots per local layer (window + verify block slack)
constexpr int MAX_ROWS = 32;     // rows of one small-batch pulse pass (GEMV regime)
constexpr int MAX_BATCH = 1024;  // sequence slots of one engine
constexpr int MAX_GAMMA = 7;     // drafts per speculative round (verify blocks of <= 8 rows)

__host__ __device__ constexpr bool is_local_layer(int l) { return l != 3 && l != 7; }

// ---- bf16 helpers ----
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float* f) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __bfloat1622float2(p[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
    uint4 v;
    __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once per pass).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// x as bf16 hi + lo halves at index i (|x - hi - lo| <= 2^-16 |x|): the activation operand of
// the tensor-core GEMMs, written by the kernel that produces x.
__device__ __forceinline__ void split_store(__nv_bfloat16* hi, __nv_bfloat16* lo, int64_t i, float x) {
    const __nv_bfloat16 h = __float2bfloat16(x);
    hi[i] = h;
    lo[i] = __float2bfloat16(x - __bfloat162float(h));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; ``red`` holds >= 32 floats of shared memory. All threads get the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
    if (warp == 0) {
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    float r = red[0];
    __syncthreads();
    return r;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.f + expf(-x)); }

// Argmax with ties to the lowest index (torch.argmax on CPU).
struct ArgMax {
    float v;
    int i;
};
__device__ __forceinline__ ArgMax argmax_merge(ArgMax a, ArgMax b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}
__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgMax b;
        b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
        b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
        a = argmax_merge(a, b);
    }
    return a;
}

}  // namespace pulsar
