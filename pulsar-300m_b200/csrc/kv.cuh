// KV-cache view shared by the per-op kernels and the persistent pulse kernel.
//   Per sequence slot and layer: K [HKV][cap][64] then V [HKV][cap][64] of type KVT (bf16
//   or fp32). Local layers are a ring of `cap` = 2048 slots addressed by pos & 2047 (or by
//   pos when the whole context fits); global layers are addressed by pos.
#pragma once

#include "common.cuh"

namespace pulsar {

constexpr int LORA_R = 24;          // 3 pulses x rank 8
constexpr int ATT_CHUNK = 128;      // keys per split-K attention block
constexpr int PART = 2 + DH;        // (m, l, o[64]) per head per chunk

struct KVLayer {
    void* base;          // this layer's block inside slot 0
    int64_t slot_stride; // elements between slots
    int cap;             // positions per head
    int mask;            // position -> index mask (ring) or -1 (identity)
};

template <typename KVT>
__device__ __forceinline__ KVT* kv_k(const KVLayer& L, int slot, int g, int pos) {
    const int idx = pos & L.mask;
    return reinterpret_cast<KVT*>(L.base) + (int64_t)slot * L.slot_stride + ((int64_t)g * L.cap + idx) * DH;
}
template <typename KVT>
__device__ __forceinline__ KVT* kv_v(const KVLayer& L, int slot, int g, int pos) {
    return kv_k<KVT>(L, slot, g, pos) + (int64_t)HKV * L.cap * DH;
}

__device__ __forceinline__ float kv_load(const float* p) { return *p; }
__device__ __forceinline__ float kv_load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__nv_bfloat16* p, float v) { *p = __float2bfloat16(v); }
// The value a store of v to a cache of element type KVT reads back as.
template <typename KVT>
__device__ __forceinline__ float kv_round(float v);
template <>
__device__ __forceinline__ float kv_round<float>(float v) { return v; }
template <>
__device__ __forceinline__ float kv_round<__nv_bfloat16>(float v) { return __bfloat162float(__float2bfloat16(v)); }

}  // namespace pulsar
