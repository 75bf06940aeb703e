// Instantiations and the cooperative launcher of the persistent pulse kernel.
#include <cuda_runtime.h>

#include "capi_util.h"
#include "mega_launch.h"
#include "megakernel.cuh"

namespace pulsar {

size_t mega_smem_bytes() { return sizeof(MegaSmem) + 128; }

template <int R, typename KVT>
static int launch_one(const MegaArgs& a, int grid, cudaStream_t st) {
    auto fn = k_mega_pulse<R, KVT>;
    PULSAR_TRY(ensure_smem_attr(reinterpret_cast<const void*>(fn), (int)mega_smem_bytes(), "cudaFuncSetAttribute(mega)"));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MEGA_THREADS);
    cfg.dynamicSmemBytes = mega_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, fn, a), "launch k_mega_pulse");
}

template <typename KVT>
static int launch_r(const MegaArgs& a, int grid, cudaStream_t st) {
    switch (a.R) {
        case 1: return launch_one<1, KVT>(a, grid, st);
        case 2: return launch_one<2, KVT>(a, grid, st);
        case 3: return launch_one<3, KVT>(a, grid, st);
        case 4: return launch_one<4, KVT>(a, grid, st);
        case 5: return launch_one<5, KVT>(a, grid, st);
        default:
            set_error("megakernel: R=%d outside [1, %d]", a.R, MEGA_RMAX);
            return PULSAR_ERR_INVALID;
    }
}

// The barrier counter starts at zero: zeroed at engine creation and re-armed by the last CTA
// of every launch.
int launch_mega(const MegaArgs& a, bool kv32, int grid, cudaStream_t st) {
    return kv32 ? launch_r<float>(a, grid, st) : launch_r<__nv_bfloat16>(a, grid, st);
}

int mega_occupancy(bool kv32, int* blocks_per_sm) {
    auto fn = kv32 ? k_mega_pulse<5, float> : k_mega_pulse<5, __nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mega_smem_bytes());
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(mega)");
    return cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, fn, MEGA_THREADS, mega_smem_bytes()),
                       "occupancy(mega)");
}

}  // namespace pulsar
