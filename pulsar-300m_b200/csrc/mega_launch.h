// Host interface of the persistent pulse kernel (implemented in mega.cu).
#pragma once

#include <cuda_runtime.h>

#include "megakernel.cuh"

namespace pulsar {

size_t mega_smem_bytes();
// Zero the grid-barrier counter and launch k_mega_pulse<a.R, KV> cooperatively on `grid` CTAs.
int launch_mega(const MegaArgs& a, bool kv32, int grid, cudaStream_t st);
int mega_occupancy(bool kv32, int* blocks_per_sm);

}  // namespace pulsar
