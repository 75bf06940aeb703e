// Host-side helpers shared by the C-ABI translation units: thread-local error text and
// argument / launch checking that turns failures into PULSAR_ERR_* codes.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <string>

#include "../../include/pulsar_b200.h"

namespace pulsar {

void set_error(const char* fmt, ...);
void clear_error();

// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, bytes) once per (kernel, device): the
// attribute belongs to the device current when it is set, so each GPU a process uses needs it.
int ensure_smem_attr(const void* fn, int bytes, const char* what);

inline int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return PULSAR_OK;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? PULSAR_ERR_OOM : PULSAR_ERR_CUDA;
}

// Check the most recent launch (configuration errors surface here, asynchronous faults on
// the next synchronising call).
inline int launch_status(const char* kernel) {
    return cuda_status(cudaGetLastError(), kernel);
}

}  // namespace pulsar

#define PULSAR_CHECK_ARG(cond, ...)               \
    do {                                          \
        if (!(cond)) {                            \
            ::pulsar::set_error(__VA_ARGS__);     \
            return PULSAR_ERR_INVALID;            \
        }                                         \
    } while (0)

#define PULSAR_TRY(expr)                   \
    do {                                   \
        int _st = (expr);                  \
        if (_st != PULSAR_OK) return _st;  \
    } while (0)

#define PULSAR_LAUNCH_CHECK(name) PULSAR_TRY(::pulsar::launch_status(name))
