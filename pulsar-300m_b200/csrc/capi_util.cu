// Thread-local error text, the per-device kernel attribute record and the ABI version query.
#include "capi_util.h"

#include <mutex>
#include <set>
#include <utility>

namespace pulsar {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

int ensure_smem_attr(const void* fn, int bytes, const char* what) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;   // (kernel, device) pairs already set
    int dev = 0;
    int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (st) return st;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({fn, dev})) return PULSAR_OK;
    st = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
    if (st == PULSAR_OK) done.insert({fn, dev});
    return st;
}

}  // namespace pulsar

extern "C" const char* pulsar_last_error(void) { return pulsar::g_last_error.c_str(); }

extern "C" int pulsar_abi_version(void) { return 100; }
