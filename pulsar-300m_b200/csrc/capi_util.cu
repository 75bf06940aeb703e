// Thread-local error text and the ABI version query.
#include "capi_util.h"

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

}  // namespace pulsar

extern "C" const char* pulsar_last_error(void) { return pulsar::g_last_error.c_str(); }

extern "C" int pulsar_abi_version(void) { return 100; }
