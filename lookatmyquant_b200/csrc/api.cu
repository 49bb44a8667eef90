// ABI version and per-thread error text for the lamq_b200 C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "lamq_common.cuh"

namespace lamq {

static thread_local char g_error[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

}  // namespace lamq

extern "C" int lamq_abi_version(void) { return 4; }

extern "C" const char *lamq_last_error(void) { return lamq::g_error; }
