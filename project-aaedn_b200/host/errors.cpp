// errors.cpp — per-thread last-error state of the C ABI.
#include "aaedn_b200.h"
#include "host_common.hpp"

#include <cstdarg>
#include <cstdio>

namespace aaedn_host
{

static thread_local char t_last_error[512] = "";

int set_error(int code, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return code;
}

} // namespace aaedn_host

extern "C" const char* aaedn_last_error(void) { return aaedn_host::t_last_error; }

extern "C" int aaedn_version(void) { return 1; }
