// Library-wide ABI: error buffer and version.
#include "common.cuh"
#include "../../include/rl2.h"

namespace rl2 {
namespace {
thread_local char g_last_error[512] = "";
}

void set_error(const char* format, ...) noexcept {
    va_list args;
    va_start(args, format);
    std::vsnprintf(g_last_error, sizeof(g_last_error), format, args);
    va_end(args);
}

void clear_error() noexcept { g_last_error[0] = '\0'; }

const char* last_error() noexcept { return g_last_error; }
}  // namespace rl2

extern "C" const char* rl2_last_error(void) { return rl2::last_error(); }

extern "C" int rl2_abi_version(void) { return 1; }
