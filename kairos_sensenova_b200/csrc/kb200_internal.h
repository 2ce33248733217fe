// kb200_internal.h -- host-side helpers shared by the C-ABI entry points.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include "../../include/kb200.h"

namespace kb {
// Records a message for kb200_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }
// Checks the result of the launches just issued.
int check_launch(const char* what);
}  // namespace kb
