// Explicit instantiation of the f16, D=64, profiler-enabled kernel variants (one
// translation unit per group so the variants compile in parallel).
#include "dispatch.cuh"

namespace attnprof {
ATTNPROF_INSTANTIATE(__half, 64, true)
}  // namespace attnprof
