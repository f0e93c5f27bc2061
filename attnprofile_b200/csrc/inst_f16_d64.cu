// Explicit instantiation of the f16, D=64 kernel variants (one
// translation unit per group so the variants compile in parallel).
#include "dispatch.cuh"

namespace attnprof {
ATTNPROF_INSTANTIATE(__half, 64, false)
}  // namespace attnprof
