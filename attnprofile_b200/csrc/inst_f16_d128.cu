// Explicit instantiation of the f16, D=128 kernel variants (one
// translation unit per group so the variants compile in parallel).
#include "dispatch.cuh"

namespace attnprof {
ATTNPROF_INSTANTIATE(__half, 128, false)
}  // namespace attnprof
