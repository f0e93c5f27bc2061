// Explicit instantiation of the bf16, D=64, profiler-enabled kernel variants (one
// translation unit per group so the variants compile in parallel).
#include "dispatch.cuh"

namespace attnprof {
ATTNPROF_INSTANTIATE(__nv_bfloat16, 64, true)
}  // namespace attnprof
