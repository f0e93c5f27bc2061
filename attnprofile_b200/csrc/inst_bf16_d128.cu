// Explicit instantiation of the bf16, D=128 kernel variants (one
// translation unit per group so the variants compile in parallel).
#include "dispatch.cuh"

namespace attnprof {
ATTNPROF_INSTANTIATE(__nv_bfloat16, 128, false)
}  // namespace attnprof
