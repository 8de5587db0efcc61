// Instantiation of the large-n bilinear kernels (bilinear_wide.cuh) for one
// sum; the three sums compile in parallel as separate units.
#include "bilinear_wide.cuh"

namespace cb {
template int bilinear_wide<CB_MODE_FWD>(int, const float *, const float *, float *, int64_t, int,
                               uint32_t, uint32_t, cudaStream_t);
}  // namespace cb
