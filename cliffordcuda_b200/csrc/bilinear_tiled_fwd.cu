// Instantiates the tiled bilinear kernels for CB_MODE_FWD.
#include "bilinear_tiled.cuh"

namespace cb {
template int bilinear_tiled<CB_MODE_FWD>(int, const float *, const float *, float *, int64_t, int,
                                uint32_t, uint32_t, cudaStream_t);
template int bilinear_tiled_cl61<CB_MODE_FWD>(const float *, const float *, float *, int64_t,
                                          cudaStream_t);
}  // namespace cb
