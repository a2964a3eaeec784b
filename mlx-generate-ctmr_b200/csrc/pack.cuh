// Weight packing launcher (see pack.cu).
#pragma once

#include <cuda_runtime.h>

namespace ctmr {

cudaError_t launch_pack_weight(const float* w, int O, int C, int k, int upsample, int opad, int cpad, int split,
                               void* out, void* out_lo, cudaStream_t stream);

}  // namespace ctmr
