// Weight packing launcher (see pack.cu).
#pragma once

#include <cuda_runtime.h>

namespace ctmr {

enum PackKind : int { kPackBF16 = 0, kPackSplitF16 = 1, kPackF16 = 2 };

cudaError_t launch_pack_weight(const float* w, int O, int C, int k, int upsample, int opad, int cpad, int kind,
                               void* out, void* out_lo, cudaStream_t stream);

}  // namespace ctmr
