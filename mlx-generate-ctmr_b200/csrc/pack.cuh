// Weight packing launcher (see pack.cu).
#pragma once

#include <cuda_runtime.h>

namespace ctmr {

// kPackTF32: fp32 values rounded to TF32 (cpad then counts fp32 values).
enum PackKind : int { kPackBF16 = 0, kPackSplitF16 = 1, kPackF16 = 2, kPackTF32 = 3 };

// `channels_last`: the source is (O, k, k, k, C) (the channels-last layout of
// released checkpoints) instead of Torch's (O, C, k, k, k).
cudaError_t launch_pack_weight(const float* w, int O, int C, int k, int upsample, int opad, int cpad, int kind,
                               void* out, void* out_lo, cudaStream_t stream, int channels_last = 0);

}  // namespace ctmr
