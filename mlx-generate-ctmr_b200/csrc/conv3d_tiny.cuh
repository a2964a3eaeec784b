// Parameters of the tiny-input direct convolution (see conv3d_tiny.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ctmr {

struct TinyParams {
  const void* x;            // fp32 NDHWC input, x_cstride elements per voxel row
  long long x_cstride;
  int vec4;                 // x and x_cstride allow 16-byte loads of four channels
  int batch, d, h, w, cin, cout;
  const float* affine;      // (B, C, 2) scale/offset or null
  int silu;
  const __half* w_hi;       // split-fp32 packed weights [27][opad][cpad]
  const __half* w_lo;
  int opad, cpad;
  const float* bias;        // (cout) or (B, cout) or null
  int bias_bstride;
  const float* res;         // fp32 residual NDHWC on the output grid or null
  long long res_cstride;
  float* y;                 // fp32 NDHWC output
  long long y_cstride;
};

cudaError_t launch_tiny_conv(const TinyParams& p, cudaStream_t stream);

}  // namespace ctmr
