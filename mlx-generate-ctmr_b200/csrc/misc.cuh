// Launchers of the small memory-bound kernels (see misc.cu).
#pragma once

#include <cuda_runtime.h>

namespace ctmr {

struct WindowParams {
  const void* pred;          // NDHWC window prediction (B, wd, wh, ww, C)
  int pred_bf16;
  long long pred_cstride;
  int batch, channels;
  int wd, wh, ww;            // window extent (output voxels)
  int z0, y0, x0;            // window origin in the output grid
  int od, oh, ow;            // output grid
  const float* gz;           // 1-D Gaussian tables over the latent ROI
  const float* gy;
  const float* gx;
  int scale;                 // latent -> output upsampling factor (nearest resize of the weights)
  float floor_value;
  float* acc;                // NDHWC fp32 (B, od, oh, ow, C)
  float* wsum;               // fp32 (od, oh, ow)
};

cudaError_t launch_transpose_cs(const void* in, int in_bf16, void* out, int out_bf16, int batch, int rows, int cols,
                                cudaStream_t stream);
cudaError_t launch_window_accumulate(const WindowParams& p, cudaStream_t stream);
cudaError_t launch_window_finalize(const float* acc, const float* wsum, float* out, int batch, int channels, int od,
                                   int oh, int ow, int cz0, int cy0, int cx0, int cd, int ch, int cw,
                                   cudaStream_t stream);
cudaError_t launch_rflow_step(const float* z, const float* vel, long long n, float guidance, int guided, float dt,
                              const float* dt_device, float* out, cudaStream_t stream);

}  // namespace ctmr
