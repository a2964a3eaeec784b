// Parameters of the GroupNorm statistics kernels (see groupnorm.cu).
#pragma once

#include <cuda_runtime.h>

#include "prepare.cuh"

namespace ctmr {

struct GnParams {
  PrepSource src[2];      // virtual channel concat (src[1].channels == 0 when unused)
  int batch;
  long long voxels;       // voxels per batch item
  int groups;
  float eps;
  const float* gamma;     // [C] or null (1)
  const float* beta;      // [C] or null (0)
  float* affine;          // out: [batch][C][2] (scale, offset)
  float* partials;        // workspace: [batch][chunks][groups][3]
  int chunks;
};

int gn_max_chunks(int batch);
int gn_chunks_for(int batch, long long voxels, int channels);
cudaError_t launch_group_norm_affine(const GnParams& p, cudaStream_t stream);

}  // namespace ctmr
