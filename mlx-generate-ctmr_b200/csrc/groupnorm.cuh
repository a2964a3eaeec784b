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

// Affine from convolution output statistics: moments float[batch][slots][channels][3]
// of up to two sources (the virtual concat a ++ b).
struct GnStatsParams {
  const float* stats[2];
  int channels[2];
  int slots, batch, groups;
  float eps;
  const float* gamma;
  const float* beta;
  float* affine;          // out: [batch][C][2]
};

// Affine from per-part moments float[parts][batch][groups][3] (count, mean, M2).
struct GnMomentsParams {
  const float* moments;
  int parts, batch, channels, groups;
  float eps;
  const float* gamma;
  const float* beta;
  float* affine;          // out: [batch][channels][2]
};

int gn_max_chunks(int batch);
cudaError_t launch_group_norm_moments(const GnParams& p, float* moments, cudaStream_t stream);
cudaError_t launch_group_norm_from_moments(const GnMomentsParams& p, cudaStream_t stream);
cudaError_t launch_group_norm_from_stats(const GnStatsParams& p, cudaStream_t stream);
int gn_chunks_for(int batch, long long voxels, int channels);
cudaError_t launch_group_norm_affine(const GnParams& p, cudaStream_t stream);
// launch_group_norm_affine makes one launch (the small-tensor kernel) instead of two.
bool gn_direct_fits(long long voxels, int channels, int groups);

}  // namespace ctmr
