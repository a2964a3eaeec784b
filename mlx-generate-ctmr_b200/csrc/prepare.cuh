// Parameters of the conv-input preparation pass (see prepare.cu).
#pragma once

#include <cuda_runtime.h>

namespace ctmr {

enum PrepMode : int { kPrepCopy = 0, kPrepTrilinear = 1, kPrepAvgPool = 2 };
// kPrepOutTF32: fp32 rows of values rounded to TF32 (the kind::tf32 operand).
enum PrepOut : int { kPrepOutBF16 = 0, kPrepOutSplitF16 = 1, kPrepOutF32 = 2, kPrepOutF16 = 3, kPrepOutTF32 = 4 };

struct PrepSource {
  const void* ptr;       // NDHWC rows, `cstride` elements apart
  int bf16;              // 1: bf16 elements, 0: fp32, 2: int16 label ids read as 8 bit-plane channels
  int channels;          // channels taken from this source (0: unused)
  long long cstride;
};

struct PrepParams {
  PrepSource src[2];     // virtual channel concat src[0] ++ src[1]
  int batch;
  int sd, sh, sw;        // source grid
  int od, oh, ow;        // output grid
  int mode;
  const float* affine;   // [batch][channels][2] (scale, offset) or null
  int silu;
  int cpad;              // output channels (zero padded past the sources)
  long long out_cstride; // elements between output voxel rows (>= cpad)
  int out_kind;
  void* out;             // bf16 / fp16 hi / fp32 plane
  void* out_lo;          // fp16 lo plane for kPrepOutSplitF16
};

cudaError_t launch_prepare(const PrepParams& p, cudaStream_t stream);

// Copy-mode operand with its GroupNorm computed in the same kernel (one block per
// (group, batch item)); only for tensors whose groups are small, see
// gn_prepare_small_fits (voxels x channels-per-group <= kGnPrepSmallElems). With
// one block per group it has less parallelism than the separate statistics and
// operand passes, which measured faster on the MAISI UNet; the conv uses it only
// when CTMR_GN_FUSED is set.
constexpr long long kGnPrepSmallElems = 32768;
bool gn_prepare_small_fits(long long voxels, int channels, int groups);
cudaError_t launch_gn_prepare_small(const PrepParams& p, const float* gamma, const float* beta, int groups, float eps,
                                    cudaStream_t stream);

// im2col expansion of a stride-1 3x3x3 convolution input with cin <= 4 channels
// (src[0] only; od/oh/ow is the grid) into kdense-column rows, and the matching
// repack of [27][opad][cpad_src] packed weights into [opad][kdense].
cudaError_t launch_im2col(const PrepParams& p, int cin, int kdense, cudaStream_t stream);
cudaError_t launch_repack_im2col(const void* hi, const void* lo, int opad, int cpad_src, int cin, int kdense,
                                 void* out_hi, void* out_lo, cudaStream_t stream);

}  // namespace ctmr
