// Weight packing for the implicit-GEMM convolution: Torch (O, C, k, k, k) fp32,
// or the channels-last (O, k, k, k, C) of released checkpoints, -> K-major taps
// [T][O_pad][C_pad] in bf16 or fp16, TF32-rounded fp32, or in fp16 hi/lo planes for
// the split-fp32 mode. Counterpart of `pack_weight` / `pack_upsample_weight`
// (`_nax_conv.py:391-445`), with the tap-major rows transposed to the K-major
// operand layout the tensor cores read.
//
// For a nearest-2x-upsampled input (T = 64 = 8 parities x 8 taps) the three
// taps of each axis fold into two per output parity p: output 2m + p reads
// upsampled 2m + p - 1 + k = source m - 1, m, m (p = 0) or m, m, m + 1 (p = 1),
// so tap t of parity p (source offset p + t - 1) sums the kernel taps
// {0} / {1, 2} for p = 0 and {0, 1} / {2} for p = 1. The folded sums are
// formed in fp32 before rounding or splitting, as in the reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "pack.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

__device__ __forceinline__ void fold_range(int p, int t, int& k0, int& k1) {
  // Kernel taps [k0, k1] merged into folded tap t of parity p.
  if (p == 0) {
    k0 = t == 0 ? 0 : 1;
    k1 = t == 0 ? 0 : 2;
  } else {
    k0 = t == 0 ? 0 : 2;
    k1 = t == 0 ? 1 : 2;
  }
}

__global__ void pack_weight_kernel(const float* __restrict__ w, int O, int C, int k, int upsample, int opad,
                                   int cpad, int kind, void* __restrict__ out, void* __restrict__ out_lo,
                                   int channels_last) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int taps = upsample ? 64 : k * k * k;
  const long long total = static_cast<long long>(taps) * opad * cpad;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cpad);
    const int o = static_cast<int>((i / cpad) % opad);
    const int tap = static_cast<int>(i / (static_cast<long long>(cpad) * opad));
    float v = 0.f;
    if (o < O && c < C) {
      // Kernel tap q of (o, c): Torch src[q], channels-last src[q * C].
      const long long k3 = static_cast<long long>(k) * k * k;
      const float* src = channels_last ? w + static_cast<long long>(o) * k3 * C + c : w + (static_cast<long long>(o) * C + c) * k3;
      const long long step = channels_last ? C : 1;
      if (!upsample) {
        v = src[tap * step];
      } else {
        const int phase = tap >> 3, t = tap & 7;
        int d0, d1, h0, h1, w0, w1;
        fold_range(phase >> 2, t >> 2, d0, d1);
        fold_range((phase >> 1) & 1, (t >> 1) & 1, h0, h1);
        fold_range(phase & 1, t & 1, w0, w1);
        for (int kd = d0; kd <= d1; ++kd)
          for (int kh = h0; kh <= h1; ++kh)
            for (int kw = w0; kw <= w1; ++kw) v += src[((kd * 3 + kh) * 3 + kw) * step];
      }
    }
    if (kind == kPackSplitF16) {
      const __half hi = __float2half_rn(v);
      const __half lo = __float2half_rn((v - __half2float(hi)) * 2048.f);
      static_cast<__half*>(out)[i] = hi;
      static_cast<__half*>(out_lo)[i] = lo;
    } else if (kind == kPackF16) {
      static_cast<__half*>(out)[i] = __float2half_rn(v);
    } else if (kind == kPackTF32) {
      static_cast<float*>(out)[i] = round_tf32(v);
    } else {
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace

cudaError_t launch_pack_weight(const float* w, int O, int C, int k, int upsample, int opad, int cpad, int kind,
                               void* out, void* out_lo, cudaStream_t stream, int channels_last) {
  const int taps = upsample ? 64 : k * k * k;
  const long long total = static_cast<long long>(taps) * opad * cpad;
  long long blocks = (total + 255) / 256;
  if (blocks > 32LL * device_sm_count()) blocks = 32LL * device_sm_count();
  if (blocks < 1) blocks = 1;
  launch_kernel(pack_weight_kernel, static_cast<unsigned>(blocks), 256, 0, stream, w, O, C, k, upsample, opad, cpad, kind,
                out, out_lo, channels_last);
  return cudaGetLastError();
}

}  // namespace ctmr
