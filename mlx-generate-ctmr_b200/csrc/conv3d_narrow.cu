// Direct 3x3x3 (padding 1, stride 1) convolution for narrow outputs (C_out <= 4):
// the MAISI output convolutions (UNet out.2: 64 -> 4, VAE decoder: 64 -> 1).
//
// With one to four output channels a tensor-core GEMM tile is almost all padding
// and its per-tap operand reloads dominate (27 taps x C_in x 2 bytes per output
// voxel). Here a CTA stages a halo block of the input once per 8-channel slice
// in shared memory — applying the group-norm affine and SiLU as it loads, with
// zeros outside the volume (the padding acts on the normalised input) — and
// every thread computes four consecutive w positions for all output channels
// with fp32 FMAs, reusing each staged value across the three kw taps. The
// weights are the split-fp32 packing (hi + lo * 2^-11 reassembles them to
// ~2^-22), the activations are used unrounded, and the input is read from HBM
// once plus the halo.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "conv3d_narrow.cuh"

namespace ctmr {
namespace {

constexpr int kTD = 2, kTH = 8, kTW = 32;   // output block per CTA
constexpr int kCS = 8;                      // channels staged per pass (static smem < 48 KB)
constexpr int kHD = kTD + 2, kHH = kTH + 2, kHW = kTW + 2;
constexpr int kWPT = 4;                     // consecutive w outputs per thread
constexpr int kThreads = kTD * kTH * (kTW / kWPT);  // 128

__device__ __forceinline__ float silu_exact(float t) { return t / (1.f + expf(-t)); }

template <int CO>
__global__ void __launch_bounds__(kThreads) narrow_conv_kernel(const NarrowParams p) {
  // Staged input [c][d][h][w] (w fastest, padded by one to spread banks) and weights [c][tap][co].
  __shared__ float s_in[kCS][kHD][kHH][kHW + 1];
  __shared__ float s_w[kCS][27][CO];
  const int tiles_w = (p.w + kTW - 1) / kTW, tiles_h = (p.h + kTH - 1) / kTH;
  int t = blockIdx.x;
  const int tw = t % tiles_w; t /= tiles_w;
  const int th = t % tiles_h; t /= tiles_h;
  const int td = t;
  const int b = blockIdx.y;
  const int w0 = tw * kTW, h0 = th * kTH, d0 = td * kTD;
  const int tid = threadIdx.x;
  const int lw = (tid % (kTW / kWPT)) * kWPT;
  const int lh = (tid / (kTW / kWPT)) % kTH;
  const int ld = tid / ((kTW / kWPT) * kTH);

  float acc[kWPT][CO];
#pragma unroll
  for (int i = 0; i < kWPT; ++i)
#pragma unroll
    for (int o = 0; o < CO; ++o) acc[i][o] = 0.f;

  const long long vox_b = static_cast<long long>(b) * p.d * p.h * p.w;
  for (int c0 = 0; c0 < p.cin; c0 += kCS) {
    const int cn = min(kCS, p.cin - c0);
    __syncthreads();
    // Stage the halo block: one (voxel, channel) element per step, channels fastest
    // so consecutive threads read consecutive addresses of a voxel row.
    constexpr int kHalo = kHD * kHH * kHW;
    for (int e = tid; e < kHalo * kCS; e += kThreads) {
      const int c = e % kCS;
      const int hv = e / kCS;
      const int x = hv % kHW, y = (hv / kHW) % kHH, z = hv / (kHW * kHH);
      const int gx = w0 + x - 1, gy = h0 + y - 1, gz = d0 + z - 1;
      float v = 0.f;
      if (c < cn && gx >= 0 && gx < p.w && gy >= 0 && gy < p.h && gz >= 0 && gz < p.d) {
        const int ch = c0 + c;
        v = __ldg(static_cast<const float*>(p.x) + (vox_b + (static_cast<long long>(gz) * p.h + gy) * p.w + gx) *
                                                       p.x_cstride + ch);
        if (p.affine != nullptr) {
          const float* a = p.affine + (static_cast<long long>(b) * p.cin + ch) * 2;
          v = fmaf(v, __ldg(a), __ldg(a + 1));
        }
        if (p.silu) v = silu_exact(v);
      }
      s_in[c][z][y][x] = v;
    }
    for (int e = tid; e < kCS * 27 * CO; e += kThreads) {
      const int o = e % CO, tap = (e / CO) % 27, c = e / (CO * 27);
      float wv = 0.f;
      if (c < cn && o < p.cout) {
        const long long k = (static_cast<long long>(tap) * p.opad + o) * p.cpad + c0 + c;
        wv = __half2float(p.w_hi[k]) + __half2float(p.w_lo[k]) * (1.f / 2048.f);
      }
      s_w[c][tap][o] = wv;
    }
    __syncthreads();
    for (int c = 0; c < cn; ++c) {
#pragma unroll
      for (int kd = 0; kd < 3; ++kd) {
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
          float row[kWPT + 2];
#pragma unroll
          for (int i = 0; i < kWPT + 2; ++i) row[i] = s_in[c][ld + kd][lh + kh][lw + i];
#pragma unroll
          for (int kw = 0; kw < 3; ++kw) {
#pragma unroll
            for (int o = 0; o < CO; ++o) {
              const float wv = s_w[c][(kd * 3 + kh) * 3 + kw][o];
#pragma unroll
              for (int i = 0; i < kWPT; ++i) acc[i][o] = fmaf(row[i + kw], wv, acc[i][o]);
            }
          }
        }
      }
    }
  }
  const int od = d0 + ld, oh = h0 + lh;
  if (od >= p.d || oh >= p.h) return;
#pragma unroll
  for (int i = 0; i < kWPT; ++i) {
    const int ow = w0 + lw + i;
    if (ow >= p.w) continue;
    const long long vox = vox_b + (static_cast<long long>(od) * p.h + oh) * p.w + ow;
#pragma unroll
    for (int o = 0; o < CO; ++o) {
      if (o >= p.cout) continue;
      float v = acc[i][o];
      if (p.bias != nullptr) v += __ldg(p.bias + static_cast<long long>(b) * p.bias_bstride + o);
      if (p.res != nullptr) {
        long long rv = vox;
        if (p.res_up) {
          const int rd = p.d / 2, rh = p.h / 2, rw = p.w / 2;
          rv = ((static_cast<long long>(b) * rd + (od >> 1)) * rh + (oh >> 1)) * rw + (ow >> 1);
        }
        v += __ldg(p.res + rv * p.res_cstride + o);
      }
      p.y[vox * p.y_cstride + o] = v;
    }
  }
}

}  // namespace

cudaError_t launch_narrow_conv(const NarrowParams& p, cudaStream_t stream) {
  if (p.cout < 1 || p.cout > 4) return cudaErrorInvalidValue;
  const int tiles = ((p.w + kTW - 1) / kTW) * ((p.h + kTH - 1) / kTH) * ((p.d + kTD - 1) / kTD);
  const dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(p.batch));
  if (p.cout == 1) narrow_conv_kernel<1><<<grid, kThreads, 0, stream>>>(p);
  else narrow_conv_kernel<4><<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ctmr
