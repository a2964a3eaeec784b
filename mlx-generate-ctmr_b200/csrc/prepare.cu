// Conv-input preparation: one HBM pass that turns NDHWC activations into the
// operand the tensor-core convolution reads.
//
// Per output voxel and channel it computes, in fp32,
//   v = source value                       (mode copy)
//     | trilinear 2x of the source          (mode trilinear; half-pixel, clamped)
//     | mean of transform(2x2x2 block)      (mode avgpool)
//   transform(v) = silu?(v * scale[b,c] + offset[b,c])   (group-norm affine optional)
// and stores it as bf16, as fp16 hi/lo planes (hi = half(y), lo = half((y-hi)*2^11)),
// or as fp32/bf16 without padding. The input may be a virtual channel concat of
// two tensors (the UNet up path's cat(hidden, skip)), and the output row is
// zero-padded to `cpad` channels. This is the counterpart of the reference's
// pack kernel (`_nax_conv.py:144-197`, trilinear at `:115-141`); the avgpool
// mode fuses `fast_fp32.py:250-255`.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "prepare.cuh"

namespace ctmr {
namespace {

__device__ __forceinline__ float load_ch(const void* base, int bf16, long long idx) {
  if (bf16) return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(base) + idx)) << 16);
  return __ldg(static_cast<const float*>(base) + idx);
}

// 8 consecutive channels of one source voxel (vectorised when aligned).
__device__ __forceinline__ void load8(const PrepSource& s, long long vox, int c, int cnt, float (&v)[8]) {
  const long long idx = vox * s.cstride + c;
  if (cnt == 8) {
    if (s.bf16) {
      const uint16_t* p = static_cast<const uint16_t*>(s.ptr) + idx;
      if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = __uint_as_float(w[i] << 16);
          v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
        return;
      }
    } else {
      const float* p = static_cast<const float*>(s.ptr) + idx;
      if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        return;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = i < cnt ? load_ch(s.ptr, s.bf16, idx + i) : 0.f;
}

// 8 channels [c0, c0+8) of the virtual concat at one voxel; channels past the end read 0.
__device__ __forceinline__ void load8_cat(const PrepParams& p, bool single, const PrepSource& s, long long vox,
                                          int c0, int cs, int cnt, float (&v)[8]) {
  if (single) {
    load8(s, vox, cs, cnt, v);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = c0 + i;
    if (i >= cnt) {
      v[i] = 0.f;
    } else if (c < p.src[0].channels) {
      v[i] = load_ch(p.src[0].ptr, p.src[0].bf16, vox * p.src[0].cstride + c);
    } else {
      v[i] = load_ch(p.src[1].ptr, p.src[1].bf16, vox * p.src[1].cstride + (c - p.src[0].channels));
    }
  }
}

// Linear-interpolation weights along one axis for the half-pixel 2x upsampling:
// output o samples source coordinate max(0, o/2 - 1/4), clamped at the far edge.
__device__ __forceinline__ void tri_axis(int o, int n, int& i0, int& i1, float& a) {
  const float f = fmaxf(0.f, static_cast<float>(o) * 0.5f - 0.25f);
  i0 = static_cast<int>(f);
  i1 = min(i0 + 1, n - 1);
  a = f - static_cast<float>(i0);
}

__device__ __forceinline__ float lerp_ref(float lo, float hi, float a) {
  // (1 - a) * lo + a * hi with the product a*hi rounded before the fused add.
  return __fmaf_rn(1.f - a, lo, __fmul_rn(a, hi));
}

// SiLU y / (1 + e^-y). FAST (16-bit outputs, rounded afterwards anyway) uses
// the hardware exponential and reciprocal; the fp32 modes use expf and an IEEE
// division.
template <bool FAST>
__device__ __forceinline__ float silu_f(float t) {
  if (FAST) return __fdividef(t, 1.f + __expf(-t));
  return t / (1.f + expf(-t));
}

__device__ __forceinline__ void store8(const PrepParams& p, long long oidx, int c0, const float (&out)[8]) {
  if (p.out_kind == kPrepOutBF16) {
    uint16_t* o = static_cast<uint16_t*>(p.out) + oidx;
    const int n = min(8, p.cpad - c0);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(out[2 * i], out[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    if (n == 8 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      *reinterpret_cast<uint4*>(o) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int i = 0; i < n; ++i) o[i] = static_cast<uint16_t>(w[i / 2] >> (16 * (i % 2)));
    }
  } else if (p.out_kind == kPrepOutF16) {
    uint16_t* o = static_cast<uint16_t*>(p.out) + oidx;
    const int n = min(8, p.cpad - c0);
    uint32_t hw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      hw[i] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(out[2 * i]))) |
              (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(out[2 * i + 1]))) << 16);
    }
    if (n == 8 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      *reinterpret_cast<uint4*>(o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    } else {
      for (int i = 0; i < n; ++i) o[i] = static_cast<uint16_t>(hw[i / 2] >> (16 * (i % 2)));
    }
  } else if (p.out_kind == kPrepOutSplitF16) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half h0 = __float2half_rn(out[2 * i]);
      const __half h1 = __float2half_rn(out[2 * i + 1]);
      const __half l0 = __float2half_rn((out[2 * i] - __half2float(h0)) * 2048.f);
      const __half l1 = __float2half_rn((out[2 * i + 1] - __half2float(h1)) * 2048.f);
      hw[i] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
      lw[i] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + oidx) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out_lo) + oidx) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  } else {
    float* o = static_cast<float*>(p.out) + oidx;
    const int n = min(8, p.cpad - c0);
    if (n == 8 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      reinterpret_cast<float4*>(o)[0] = make_float4(out[0], out[1], out[2], out[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(out[4], out[5], out[6], out[7]);
    } else {
      for (int i = 0; i < n; ++i) o[i] = out[i];
    }
  }
}

// One item = one output voxel x 8 channels. All index arithmetic is 32-bit
// (voxel counts per batch item fit comfortably; the host checks), and the copy
// mode needs no spatial decomposition because output voxel v is input voxel v.
template <int MODE, bool FAST>
__global__ void __launch_bounds__(256) prepare_kernel(const PrepParams p, const unsigned chunks_log2,
                                                      const unsigned vox_out) {
  const unsigned chunks = 1u << chunks_log2;
  const unsigned items_per_batch = vox_out << chunks_log2;
  const unsigned total = items_per_batch * static_cast<unsigned>(p.batch);
  const int ctot = p.src[0].channels + p.src[1].channels;
  const unsigned vox_in = static_cast<unsigned>(p.sd) * p.sh * p.sw;
  for (unsigned item = blockIdx.x * blockDim.x + threadIdx.x; item < total; item += gridDim.x * blockDim.x) {
    const unsigned b = item / items_per_batch;
    const unsigned rem = item - b * items_per_batch;
    const unsigned v = rem >> chunks_log2;
    const int c0 = static_cast<int>(rem & (chunks - 1)) * 8;
    if (c0 >= p.cpad) continue;  // chunk slots past the row when the chunk count is not a power of two
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = 0.f;
    if (c0 < ctot) {
      const int cnt = min(8, ctot - c0);
      const bool in1 = c0 >= p.src[0].channels;
      const bool single = (c0 + cnt <= p.src[0].channels) || in1;
      const PrepSource& s = p.src[in1 ? 1 : 0];
      const int cs = in1 ? c0 - p.src[0].channels : c0;
      float sc[8], of[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sc[i] = 1.f;
        of[i] = 0.f;
      }
      if (p.affine != nullptr) {
        const float* a = p.affine + (static_cast<long long>(b) * ctot + c0) * 2;
        if (cnt == 8 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 q = __ldg(reinterpret_cast<const float4*>(a) + i);
            sc[2 * i] = q.x;
            of[2 * i] = q.y;
            sc[2 * i + 1] = q.z;
            of[2 * i + 1] = q.w;
          }
        } else {
          for (int i = 0; i < cnt; ++i) {
            sc[i] = __ldg(a + 2 * i);
            of[i] = __ldg(a + 2 * i + 1);
          }
        }
      }
      const long long bvox = static_cast<long long>(b) * vox_in;
      if (MODE == kPrepCopy) {
        float r[8];
        load8_cat(p, single, s, bvox + v, c0, cs, cnt, r);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float t = fmaf(r[c], sc[c], of[c]);
          if (p.silu) t = silu_f<FAST>(t);
          out[c] = t;
        }
      } else {
        const unsigned x = v % static_cast<unsigned>(p.ow);
        const unsigned yz = v / static_cast<unsigned>(p.ow);
        const unsigned y = yz % static_cast<unsigned>(p.oh);
        const unsigned z = yz / static_cast<unsigned>(p.oh);
        if (MODE == kPrepTrilinear) {
          int z0, z1, y0, y1, x0, x1;
          float az, ay, ax;
          tri_axis(static_cast<int>(z), p.sd, z0, z1, az);
          tri_axis(static_cast<int>(y), p.sh, y0, y1, ay);
          tri_axis(static_cast<int>(x), p.sw, x0, x1, ax);
          float r[2][2][2][8];
          const int zs[2] = {z0, z1}, ys[2] = {y0, y1}, xs[2] = {x0, x1};
#pragma unroll
          for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int k = 0; k < 2; ++k)
                load8_cat(p, single, s, bvox + (static_cast<long long>(zs[i]) * p.sh + ys[j]) * p.sw + xs[k], c0, cs,
                          cnt, r[i][j][k]);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float r00 = lerp_ref(r[0][0][0][c], r[0][0][1][c], ax);
            const float r01 = lerp_ref(r[0][1][0][c], r[0][1][1][c], ax);
            const float r10 = lerp_ref(r[1][0][0][c], r[1][0][1][c], ax);
            const float r11 = lerp_ref(r[1][1][0][c], r[1][1][1][c], ax);
            const float p0 = lerp_ref(r00, r01, ay);
            const float p1 = lerp_ref(r10, r11, ay);
            out[c] = lerp_ref(p0, p1, az);
          }
        } else {  // kPrepAvgPool
          float acc[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
          for (int dz = 0; dz < 2; ++dz)
#pragma unroll
            for (int dy = 0; dy < 2; ++dy)
#pragma unroll
              for (int dx = 0; dx < 2; ++dx) {
                float r[8];
                load8_cat(p, single, s,
                          bvox + (static_cast<long long>(2 * z + dz) * p.sh + 2 * y + dy) * p.sw + 2 * x + dx, c0, cs,
                          cnt, r);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                  float t = fmaf(r[c], sc[c], of[c]);
                  if (p.silu) t = silu_f<FAST>(t);
                  acc[c] += t;
                }
              }
#pragma unroll
          for (int c = 0; c < 8; ++c) out[c] = acc[c] * 0.125f;
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c >= cnt) out[c] = 0.f;
    }
    store8(p, (static_cast<long long>(b) * vox_out + v) * p.out_cstride + c0, c0, out);
  }
}

}  // namespace

cudaError_t launch_prepare(const PrepParams& p, cudaStream_t stream) {
  const int chunks = (p.cpad + 7) >> 3;
  unsigned log2 = 0;
  while ((1 << log2) < chunks) ++log2;
  const long long vox_out = static_cast<long long>(p.od) * p.oh * p.ow;
  const long long total = static_cast<long long>(p.batch) * (vox_out << log2);
  if (total <= 0) return cudaSuccess;
  if (total >= (1LL << 31) || static_cast<long long>(p.sd) * p.sh * p.sw >= (1LL << 31))
    return cudaErrorInvalidValue;  // the 32-bit item space of prepare_kernel
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  const bool fast = p.out_kind == kPrepOutBF16 || p.out_kind == kPrepOutF16;
  const dim3 grid(static_cast<unsigned>(blocks));
  const unsigned vo = static_cast<unsigned>(vox_out);
#define CTMR_PREP(MODE)                                                         \
  if (fast) prepare_kernel<MODE, true><<<grid, threads, 0, stream>>>(p, log2, vo); \
  else prepare_kernel<MODE, false><<<grid, threads, 0, stream>>>(p, log2, vo);
  if (p.mode == kPrepTrilinear) {
    CTMR_PREP(kPrepTrilinear)
  } else if (p.mode == kPrepAvgPool) {
    CTMR_PREP(kPrepAvgPool)
  } else {
    CTMR_PREP(kPrepCopy)
  }
#undef CTMR_PREP
  return cudaGetLastError();
}

}  // namespace ctmr
