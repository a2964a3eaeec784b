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
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

__device__ __forceinline__ float load_ch(const void* base, int bf16, long long idx) {
  if (bf16) return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(base) + idx)) << 16);
  return __ldg(static_cast<const float*>(base) + idx);
}

// 8 consecutive channels of one source voxel (vectorised when aligned). A label
// source holds one int16 id per voxel; its channel k is bit k of the id.
__device__ __forceinline__ void load8(const PrepSource& s, long long vox, int c, int cnt, float (&v)[8]) {
  if (s.bf16 == 2) {
    const int id = __ldg(static_cast<const int16_t*>(s.ptr) + vox * s.cstride);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i < cnt ? static_cast<float>((id >> (c + i)) & 1) : 0.f;
    return;
  }
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
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = p.out_kind == kPrepOutTF32 ? round_tf32(out[i]) : out[i];
    if (n == 8 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      reinterpret_cast<float4*>(o)[0] = make_float4(r[0], r[1], r[2], r[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(r[4], r[5], r[6], r[7]);
    } else {
      for (int i = 0; i < n; ++i) o[i] = r[i];
    }
  }
}

// One item = one output voxel x 8 channels. All index arithmetic is 32-bit
// (voxel counts per batch item fit comfortably; the host checks), and the copy
// mode needs no spatial decomposition because output voxel v is input voxel v.
template <int MODE, bool FAST>
__global__ void __launch_bounds__(256) prepare_kernel(const PrepParams p, const unsigned chunks_log2,
                                                      const unsigned vox_out) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
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
      const PrepSource s{in1 ? p.src[1].ptr : p.src[0].ptr, in1 ? p.src[1].bf16 : p.src[0].bf16,
                         in1 ? p.src[1].channels : p.src[0].channels, in1 ? p.src[1].cstride : p.src[0].cstride};
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

// ---------------------------------------------------------------- vectorised fast paths
// Division by a runtime divisor d as a multiply-high and shift (Granlund and
// Montgomery's round-up method): q = (umulhi(m, n) + n) >> l with l = ceil(log2 d)
// and m = floor(2^32 (2^l - d) / d) + 1, exact for every 32-bit n.
struct FastDiv {
  uint32_t d, m, l;
};

FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{d, static_cast<uint32_t>(m), l};
}

__device__ __forceinline__ uint32_t fdiv(const FastDiv& f, uint32_t n) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(f.m, n)) + n) >> f.l);
}

template <int OUTK, int N>
__device__ __forceinline__ void store_vec(const PrepParams& p, long long oidx, const float (&v)[N]) {
  static_assert(N == 4 || N == 8, "4 or 8 channels");
  if (OUTK == kPrepOutF32 || OUTK == kPrepOutTF32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.out) + oidx);
    float r[N];
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = OUTK == kPrepOutTF32 ? round_tf32(v[i]) : v[i];
#pragma unroll
    for (int i = 0; i < N / 4; ++i) o[i] = make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
  } else {
    uint32_t hw[N / 2], lw[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      if (OUTK == kPrepOutBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        hw[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        const __half h0 = __float2half_rn(v[2 * i]);
        const __half h1 = __float2half_rn(v[2 * i + 1]);
        hw[i] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
        if (OUTK == kPrepOutSplitF16) {
          const __half l0 = __float2half_rn((v[2 * i] - __half2float(h0)) * 2048.f);
          const __half l1 = __float2half_rn((v[2 * i + 1] - __half2float(h1)) * 2048.f);
          lw[i] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
        }
      }
    }
    uint16_t* o = static_cast<uint16_t*>(p.out) + oidx;
    if constexpr (N == 8) {
      *reinterpret_cast<uint4*>(o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      if (OUTK == kPrepOutSplitF16)
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out_lo) + oidx) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    } else {
      *reinterpret_cast<uint2*>(o) = make_uint2(hw[0], hw[1]);
      if (OUTK == kPrepOutSplitF16)
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out_lo) + oidx) = make_uint2(lw[0], lw[1]);
    }
  }
}

// N consecutive fp32 channels [c0, c0 + N) of the virtual concat at one voxel
// (the concat boundary and the channel count are multiples of N; past the
// channels the value is 0).
template <int N>
__device__ __forceinline__ void load_vec(const PrepParams& p, int ctot, long long vox, int c0, float (&v)[N]) {
  if (c0 >= ctot) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = 0.f;
    return;
  }
  const bool in1 = c0 >= p.src[0].channels;
  // Field selects (not a runtime index into the parameter array, which would copy it to local memory).
  const void* ptr = in1 ? p.src[1].ptr : p.src[0].ptr;
  const long long cstride = in1 ? p.src[1].cstride : p.src[0].cstride;
  const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(ptr) + vox * cstride +
                                                    (in1 ? c0 - p.src[0].channels : c0));
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const float4 a = __ldg(q + i);
    v[4 * i] = a.x;
    v[4 * i + 1] = a.y;
    v[4 * i + 2] = a.z;
    v[4 * i + 3] = a.w;
  }
}

// Copy mode, 8 channels per item, two items in flight per thread; batch item
// on grid y. Preconditions (checked by the launcher): fp32 sources, channel
// counts, strides and cpad multiples of 8, 16-byte aligned rows; the grid's
// thread count a multiple of the chunks per voxel, so every item of a thread
// has the same 8-channel chunk and its GroupNorm scale / offset pairs are loaded
// once (16 registers held; four blocks of 256 threads per SM at 64 registers).
template <int OUTK, bool FAST>
__global__ void __launch_bounds__(256, 4) prepare_copy_kernel(const PrepParams p, const FastDiv qdiv,
                                                           const unsigned vox) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int b = blockIdx.y;
  const int ctot = p.src[0].channels + p.src[1].channels;
  const long long bvox = static_cast<long long>(b) * vox;
  const unsigned first = blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned v0 = fdiv(qdiv, first);
  const int c0 = static_cast<int>(first - v0 * qdiv.d) * 8;  // this thread's chunk, for all its items
  const unsigned vstep = fdiv(qdiv, gridDim.x * blockDim.x);  // voxels between a thread's items
  const bool live = c0 < ctot;
  float sc[8], of[8];
  const bool aff = live && p.affine != nullptr;
  if (aff) {
    const float4* a = reinterpret_cast<const float4*>(p.affine + (static_cast<long long>(b) * ctot + c0) * 2);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 q = __ldg(a + i);
      sc[2 * i] = q.x, of[2 * i] = q.y, sc[2 * i + 1] = q.z, of[2 * i + 1] = q.w;
    }
  }
  for (unsigned v = v0; v < vox; v += 2 * vstep) {
    float r[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (v + k * vstep < vox) load_vec<8>(p, ctot, bvox + v + k * vstep, c0, r[k]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const unsigned vk = v + k * vstep;
      if (vk >= vox) break;
      if (live) {
        if (aff) {
#pragma unroll
          for (int i = 0; i < 8; ++i) r[k][i] = fmaf(r[k][i], sc[i], of[i]);
        }
        if (p.silu) {
#pragma unroll
          for (int i = 0; i < 8; ++i) r[k][i] = silu_f<FAST>(r[k][i]);
        }
      }
      store_vec<OUTK, 8>(p, (bvox + vk) * p.out_cstride + c0, r[k]);
    }
  }
}

// Trilinear 2x (half-pixel, clamped; no transform), 4 channels per item. An item is one
// column: a source (h, w) position and channel chunk, whose 2 (h) x 2 (w) output block the
// thread produces at every output depth. Walking the source depths once, it reads the 3 x 3
// source neighbourhood of each depth (9 loads for 8 outputs), lerps it along w then h into
// that depth's 2 x 2 block, and emits every output depth whose two source depths it now
// holds (2 zs - 1 and 2 zs, output 0 at zs = 1, the last output at the last depth). Each
// output uses exactly the source pair and weight of tri_axis and the same lerp order (w,
// then h, then d) as the general path, so results are bitwise equal.
template <int OUTK>
__global__ void __launch_bounds__(128) prepare_tri_kernel(const PrepParams p, const FastDiv qdiv, const FastDiv xdiv,
                                                          const unsigned items) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int b = blockIdx.y;
  const int ctot = p.src[0].channels + p.src[1].channels;
  const long long bsrc = static_cast<long long>(b) * p.sd * p.sh * p.sw;
  const long long bout = static_cast<long long>(b) * p.od * p.oh * p.ow;
  for (unsigned item = blockIdx.x * blockDim.x + threadIdx.x; item < items; item += gridDim.x * blockDim.x) {
    const unsigned r1 = fdiv(qdiv, item);
    const int c0 = static_cast<int>(item - r1 * qdiv.d) * 4;
    const unsigned yj_u = fdiv(xdiv, r1);
    const int xi = static_cast<int>(r1 - yj_u * xdiv.d);  // source w index = output w pair
    const int yj = static_cast<int>(yj_u);               // source h index = output h pair
    const int xs[3] = {max(xi - 1, 0), xi, min(xi + 1, p.sw - 1)};
    const int ys[3] = {max(yj - 1, 0), yj, min(yj + 1, p.sh - 1)};
    // Output pair element e (0: 2i, 1: 2i + 1) uses slots (lo, hi) and weight a:
    // e = 0: (0, 1, 0.75) for i >= 1, (1, 2, 0) for i = 0; e = 1: (1, 2, 0.25).
    int xo[2], yo[2];
    float ax[2], ay[2];
    {
      int i0, i1;
      tri_axis(2 * xi, p.sw, i0, i1, ax[0]);
      tri_axis(2 * xi + 1, p.sw, i0, i1, ax[1]);
      tri_axis(2 * yj, p.sh, i0, i1, ay[0]);
      tri_axis(2 * yj + 1, p.sh, i0, i1, ay[1]);
      xo[0] = xi >= 1 ? 0 : 1;
      xo[1] = 1;
      yo[0] = yj >= 1 ? 0 : 1;
      yo[1] = 1;
    }
    // The 2 x 2 output block of output depth o from the w-then-h lerped blocks of its source depths.
    auto emit = [&](int o, const float (&lo)[2][2][4], const float (&hi)[2][2][4], float az) {
      float v[4];
#pragma unroll
      for (int f = 0; f < 2; ++f)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) v[ch] = lerp_ref(lo[f][e][ch], hi[f][e][ch], az);
          const long long ov = bout + (static_cast<long long>(o) * p.oh + 2 * yj + f) * p.ow + 2 * xi + e;
          store_vec<OUTK, 4>(p, ov * p.out_cstride + c0, v);
        }
    };
    float prev[2][2][4], cur[2][2][4];  // [h pair][w pair][channel] of source depths zs - 1 and zs
    for (int zs = 0; zs < p.sd; ++zs) {
      float sv[3][3][4];
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          load_vec<4>(p, ctot, bsrc + (static_cast<long long>(zs) * p.sh + ys[a]) * p.sw + xs[c], c0, sv[a][c]);
      // w lerps for every source row, both output w elements; then the h lerps.
      float wl[3][2][4];
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const float lo = xo[e] == 0 ? sv[a][0][ch] : sv[a][1][ch];
            const float hi = xo[e] == 0 ? sv[a][1][ch] : sv[a][2][ch];
            wl[a][e][ch] = lerp_ref(lo, hi, ax[e]);
          }
#pragma unroll
      for (int f = 0; f < 2; ++f)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const float lo = yo[f] == 0 ? wl[0][e][ch] : wl[1][e][ch];
            const float hi = yo[f] == 0 ? wl[1][e][ch] : wl[2][e][ch];
            cur[f][e][ch] = lerp_ref(lo, hi, ay[f]);
          }
      int z0, z1;
      float az;
      if (zs >= 1) {
        if (zs == 1) {  // output 0: source depths (0, 1), weight 0
          tri_axis(0, p.sd, z0, z1, az);
          emit(0, prev, cur, az);
        }
        tri_axis(2 * zs - 1, p.sd, z0, z1, az);  // (zs - 1, zs)
        emit(2 * zs - 1, prev, cur, az);
        tri_axis(2 * zs, p.sd, z0, z1, az);      // (zs - 1, zs)
        emit(2 * zs, prev, cur, az);
      }
      if (zs == p.sd - 1) {
        if (zs == 0) {  // a single source depth: outputs 0 and 1 both read it twice
          tri_axis(0, p.sd, z0, z1, az);
          emit(0, cur, cur, az);
        }
        tri_axis(2 * zs + 1, p.sd, z0, z1, az);  // (zs, zs): the far edge clamps
        emit(2 * zs + 1, cur, cur, az);
      }
#pragma unroll
      for (int f = 0; f < 2; ++f)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) prev[f][e][ch] = cur[f][e][ch];
    }
  }
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// Whether the vectorised paths apply: fp32 sources whose channel counts,
// strides and row starts allow `vec`-channel loads, and an output whose rows
// take vec-channel stores.
bool vec_ok(const PrepParams& p, int vec) {
  for (int i = 0; i < 2; ++i) {
    const PrepSource& s = p.src[i];
    if (s.channels == 0) continue;
    if (s.bf16 || s.channels % vec || s.cstride % 4 || !aligned16(s.ptr)) return false;
  }
  const int obytes = (p.out_kind == kPrepOutF32 || p.out_kind == kPrepOutTF32) ? 4 : 2;
  if (p.cpad % vec || (p.out_cstride * obytes) % 16 || !aligned16(p.out)) return false;
  if (p.out_kind == kPrepOutSplitF16 && !aligned16(p.out_lo)) return false;
  if (p.affine != nullptr && !aligned16(p.affine)) return false;
  return true;
}

// Blocks of `kern` resident on the whole GPU at once (SMs x blocks per SM).
template <typename K>
long long resident_blocks(K kern, int threads, size_t smem) {
  const int sms = device_sm_count();
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return static_cast<long long>(sms) * per_sm;
}

cudaError_t launch_copy_fast(const PrepParams& p, cudaStream_t stream) {
  const unsigned vox = static_cast<unsigned>(static_cast<long long>(p.od) * p.oh * p.ow);
  const FastDiv q = make_fastdiv(static_cast<uint32_t>(p.cpad / 8));
  const long long items = static_cast<long long>(vox) * q.d;
  long long blocks = (items + 511) / 512;
  // One resident wave over all batch items (a second, partial wave would idle most SMs).
  static const long long resident = resident_blocks(prepare_copy_kernel<kPrepOutF16, true>, 256, 0);
  const long long cap = resident / p.batch > 0 ? resident / p.batch : 1;
  if (blocks > cap) blocks = cap;
  // The grid's thread count a multiple of the chunks per voxel: blocks a multiple of q / gcd(q, 256).
  long long g = q.d, r = 256;
  while (r != 0) {
    const long long t = g % r;
    g = r;
    r = t;
  }
  const long long unit = q.d / g;
  blocks = blocks < unit ? unit : blocks / unit * unit;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(p.batch));
  switch (p.out_kind) {
    case kPrepOutBF16: launch_kernel(prepare_copy_kernel<kPrepOutBF16, true>, grid, 256, 0, stream, p, q, vox); break;
    case kPrepOutF16: launch_kernel(prepare_copy_kernel<kPrepOutF16, true>, grid, 256, 0, stream, p, q, vox); break;
    case kPrepOutSplitF16: launch_kernel(prepare_copy_kernel<kPrepOutSplitF16, false>, grid, 256, 0, stream, p, q, vox); break;
    case kPrepOutTF32: launch_kernel(prepare_copy_kernel<kPrepOutTF32, true>, grid, 256, 0, stream, p, q, vox); break;
    default: launch_kernel(prepare_copy_kernel<kPrepOutF32, false>, grid, 256, 0, stream, p, q, vox); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_tri_fast(const PrepParams& p, cudaStream_t stream) {
  const FastDiv q = make_fastdiv(static_cast<uint32_t>(p.cpad / 4));
  const FastDiv xd = make_fastdiv(static_cast<uint32_t>(p.sw));
  const long long items = static_cast<long long>(p.sh) * p.sw * q.d;  // columns: every output depth per item
  long long blocks = (items + 127) / 128;
  static const long long resident = resident_blocks(prepare_tri_kernel<kPrepOutF16>, 128, 0);
  const long long cap = resident / p.batch > 0 ? resident / p.batch : 1;
  if (blocks > cap) blocks = cap;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(p.batch));
  const unsigned n = static_cast<unsigned>(items);
  switch (p.out_kind) {
    case kPrepOutBF16: launch_kernel(prepare_tri_kernel<kPrepOutBF16>, grid, 128, 0, stream, p, q, xd, n); break;
    case kPrepOutF16: launch_kernel(prepare_tri_kernel<kPrepOutF16>, grid, 128, 0, stream, p, q, xd, n); break;
    case kPrepOutSplitF16: launch_kernel(prepare_tri_kernel<kPrepOutSplitF16>, grid, 128, 0, stream, p, q, xd, n); break;
    case kPrepOutTF32: launch_kernel(prepare_tri_kernel<kPrepOutTF32>, grid, 128, 0, stream, p, q, xd, n); break;
    default: launch_kernel(prepare_tri_kernel<kPrepOutF32>, grid, 128, 0, stream, p, q, xd, n); break;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- im2col for tiny inputs
// A 3x3x3 stride-1 convolution of a C <= 4 channel input as a 1x1x1 convolution
// of its im2col expansion: row v holds transform(x[v + tap])[c] at column
// tap * C + c (tap = kd * 9 + kh * 3 + kw, zero outside the volume and past
// 27 * C up to kdense), so the GEMM's K is 27 * C rounded up to 16 instead of
// 27 taps x 16 padded channels.
template <int OUTK>
__global__ void __launch_bounds__(256) im2col_kernel(const PrepParams p, const int cin, const int kdense) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int b = blockIdx.y;
  const unsigned vox = static_cast<unsigned>(p.od) * p.oh * p.ow;
  const int chunks = kdense / 8;
  const unsigned items = vox * static_cast<unsigned>(chunks);
  const PrepSource& s = p.src[0];
  for (unsigned item = blockIdx.x * blockDim.x + threadIdx.x; item < items; item += gridDim.x * blockDim.x) {
    const unsigned v = item / static_cast<unsigned>(chunks);
    const int k0 = static_cast<int>(item - v * static_cast<unsigned>(chunks)) * 8;
    const int x = static_cast<int>(v % static_cast<unsigned>(p.ow));
    const unsigned yz = v / static_cast<unsigned>(p.ow);
    const int y = static_cast<int>(yz % static_cast<unsigned>(p.oh));
    const int z = static_cast<int>(yz / static_cast<unsigned>(p.oh));
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = k0 + i;
      const int tap = k / cin, c = k - tap * cin;
      float t = 0.f;
      if (tap < 27) {
        const int gz = z + tap / 9 - 1, gy = y + (tap / 3) % 3 - 1, gx = x + tap % 3 - 1;
        if (gz >= 0 && gz < p.od && gy >= 0 && gy < p.oh && gx >= 0 && gx < p.ow) {
          const long long src = ((static_cast<long long>(b) * p.od + gz) * p.oh + gy) * p.ow + gx;
          t = load_ch(s.ptr, s.bf16, src * s.cstride + c);
          if (p.affine != nullptr) {
            const float* a = p.affine + (static_cast<long long>(b) * cin + c) * 2;
            t = fmaf(t, __ldg(a), __ldg(a + 1));
          }
          if (p.silu) t = silu_f<false>(t);
        }
      }
      out[i] = t;
    }
    store_vec<OUTK, 8>(p, (static_cast<long long>(b) * vox + v) * p.out_cstride + k0, out);
  }
}

// ---------------------------------------------------------------- small-tensor GroupNorm + operand
// One kernel for a copy-mode operand with its GroupNorm computed in place, for
// tensors small enough that one block per (group, batch item) reads its group
// twice from L2: pass 1 reduces (count, mean, M2) (pivot-shifted per thread,
// Chan merges in double in a fixed order), pass 2 applies the affine (computed as
// ctmr_group_norm_affine does) and the optional SiLU and writes the operand. The
// block of the last group also writes the zero channels [ctot, cpad).
struct MomD {
  double n, mean, m2;
};

__device__ __forceinline__ MomD mom_merge(MomD a, MomD b) {
  if (b.n == 0.0) return a;
  if (a.n == 0.0) return b;
  const double n = a.n + b.n, delta = b.mean - a.mean, fb = b.n / n;
  return MomD{n, a.mean + delta * fb, a.m2 + b.m2 + delta * delta * a.n * fb};
}

constexpr int kGnPrepThreads = 256;

template <int OUTK, bool FAST>
__global__ void __launch_bounds__(kGnPrepThreads) gn_prepare_small_kernel(const PrepParams p, const float* gamma,
                                                                          const float* beta, const float eps,
                                                                          const FastDiv cdiv) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  __shared__ double s_m[kGnPrepThreads / 32][3];
  __shared__ float s_scale[64], s_offset[64];
  const int g = blockIdx.x, b = blockIdx.y;
  const int groups = gridDim.x;
  const int c0s = p.src[0].channels;
  const int ctot = c0s + p.src[1].channels;
  const int cpg = static_cast<int>(cdiv.d);
  const int cbase = g * cpg;
  const unsigned vox = static_cast<unsigned>(p.od) * p.oh * p.ow;
  const unsigned elems = vox * static_cast<unsigned>(cpg);
  const long long bvox = static_cast<long long>(b) * vox;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto load = [&](unsigned e, int& c) -> float {
    const unsigned v = fdiv(cdiv, e);
    c = cbase + static_cast<int>(e - v * cdiv.d);
    const bool second = c >= c0s;
    const void* ptr = second ? p.src[1].ptr : p.src[0].ptr;
    const int bf = second ? p.src[1].bf16 : p.src[0].bf16;
    const long long cs = second ? p.src[1].cstride : p.src[0].cstride;
    return load_ch(ptr, bf, (bvox + v) * cs + (second ? c - c0s : c));
  };
  // Pass 1: moments of the group.
  // Eight elements' loads in flight per thread (the loops are latency-bound).
  float pivot = 0.f, sd = 0.f, sq = 0.f, n = 0.f;
  if (tid < elems) {
    int c;
    pivot = load(tid, c);
  }
#pragma unroll 8
  for (unsigned e = tid; e < elems; e += kGnPrepThreads) {
    int c;
    const float x = load(e, c);
    const float d = x - pivot;
    sd += d;
    sq = fmaf(d, d, sq);
    n += 1.f;
  }
  MomD m{0.0, 0.0, 0.0};
  if (n > 0.f) {
    const double md = static_cast<double>(sd) / n;
    m = MomD{n, pivot + md, fmax(0.0, static_cast<double>(sq) - static_cast<double>(sd) * md)};
  }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const MomD o{__shfl_down_sync(0xffffffffu, m.n, off), __shfl_down_sync(0xffffffffu, m.mean, off),
                 __shfl_down_sync(0xffffffffu, m.m2, off)};
    if ((lane & (2 * off - 1)) == 0) m = mom_merge(m, o);
  }
  if (lane == 0) {
    s_m[warp][0] = m.n;
    s_m[warp][1] = m.mean;
    s_m[warp][2] = m.m2;
  }
  __syncthreads();
  if (tid < cpg) {
    MomD t{0.0, 0.0, 0.0};
    for (int w = 0; w < kGnPrepThreads / 32; ++w) t = mom_merge(t, MomD{s_m[w][0], s_m[w][1], s_m[w][2]});
    const double var = t.n > 0.0 ? t.m2 / t.n : 0.0;
    const double rstd = 1.0 / sqrt(var + static_cast<double>(eps));
    const int c = cbase + tid;
    const double gam = gamma != nullptr ? static_cast<double>(gamma[c]) : 1.0;
    const double bet = beta != nullptr ? static_cast<double>(beta[c]) : 0.0;
    const double scale = gam * rstd;
    s_scale[tid] = static_cast<float>(scale);
    s_offset[tid] = static_cast<float>(bet - t.mean * scale);
  }
  __syncthreads();
  // Pass 2: the operand.
#pragma unroll 8
  for (unsigned e = tid; e < elems; e += kGnPrepThreads) {
    int c;
    const float x = load(e, c);
    float t = fmaf(x, s_scale[c - cbase], s_offset[c - cbase]);
    if (p.silu) t = silu_f<FAST>(t);
    const unsigned v = fdiv(cdiv, e);
    const long long o = (bvox + v) * p.out_cstride + c;
    if (OUTK == kPrepOutBF16) {
      __nv_bfloat16 h = __float2bfloat16_rn(t);
      static_cast<uint16_t*>(p.out)[o] = *reinterpret_cast<uint16_t*>(&h);
    } else {
      const __half h = __float2half_rn(t);
      static_cast<__half*>(p.out)[o] = h;
      if (OUTK == kPrepOutSplitF16) static_cast<__half*>(p.out_lo)[o] = __float2half_rn((t - __half2float(h)) * 2048.f);
    }
  }
  if (g == groups - 1 && p.cpad > ctot) {
    const int pad = p.cpad - ctot;
    for (unsigned e = tid; e < vox * static_cast<unsigned>(pad); e += kGnPrepThreads) {
      const unsigned v = e / static_cast<unsigned>(pad);
      const long long o = (bvox + v) * p.out_cstride + ctot + static_cast<int>(e - v * pad);
      static_cast<uint16_t*>(p.out)[o] = 0;
      if (OUTK == kPrepOutSplitF16) static_cast<uint16_t*>(p.out_lo)[o] = 0;
    }
  }
}

// Four input channels (the 4-channel latent): one item = one voxel x two taps,
// i.e. the 8 consecutive columns [8p, 8p + 8) written as one 16-byte store, from
// two 16-byte neighbour loads (tap 27 is the zero padding up to 112 columns).
template <int OUTK>
__global__ void __launch_bounds__(256) im2col4_kernel(const PrepParams p, const FastDiv pdiv, const FastDiv wdiv,
                                                      const FastDiv hdiv, const unsigned items) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int b = blockIdx.y;
  const unsigned vox = static_cast<unsigned>(p.od) * p.oh * p.ow;
  const PrepSource& s = p.src[0];
  for (unsigned item = blockIdx.x * blockDim.x + threadIdx.x; item < items; item += gridDim.x * blockDim.x) {
    const unsigned v = fdiv(pdiv, item);
    const int pair = static_cast<int>(item - v * pdiv.d);
    const unsigned yz = fdiv(wdiv, v);
    const int x = static_cast<int>(v - yz * wdiv.d);
    const unsigned z = fdiv(hdiv, yz);
    const int y = static_cast<int>(yz - z * hdiv.d);
    float out[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tap = 2 * pair + h;
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tap < 27) {
        const int gz = static_cast<int>(z) + tap / 9 - 1, gy = y + (tap / 3) % 3 - 1, gx = x + tap % 3 - 1;
        if (gz >= 0 && gz < p.od && gy >= 0 && gy < p.oh && gx >= 0 && gx < p.ow) {
          const long long src = ((static_cast<long long>(b) * p.od + gz) * p.oh + gy) * p.ow + gx;
          q = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(s.ptr) + src * s.cstride));
          float t[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (p.affine != nullptr) {
              const float* a = p.affine + (static_cast<long long>(b) * 4 + c) * 2;
              t[c] = fmaf(t[c], __ldg(a), __ldg(a + 1));
            }
            if (p.silu) t[c] = silu_f<false>(t[c]);
          }
          q = make_float4(t[0], t[1], t[2], t[3]);
        }
      }
      out[4 * h] = q.x;
      out[4 * h + 1] = q.y;
      out[4 * h + 2] = q.z;
      out[4 * h + 3] = q.w;
    }
    store_vec<OUTK, 8>(p, (static_cast<long long>(b) * vox + v) * p.out_cstride + 8 * pair, out);
  }
}

// Packed weights [27][opad][cpad_src] (hi and, for the split kind, lo) ->
// [opad][kdense] with column tap * cin + c, zero past 27 * cin.
__global__ void repack_im2col_kernel(const uint16_t* __restrict__ hi, const uint16_t* __restrict__ lo, int opad,
                                     int cpad_src, int cin, int kdense, uint16_t* __restrict__ out_hi,
                                     uint16_t* __restrict__ out_lo) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int n = opad * kdense;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int o = i / kdense, k = i - o * kdense;
    const int tap = k / cin, c = k - tap * cin;
    uint16_t h = 0, l = 0;
    if (tap < 27) {
      const long long src = (static_cast<long long>(tap) * opad + o) * cpad_src + c;
      h = hi[src];
      if (lo != nullptr) l = lo[src];
    }
    out_hi[i] = h;
    if (out_lo != nullptr) out_lo[i] = l;
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
  if (p.mode == kPrepCopy && p.od == p.sd && p.oh == p.sh && p.ow == p.sw && vec_ok(p, 8))
    return launch_copy_fast(p, stream);
  if (p.mode == kPrepTrilinear && p.affine == nullptr && !p.silu && p.od == 2 * p.sd && p.oh == 2 * p.sh &&
      p.ow == 2 * p.sw && vec_ok(p, 4))
    return launch_tri_fast(p, stream);
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 16LL * device_sm_count()) blocks = 16LL * device_sm_count();
  const bool fast = p.out_kind == kPrepOutBF16 || p.out_kind == kPrepOutF16 || p.out_kind == kPrepOutTF32;
  const dim3 grid(static_cast<unsigned>(blocks));
  const unsigned vo = static_cast<unsigned>(vox_out);
#define CTMR_PREP(MODE)                                                         \
  if (fast) launch_kernel(prepare_kernel<MODE, true>, grid, threads, 0, stream, p, log2, vo); \
  else launch_kernel(prepare_kernel<MODE, false>, grid, threads, 0, stream, p, log2, vo);
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

namespace ctmr {

cudaError_t launch_im2col(const PrepParams& p, int cin, int kdense, cudaStream_t stream) {
  if (cin < 1 || cin > 4 || kdense % 8 || kdense < 27 * cin || p.out_cstride % 8) return cudaErrorInvalidValue;
  const PrepSource& s0 = p.src[0];
  if (cin == 4 && kdense == 112 && !s0.bf16 && s0.cstride % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(s0.ptr) & 15) == 0 && p.out_kind != kPrepOutF32) {
    const FastDiv pd = make_fastdiv(14), wd = make_fastdiv(static_cast<uint32_t>(p.ow)),
                  hd = make_fastdiv(static_cast<uint32_t>(p.oh));
    const long long items = static_cast<long long>(p.od) * p.oh * p.ow * 14;
    if (items >= (1LL << 31)) return cudaErrorInvalidValue;
    long long blocks = (items + 255) / 256;
    static const long long resident = resident_blocks(im2col4_kernel<kPrepOutF16>, 256, 0);
    const long long cap = resident / p.batch > 0 ? resident / p.batch : 1;
    if (blocks > cap) blocks = cap;
    const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(p.batch));
    const unsigned n = static_cast<unsigned>(items);
    switch (p.out_kind) {
      case kPrepOutBF16: launch_kernel(im2col4_kernel<kPrepOutBF16>, grid, 256, 0, stream, p, pd, wd, hd, n); break;
      case kPrepOutF16: launch_kernel(im2col4_kernel<kPrepOutF16>, grid, 256, 0, stream, p, pd, wd, hd, n); break;
      default: launch_kernel(im2col4_kernel<kPrepOutSplitF16>, grid, 256, 0, stream, p, pd, wd, hd, n); break;
    }
    return cudaGetLastError();
  }
  const long long items = static_cast<long long>(p.od) * p.oh * p.ow * (kdense / 8);
  if (items >= (1LL << 31)) return cudaErrorInvalidValue;
  long long blocks = (items + 255) / 256;
  const long long cap = 8LL * device_sm_count() / p.batch + 1;
  if (blocks > cap) blocks = cap;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(p.batch));
  switch (p.out_kind) {
    case kPrepOutBF16: launch_kernel(im2col_kernel<kPrepOutBF16>, grid, 256, 0, stream, p, cin, kdense); break;
    case kPrepOutF16: launch_kernel(im2col_kernel<kPrepOutF16>, grid, 256, 0, stream, p, cin, kdense); break;
    case kPrepOutSplitF16: launch_kernel(im2col_kernel<kPrepOutSplitF16>, grid, 256, 0, stream, p, cin, kdense); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_repack_im2col(const void* hi, const void* lo, int opad, int cpad_src, int cin, int kdense,
                                 void* out_hi, void* out_lo, cudaStream_t stream) {
  const int n = opad * kdense;
  launch_kernel(repack_im2col_kernel, (n + 255) / 256, 256, 0, stream, 
      static_cast<const uint16_t*>(hi), static_cast<const uint16_t*>(lo), opad, cpad_src, cin, kdense,
      static_cast<uint16_t*>(out_hi), static_cast<uint16_t*>(out_lo));
  return cudaGetLastError();
}

}  // namespace ctmr

namespace ctmr {

bool gn_prepare_small_fits(long long voxels, int channels, int groups) {
  if (groups <= 0 || channels % groups != 0 || channels / groups > 64) return false;
  return voxels * (channels / groups) <= kGnPrepSmallElems;
}

cudaError_t launch_gn_prepare_small(const PrepParams& p, const float* gamma, const float* beta, int groups, float eps,
                                    cudaStream_t stream) {
  const int ctot = p.src[0].channels + p.src[1].channels;
  const long long vox = static_cast<long long>(p.od) * p.oh * p.ow;
  if (p.mode != kPrepCopy || p.od != p.sd || p.oh != p.sh || p.ow != p.sw || p.affine != nullptr ||
      !gn_prepare_small_fits(vox, ctot, groups))
    return cudaErrorInvalidValue;
  const FastDiv cd = make_fastdiv(static_cast<uint32_t>(ctot / groups));
  const dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(p.batch));
  switch (p.out_kind) {
    case kPrepOutBF16:
      return launch_kernel(gn_prepare_small_kernel<kPrepOutBF16, true>, grid, dim3(kGnPrepThreads), 0, stream, p,
                           gamma, beta, eps, cd);
    case kPrepOutF16:
      return launch_kernel(gn_prepare_small_kernel<kPrepOutF16, true>, grid, dim3(kGnPrepThreads), 0, stream, p,
                           gamma, beta, eps, cd);
    case kPrepOutSplitF16:
      return launch_kernel(gn_prepare_small_kernel<kPrepOutSplitF16, false>, grid, dim3(kGnPrepThreads), 0, stream,
                           p, gamma, beta, eps, cd);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace ctmr
