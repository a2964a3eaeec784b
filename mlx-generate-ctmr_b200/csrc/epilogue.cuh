// Epilogue helpers shared by the implicit-GEMM kernels: residual add and the
// store of 16 output columns of one voxel row (vectorised when aligned).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "conv3d_umma.cuh"

namespace ctmr {

__device__ __forceinline__ float bf16_to_f32(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Add the residual and store 16 output columns [n, n+16) of one voxel row. Residual loads go
// through L2 (ld.global.cg), not the read-only path, so an in-place residual add (residual ==
// output, each element read before it is written) is defined.
__device__ __forceinline__ void store_row16(const ConvGeom& g, float (&v)[16], int n, long long out_off,
                                            long long res_off) {
  const int cnt = min(16, g.cout - n);
  if (cnt <= 0) return;
  if (g.res != nullptr) {
    if (g.res_bf16) {
      const uint16_t* r = static_cast<const uint16_t*>(g.res) + res_off;
      if (cnt == 16 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
        const uint4 q0 = __ldcg(reinterpret_cast<const uint4*>(r));
        const uint4 q1 = __ldcg(reinterpret_cast<const uint4*>(r) + 1);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[2 * i] += bf16_to_f32(static_cast<uint16_t>(w[i] & 0xFFFFu));
          v[2 * i + 1] += bf16_to_f32(static_cast<uint16_t>(w[i] >> 16));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < cnt) v[i] += bf16_to_f32(r[i]);
      }
    } else {
      const float* r = static_cast<const float*>(g.res) + res_off;
      if (cnt == 16 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 q = __ldcg(reinterpret_cast<const float4*>(r) + i);
          v[4 * i] += q.x;
          v[4 * i + 1] += q.y;
          v[4 * i + 2] += q.z;
          v[4 * i + 3] += q.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < cnt) v[i] += __ldcg(r + i);
      }
    }
  }
  if (g.out_bf16) {
    uint16_t* o = static_cast<uint16_t*>(g.out) + out_off;
    if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      uint4 q0, q1;
      q0.x = pack_bf16x2(v[0], v[1]);
      q0.y = pack_bf16x2(v[2], v[3]);
      q0.z = pack_bf16x2(v[4], v[5]);
      q0.w = pack_bf16x2(v[6], v[7]);
      q1.x = pack_bf16x2(v[8], v[9]);
      q1.y = pack_bf16x2(v[10], v[11]);
      q1.z = pack_bf16x2(v[12], v[13]);
      q1.w = pack_bf16x2(v[14], v[15]);
      reinterpret_cast<uint4*>(o)[0] = q0;
      reinterpret_cast<uint4*>(o)[1] = q1;
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < cnt) {
          __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
          o[i] = *reinterpret_cast<uint16_t*>(&h);
        }
      }
    }
  } else {
    float* o = static_cast<float*>(g.out) + out_off;
    if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < cnt) o[i] = v[i];
    }
  }
}

// Store 16 finished output columns [n, n+16) of one voxel row.
__device__ __forceinline__ void store16(const ConvGeom& g, const float (&v)[16], int n, long long out_off) {
  const int cnt = min(16, g.cout - n);
  if (g.out_bf16) {
    uint16_t* o = static_cast<uint16_t*>(g.out) + out_off;
    if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      uint4 q0, q1;
      q0.x = pack_bf16x2(v[0], v[1]);
      q0.y = pack_bf16x2(v[2], v[3]);
      q0.z = pack_bf16x2(v[4], v[5]);
      q0.w = pack_bf16x2(v[6], v[7]);
      q1.x = pack_bf16x2(v[8], v[9]);
      q1.y = pack_bf16x2(v[10], v[11]);
      q1.z = pack_bf16x2(v[12], v[13]);
      q1.w = pack_bf16x2(v[14], v[15]);
      reinterpret_cast<uint4*>(o)[0] = q0;
      reinterpret_cast<uint4*>(o)[1] = q1;
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < cnt) {
          __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
          o[i] = *reinterpret_cast<uint16_t*>(&h);
        }
      }
    }
  } else {
    float* o = static_cast<float*>(g.out) + out_off;
    if (cnt == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < cnt) o[i] = v[i];
    }
  }
}

// Issue the residual loads for output columns [n, n + 64) of one voxel row into
// raw 32-bit words (fp32: one column per word; bf16: two columns per word), so
// that their latency overlaps the accumulator wait and the previous block.
__device__ __forceinline__ void res_issue64(const ConvGeom& g, int n, long long res_off, uint32_t (&w)[64]) {
  const int cnt = min(64, g.cout - n);
  if (cnt <= 0) return;
  if (g.res_bf16) {
    const uint16_t* r = static_cast<const uint16_t*>(g.res) + res_off;
    if (cnt == 64 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 q = __ldcg(reinterpret_cast<const uint4*>(r) + i);
        w[4 * i] = q.x;
        w[4 * i + 1] = q.y;
        w[4 * i + 2] = q.z;
        w[4 * i + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint32_t lo = 2 * i < cnt ? r[2 * i] : 0u;
        const uint32_t hi = 2 * i + 1 < cnt ? r[2 * i + 1] : 0u;
        w[i] = lo | (hi << 16);
      }
    }
  } else {
    const float* r = static_cast<const float*>(g.res) + res_off;
    if (cnt == 64 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 q = __ldcg(reinterpret_cast<const uint4*>(r) + i);
        w[4 * i] = q.x;
        w[4 * i + 1] = q.y;
        w[4 * i + 2] = q.z;
        w[4 * i + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) w[i] = i < cnt ? __float_as_uint(__ldcg(r + i)) : 0u;
    }
  }
}

// Residual column j (0..63) of a block loaded by res_issue64.
__device__ __forceinline__ float res_word(const ConvGeom& g, const uint32_t (&w)[64], int j) {
  if (g.res_bf16) return __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
  return __uint_as_float(w[j]);
}

// ---------------------------------------------------------------- output statistics
// Chan et al.'s pairwise update of (count, mean, M2) moments.
__device__ __forceinline__ void chan_merge(float* m, float nb, float meanb, float m2b) {
  if (nb == 0.f) return;
  const float na = m[0];
  if (na == 0.f) {
    m[0] = nb;
    m[1] = meanb;
    m[2] = m2b;
    return;
  }
  const float n = na + nb;
  const float delta = meanb - m[1];
  const float fb = nb / n;
  m[1] = fmaf(delta, fb, m[1]);
  m[2] = m[2] + m2b + delta * delta * na * fb;
  m[0] = n;
}

// Reduce-scatter of 16 per-lane columns over the warp (16 shuffles, fixed
// order): lane l ends up with the warp total of column stat_col(l).
__device__ __forceinline__ int stat_col(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
__device__ __forceinline__ int stat_src(int col) {
  return (((col >> 3) & 1) << 4) | (((col >> 2) & 1) << 3) | (((col >> 1) & 1) << 2) | ((col & 1) << 1);
}
__device__ __forceinline__ float reduce_scatter16(const float (&x)[16], int lane) {
  float a[8], b[4], c[2];
  const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4, h1 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = (h4 ? x[i + 8] : x[i]) + __shfl_xor_sync(0xffffffffu, h4 ? x[i] : x[i + 8], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) b[i] = (h3 ? a[i + 4] : a[i]) + __shfl_xor_sync(0xffffffffu, h3 ? a[i] : a[i + 4], 8);
#pragma unroll
  for (int i = 0; i < 2; ++i) c[i] = (h2 ? b[i + 2] : b[i]) + __shfl_xor_sync(0xffffffffu, h2 ? b[i] : b[i + 2], 4);
  const float d = (h1 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, h1 ? c[0] : c[1], 2);
  return d + __shfl_xor_sync(0xffffffffu, d, 1);
}

// Moments of 16 output columns over this warp's valid rows (two passes: means,
// then squared deviations), merged into the warp-private accumulator `acc`
// (column i at acc + 3 * i) for the first `cnt` columns. Warp-collective.
__device__ __forceinline__ void warp_stats16(const float (&v)[16], bool valid, int cnt, float* acc) {
  const int lane = threadIdx.x & 31;
  const unsigned vm = __ballot_sync(0xffffffffu, valid);
  if (vm == 0u) return;
  const float nw = static_cast<float>(__popc(vm));
  float x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = valid ? v[i] : 0.f;
  const float mean = reduce_scatter16(x, lane) / nw;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float mi = __shfl_sync(0xffffffffu, mean, stat_src(i));
    const float d = valid ? v[i] - mi : 0.f;
    x[i] = d * d;
  }
  const float m2 = reduce_scatter16(x, lane);
  const int col = stat_col(lane);
  if ((lane & 1) == 0 && col < cnt) chan_merge(acc + 3 * col, nw, mean, m2);
  __syncwarp();
}

}  // namespace ctmr
