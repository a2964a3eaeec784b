// Direct 3x3x3 (padding 1, stride 1) convolution for tiny inputs (C_in <= 4) in
// the fp32 mode: the conv_in of the UNet, the ControlNet and the VAE decoder on
// the 4-channel latent.
//
// With four input channels the whole reduction is 108 products per output, far
// too short for a tensor-core pipeline to pay for its operand staging. Here a
// block owns 64 output channels (one warp per 16) over tiles of 128 voxels; each
// thread handles 4 voxels: it reads their 27 neighbour rows of C_in values
// (16-byte loads, shared through L1), applies the optional group-norm affine and
// SiLU, and accumulates with fp32 FMAs against weights held in shared memory as
// [tap][c][o] (the split-fp32 packing reassembled, hi + lo * 2^-11); each
// broadcast weight load feeds 16 FMAs, and the next tap's rows are loaded while
// the current one is accumulated. The results are transposed
// through shared memory so that the stores are coalesced 16-byte writes of
// consecutive voxel rows, bias and residual added on the way.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "conv3d_tiny.cuh"
#include "launch.cuh"

namespace ctmr {
namespace {

constexpr int kThreads = 128;          // 4 warps x 16 output channels
constexpr int kOG = 64;                // output channels per block
constexpr int kVPT = 4;                // voxels per thread
constexpr int kTile = 32 * kVPT;       // voxels per block tile

__global__ void __launch_bounds__(kThreads) tiny_conv_kernel(const TinyParams p) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  extern __shared__ __align__(16) float smem[];
  float* s_w = smem;                                                    // [tap][c][o]
  float (*s_out)[kOG + 4] = reinterpret_cast<float (*)[kOG + 4]>(smem + 27 * 4 * kOG);  // [kTile] epilogue rows
  const int og = blockIdx.y, b = blockIdx.z;
  const int o0 = og * kOG;
  // Weights: per tap the packed block [o0, o0 + 64) x cpad is contiguous; read it
  // in 8-half pieces (coalesced) and keep channels < cin as fp32 [tap][c][o].
  {
    const int pieces = kOG * p.cpad / 8;  // per tap
    for (int e = threadIdx.x; e < 27 * pieces; e += kThreads) {
      const int tap = e / pieces, r = e - tap * pieces;
      const int o = (r * 8) / p.cpad, c0 = (r * 8) % p.cpad;
      if (c0 >= 4) continue;
      const long long k = (static_cast<long long>(tap) * p.opad + o0 + o) * p.cpad + c0;
      const bool valid = o0 + o < p.opad;
      uint4 qh = make_uint4(0, 0, 0, 0), ql = qh;
      if (valid) {
        qh = __ldg(reinterpret_cast<const uint4*>(p.w_hi + k));
        ql = __ldg(reinterpret_cast<const uint4*>(p.w_lo + k));
      }
      const __half* hh = reinterpret_cast<const __half*>(&qh);
      const __half* hl = reinterpret_cast<const __half*>(&ql);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool use = valid && c < p.cin && o0 + o < p.cout;
        s_w[(tap * 4 + c) * kOG + o] = use ? __half2float(hh[c]) + __half2float(hl[c]) * (1.f / 2048.f) : 0.f;
      }
    }
  }
  float sc[4] = {1.f, 1.f, 1.f, 1.f}, of[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.affine != nullptr) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c < p.cin) {
        sc[c] = __ldg(p.affine + (static_cast<long long>(b) * p.cin + c) * 2);
        of[c] = __ldg(p.affine + (static_cast<long long>(b) * p.cin + c) * 2 + 1);
      }
    }
  }
  __syncthreads();

  const long long vox_n = static_cast<long long>(p.d) * p.h * p.w;
  const long long tiles = (vox_n + kTile - 1) / kTile;
  const float* xin = static_cast<const float*>(p.x);
  const long long vox_b = static_cast<long long>(b) * vox_n;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ob = warp * 16;  // this warp's 16 output channels within the group
  // Blocks walk tiles of 128 voxels so the weights are staged once per block.
  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    int vz[kVPT], vy[kVPT], vx[kVPT];
#pragma unroll
    for (int i = 0; i < kVPT; ++i) {
      long long v = tile * kTile + i * 32 + lane;  // consecutive lanes, consecutive voxels
      if (v >= vox_n) v = vox_n - 1;  // past the end: computed, not stored
      vx[i] = static_cast<int>(v % p.w);
      const long long yz = v / p.w;
      vy[i] = static_cast<int>(yz % p.h);
      vz[i] = static_cast<int>(yz / p.h);
    }
    float2 acc[kVPT][8];
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = make_float2(0.f, 0.f);

    // Input rows of tap t + 1 are loaded while tap t is accumulated.
    float raw[kVPT][4];
    bool inb[kVPT];  // the row lies inside the volume (else it is zero padding)
    auto load_tap = [&](int tap) {
      const int dz = tap / 9 - 1, dy = (tap / 3) % 3 - 1, dx = tap % 3 - 1;
#pragma unroll
      for (int i = 0; i < kVPT; ++i) {
        const int gz = vz[i] + dz, gy = vy[i] + dy, gx = vx[i] + dx;
        const bool in = gz >= 0 && gz < p.d && gy >= 0 && gy < p.h && gx >= 0 && gx < p.w;
        const float* src = xin + (vox_b + (static_cast<long long>(in ? gz : 0) * p.h + (in ? gy : 0)) * p.w +
                                  (in ? gx : 0)) * p.x_cstride;
        if (p.vec4 && p.cin == 4) {
          const float4 q = in ? __ldg(reinterpret_cast<const float4*>(src)) : make_float4(0.f, 0.f, 0.f, 0.f);
          raw[i][0] = q.x;
          raw[i][1] = q.y;
          raw[i][2] = q.z;
          raw[i][3] = q.w;
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) raw[i][c] = (in && c < p.cin) ? __ldg(src + c) : 0.f;
        }
        inb[i] = in;
      }
    };
    load_tap(0);
#pragma unroll 1
    for (int tap = 0; tap < 27; ++tap) {
      float u[kVPT][4];
#pragma unroll
      for (int i = 0; i < kVPT; ++i) {
        const bool in = inb[i];  // zero padding acts on the transformed input
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float t = fmaf(raw[i][c], sc[c], of[c]);
          if (p.silu) t = t / (1.f + expf(-t));
          u[i][c] = (in && c < p.cin) ? t : 0.f;
        }
      }
      if (tap + 1 < 27) load_tap(tap + 1);
      const float4* wt = reinterpret_cast<const float4*>(s_w + tap * 4 * kOG + ob);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 w4 = wt[c * (kOG / 4) + j];  // one broadcast load feeds kVPT x 4 FMAs
#pragma unroll
          for (int i = 0; i < kVPT; ++i) {
            acc[i][2 * j].x = fmaf(u[i][c], w4.x, acc[i][2 * j].x);
            acc[i][2 * j].y = fmaf(u[i][c], w4.y, acc[i][2 * j].y);
            acc[i][2 * j + 1].x = fmaf(u[i][c], w4.z, acc[i][2 * j + 1].x);
            acc[i][2 * j + 1].y = fmaf(u[i][c], w4.w, acc[i][2 * j + 1].y);
          }
        }
      }
    }

    // Epilogue: the tile's 128 x 64 results go through shared memory so that the
    // stores are whole 16-byte pieces of consecutive voxel rows.
    __syncthreads();  // the previous tile's rows are stored
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4*>(&s_out[i * 32 + lane][ob + 4 * j]) =
            make_float4(acc[i][2 * j].x, acc[i][2 * j].y, acc[i][2 * j + 1].x, acc[i][2 * j + 1].y);
    __syncthreads();
    const int cnt = min(kOG, p.cout - o0);
    const float* bias = p.bias != nullptr ? p.bias + static_cast<long long>(b) * p.bias_bstride + o0 : nullptr;
    for (int e = threadIdx.x; e < kTile * (kOG / 4); e += kThreads) {
      const int r = e / (kOG / 4), q = e % (kOG / 4);
      const long long vr = tile * kTile + r;
      const int o = 4 * q;
      if (vr >= vox_n || o >= cnt) continue;
      const long long vox = vox_b + vr;
      const float4 a = *reinterpret_cast<const float4*>(&s_out[r][o]);
      float val[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (o + i >= cnt) break;
        if (bias != nullptr) val[i] += __ldg(bias + o + i);
        if (p.res != nullptr) val[i] += __ldg(p.res + vox * p.res_cstride + o0 + o + i);
      }
      float* dst = p.y + vox * p.y_cstride + o0 + o;
      if (o + 4 <= cnt && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<float4*>(dst) = make_float4(val[0], val[1], val[2], val[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (o + i < cnt) dst[i] = val[i];
      }
    }
  }
}

}  // namespace

cudaError_t launch_tiny_conv(const TinyParams& p, cudaStream_t stream) {
  if (p.cin < 1 || p.cin > 4 || p.cout < 1) return cudaErrorInvalidValue;
  const long long vox = static_cast<long long>(p.d) * p.h * p.w;
  // About three blocks per SM over the whole grid (each stages the weights once).
  const long long groups = static_cast<long long>((p.cout + kOG - 1) / kOG) * p.batch;
  long long blocks = (vox + kTile - 1) / kTile;
  const long long cap = (3LL * device_sm_count() + groups - 1) / groups;
  if (blocks > cap) blocks = cap;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>((p.cout + kOG - 1) / kOG),
                  static_cast<unsigned>(p.batch));
  const size_t smem = (27 * 4 * kOG + kTile * (kOG + 4)) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(tiny_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  launch_kernel(tiny_conv_kernel, grid, kThreads, smem, stream, p);
  return cudaGetLastError();
}

}  // namespace ctmr
