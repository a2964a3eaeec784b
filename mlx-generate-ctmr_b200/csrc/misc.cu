// Small memory-bound kernels around the convolution stack: layout transposes
// at the API boundary, the sliding-window Gaussian blend of the VAE decode
// (`decode.py:115-184`), and the guided rectified-flow Euler update
// (`image.py:163-175` + `rflow.py:101-121`).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "misc.cuh"
#include "launch.cuh"

namespace ctmr {
namespace {

__device__ __forceinline__ float ld_any(const void* p, int bf16, long long i) {
  if (bf16) return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p)[i]) << 16);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_any(void* p, int bf16, long long i, float v) {
  if (bf16) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<float*>(p)[i] = v;
  }
}

// (B, C, S) <-> (B, S, C) through a 32x33 shared tile; one batch item per grid.z.
__global__ void transpose_cs_kernel(const void* __restrict__ in, int in_bf16, void* __restrict__ out, int out_bf16,
                                    int rows, int cols) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  __shared__ float tile[32][33];
  const long long boff = static_cast<long long>(blockIdx.z) * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = ld_any(in, in_bf16, boff + static_cast<long long>(r) * cols + c);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) st_any(out, out_bf16, boff + static_cast<long long>(c) * rows + r, tile[threadIdx.x][i]);
  }
}

// acc[b, z0+z, y0+y, x0+x, c] += pred[b, z, y, x, c] * w(z, y, x); wsum[...] += w once per voxel.
// w = max(gz[z/scale] * gy[y/scale] * gx[x/scale], floor), the nearest-resized
// Gaussian importance map of `decode.py:88-112` / `:164`.
__global__ void window_accumulate_kernel(const WindowParams p) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const long long per_b = static_cast<long long>(p.wd) * p.wh * p.ww;
  const long long total = per_b * p.batch * p.channels;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % p.channels);
    long long v = i / p.channels;
    const int x = static_cast<int>(v % p.ww); v /= p.ww;
    const int y = static_cast<int>(v % p.wh); v /= p.wh;
    const int z = static_cast<int>(v % p.wd);
    const int b = static_cast<int>(v / p.wd);
    const float w = fmaxf(p.gz[z / p.scale] * p.gy[y / p.scale] * p.gx[x / p.scale], p.floor_value);
    const long long src = (((static_cast<long long>(b) * p.wd + z) * p.wh + y) * p.ww + x) * p.pred_cstride + c;
    const long long dvox = ((static_cast<long long>(b) * p.od + (p.z0 + z)) * p.oh + (p.y0 + y)) * p.ow + (p.x0 + x);
    p.acc[dvox * p.channels + c] += ld_any(p.pred, p.pred_bf16, src) * w;
    if (c == 0 && b == 0) {
      const long long wv = (static_cast<long long>(p.z0 + z) * p.oh + (p.y0 + y)) * p.ow + (p.x0 + x);
      p.wsum[wv] += w;
    }
  }
}

__global__ void window_finalize_kernel(const float* __restrict__ acc, const float* __restrict__ wsum,
                                       float* __restrict__ out, int batch, int channels, int od, int oh, int ow,
                                       int cz0, int cy0, int cx0, int cd, int ch, int cw) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  // out is NCDHW (B, C, cd, ch, cw): the cropped blend, acc / wsum.
  const long long total = static_cast<long long>(batch) * channels * cd * ch * cw;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long v = i;
    const int x = static_cast<int>(v % cw); v /= cw;
    const int y = static_cast<int>(v % ch); v /= ch;
    const int z = static_cast<int>(v % cd); v /= cd;
    const int c = static_cast<int>(v % channels);
    const int b = static_cast<int>(v / channels);
    const long long wv = (static_cast<long long>(cz0 + z) * oh + (cy0 + y)) * ow + (cx0 + x);
    const long long av = ((static_cast<long long>(b) * od + (cz0 + z)) * oh + (cy0 + y)) * ow + (cx0 + x);
    out[i] = acc[av * channels + c] / wsum[wv];
  }
}

// z_next = z + dt * v, v = u + s * (c - u) with c = vel[:n], u = vel[n:] (or v = vel when s < 0).
__global__ void rflow_step_kernel(const float* z, const float* __restrict__ vel, long long n, float guidance,
                                  int guided, float dt, const float* __restrict__ dt_device, float* out) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  if (dt_device != nullptr) dt = *dt_device;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v = vel[i];
    if (guided) {
      const float u = vel[n + i];
      v = u + guidance * (v - u);
    }
    out[i] = z[i] + v * dt;
  }
}

unsigned grid_for(long long total, int threads) {
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 32LL * device_sm_count()) blocks = 32LL * device_sm_count();
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace

cudaError_t launch_transpose_cs(const void* in, int in_bf16, void* out, int out_bf16, int batch, int rows, int cols,
                                cudaStream_t stream) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return cudaSuccess;
  const dim3 grid((cols + 31) / 32, (rows + 31) / 32, batch);
  launch_kernel(transpose_cs_kernel, grid, dim3(32, 8), 0, stream, in, in_bf16, out, out_bf16, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_window_accumulate(const WindowParams& p, cudaStream_t stream) {
  const long long total = static_cast<long long>(p.wd) * p.wh * p.ww * p.batch * p.channels;
  launch_kernel(window_accumulate_kernel, grid_for(total, 256), dim3(256), 0, stream, p);
  return cudaGetLastError();
}

cudaError_t launch_window_finalize(const float* acc, const float* wsum, float* out, int batch, int channels, int od,
                                   int oh, int ow, int cz0, int cy0, int cx0, int cd, int ch, int cw,
                                   cudaStream_t stream) {
  const long long total = static_cast<long long>(batch) * channels * cd * ch * cw;
  launch_kernel(window_finalize_kernel, grid_for(total, 256), dim3(256), 0, stream, acc, wsum, out, batch, channels, od, oh, ow, cz0,
                                                                    cy0, cx0, cd, ch, cw);
  return cudaGetLastError();
}

cudaError_t launch_rflow_step(const float* z, const float* vel, long long n, float guidance, int guided, float dt,
                              const float* dt_device, float* out, cudaStream_t stream) {
  launch_kernel(rflow_step_kernel, grid_for(n, 256), dim3(256), 0, stream, z, vel, n, guidance, guided, dt, dt_device, out);
  return cudaGetLastError();
}

}  // namespace ctmr
