// Direct 3x3x3 (padding 1, stride 1) convolution for narrow outputs (C_out <= 4):
// the MAISI output convolutions (UNet out.2: 64 -> 4, VAE decoder: 64 -> 1).
//
// With one to four output channels a tensor-core GEMM tile is almost all padding
// and its per-tap operand reloads dominate (27 taps x C_in x 2 bytes per output
// voxel), so this is an fp32 FMA kernel that streams the input along depth.
//
// A CTA owns a 16 (h) x 32 (w) column of outputs over a chunk of depths. It walks
// the input planes of that chunk (plus one on either side) once: each plane's
// 18 x 34 halo is staged in shared memory 32 channels at a time with 16-byte
// loads of whole 128-byte channel runs (so every DRAM line fetched is used in
// full), the group-norm affine and SiLU applied once per staged value and zeros
// outside the volume (the padding acts on the normalised input). A thread holds a
// 4 (h) x 2 (w) output block for the three output depths a plane feeds (kd = 0,
// 1, 2) in registers; per channel it reads the plane's 6 x 4 window and the 27
// weights once and applies all 27 taps (under half a shared-memory byte per
// FMA). When an output depth has received its last plane it is written (with
// bias and residual) and the three accumulators rotate.
//
// Thread groups (64 threads each): for one output channel the four groups split
// each 32-channel slice (8 channels each) and their partial sums are added in
// group order in shared memory; for two to four output channels group g
// computes channel g.
// The weights are the split-fp32 packing (hi + lo * 2^-11 reassembles them to
// ~2^-22), staged once per CTA; the activations are used unrounded.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "conv3d_narrow.cuh"
#include "launch.cuh"

namespace ctmr {
namespace {

constexpr int kTH = 16, kTW = 32;          // output column per CTA (h, w)
constexpr int kHH = kTH + 2, kHW = kTW + 2;
constexpr int kRow = 36;                   // staged row stride in floats (16-byte aligned rows)
constexpr int kPlane = kHH * kRow;         // floats per staged channel plane
constexpr int kCS = 32;                    // channels staged per pass
constexpr int kQW = 2;                     // outputs per thread along w (4 along h)
constexpr int kGroupThreads = (kTH / 4) * (kTW / kQW);  // 64 threads cover the column
constexpr int kThreads = 4 * kGroupThreads;             // 4 groups (channel quarters or output channels)
constexpr int kSpatial = kTH * kTW;        // 512 outputs per depth
constexpr int kWTap = 28;                  // weight row stride (27 taps, 16-byte aligned rows)

size_t narrow_smem_bytes(int cin, int co) {
  const size_t stage = static_cast<size_t>(kCS) * kPlane * 4;
  const size_t red = co == 1 ? static_cast<size_t>(4) * kSpatial * 4 : 0;
  const size_t w = static_cast<size_t>(cin) * kWTap * co * 4;
  const size_t aff = static_cast<size_t>(cin) * 8;
  return stage + red + w + aff;
}

// SiLU t * sigmoid(t) with the hardware exponential and a fast divide
// (relative error a few ulp, well inside the fp32 budget).
__device__ __forceinline__ float silu_fast(float t) { return __fdividef(t, 1.f + __expf(-t)); }

// Two fp32 FMAs in one instruction (fma.rn.f32x2, sm_100): each lane is an
// IEEE fma, bit-identical to fmaf.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

template <int CO>
__global__ void __launch_bounds__(kThreads) narrow_conv_kernel(const NarrowParams p, const int chunk_d) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  extern __shared__ __align__(16) float smem[];
  float* s_in = smem;                                        // [kCS][kHH][kRow]
  float* s_red = s_in + kCS * kPlane;                        // [4][kSpatial] (CO == 1)
  float* s_w = s_red + (CO == 1 ? 4 * kSpatial : 0);         // [CO][cin][kWTap]
  float2* s_aff = reinterpret_cast<float2*>(s_w + p.cin * kWTap * CO);  // [cin] (scale, offset)

  const int tiles_w = (p.w + kTW - 1) / kTW, tiles_h = (p.h + kTH - 1) / kTH;
  int t = blockIdx.x;
  const int tw = t % tiles_w; t /= tiles_w;
  const int th = t % tiles_h; t /= tiles_h;
  const int d0 = t * chunk_d;
  const int d1 = min(p.d, d0 + chunk_d);
  const int b = blockIdx.y;
  const int w0 = tw * kTW, h0 = th * kTH;
  const int tid = threadIdx.x;
  const int sp = tid % kGroupThreads, grp = tid / kGroupThreads;
  const int lw = (sp % (kTW / kQW)) * kQW, lh = (sp / (kTW / kQW)) * 4;

  // Weights for every input channel, fp32 [o][c][tap] (rows of kWTap).
  for (int e = tid; e < p.cin * kWTap * CO; e += kThreads) {
    const int tap = e % kWTap, c = (e / kWTap) % p.cin, o = e / (kWTap * p.cin);
    float wv = 0.f;
    if (o < p.cout && tap < 27) {
      const long long k = (static_cast<long long>(tap) * p.opad + o) * p.cpad + c;
      wv = __half2float(p.w_hi[k]) + __half2float(p.w_lo[k]) * (1.f / 2048.f);
    }
    s_w[e] = wv;
  }
  for (int c = tid; c < p.cin; c += kThreads) {
    float2 a = make_float2(1.f, 0.f);
    if (p.affine != nullptr) {
      const float* src = p.affine + (static_cast<long long>(b) * p.cin + c) * 2;
      a = make_float2(__ldg(src), __ldg(src + 1));
    }
    s_aff[c] = a;
  }

  static_assert(kQW == 2, "one f32x2 accumulator pair per output row");
  float2 acc[3][4];  // [output depth z+1, z, z-1 for input plane z][h] -> (w, w + 1)
#pragma unroll
  for (int k = 0; k < 3; ++k)
#pragma unroll
    for (int a = 0; a < 4; ++a) acc[k][a] = make_float2(0.f, 0.f);

  const float* x = static_cast<const float*>(p.x);
  const long long vox_b = static_cast<long long>(b) * p.d * p.h * p.w;
  const int co = CO == 1 ? 0 : grp;  // output channel of this thread

  for (int z = d0 - 1; z <= d1; ++z) {
    if (z >= 0 && z < p.d) {
      for (int c0 = 0; c0 < p.cin; c0 += kCS) {
        const int cn = min(kCS, p.cin - c0);
        __syncthreads();  // the previous pass's reads of s_in are done (and s_w is written)
        // Stage: item = (8-channel octet, halo voxel), voxel fastest so that a warp's
        // stores land on consecutive banks; each thread issues kBatch items' loads
        // before transforming any of them.
        constexpr int kVox = kHH * kHW;
        constexpr int kItems = kVox * (kCS / 8);
        constexpr int kBatch = 5;
        for (int base = tid; base < kItems; base += kBatch * kThreads) {
          float4 v[kBatch][2];
          int dst[kBatch];
          int cq[kBatch];
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            const int e = base + k * kThreads;
            const int oct = e / kVox, vox = e - oct * kVox;
            const int hy = vox / kHW, hx = vox - hy * kHW;
            const int gx = w0 + hx - 1, gy = h0 + hy - 1;
            const int c = oct * 8;
            cq[k] = c;
            dst[k] = e < kItems ? c * kPlane + hy * kRow + hx : -1;
            v[k][0] = make_float4(0.f, 0.f, 0.f, 0.f);
            v[k][1] = v[k][0];
            if (e < kItems && c < cn && gx >= 0 && gx < p.w && gy >= 0 && gy < p.h) {
              const float* src = x + (vox_b + (static_cast<long long>(z) * p.h + gy) * p.w + gx) * p.x_cstride + c0 + c;
              if (p.vec4 && c + 8 <= cn) {
                v[k][0] = __ldg(reinterpret_cast<const float4*>(src));
                v[k][1] = __ldg(reinterpret_cast<const float4*>(src) + 1);
              } else {
                float* f = reinterpret_cast<float*>(v[k]);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (c + i < cn) f[i] = __ldg(src + i);
              }
            } else {
              cq[k] = -1;  // padding or past the channels: stays zero
            }
          }
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            if (dst[k] < 0) continue;
            float u[8] = {v[k][0].x, v[k][0].y, v[k][0].z, v[k][0].w, v[k][1].x, v[k][1].y, v[k][1].z, v[k][1].w};
            if (cq[k] >= 0) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                if (cq[k] + i < cn) {
                  const float2 a = s_aff[c0 + cq[k] + i];
                  const float t = fmaf(u[i], a.x, a.y);
                  u[i] = p.silu ? silu_fast(t) : t;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) s_in[dst[k] + i * kPlane] = u[i];
          }
        }
        __syncthreads();
        // Channels of this slice for this thread: a quarter (one output) or all of them.
        const int cb = CO == 1 ? grp * (kCS / 4) : 0;
        const int ce = CO == 1 ? min(cn, cb + kCS / 4) : cn;
#pragma unroll 1
        for (int c = cb; c < ce; ++c) {
          const float* plane = s_in + c * kPlane;
          float2 r[6][3];  // per window row: (w, w+1), (w+1, w+2), (w+2, w+3)
#pragma unroll
          for (int a = 0; a < 6; ++a) {
            const float* row = plane + (lh + a) * kRow + lw;
            r[a][0] = *reinterpret_cast<const float2*>(row);
            r[a][2] = *reinterpret_cast<const float2*>(row + 2);
            r[a][1] = make_float2(r[a][0].y, r[a][2].x);
          }
          float wv[kWTap];
          const float4* wrow = reinterpret_cast<const float4*>(s_w + (static_cast<long long>(co) * p.cin + c0 + c) * kWTap);
#pragma unroll
          for (int j = 0; j < kWTap / 4; ++j) {
            const float4 q = wrow[j];
            wv[4 * j] = q.x;
            wv[4 * j + 1] = q.y;
            wv[4 * j + 2] = q.z;
            wv[4 * j + 3] = q.w;
          }
#pragma unroll
          for (int kd = 0; kd < 3; ++kd) {
            // Input plane z feeds output depth z + 1 - kd, held in acc[kd].
            const int od = z + 1 - kd;
            if (od < d0 || od >= d1) continue;
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
              for (int kw = 0; kw < 3; ++kw) {
                const float w = wv[(kd * 3 + kh) * 3 + kw];
                const float2 w2 = make_float2(w, w);
#pragma unroll
                for (int a = 0; a < 4; ++a) acc[kd][a] = ffma2(r[a + kh][kw], w2, acc[kd][a]);
              }
          }
        }
      }
    }
    // Output depth z - 1 (acc[2]) has all its planes.
    const int od = z - 1;
    if (od >= d0 && od < d1) {
      float out[4][kQW];
      if (CO == 1) {
        __syncthreads();  // s_red is free
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int q = 0; q < kQW; ++q) s_red[grp * kSpatial + (lh + a) * kTW + lw + q] = q == 0 ? acc[2][a].x : acc[2][a].y;
        __syncthreads();
      } else {
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int q = 0; q < kQW; ++q) out[a][q] = q == 0 ? acc[2][a].x : acc[2][a].y;
      }
      if (CO == 1) {
        // 512 outputs, two per thread, summed over the four channel quarters in order.
#pragma unroll
        for (int i = 0; i < kSpatial / kThreads; ++i) {
          const int s = tid + i * kThreads;
          const int oh = h0 + s / kTW, ow = w0 + s % kTW;
          float v = ((s_red[s] + s_red[kSpatial + s]) + s_red[2 * kSpatial + s]) + s_red[3 * kSpatial + s];
          if (oh < p.h && ow < p.w) {
            const long long vox = vox_b + (static_cast<long long>(od) * p.h + oh) * p.w + ow;
            if (p.bias != nullptr) v += __ldg(p.bias + static_cast<long long>(b) * p.bias_bstride);
            if (p.res != nullptr) {
              long long rv = vox;
              if (p.res_up)
                rv = ((static_cast<long long>(b) * (p.d / 2) + (od >> 1)) * (p.h / 2) + (oh >> 1)) * (p.w / 2) +
                     (ow >> 1);
              v += __ldg(p.res + rv * p.res_cstride);
            }
            p.y[vox * p.y_cstride] = v;
          }
        }
      } else if (co < p.cout) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const int oh = h0 + lh + a;
#pragma unroll
          for (int q = 0; q < kQW; ++q) {
            const int ow = w0 + lw + q;
            if (oh >= p.h || ow >= p.w) continue;
            const long long vox = vox_b + (static_cast<long long>(od) * p.h + oh) * p.w + ow;
            float v = out[a][q];
            if (p.bias != nullptr) v += __ldg(p.bias + static_cast<long long>(b) * p.bias_bstride + co);
            if (p.res != nullptr) {
              long long rv = vox;
              if (p.res_up)
                rv = ((static_cast<long long>(b) * (p.d / 2) + (od >> 1)) * (p.h / 2) + (oh >> 1)) * (p.w / 2) +
                     (ow >> 1);
              v += __ldg(p.res + rv * p.res_cstride + co);
            }
            p.y[vox * p.y_cstride + co] = v;
          }
        }
      }
    }
    // Rotate: acc[2] <- acc[1] <- acc[0] <- 0 (output depths z, z + 1, z + 2 for plane z + 1).
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      acc[2][a] = acc[1][a];
      acc[1][a] = acc[0][a];
      acc[0][a] = make_float2(0.f, 0.f);
    }
  }
}

template <int CO>
cudaError_t launch_typed(const NarrowParams& p, cudaStream_t stream) {
  auto kern = narrow_conv_kernel<CO>;
  const size_t smem = narrow_smem_bytes(p.cin, CO);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // Depth chunks: about two CTAs per SM over the whole grid, so one wave.
  const int cols = ((p.w + kTW - 1) / kTW) * ((p.h + kTH - 1) / kTH) * p.batch;
  int per_col = (2 * device_sm_count()) / cols;
  if (per_col < 1) per_col = 1;
  const int chunk_d = (p.d + per_col - 1) / per_col;
  const int chunks = (p.d + chunk_d - 1) / chunk_d;
  const int tiles = ((p.w + kTW - 1) / kTW) * ((p.h + kTH - 1) / kTH) * chunks;
  const dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(p.batch));
  launch_kernel(kern, grid, kThreads, smem, stream, p, chunk_d);
  return cudaGetLastError();
}

}  // namespace

bool narrow_conv_supported(int cin, int cout) {
  return cout >= 1 && cout <= 4 && cin >= 1 && narrow_smem_bytes(cin, cout == 1 ? 1 : 4) <= 200 * 1024;
}

cudaError_t launch_narrow_conv(const NarrowParams& p, cudaStream_t stream) {
  if (!narrow_conv_supported(p.cin, p.cout)) return cudaErrorInvalidValue;
  if (p.cout == 1) return launch_typed<1>(p, stream);
  return launch_typed<4>(p, stream);
}

}  // namespace ctmr
