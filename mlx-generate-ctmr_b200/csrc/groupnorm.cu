// GroupNorm statistics over NDHWC activations -> per-channel (scale, offset)
// pairs, the operand of the conv prologue. Counterpart of the external
// `medmlx_core.group_norm.group_norm_affine` the reference calls at
// `fast_fp32.py:183-189` (layout (B*C*2), consumed at `_nax_conv.py:174-176`).
//
// Pass 1 (grid chunks x batch): each block reads a contiguous voxel range with
// 16-byte loads (every voxel row is C contiguous channels). A thread owns one
// 8-channel slice and a voxel lane; it accumulates sums of (x - pivot) and
// (x - pivot)^2 around one pivot per channel shared by the block (the chunk's
// first voxel), so lanes combine by plain addition: a shuffle-xor tree inside
// each warp, then the warps in order through shared memory. Channels then merge
// into groups in a fixed order (Chan et al.'s pairwise update), one (n, mean,
// M2) partial per group.
// Pass 2 (grid groups x batch): one block per group merges the chunk partials as
// double-precision sums (n, n mean, M2 + n mean^2: each thread its strided chunks
// in order, a fixed shuffle-xor tree per warp, then the warps in order; one
// division at the end), then writes scale = gamma * rstd and offset =
// beta - mean * scale for each channel. The fixed merge order makes the result
// bitwise reproducible run to run.
// Small tensors (a group that 1024 threads read with at most eight loads each) skip
// both passes: one block per (group, batch item) reads its group and writes the
// affine directly (gn_direct_kernel), one launch instead of two.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

#include "groupnorm.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

constexpr int kGnThreads = 256;
// Bulk-staged pass 1 (dense fp32 rows): the block's voxel range streams through a ring of
// kGnStages shared-memory segments of at most kGnSegBytes, filled by cp.async.bulk copies.
constexpr int kGnStages = 4;
constexpr int kGnSegBytes = 16 << 10;

__device__ __forceinline__ float gn_load(const PrepSource& s, long long vox, int c) {
  const long long i = vox * s.cstride + c;
  if (s.bf16) return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(s.ptr) + i)) << 16);
  return __ldg(static_cast<const float*>(s.ptr) + i);
}

__device__ __forceinline__ void gn_load8(const GnParams& p, long long vox, int c0, float (&v)[8], int& cnt) {
  const int ctot = p.src[0].channels + p.src[1].channels;
  cnt = min(8, ctot - c0);
  const PrepSource& s0 = p.src[0];
  if (cnt == 8 && c0 + 8 <= s0.channels && !s0.bf16) {
    const float* ptr = static_cast<const float*>(s0.ptr) + vox * s0.cstride + c0;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(ptr));
      const float4 b = __ldg(reinterpret_cast<const float4*>(ptr) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      return;
    }
  }
  if (cnt == 8 && c0 + 8 <= s0.channels && s0.bf16) {
    const uint16_t* ptr = static_cast<const uint16_t*>(s0.ptr) + vox * s0.cstride + c0;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(ptr));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = c0 + i;
    if (i >= cnt) v[i] = 0.f;
    else if (c < s0.channels) v[i] = gn_load(s0, vox, c);
    else v[i] = gn_load(p.src[1], vox, c - s0.channels);
  }
}

struct Moments {
  float n, mean, m2;
};

__device__ __forceinline__ Moments merge(Moments a, Moments b) {
  if (b.n == 0.f) return a;
  if (a.n == 0.f) return b;
  const float n = a.n + b.n;
  const float delta = b.mean - a.mean;
  const float fb = b.n / n;
  Moments r;
  r.n = n;
  r.mean = fmaf(delta, fb, a.mean);
  r.m2 = a.m2 + b.m2 + delta * delta * a.n * fb;
  return r;
}

// BULK: the sources are dense fp32 rows (cstride == channels, channel counts multiples of 8,
// 16-byte aligned): the voxels come through the shared-memory ring instead of per-thread loads,
// so the bytes in flight do not depend on registers. Same per-thread arithmetic either way.
template <bool BULK>
__global__ void __launch_bounds__(kGnThreads) gn_partial_kernel(const GnParams p) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  __shared__ float s_sum[kGnThreads][8];   // per thread, then per warp: sums of (x - pivot)
  __shared__ float s_sq[kGnThreads][8];    // ... of (x - pivot)^2
  __shared__ float s_n[kGnThreads];
  __shared__ uint64_t s_full[kGnStages];   // BULK: a ring segment has landed
  extern __shared__ float s_chan[];        // [ctot][3]: (count, mean, M2) per channel; BULK: then the ring
  const int ctot = p.src[0].channels + p.src[1].channels;
  const int nslices = (ctot + 7) / 8;
  const int lanes = kGnThreads / nslices;
  const int tid = threadIdx.x;
  const int slice = tid % nslices;
  const int lane = tid / nslices;
  const int b = blockIdx.y;
  const long long per = (p.voxels + p.chunks - 1) / p.chunks;
  const long long v_begin = min(p.voxels, per * blockIdx.x);
  const long long v_end = min(p.voxels, v_begin + per);
  const long long base = static_cast<long long>(b) * p.voxels;

  // One pivot per channel for the whole block (the chunk's first voxel), so that the
  // shifted sums of all lanes add without rescaling: n, S = sum(x - p), Q = sum((x - p)^2)
  // give mean = p + S / n and M2 = Q - S^2 / n.
  float pivot[8], s[8], q[8];
  float n = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    pivot[i] = 0.f;
    s[i] = 0.f;
    q[i] = 0.f;
  }
  if (v_begin < v_end) {
    int cnt;
    gn_load8(p, base + v_begin, slice * 8, pivot, cnt);
  }
  if (BULK) {
    const int c0n = p.src[0].channels, c1n = p.src[1].channels;
    const int seg = max(1, kGnSegBytes / (ctot * 4));  // voxels per segment
    const long long nvox = v_end - v_begin;
    const int nseg = static_cast<int>((nvox + seg - 1) / seg);
    float* ring = s_chan + ((ctot * 3 + 3) & ~3);     // 16-byte aligned after the channel moments
    const int stage_floats = seg * ctot;
    if (tid == 0) {
      for (int i = 0; i < kGnStages; ++i) mbar_init(&s_full[i], 1);
      fence_barrier_init();
    }
    __syncthreads();
    int issued = 0;
    auto issue = [&](int k) {  // segment k into ring slot k % kGnStages (thread 0)
      const int st = k % kGnStages;
      const long long v0 = v_begin + static_cast<long long>(k) * seg;
      const int nv = static_cast<int>(min(static_cast<long long>(seg), v_end - v0));
      const uint32_t b0 = static_cast<uint32_t>(nv * c0n * 4), b1 = static_cast<uint32_t>(nv * c1n * 4);
      float* dst = ring + static_cast<size_t>(st) * stage_floats;
      mbar_arrive_expect_tx(&s_full[st], b0 + b1);
      bulk_load(dst, static_cast<const float*>(p.src[0].ptr) + (base + v0) * c0n, b0, &s_full[st]);
      if (c1n > 0)
        bulk_load(dst + seg * c0n, static_cast<const float*>(p.src[1].ptr) + (base + v0) * c1n, b1, &s_full[st]);
      ++issued;
    };
    if (tid == 0)
      for (int k = 0; k < nseg && k < kGnStages; ++k) issue(k);
    bool ok = true;
    int consumed = 0;
    for (int k = 0; k < nseg; ++k) {
      const int st = k % kGnStages;
      ok = ok && mbar_wait_bounded(&s_full[st], static_cast<uint32_t>(k / kGnStages) & 1u, kErrWaitFull);
      if (ok && lane < lanes) {
        const long long v0 = v_begin + static_cast<long long>(k) * seg;
        const int nv = static_cast<int>(min(static_cast<long long>(seg), v_end - v0));
        const int c = slice * 8;
        const float* row0 = ring + static_cast<size_t>(st) * stage_floats +
                            (c < c0n ? c : seg * c0n + (c - c0n));
        const int pitch = c < c0n ? c0n : c1n;
        for (int j = lane; j < nv; j += lanes) {
          const float4 a = reinterpret_cast<const float4*>(row0 + j * pitch)[0];
          const float4 bq = reinterpret_cast<const float4*>(row0 + j * pitch)[1];
          const float x[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float d = x[i] - pivot[i];
            s[i] += d;
            q[i] = fmaf(d, d, q[i]);
          }
          n += 1.f;
        }
      }
      ++consumed;
      __syncthreads();  // every thread is done with slot st
      if (tid == 0 && ok && k + kGnStages < nseg) issue(k + kGnStages);
    }
    // A copy still in flight (only after a timed-out wait) lands before the block can exit.
    if (tid == 0)
      for (int k = consumed; k < issued; ++k)
        mbar_wait_bounded(&s_full[k % kGnStages], static_cast<uint32_t>(k / kGnStages) & 1u, kErrWaitDrain);
  } else if (lane < lanes) {
    long long v = v_begin + lane;
    // Four voxels per step, all loads issued before any accumulation.
    for (; v + 3 * lanes < v_end; v += 4 * lanes) {
      float x[4][8];
      int cnt;
#pragma unroll
      for (int k = 0; k < 4; ++k) gn_load8(p, base + v + k * lanes, slice * 8, x[k], cnt);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = x[k][i] - pivot[i];
          s[i] += d;
          q[i] = fmaf(d, d, q[i]);
        }
      }
      n += 4.f;
    }
    for (; v < v_end; v += lanes) {
      float x[8];
      int cnt;
      gn_load8(p, base + v, slice * 8, x, cnt);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = x[i] - pivot[i];
        s[i] += d;
        q[i] = fmaf(d, d, q[i]);
      }
      n += 1.f;
    }
  }
  // Lanes -> channels. With a power-of-two slice count below 32 the lanes of one
  // slice sit nslices apart in a warp: a shuffle-xor tree sums them, then the
  // warps add in order through shared memory. Otherwise every thread's sums go
  // through shared memory and add in lane order. Fixed order either way.
  const bool shfl = (nslices & (nslices - 1)) == 0 && nslices < 32;
  if (shfl) {
    for (int off = nslices; off < 32; off <<= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s[i] += __shfl_xor_sync(0xffffffffu, s[i], off);
        q[i] += __shfl_xor_sync(0xffffffffu, q[i], off);
      }
      n += __shfl_xor_sync(0xffffffffu, n, off);
    }
    const int wl = tid & 31;
    if (wl < nslices) {
      const int row = (tid >> 5) * nslices + wl;  // [warp][slice]
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s_sum[row][i] = s[i];
        s_sq[row][i] = q[i];
      }
      s_n[row] = n;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s_sum[tid][i] = s[i];
      s_sq[tid][i] = q[i];
    }
    s_n[tid] = lane < lanes ? n : 0.f;
  }
  __syncthreads();
  const int rows = shfl ? kGnThreads / 32 : lanes;  // partial sums per slice
  for (int c = tid; c < ctot; c += kGnThreads) {
    const int sl = c / 8, i = c % 8;
    float nn = 0.f, ss = 0.f, qq = 0.f;
    for (int r = 0; r < rows; ++r) {
      const int t = r * nslices + sl;
      nn += s_n[t];
      ss += s_sum[t][i];
      qq += s_sq[t][i];
    }
    // The pivot of channel c (every thread of its slice loaded the same value).
    float pv = 0.f;
    if (v_begin < v_end) {
      float x[8];
      int cnt;
      gn_load8(p, base + v_begin, sl * 8, x, cnt);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k == i) pv = x[k];
    }
    const float mean_d = nn > 0.f ? ss / nn : 0.f;
    s_chan[3 * c] = nn;
    s_chan[3 * c + 1] = pv + mean_d;
    s_chan[3 * c + 2] = fmaxf(0.f, qq - ss * mean_d);
  }
  __syncthreads();
  // Channels -> groups (fixed channel order, Chan et al.'s pairwise update).
  const int cpg = ctot / p.groups;
  for (int g = tid; g < p.groups; g += kGnThreads) {
    Moments m{0.f, 0.f, 0.f};
    for (int c = g * cpg; c < (g + 1) * cpg; ++c) m = merge(m, Moments{s_chan[3 * c], s_chan[3 * c + 1], s_chan[3 * c + 2]});
    float* out = p.partials + ((static_cast<long long>(b) * p.chunks + blockIdx.x) * p.groups + g) * 3;
    out[0] = m.n;
    out[1] = m.mean;
    out[2] = m.m2;
  }
}

struct MomentsD {
  double n, mean, m2;
};

__device__ __forceinline__ MomentsD merge_d(MomentsD a, MomentsD b) {
  if (b.n == 0.0) return a;
  if (a.n == 0.0) return b;
  const double n = a.n + b.n;
  const double delta = b.mean - a.mean;
  const double fb = b.n / n;
  return MomentsD{n, a.mean + delta * fb, a.m2 + b.m2 + delta * delta * a.n * fb};
}

__device__ __forceinline__ MomentsD shfl_down_moments(const MomentsD& m, int off) {
  return MomentsD{__shfl_down_sync(0xffffffffu, m.n, off), __shfl_down_sync(0xffffffffu, m.mean, off),
                  __shfl_down_sync(0xffffffffu, m.m2, off)};
}

// One block per (group, batch item): thread i merges chunks i, i + 128, ... in
// order (all of its loads issued before the merges), then a fixed shuffle tree
// joins the lanes of each warp and thread 0 joins the four warps in order (double
// precision, deterministic).
constexpr int kFinThreads = 128;
constexpr int kFinPerThread = 5;  // ceil(gn_max_chunks(1) / kFinThreads)

// The (count, mean, M2) of group g of batch item b over all chunk partials, merged in a
// fixed order (per thread its strided chunks, a shuffle tree per warp, then the warps in
// order) in double precision; the result is valid in thread 0.
// The chunk partials of group g, batch item b, merged in a fixed order: each (n, mean, M2) becomes
// (n, S = n mean, Q = M2 + n mean^2) in double, which add without a division (each thread its
// strided chunks in order, a shuffle-xor tree per warp, then the warps in order); the whole group's
// (n, mean, M2) follows from one division at the end. In double the final Q - S mean loses
// log2(mean^2 / var) of 53 bits, harmless for activations. Valid in thread 0.
__device__ __forceinline__ MomentsD merge_chunks(const GnParams& p, int g, int b, double (*s_m)[3]) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float q[kFinPerThread][3];
#pragma unroll
  for (int j = 0; j < kFinPerThread; ++j) {
    const int k = tid + j * kFinThreads;
    if (k < p.chunks) {
      const float* src = p.partials + ((static_cast<long long>(b) * p.chunks + k) * p.groups + g) * 3;
      q[j][0] = src[0];
      q[j][1] = src[1];
      q[j][2] = src[2];
    } else {
      q[j][0] = 0.f;
      q[j][1] = 0.f;
      q[j][2] = 0.f;
    }
  }
  double n = 0.0, sum = 0.0, sq = 0.0;
#pragma unroll
  for (int j = 0; j < kFinPerThread; ++j) {
    const double nn = q[j][0], mm = q[j][1];
    n += nn;
    sum += nn * mm;
    sq += static_cast<double>(q[j][2]) + nn * mm * mm;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    n += __shfl_xor_sync(0xffffffffu, n, off);
    sum += __shfl_xor_sync(0xffffffffu, sum, off);
    sq += __shfl_xor_sync(0xffffffffu, sq, off);
  }
  if (lane == 0) {
    s_m[warp][0] = n;
    s_m[warp][1] = sum;
    s_m[warp][2] = sq;
  }
  __syncthreads();
  MomentsD t{0.0, 0.0, 0.0};
  if (tid == 0) {
    double tn = 0.0, ts = 0.0, tq = 0.0;
    for (int w = 0; w < kFinThreads / 32; ++w) {
      tn += s_m[w][0];
      ts += s_m[w][1];
      tq += s_m[w][2];
    }
    if (tn > 0.0) {
      const double mean = ts / tn;
      t = MomentsD{tn, mean, fmax(0.0, tq - ts * mean)};
    }
  }
  return t;
}

__device__ __forceinline__ void write_group_affine(double mean, double rstd, int g, int b, int ctot, int cpg,
                                                   const float* gamma, const float* beta, float* affine) {
  for (int c = g * cpg + static_cast<int>(threadIdx.x); c < (g + 1) * cpg; c += kFinThreads) {
    const double gam = gamma != nullptr ? static_cast<double>(gamma[c]) : 1.0;
    const double bet = beta != nullptr ? static_cast<double>(beta[c]) : 0.0;
    const double scale = gam * rstd;
    float* a = affine + (static_cast<long long>(b) * ctot + c) * 2;
    a[0] = static_cast<float>(scale);
    a[1] = static_cast<float>(bet - mean * scale);
  }
}

__global__ void __launch_bounds__(kFinThreads) gn_finalize_kernel(const GnParams p) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  __shared__ double s_m[kFinThreads / 32][3];
  __shared__ double s_stat[2];
  const int g = blockIdx.x, b = blockIdx.y;
  const int ctot = p.src[0].channels + p.src[1].channels;
  const int cpg = ctot / p.groups;
  const MomentsD t = merge_chunks(p, g, b, s_m);
  if (threadIdx.x == 0) {
    const double var = t.n > 0.0 ? t.m2 / t.n : 0.0;
    s_stat[0] = t.mean;
    s_stat[1] = 1.0 / sqrt(var + static_cast<double>(p.eps));
  }
  __syncthreads();
  write_group_affine(s_stat[0], s_stat[1], g, b, ctot, cpg, p.gamma, p.beta, p.affine);
}

// Small tensors: one block per (group, batch item) reads the group once and writes its
// (scale, offset) pairs, one launch in place of pass 1 + pass 2. Thread t owns the VW-channel
// chunk t % slots of the group (VW = 4 with 16-byte loads of dense fp32 rows, else 1) and the
// voxels t / slots, t / slots + lanes, ..., all of its (at most eight) loads in flight at once: a
// group qualifies when every thread needs at most one such round (measured on the MAISI UNet step:
// 5.084 ms with one round, 5.122 with two, 5.163 with four, 5.162 with two passes everywhere). Sums of (x - pivot) and (x - pivot)^2 around each
// channel's first voxel; the lanes of a chunk add by a shuffle-xor tree and then warp by warp
// (power-of-two slot counts below 32) or in lane order through shared memory; the channels join
// in order as double (n, n mean, M2 + n mean^2) sums. Fixed order throughout: bitwise
// reproducible.
constexpr int kGnDirectThreads = 1024;
constexpr int kGnDirectInFlight = 8;

__device__ __forceinline__ float gn_load_cat(const GnParams& p, long long vox, int c) {
  const int c0n = p.src[0].channels;
  return c < c0n ? gn_load(p.src[0], vox, c) : gn_load(p.src[1], vox, c - c0n);
}

// VW consecutive channels from c (16-byte aligned when VW == 4: the launcher checked the rows).
template <int VW>
__device__ __forceinline__ void gn_load_vec(const GnParams& p, long long vox, int c, float (&x)[VW]) {
  if constexpr (VW == 4) {
    const int c0n = p.src[0].channels;
    const PrepSource& s = c < c0n ? p.src[0] : p.src[1];
    const float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(s.ptr) + vox * s.cstride +
                                                           (c < c0n ? c : c - c0n)));
    x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
  } else {
    x[0] = gn_load_cat(p, vox, c);
  }
}

template <int VW>
__global__ void __launch_bounds__(kGnDirectThreads) gn_direct_kernel(const GnParams p) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  __shared__ float s_part[kGnDirectThreads][2 * VW + 1];  // per thread, then per [warp][slot]: n, S, Q
  __shared__ double s_chan[64][3];
  __shared__ double s_stat[2];
  const int g = blockIdx.x, b = blockIdx.y;
  const int ctot = p.src[0].channels + p.src[1].channels;
  const int cpg = ctot / p.groups;  // <= 64, a multiple of VW (checked by the launcher)
  const int slots = cpg / VW;
  const int lanes = kGnDirectThreads / slots;
  const int tid = threadIdx.x;
  const int slot = tid % slots, lane = tid / slots;
  const int c = g * cpg + slot * VW;
  const long long base = static_cast<long long>(b) * p.voxels;
  float pivot[VW], s[VW], q[VW];
  float n = 0.f;
#pragma unroll
  for (int i = 0; i < VW; ++i) pivot[i] = s[i] = q[i] = 0.f;
  if (lane < lanes && p.voxels > 0) {
    gn_load_vec<VW>(p, base, c, pivot);
    for (long long v0 = lane; v0 < p.voxels; v0 += static_cast<long long>(kGnDirectInFlight) * lanes) {
      float x[kGnDirectInFlight][VW];
#pragma unroll
      for (int k = 0; k < kGnDirectInFlight; ++k) {
        const long long v = v0 + static_cast<long long>(k) * lanes;
        if (v < p.voxels) {
          gn_load_vec<VW>(p, base + v, c, x[k]);
        } else {
#pragma unroll
          for (int i = 0; i < VW; ++i) x[k][i] = pivot[i];  // adds zero
        }
      }
#pragma unroll
      for (int k = 0; k < kGnDirectInFlight; ++k) {
#pragma unroll
        for (int i = 0; i < VW; ++i) {
          const float d = x[k][i] - pivot[i];
          s[i] += d;
          q[i] = fmaf(d, d, q[i]);
        }
      }
      const long long left = (p.voxels - v0 + lanes - 1) / lanes;  // this thread's voxels from v0 on
      n += static_cast<float>(left < kGnDirectInFlight ? left : kGnDirectInFlight);
    }
  }
  const bool shfl = (slots & (slots - 1)) == 0 && slots < 32;
  int rows;  // partial sums per slot left in s_part, slot-major within a row
  if (shfl) {
    for (int off = slots; off < 32; off <<= 1) {
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        s[i] += __shfl_xor_sync(0xffffffffu, s[i], off);
        q[i] += __shfl_xor_sync(0xffffffffu, q[i], off);
      }
      n += __shfl_xor_sync(0xffffffffu, n, off);
    }
    const int wl = tid & 31;
    if (wl < slots) {
      const int row = (tid >> 5) * slots + wl;  // [warp][slot]
      s_part[row][0] = n;
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        s_part[row][1 + i] = s[i];
        s_part[row][1 + VW + i] = q[i];
      }
    }
    rows = kGnDirectThreads / 32;
  } else {
    s_part[tid][0] = n;
#pragma unroll
    for (int i = 0; i < VW; ++i) {
      s_part[tid][1 + i] = s[i];
      s_part[tid][1 + VW + i] = q[i];
    }
    rows = lanes;
  }
  __syncthreads();
  if (tid < cpg) {  // channel tid of the group: slot tid / VW, component tid % VW
    const int sl = tid / VW, i = tid % VW;
    float nn = 0.f, ss = 0.f, qq = 0.f;
    for (int r = 0; r < rows; ++r) {
      const int t = r * slots + sl;
      nn += s_part[t][0];
      ss += s_part[t][1 + i];
      qq += s_part[t][1 + VW + i];
    }
    const float pv = p.voxels > 0 ? gn_load_cat(p, base, g * cpg + tid) : 0.f;
    const float mean_d = nn > 0.f ? ss / nn : 0.f;
    const double mean = static_cast<double>(pv) + static_cast<double>(mean_d);
    const double m2 = fmax(0.0, static_cast<double>(qq) - static_cast<double>(ss) * mean_d);
    s_chan[tid][0] = nn;
    s_chan[tid][1] = static_cast<double>(nn) * mean;
    s_chan[tid][2] = m2 + static_cast<double>(nn) * mean * mean;
  }
  __syncthreads();
  if (tid == 0) {
    double tn = 0.0, ts = 0.0, tq = 0.0;
    for (int k = 0; k < cpg; ++k) {
      tn += s_chan[k][0];
      ts += s_chan[k][1];
      tq += s_chan[k][2];
    }
    const double mean = tn > 0.0 ? ts / tn : 0.0;
    const double var = tn > 0.0 ? fmax(0.0, tq - ts * mean) / tn : 0.0;
    s_stat[0] = mean;
    s_stat[1] = 1.0 / sqrt(var + static_cast<double>(p.eps));
  }
  __syncthreads();
  if (tid < cpg) {
    const int cc = g * cpg + tid;
    const double gam = p.gamma != nullptr ? static_cast<double>(p.gamma[cc]) : 1.0;
    const double bet = p.beta != nullptr ? static_cast<double>(p.beta[cc]) : 0.0;
    const double scale = gam * s_stat[1];
    float* a = p.affine + (static_cast<long long>(b) * ctot + cc) * 2;
    a[0] = static_cast<float>(scale);
    a[1] = static_cast<float>(bet - s_stat[0] * scale);
  }
}

// The merged moments themselves, float (count, mean, M2) per (batch item, group), for a
// caller that combines the moments of several parts of one tensor (depth shards).
__global__ void __launch_bounds__(kFinThreads) gn_moments_kernel(const GnParams p, float* moments) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ double s_m[kFinThreads / 32][3];
  const int g = blockIdx.x, b = blockIdx.y;
  const MomentsD t = merge_chunks(p, g, b, s_m);
  if (threadIdx.x == 0) {
    float* out = moments + (static_cast<long long>(b) * p.groups + g) * 3;
    out[0] = static_cast<float>(t.n);
    out[1] = static_cast<float>(t.mean);
    out[2] = static_cast<float>(t.m2);
  }
}

// Affine from the moments of `parts` parts, float[parts][batch][groups][3], merged in part
// order in double precision: every holder of the same moments gets the same affine, bit for bit.
__global__ void __launch_bounds__(kFinThreads) gn_affine_from_moments_kernel(const GnMomentsParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ double s_stat[2];
  const int g = blockIdx.x, b = blockIdx.y;
  const int cpg = p.channels / p.groups;
  if (threadIdx.x == 0) {
    MomentsD t{0.0, 0.0, 0.0};
    for (int k = 0; k < p.parts; ++k) {
      const float* q = p.moments + ((static_cast<long long>(k) * p.batch + b) * p.groups + g) * 3;
      t = merge_d(t, MomentsD{q[0], q[1], q[2]});
    }
    const double var = t.n > 0.0 ? t.m2 / t.n : 0.0;
    s_stat[0] = t.mean;
    s_stat[1] = 1.0 / sqrt(var + static_cast<double>(p.eps));
  }
  __syncthreads();
  write_group_affine(s_stat[0], s_stat[1], g, b, p.channels, cpg, p.gamma, p.beta, p.affine);
}

__global__ void __launch_bounds__(kFinThreads) gn_from_stats_kernel(const GnStatsParams p) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ double s_m[kFinThreads / 32][3];
  __shared__ double s_stat[2];
  const int g = blockIdx.x, b = blockIdx.y;
  const int ctot = p.channels[0] + p.channels[1];
  const int cpg = ctot / p.groups;
  const int c_begin = g * cpg;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int entries = p.slots * cpg;
  MomentsD m{0.0, 0.0, 0.0};
  for (int e = tid; e < entries; e += kFinThreads) {
    const int slot = e / cpg, cl = e - slot * cpg;
    const int c = c_begin + cl;
    const bool second = c >= p.channels[0];
    const int cs = second ? c - p.channels[0] : c;
    const float* base = second ? p.stats[1] : p.stats[0];
    const int nch = second ? p.channels[1] : p.channels[0];
    const float* q = base + ((static_cast<long long>(b) * p.slots + slot) * nch + cs) * 3;
    m = merge_d(m, MomentsD{q[0], q[1], q[2]});
  }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const MomentsD o = shfl_down_moments(m, off);
    if ((lane & (2 * off - 1)) == 0) m = merge_d(m, o);
  }
  if (lane == 0) {
    s_m[warp][0] = m.n;
    s_m[warp][1] = m.mean;
    s_m[warp][2] = m.m2;
  }
  __syncthreads();
  if (tid == 0) {
    MomentsD t{0.0, 0.0, 0.0};
    for (int w = 0; w < kFinThreads / 32; ++w) t = merge_d(t, MomentsD{s_m[w][0], s_m[w][1], s_m[w][2]});
    const double var = t.n > 0.0 ? t.m2 / t.n : 0.0;
    s_stat[0] = t.mean;
    s_stat[1] = 1.0 / sqrt(var + static_cast<double>(p.eps));
  }
  __syncthreads();
  const double mean = s_stat[0], rstd = s_stat[1];
  for (int c = c_begin + tid; c < c_begin + cpg; c += kFinThreads) {
    const double gam = p.gamma != nullptr ? static_cast<double>(p.gamma[c]) : 1.0;
    const double bet = p.beta != nullptr ? static_cast<double>(p.beta[c]) : 0.0;
    const double scale = gam * rstd;
    float* a = p.affine + (static_cast<long long>(b) * ctot + c) * 2;
    a[0] = static_cast<float>(scale);
    a[1] = static_cast<float>(bet - mean * scale);
  }
}

}  // namespace

int gn_max_chunks(int batch) { return (2 * 296 + batch - 1) / batch; }

// About 32 KB of input per block (small tensors still spread over many SMs), at
// least 16 voxels, at most one resident wave of blocks over all batch items (a
// second, partial wave measured slower than fewer, longer blocks).
int gn_chunks_for(int batch, long long voxels, int channels) {
  static const int wave = [] {
    const int sms = device_sm_count();
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gn_partial_kernel<false>, kGnThreads, 1024) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    return sms * per_sm;
  }();
  long long chunks = (voxels * channels * 4 + (32 << 10) - 1) / (32 << 10);
  if (chunks > gn_max_chunks(batch)) chunks = gn_max_chunks(batch);
  if (chunks > wave / batch) chunks = wave / batch;
  if (chunks > (voxels + 15) / 16) chunks = (voxels + 15) / 16;
  if (chunks < 1) chunks = 1;
  return static_cast<int>(chunks);
}

namespace {
// Whether pass 1 can stream the sources through the shared-memory ring: dense fp32 rows whose
// channel counts (and the concat boundary) are multiples of 8, 16-byte aligned.
bool gn_bulk_ok(const GnParams& p) {
  for (int i = 0; i < 2; ++i) {
    const PrepSource& q = p.src[i];
    if (q.channels == 0) continue;
    if (q.bf16 || q.cstride != q.channels || q.channels % 8 || (reinterpret_cast<uintptr_t>(q.ptr) & 15)) return false;
  }
  return p.src[0].channels > 0;
}

// Pass 1 over all chunks: the bulk-staged kernel where it applies (its dynamic shared memory is the
// channel moments, then the ring), the per-thread-load kernel otherwise.
cudaError_t launch_gn_partial(const GnParams& p, cudaStream_t stream) {
  const int ctot = p.src[0].channels + p.src[1].channels;
  const size_t chan_smem = static_cast<size_t>(ctot) * 3 * sizeof(float);
  const bool bulk = gn_bulk_ok(p);
  const int seg = bulk ? std::max(1, kGnSegBytes / (ctot * 4)) : 0;
  const size_t smem = bulk ? ((chan_smem + 15) & ~static_cast<size_t>(15)) +
                                 static_cast<size_t>(kGnStages) * seg * ctot * sizeof(float)
                           : chan_smem;
  auto kern = bulk ? gn_partial_kernel<true> : gn_partial_kernel<false>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  if (bulk) {  // two ring-holding blocks per SM need the whole unified L1 as shared memory
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
  }
  launch_kernel(kern, dim3(p.chunks, p.batch), dim3(kGnThreads), smem, stream, p);
  return cudaGetLastError();
}
}  // namespace

// The vector width of the one-launch small-tensor kernel for these sources (4: dense 16-byte
// aligned fp32 rows and channel counts that are multiples of 4, else 1).
static int gn_direct_width(const GnParams& p, int cpg) {
  if (cpg % 4 != 0) return 1;
  for (int i = 0; i < 2; ++i) {
    const PrepSource& s = p.src[i];
    if (s.channels == 0) continue;
    if (s.bf16 || s.channels % 4 != 0 || s.cstride % 4 != 0 || (reinterpret_cast<uintptr_t>(s.ptr) & 15)) return 1;
  }
  return 4;
}

// Whether the one-launch small-tensor kernel takes a GroupNorm of this size, with loads of `width`
// channels (CTMR_DISABLE_GN_DIRECT=1: never).
static bool gn_direct_fits_width(long long voxels, int channels, int groups, int width) {
  if (std::getenv("CTMR_DISABLE_GN_DIRECT") != nullptr || groups <= 0 || channels % groups != 0) return false;
  const int cpg = channels / groups;
  if (cpg < 1 || cpg > 64 || cpg % width != 0) return false;
  const long long slots = cpg / width, lanes = kGnDirectThreads / slots;
  return (voxels + lanes - 1) / lanes <= kGnDirectInFlight;
}

bool gn_direct_fits(long long voxels, int channels, int groups) {
  return gn_direct_fits_width(voxels, channels, groups, channels / (groups > 0 ? groups : 1) % 4 == 0 ? 4 : 1);
}

cudaError_t launch_group_norm_affine(const GnParams& p, cudaStream_t stream) {
  const int ctot = p.src[0].channels + p.src[1].channels;
  if (p.groups > 0 && ctot % p.groups == 0) {
    const int width = gn_direct_width(p, ctot / p.groups);
    if (gn_direct_fits_width(p.voxels, ctot, p.groups, width)) {
      if (width == 4) launch_kernel(gn_direct_kernel<4>, dim3(p.groups, p.batch), dim3(kGnDirectThreads), 0, stream, p);
      else launch_kernel(gn_direct_kernel<1>, dim3(p.groups, p.batch), dim3(kGnDirectThreads), 0, stream, p);
      return cudaGetLastError();
    }
  }
  cudaError_t e = launch_gn_partial(p, stream);
  if (e != cudaSuccess) return e;
  if (p.chunks > kFinThreads * kFinPerThread) return cudaErrorInvalidValue;
  launch_kernel(gn_finalize_kernel, dim3(p.groups, p.batch), dim3(kFinThreads), 0, stream, p);
  return cudaGetLastError();
}

}  // namespace ctmr

namespace ctmr {

cudaError_t launch_group_norm_from_stats(const GnStatsParams& p, cudaStream_t stream) {
  return launch_kernel(gn_from_stats_kernel, dim3(p.groups, p.batch), dim3(kFinThreads), 0, stream, p);
}

cudaError_t launch_group_norm_moments(const GnParams& p, float* moments, cudaStream_t stream) {
  if (p.chunks > kFinThreads * kFinPerThread) return cudaErrorInvalidValue;
  cudaError_t e = launch_gn_partial(p, stream);
  if (e != cudaSuccess) return e;
  launch_kernel(gn_moments_kernel, dim3(p.groups, p.batch), dim3(kFinThreads), 0, stream, p, moments);
  return cudaGetLastError();
}

cudaError_t launch_group_norm_from_moments(const GnMomentsParams& p, cudaStream_t stream) {
  return launch_kernel(gn_affine_from_moments_kernel, dim3(p.groups, p.batch), dim3(kFinThreads), 0, stream, p);
}

}  // namespace ctmr
