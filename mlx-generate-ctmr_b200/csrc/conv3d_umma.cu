// Implicit-GEMM 3-D convolution on the sm_100a tensor cores (tcgen05 + TMEM),
// fed by TMA tiled loads. Activations are channels-last (NDHWC).
//
// GEMM view (the reference computes the same contraction, `_nax_conv.py:200-317`):
//   rows    M = output voxels, one 128-voxel box (tile_w x tile_h x tile_d) per CTA
//   columns N = output channels, one N tile of `bn` per CTA
//   depth   K = taps x padded input channels, walked tap-major in KC-channel blocks
// For each (tap, channel block) one TMA load brings the input box shifted by the
// tap offset; coordinates that fall outside the volume are zero-filled by the
// TMA unit, which is exactly the convolution's zero padding, so no padded copy
// and no im2col buffer exist. Weights are packed [tap][Cout_pad][Cin_pad]
// (K-major) and loaded as a bn x KC box.
//
// Warp roles (192 threads): warp 0 lane 0 issues TMA loads, warp 1 owns TMEM
// and lane 0 issues tcgen05.mma, warps 2-5 drain the accumulator: TMEM ->
// registers -> +bias (per channel or per batch item) -> +residual -> store.
//
// Precision modes:
//   bf16/fp16: bf16 x bf16 or fp16 x fp16 products, fp32 accumulation, one rounding at the store.
//   fp32 (EXACT): every fp32 operand v is carried as fp16 hi = half(v) and
//             lo = half((v - hi) * 2^11); three MMAs per K step accumulate
//             hi*hi into one TMEM accumulator and hi*lo + lo*hi into a second,
//             which the epilogue folds in at 2^-11 before any addition. This is
//             the split-precision scheme of Ootomo & Yokota (2022, "Recovering
//             single precision accuracy from Tensor Cores while surpassing the
//             FP32 theoretical peak performance"), the same operand split the
//             reference uses (`_nax_conv.py:27-35`): ~2^-22 relative product error.
#include "conv3d_umma.cuh"
#include "epilogue.cuh"
#include "ptx.cuh"
#include "launch.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace ctmr {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr int kThreads = 192;
constexpr int kRows = 128;

__host__ __device__ constexpr uint32_t round_up_u32(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// EXACT with at most 64 output columns per tile ("paired"): hi*hi and hi*lo come from one N = 2 bn
// MMA whose B is the weight blocks [hi; lo] (or [lo; hi]) stacked along N, with its D the hi chunk
// buffer and the lo accumulator side by side in TMEM; lo*hi is a second MMA. Two MMAs per K step
// instead of three, where an N <= 64 MMA costs about as much as an N = 128 one. The stacked blocks
// must be contiguous whole swizzle atoms: bn * kc * 2 bytes a multiple of 1024.
__host__ __device__ constexpr bool exact_pair(int kc, int bn, bool exact) {
  return exact && bn <= 64 && (bn * kc * 2) % 1024 == 0;
}

struct StageLayout {
  uint32_t a_bytes, b_bytes, stage_bytes;
  __host__ __device__ StageLayout(int kc, int bn, bool exact) {
    a_bytes = round_up_u32(kRows * kc * 2, 1024);
    b_bytes = round_up_u32(static_cast<uint32_t>(bn) * kc * 2, 1024);
    // Paired: the weight blocks [hi; lo; hi], so that both [hi; lo] and [lo; hi] are contiguous.
    stage_bytes = exact ? 2u * a_bytes + (exact_pair(kc, bn, exact) ? 3u : 2u) * b_bytes : a_bytes + b_bytes;
  }
};

// 16 zero columns into this warp's 32 TMEM lanes (completed by tcgen05.wait::st).
__device__ __forceinline__ void tmem_zero16(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(0u)
      : "memory");
}

template <int KC, bool EXACT, bool TF32, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    conv3d_umma_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvGeom g) {
  static_assert(!PAIR || EXACT, "the paired products are the split mode's");
  constexpr uint32_t kRowBytes = KC * 2;
  constexpr int kSteps = KC / 16;  // K=16 MMAs per channel block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(round_up_u32(smem_u32(smem_raw), 1024) - smem_u32(smem_raw) +
                                             reinterpret_cast<uintptr_t>(smem_raw));
  const StageLayout L(KC, g.bn, EXACT);
  const int S = g.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * L.stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* chunk_full = acc_full + 1;   // [2]: a promotion chunk of the hi accumulator is complete
  uint64_t* chunk_empty = chunk_full + 2;  // [2]: the epilogue has drained that chunk buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(chunk_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Tile coordinates: w fastest, then h, d, batch item, parity phase.
  int t = blockIdx.x;
  const int tw_i = t % g.tiles_w; t /= g.tiles_w;
  const int th_i = t % g.tiles_h; t /= g.tiles_h;
  const int td_i = t % g.tiles_d; t /= g.tiles_d;
  const int b = t % g.batch; t /= g.batch;
  const int phase = t;
  const int w0 = tw_i * g.tile_w, h0 = th_i * g.tile_h, d0 = td_i * g.tile_d;
  const int n0 = blockIdx.y * g.bn;
  // Split-K: this CTA accumulates K iterations [it_begin, it_begin + n_iter) of the tap-major walk.
  const int n_iter_all = g.taps * g.kblocks;
  const int it_begin = static_cast<int>(static_cast<long long>(n_iter_all) * blockIdx.z / g.ksplit);
  const int n_iter = static_cast<int>(static_cast<long long>(n_iter_all) * (blockIdx.z + 1) / g.ksplit) - it_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&chunk_full[i], 1);
      mbar_init(&chunk_empty[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, g.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Barrier and TMEM set-up above overlaps the preceding kernel's tail; global
  // memory (TMA loads, epilogue stores) only from here on. Dependents are
  // released once every CTA holds its TMEM.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    const int nmaps = g.mode == kModeStride2 ? 8 : 1;
    for (int i = 0; i < nmaps; ++i) {
      tma_prefetch_desc(&maps.a[i]);
      if (EXACT) tma_prefetch_desc(&maps.a_lo[i]);
    }
    tma_prefetch_desc(&maps.b);
    if (EXACT) tma_prefetch_desc(&maps.b_lo);
    const int pd = phase >> 2, ph = (phase >> 1) & 1, pw = phase & 1;
    int issued = 0;
    for (int it = 0; it < n_iter; ++it) {
      const int s = it % S;
      const uint32_t round = static_cast<uint32_t>(it / S);
      if (it >= S && !mbar_wait_bounded(&empty[s], (round - 1) & 1u, kErrWaitEmpty)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      const int tap = (it_begin + it) / g.kblocks;
      const int c = (it_begin + it - tap * g.kblocks) * KC;
      int map = 0, x = w0, y = h0, z = d0, btap = tap;
      if (g.mode == kModeConv3) {
        z += tap / 9 - 1;
        y += (tap / 3) % 3 - 1;
        x += tap % 3 - 1;
      } else if (g.mode == kModeUp2) {
        z += pd + (tap >> 2) - 1;
        y += ph + ((tap >> 1) & 1) - 1;
        x += pw + (tap & 1) - 1;
        btap = phase * 8 + tap;
      } else if (g.mode == kModeStride2) {
        // Input index 2o + k - 1: k = 1 is even element o, k = 0 / 2 are odd elements o - 1 / o.
        const int kd = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
        map = (kd != 1) * 4 + (kh != 1) * 2 + (kw != 1);
        z -= (kd == 0);
        y -= (kh == 0);
        x -= (kw == 0);
      }
      uint8_t* st = smem + static_cast<size_t>(s) * L.stage_bytes;
      mbar_arrive_expect_tx(&full[s], (kRows * (EXACT ? 2u : 1u) + static_cast<uint32_t>(g.bn) * (PAIR ? 3u : (EXACT ? 2u : 1u))) *
                                          kRowBytes);
      tma_load_5d(st, &maps.a[map], &full[s], c, x, y, z, b);
      if (EXACT) tma_load_5d(st + L.a_bytes, &maps.a_lo[map], &full[s], c, x, y, z, b);
      uint8_t* bs = st + L.a_bytes * (EXACT ? 2 : 1);
      tma_load_3d(bs, &maps.b, &full[s], c, n0, btap);
      if (EXACT) tma_load_3d(bs + L.b_bytes, &maps.b_lo, &full[s], c, n0, btap);
      if (PAIR) tma_load_3d(bs + 2 * L.b_bytes, &maps.b, &full[s], c, n0, btap);
      ++issued;
    }
    // Drain: the newest load of every stage must land before the CTA can exit.
    for (int k = max(0, issued - S); k < issued; ++k) {
      if (!mbar_wait_bounded(&full[k % S], static_cast<uint32_t>(k / S) & 1u, kErrWaitDrain)) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    // EXACT: the hi*hi products accumulate in chunks of `chunk_iters` iterations,
    // alternating between two TMEM buffers; the epilogue warps add each finished
    // chunk into fp32 registers with round-to-nearest adds while the next chunk
    // accumulates. This bounds how long the tensor core's own fp32 accumulation
    // runs, whose rounding error otherwise grows with K (27 * C_in products).
    static_assert(!(EXACT && TF32), "the split mode has fp16 operands");
    const uint32_t idesc = idesc_f16(!EXACT && g.operand_bf16 != 0, kRows, static_cast<uint32_t>(g.bn), TF32);
    const uint32_t idesc_pair = idesc_f16(false, kRows, 2u * static_cast<uint32_t>(g.bn));
    const uint32_t bn = static_cast<uint32_t>(g.bn);
    // TMEM: [hi0 | hi1 | lo], or paired [hi0 | lo | hi1] (each hi buffer adjacent to lo).
    const uint32_t acc_lo = tmem + (PAIR ? 1u : 2u) * bn;
    const int T = EXACT ? g.chunk_iters : n_iter;
    for (int it = 0; it < n_iter; ++it) {
      const int s = it % S;
      const int chunk = it / T;
      const int buf = chunk & 1;
      const bool chunk_start = it - chunk * T == 0;
      // The hi buffer about to be reused must be drained (paired: and zeroed; the epilogue also zeroes
      // buffer 1 once before its first use, which is that buffer's first completion).
      if (EXACT && chunk_start && (PAIR ? chunk >= 1 : chunk >= 2) &&
          !mbar_wait_bounded(&chunk_empty[buf],
                             static_cast<uint32_t>(PAIR && buf == 1 ? (chunk - 1) >> 1 : (chunk >> 1) - 1) & 1u,
                             kErrWaitAcc)) {
        *abort_flag = 1;
        break;
      }
      if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(it / S) & 1u, kErrWaitFull)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      tc_fence_after();
      const uint32_t st = smem_u32(smem + static_cast<size_t>(s) * L.stage_bytes);
      const uint64_t a_hi = smem_desc_kmajor(st, kRowBytes), a_lo = desc_advance(a_hi, L.a_bytes);
      const uint64_t b_hi = desc_advance(a_hi, L.a_bytes * (EXACT ? 2 : 1)), b_lo = desc_advance(b_hi, L.b_bytes);
      if (PAIR) {
        // Buffer 0: D = [hi0 | lo], B = [hi; lo]; buffer 1: D = [lo | hi1], B = [lo; hi] (the stage's
        // weight blocks are [hi; lo; hi]). The hi buffers restart from the epilogue's zeros, so only
        // the first product overwrites.
        const uint32_t d_pair = tmem + static_cast<uint32_t>(buf) * bn;
        const uint64_t b_pair = buf == 0 ? b_hi : b_lo;
#pragma unroll
        for (int k = 0; k < kSteps; ++k) {
          const uint32_t kd = 2u * static_cast<uint32_t>(k);
          umma_f16(d_pair, a_hi + kd, b_pair + kd, idesc_pair, (it == 0 && k == 0) ? 0u : 1u);
          umma_f16(acc_lo, a_lo + kd, b_hi + kd, idesc, 1u);
        }
      } else {
        const uint32_t acc_hi = tmem + static_cast<uint32_t>(buf) * bn;
#pragma unroll
        for (int k = 0; k < kSteps; ++k) {  // 32 bytes of K per MMA (16 fp16/bf16, 8 tf32): +2 in the address field
          const uint32_t kd = 2u * static_cast<uint32_t>(k);
          umma<TF32>(acc_hi, a_hi + kd, b_hi + kd, idesc, (chunk_start && k == 0) ? 0u : 1u);
          if (EXACT) {
            umma_f16(acc_lo, a_hi + kd, b_lo + kd, idesc, (it == 0 && k == 0) ? 0u : 1u);
            umma_f16(acc_lo, a_lo + kd, b_hi + kd, idesc, 1u);
          }
        }
      }
      umma_commit(&empty[s]);
      if (EXACT && (it - chunk * T == T - 1 || it == n_iter - 1)) umma_commit(&chunk_full[buf]);
    }
    // Signal the epilogue (also on abort, so it unwinds instead of waiting out its own limit).
    umma_commit(acc_full);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // EXACT: promote the hi chunks into fp32 registers as they complete.
    float sum[EXACT ? 128 : 1];
#pragma unroll
    for (int i = 0; i < (EXACT ? 128 : 1); ++i) sum[i] = 0.f;
    bool ok = true;
    if (EXACT) {
      const int T = g.chunk_iters;
      const int nchunks = (n_iter + T - 1) / T;
      // Paired: hi buffer 0 sits at column 0, buffer 1 at 2 bn (lo between them).
      auto hi_col = [&](int buf) { return PAIR ? buf * 2 * g.bn : buf * g.bn; };
      if (PAIR) {
        // Buffer 1's first chunk accumulates onto zeros: clear it, then hand it to the issuer.
#pragma unroll
        for (int cb = 0; cb < 4; ++cb)
          if (cb * 16 < g.bn) tmem_zero16(lane_addr + static_cast<uint32_t>(hi_col(1) + cb * 16));
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(&chunk_empty[1]);
      }
      for (int chunk = 0; chunk < nchunks && ok; ++chunk) {
        const int buf = chunk & 1;
        ok = mbar_wait_bounded(&chunk_full[buf], static_cast<uint32_t>(chunk >> 1) & 1u, kErrWaitAcc);
        tc_fence_after();
#pragma unroll
        for (int cb = 0; cb < 8; ++cb) {
          if (cb * 16 < g.bn) {
            float v[16];
            tmem_ld16(lane_addr + static_cast<uint32_t>(hi_col(buf) + cb * 16), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[(cb * 16 + i) & (EXACT ? 127 : 0)] += v[i];
            if (PAIR) tmem_zero16(lane_addr + static_cast<uint32_t>(hi_col(buf) + cb * 16));
          }
        }
        if (PAIR) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(&chunk_empty[buf]);
      }
    }
    ok = mbar_wait_bounded(acc_full, 0, kErrWaitAcc) && ok;
    tc_fence_after();
    const int ww = row % g.tile_w;
    const int hh = (row / g.tile_w) % g.tile_h;
    const int dd = row / (g.tile_w * g.tile_h);
    const int rw = w0 + ww, rh = h0 + hh, rd = d0 + dd;
    const bool valid = ok && rw < g.row_w && rh < g.row_h && rd < g.row_d;
    int ow = rw, oh = rh, od = rd;
    if (g.mode == kModeUp2) {
      od = 2 * rd + (phase >> 2);
      oh = 2 * rh + ((phase >> 1) & 1);
      ow = 2 * rw + (phase & 1);
    }
    const long long vox = ((static_cast<long long>(b) * g.out_d + od) * g.out_h + oh) * g.out_w + ow;
    const long long out_base = vox * g.out_cstride + g.out_coff;
    long long res_base = 0;
    if (g.res != nullptr) {
      const int qd = g.res_up ? od >> 1 : od, qh = g.res_up ? oh >> 1 : oh, qw = g.res_up ? ow >> 1 : ow;
      res_base = (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride;
    }
    const float* bias = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
#pragma unroll
    for (int cb = 0; cb < 8; ++cb) {
      const int c = cb * 16;
      if (c < g.bn) {
        float v[16];
        if (EXACT) {
          float l[16];
          tmem_ld16(lane_addr + static_cast<uint32_t>((PAIR ? 1 : 2) * g.bn + c), l);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = fmaf(l[i], g.lo_scale, sum[(c + i) & (EXACT ? 127 : 0)]);
        } else {
          tmem_ld16(lane_addr + static_cast<uint32_t>(c), v);
        }
        const int n = n0 + c;
        if (valid && g.ksplit > 1) {
          // Raw fp32 partial sum; bias and residual are added by the reduction.
          float* dst = g.partial + ((((static_cast<long long>(blockIdx.z) * g.batch + b) * g.row_d + rd) * g.row_h + rh) *
                                        g.row_w + rw) * g.part_cstride + n;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else if (valid && n < g.cout) {
          if (bias != nullptr) {
            const int cnt = min(16, g.cout - n);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < cnt) v[i] += __ldg(bias + n + i);
          }
          store_row16(g, v, n, out_base + n, res_base + n);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, g.tmem_cols);
  }
}

// Split-K reduction (the role of the reference's `_REDUCE`, `_nax_conv.py:320-331`):
// sums the fp32 partial planes in split order, adds bias and the residual, and
// rounds once to the output type. One thread per (row voxel, 4 channels).
__global__ void splitk_reduce_kernel(const ConvGeom g) {
  griddep_wait();  // the preceding kernel's writes are visible from here on
  griddep_launch_dependents();
  const int q4 = (g.cout + 3) / 4;
  const long long rows = static_cast<long long>(g.batch) * g.row_d * g.row_h * g.row_w;
  const long long total = rows * q4;
  const long long plane = rows * g.part_cstride;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i % q4) * 4;
    const long long r = i / q4;
    long long t = r;
    const int rw = static_cast<int>(t % g.row_w); t /= g.row_w;
    const int rh = static_cast<int>(t % g.row_h); t /= g.row_h;
    const int rd = static_cast<int>(t % g.row_d);
    const int b = static_cast<int>(t / g.row_d);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = g.partial + r * g.part_cstride + n;
    for (int z = 0; z < g.ksplit; ++z) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(src + z * plane));
      acc.x += q.x;
      acc.y += q.y;
      acc.z += q.z;
      acc.w += q.w;
    }
    float v[16] = {acc.x, acc.y, acc.z, acc.w};
    const int cnt = min(4, g.cout - n);
    if (g.bias != nullptr) {
      const float* bias = g.bias + static_cast<long long>(b) * g.bias_bstride;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k < cnt) v[k] += __ldg(bias + n + k);
    }
    const long long vox = ((static_cast<long long>(b) * g.out_d + rd) * g.out_h + rh) * g.out_w + rw;
    long long res_base = 0;
    if (g.res != nullptr) {
      const int qd = g.res_up ? rd >> 1 : rd, qh = g.res_up ? rh >> 1 : rh, qw = g.res_up ? rw >> 1 : rw;
      res_base = (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride;
    }
    ConvGeom g4 = g;
    g4.cout = n + cnt;  // store_row16 writes min(16, cout - n) columns
    store_row16(g4, v, n, vox * g.out_cstride + g.out_coff + n, res_base + n);
  }
}

}  // namespace

// ---------------------------------------------------------------- host side

template <int KC, bool EXACT>
static cudaError_t launch_typed(const ConvMaps& maps, const ConvGeom& g, dim3 grid, size_t smem,
                                cudaStream_t stream) {
  auto kern = EXACT ? (exact_pair(KC, g.bn, true) ? conv3d_umma_kernel<KC, EXACT, false, EXACT>
                                                   : conv3d_umma_kernel<KC, EXACT, false, false>)
                    : (g.operand_tf32 ? conv3d_umma_kernel<KC, EXACT, !EXACT, false>
                                      : conv3d_umma_kernel<KC, EXACT, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  launch_kernel(kern, grid, kThreads, smem, stream, maps, g);
  return cudaGetLastError();
}

// Chooses the pipeline depth for the smem budget: two CTAs per SM when at least
// three stages fit in half the SM's shared memory, otherwise one deeper CTA.
int conv_stage_plan(int kc, int bn, bool exact, bool one_cta_per_sm, size_t* smem_bytes) {
  const StageLayout L(kc, bn, exact);
  const size_t extra = 1024 /*align*/ + 256 /*barriers*/;
  const size_t half_budget = 113 * 1024;
  const size_t full_budget = 227 * 1024;
  int stages = one_cta_per_sm ? 0 : static_cast<int>((half_budget - extra) / L.stage_bytes);
  if (stages < 3) stages = static_cast<int>((full_budget - extra) / L.stage_bytes);
  if (stages > 8) stages = 8;
  if (stages < 2) return 0;
  *smem_bytes = static_cast<size_t>(stages) * L.stage_bytes + extra;
  return stages;
}

cudaError_t launch_conv3d_umma(const ConvMaps& maps, const ConvGeom& g, int kc, bool exact, size_t smem,
                               cudaStream_t stream) {
  const int n_tiles = (g.cout + g.bn - 1) / g.bn;
  const long long m_tiles = static_cast<long long>(g.tiles_w) * g.tiles_h * g.tiles_d * g.batch * g.phases;
  if (m_tiles <= 0 || m_tiles > 0x7FFFFFFFLL || n_tiles <= 0 || n_tiles > 65535) return cudaErrorInvalidValue;
  if (g.ksplit < 1 || g.ksplit > 65535 || (g.ksplit > 1 && (g.partial == nullptr || g.mode == kModeUp2)))
    return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(m_tiles), static_cast<unsigned>(n_tiles), static_cast<unsigned>(g.ksplit));
  cudaError_t e = cudaErrorInvalidValue;
  if (kc == 64) e = exact ? launch_typed<64, true>(maps, g, grid, smem, stream)
                          : launch_typed<64, false>(maps, g, grid, smem, stream);
  else if (kc == 32) e = exact ? launch_typed<32, true>(maps, g, grid, smem, stream)
                               : launch_typed<32, false>(maps, g, grid, smem, stream);
  else if (kc == 16) e = exact ? launch_typed<16, true>(maps, g, grid, smem, stream)
                               : launch_typed<16, false>(maps, g, grid, smem, stream);
  if (e != cudaSuccess || g.ksplit == 1) return e;
  const long long total = static_cast<long long>(g.batch) * g.row_d * g.row_h * g.row_w * ((g.cout + 3) / 4);
  long long blocks = (total + 255) / 256;
  if (blocks > 16LL * device_sm_count()) blocks = 16LL * device_sm_count();
  launch_kernel(splitk_reduce_kernel, static_cast<unsigned>(blocks), 256, 0, stream, g);
  return cudaGetLastError();
}

}  // namespace ctmr
