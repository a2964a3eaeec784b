// Persistent implicit-GEMM conv3d for the 16-bit operand modes that reuses
// each input box across the taps along w.
//
// The M tile is 8 (h) x 16 (w) output voxels of one depth, ordered so that each
// 8-row core group of the K-major swizzled operand (one swizzle atom: 8 rows x
// KC channels) is one w position holding 8 consecutive h. A tap shift along w
// is then a whole-atom shift of the operand start address, so one TMA box of
// (16 + TW - 1) atoms — the input rows for all TW taps along w — feeds TW MMAs
// through descriptor offsets. The TMA view of the activations puts H before W
// (dims C, H, W, D, B) so the box lands in exactly this atom order, and
// out-of-range coordinates are zero-filled (the convolution's padding).
//
// Each CTA owns MT M tiles at consecutive depths that share every weight box,
// and walks its tiles persistently: the accumulator (MT x bn fp32 columns) is
// double-buffered in TMEM so the epilogue warps drain tile i while the MMA
// issuer accumulates tile i + 1.
//
// EXACT (the fp32 mode, one depth per tile): every operand is carried as fp16 hi + lo planes
// (hi = half(v), lo = half((v - hi) * 2^11)) and each K step issues hi*hi into a chunk buffer and
// hi*lo + lo*hi into the tile's lo accumulator. The hi*hi products accumulate in chunks of at most
// 512 K terms (whole stages), alternating between two TMEM buffers that the epilogue promotes into
// fp32 registers as they complete; the lo accumulator is double-buffered across tiles. TMEM:
// [hi0 | hi1 | lo0 | lo1], bn columns each. The same split-precision scheme as the per-tap kernel
// (Ootomo & Yokota 2022), with the kw reuse of the input box.
//
// Modes: kModeConv3 (TW = 3; stages over (kd, kh)), kModeUp2 (TW = 2; stages
// over the (td, th) of each nearest-2x parity, whose taps are the folded
// weights of pack_weight(upsample=1)) and kModeConv1 (TW = 1: the 1x1x1
// convolution, one box per channel block; the kernel is then a persistent
// streaming GEMM).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv3d_umma.cuh"
#include "epilogue.cuh"
#include "ptx.cuh"
#include "launch.cuh"

namespace ctmr {
namespace {

constexpr int kThreadsV2 = 192;

__host__ __device__ constexpr uint32_t ru(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Stage: A (hi) | A lo | B (hi) | B lo; the lo planes only in EXACT.
struct V2Layout {
  uint32_t atom_bytes, a_m_bytes, a_bytes, b_tap_bytes, b_bytes, b_off, stage_bytes;
  __host__ __device__ V2Layout(int kc, int mt, int tw, int bn, bool exact = false) {
    atom_bytes = 8u * static_cast<uint32_t>(kc) * 2u;
    a_m_bytes = static_cast<uint32_t>(16 + tw - 1) * atom_bytes;
    a_bytes = ru(static_cast<uint32_t>(mt) * a_m_bytes, 1024);
    b_tap_bytes = static_cast<uint32_t>(bn) * kc * 2u;
    b_bytes = ru(static_cast<uint32_t>(tw) * b_tap_bytes, 1024);
    b_off = a_bytes * (exact ? 2u : 1u);
    stage_bytes = (a_bytes + b_bytes) * (exact ? 2u : 1u);
  }
};

// EXACT: whole stages per hi*hi promotion chunk (at most 512 K terms, at least one stage).
__host__ __device__ constexpr int v2_chunk_stages(int kc, int tw) { return 512 / (tw * kc) > 0 ? 512 / (tw * kc) : 1; }

template <int KC, int MT, int TW, bool STATS, bool TF32, bool EXACT>
__global__ void __launch_bounds__(kThreadsV2, 1)
    conv3d_umma_v2_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvGeom g) {
  static_assert(!EXACT || (MT == 1 && !STATS && !TF32), "the split mode: one depth per tile, fp16 planes");
  constexpr int CH = v2_chunk_stages(KC, TW);
  constexpr uint32_t kRowBytes = KC * 2;
  constexpr int kSteps = KC / 16;
  constexpr int KDH = TW == 3 ? 9 : (TW == 2 ? 4 : 1);  // (kd, kh) or (td, th) pairs per tile (1x1: one)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(ru(smem_u32(smem_raw), 1024) - smem_u32(smem_raw) +
                                             reinterpret_cast<uintptr_t>(smem_raw));
  const V2Layout L(KC, MT, TW, g.bn, EXACT);
  const int S = g.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * L.stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* tmem_full = empty + S;      // [2] (EXACT: the tile's lo accumulator)
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint64_t* chunk_full = tmem_empty + 2;   // [2] EXACT: a hi*hi chunk is complete
  uint64_t* chunk_empty = chunk_full + 2;  // [2] EXACT: the epilogue has promoted that chunk buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(chunk_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Output statistics: one accumulator per epilogue warp, [4][batch][cout][3].
  float* s_stats = reinterpret_cast<float*>(smem + static_cast<size_t>(S) * L.stage_bytes + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages_per_tile = KDH * g.kblocks;
  const uint32_t bn = static_cast<uint32_t>(g.bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 128);
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

  // Tile t -> (n tile fastest, then w, h, d, batch item, parity phase).
  auto decode = [&](int t, int& n0, int& w0, int& h0, int& d0, int& b, int& phase) {
    const int nt = t % g.n_tiles; t /= g.n_tiles;
    const int tw_i = t % g.tiles_w; t /= g.tiles_w;
    const int th_i = t % g.tiles_h; t /= g.tiles_h;
    const int td_i = t % g.tiles_d; t /= g.tiles_d;
    b = t % g.batch;
    phase = t / g.batch;
    n0 = nt * g.bn;
    w0 = tw_i * 16;
    h0 = th_i * 8;
    d0 = td_i * MT;
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    tma_prefetch_desc(&maps.a[0]);
    tma_prefetch_desc(&maps.b);
    if (EXACT) {
      tma_prefetch_desc(&maps.a_lo[0]);
      tma_prefetch_desc(&maps.b_lo);
    }
    int it = 0;
    int issued = 0;
    for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x) {
      int n0, w0, h0, d0, b, phase;
      decode(t, n0, w0, h0, d0, b, phase);
      const int pd = phase >> 2, ph = (phase >> 1) & 1, pw = phase & 1;
      for (int st = 0; st < stages_per_tile; ++st, ++it) {
        const int s = it % S;
        const uint32_t round = static_cast<uint32_t>(it / S);
        if (it >= S && !mbar_wait_bounded(&empty[s], (round - 1) & 1u, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        const int kdh = st / g.kblocks;
        const int c = (st - kdh * g.kblocks) * KC;
        int y, x, z, btap;
        if (TW == 3) {
          const int kd = kdh / 3, kh = kdh % 3;
          z = d0 + kd - 1;
          y = h0 + kh - 1;
          x = w0 - 1;
          btap = kd * 9 + kh * 3;
        } else if (TW == 1) {
          z = d0;
          y = h0;
          x = w0;
          btap = 0;
        } else {
          const int td = kdh >> 1, th = kdh & 1;
          z = d0 + pd + td - 1;
          y = h0 + ph + th - 1;
          x = w0 + pw - 1;
          btap = phase * 8 + td * 4 + th * 2;
        }
        uint8_t* st_base = smem + static_cast<size_t>(s) * L.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (static_cast<uint32_t>(MT) * L.a_m_bytes + static_cast<uint32_t>(TW) *
                                                                                     L.b_tap_bytes) *
                                            (EXACT ? 2u : 1u));
        tma_load_5d(st_base, &maps.a[0], &full[s], c, y, x, z, b);
        if (EXACT) tma_load_5d(st_base + L.a_bytes, &maps.a_lo[0], &full[s], c, y, x, z, b);
        tma_load_3d(st_base + L.b_off, &maps.b, &full[s], c, n0, btap);
        if (EXACT) tma_load_3d(st_base + L.b_off + L.b_bytes, &maps.b_lo, &full[s], c, n0, btap);
        ++issued;
      }
    }
    for (int k = max(0, issued - S); k < issued; ++k) {
      if (!mbar_wait_bounded(&full[k % S], static_cast<uint32_t>(k / S) & 1u, kErrWaitDrain)) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(!EXACT && g.operand_bf16 != 0, 128, bn, TF32);
    int it = 0;
    int lt = 0;
    if (EXACT) {
      int chunk = 0;  // hi*hi chunks over all of this CTA's tiles
      for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x, ++lt) {
        const int lbuf = lt & 1;
        if (lt >= 2 &&
            !mbar_wait_bounded(&tmem_empty[lbuf], static_cast<uint32_t>((lt >> 1) - 1) & 1u, kErrWaitAcc)) {
          *abort_flag = 1;
          break;
        }
        const uint32_t acc_lo = tmem + static_cast<uint32_t>(2 + lbuf) * bn;
        bool stop = false;
        for (int st = 0; st < stages_per_tile; ++st, ++it) {
          const int cs = st % CH;  // stage within the chunk
          const int cbuf = chunk & 1;
          if (cs == 0 && chunk >= 2 &&
              !mbar_wait_bounded(&chunk_empty[cbuf], static_cast<uint32_t>((chunk >> 1) - 1) & 1u, kErrWaitAcc)) {
            stop = true;
            break;
          }
          const int s = it % S;
          if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(it / S) & 1u, kErrWaitFull)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * L.stage_bytes);
          const uint64_t a_hi0 = smem_desc_kmajor(a_base, kRowBytes);
          const uint64_t a_lo0 = desc_advance(a_hi0, L.a_bytes);
          const uint64_t b_hi0 = desc_advance(a_hi0, L.b_off);
          const uint64_t b_lo0 = desc_advance(b_hi0, L.b_bytes);
          const uint32_t acc_hi = tmem + static_cast<uint32_t>(cbuf) * bn;
#pragma unroll
          for (int kw = 0; kw < TW; ++kw) {
            const uint32_t ao = static_cast<uint32_t>(kw) * L.atom_bytes, bo = static_cast<uint32_t>(kw) * L.b_tap_bytes;
            const uint64_t a_hi = desc_advance(a_hi0, ao), a_lo = desc_advance(a_lo0, ao);
            const uint64_t b_hi = desc_advance(b_hi0, bo), b_lo = desc_advance(b_lo0, bo);
#pragma unroll
            for (int k = 0; k < kSteps; ++k) {
              const uint32_t kd = 2u * static_cast<uint32_t>(k);
              umma_f16(acc_hi, a_hi + kd, b_hi + kd, idesc, (cs == 0 && kw == 0 && k == 0) ? 0u : 1u);
              umma_f16(acc_lo, a_hi + kd, b_lo + kd, idesc, (st == 0 && kw == 0 && k == 0) ? 0u : 1u);
              umma_f16(acc_lo, a_lo + kd, b_hi + kd, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
          if (cs == CH - 1 || st == stages_per_tile - 1) {  // a chunk ends with the tile at the latest
            umma_commit(&chunk_full[cbuf]);
            ++chunk;
          }
        }
        if (stop) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&tmem_full[lbuf]);
      }
    } else {
    for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (lt >= 2 &&
          !mbar_wait_bounded(&tmem_empty[buf], static_cast<uint32_t>((lt >> 1) - 1) & 1u, kErrWaitAcc)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t acc0 = tmem + static_cast<uint32_t>(buf * MT) * bn;
      for (int st = 0; st < stages_per_tile; ++st, ++it) {
        const int s = it % S;
        if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(it / S) & 1u, kErrWaitFull)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * L.stage_bytes);
        const uint64_t a_desc0 = smem_desc_kmajor(a_base, kRowBytes);
        const uint64_t b_desc0 = smem_desc_kmajor(a_base + L.a_bytes, kRowBytes);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
#pragma unroll
          for (int kw = 0; kw < TW; ++kw) {
            const uint64_t a_desc = desc_advance(a_desc0, static_cast<uint32_t>(m) * L.a_m_bytes +
                                                              static_cast<uint32_t>(kw) * L.atom_bytes);
            const uint64_t b_desc = desc_advance(b_desc0, static_cast<uint32_t>(kw) * L.b_tap_bytes);
#pragma unroll
            for (int k = 0; k < kSteps; ++k) {  // 32 bytes of K per MMA: +2 in the descriptors' address field
              umma<TF32>(acc0 + static_cast<uint32_t>(m) * bn, a_desc + 2u * k, b_desc + 2u * k, idesc,
                         (st == 0 && kw == 0 && k == 0) ? 0u : 1u);
            }
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&tmem_full[buf]);
    }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int aw = row >> 3, ih = row & 7;  // atom (w offset), row in atom (h offset)
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // Each tile is drained in blocks of (M tile m, 64 columns); the residual of
    // block k + 1 is loaded while block k is finished, and block 0's before the
    // accumulator wait, so the residual reads overlap instead of serialising.
    const int halves = (g.bn + 63) >> 6;
    const int nblk = MT * halves;
    int n0 = 0, w0 = 0, h0 = 0, d0 = 0, b = 0, phase = 0;
    auto row_of = [&](int m, bool& valid, long long& out_base, long long& res_base) {
      const int rd = d0 + m, rh = h0 + ih, rw = w0 + aw;
      valid = rw < g.row_w && rh < g.row_h && rd < g.row_d;
      int od = rd, oh = rh, ow = rw;
      if (TW == 2) {
        od = 2 * rd + (phase >> 2);
        oh = 2 * rh + ((phase >> 1) & 1);
        ow = 2 * rw + (phase & 1);
      }
      const long long vox = ((static_cast<long long>(b) * g.out_d + od) * g.out_h + oh) * g.out_w + ow;
      out_base = vox * g.out_cstride + g.out_coff;
      res_base = 0;
      if (g.res != nullptr) {
        const int qd = g.res_up ? od >> 1 : od, qh = g.res_up ? oh >> 1 : oh, qw = g.res_up ? ow >> 1 : ow;
        res_base = (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride;
      }
    };
    if (EXACT) {
      // Promote each hi*hi chunk into fp32 registers as it completes, then fold in the tile's lo
      // accumulator at 2^-11, add bias and residual, and store (the per-tap kernel's epilogue order).
      const int nch = (stages_per_tile + CH - 1) / CH;
      int chunk = 0;
      int et = 0;
      for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x, ++et) {
        const int lbuf = et & 1;
        decode(t, n0, w0, h0, d0, b, phase);
        bool ok = true;
        float sum[128];
#pragma unroll
        for (int i = 0; i < 128; ++i) sum[i] = 0.f;
        for (int c = 0; c < nch && ok; ++c, ++chunk) {
          const int cbuf = chunk & 1;
          ok = __all_sync(0xffffffffu,
                          mbar_wait_bounded(&chunk_full[cbuf], static_cast<uint32_t>(chunk >> 1) & 1u, kErrWaitAcc));
          tc_fence_after();
#pragma unroll
          for (int cb = 0; cb < 8; ++cb) {
            if (cb * 16 < g.bn) {
              float v[16];
              tmem_ld16(lane_addr + static_cast<uint32_t>(cbuf * g.bn + cb * 16), v);
#pragma unroll
              for (int i = 0; i < 16; ++i) sum[cb * 16 + i] += v[i];
            }
          }
          tc_fence_before();
          mbar_arrive(&chunk_empty[cbuf]);
        }
        ok = ok && __all_sync(0xffffffffu, mbar_wait_bounded(&tmem_full[lbuf], static_cast<uint32_t>(et >> 1) & 1u,
                                                             kErrWaitAcc));
        tc_fence_after();
        bool valid;
        long long out_base, res_base;
        row_of(0, valid, out_base, res_base);
        valid = valid && ok;
        const float* bias = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
#pragma unroll
        for (int cb = 0; cb < 8; ++cb) {
          const int c = cb * 16;
          if (c < g.bn) {
            float l[16], v[16];
            tmem_ld16(lane_addr + static_cast<uint32_t>((2 + lbuf) * g.bn + c), l);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = fmaf(l[i], g.lo_scale, sum[c + i]);
            const int n = n0 + c;
            if (valid && n < g.cout) {
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
        tc_fence_before();
        mbar_arrive(&tmem_empty[lbuf]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
    auto issue = [&](int k, uint32_t(&w)[64]) {
      if (g.res == nullptr) return;
      const int m = k / halves, c0 = (k - m * halves) * 64;
      bool valid;
      long long out_base, res_base;
      row_of(m, valid, out_base, res_base);
      if (valid) res_issue64(g, n0 + c0, res_base + n0 + c0, w);
    };
    int lt = 0;
    auto finish = [&](int k, const uint32_t(&w)[64]) {
      const int m = k / halves, c0 = (k - m * halves) * 64;
      bool valid;
      long long out_base, res_base;
      row_of(m, valid, out_base, res_base);
      const float* bias = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
      const uint32_t acc = lane_addr + static_cast<uint32_t>((lt & 1) * MT + m) * bn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + 16 * j;
        if (c >= g.bn) break;
        float v[16];
        tmem_ld16(acc + static_cast<uint32_t>(c), v);  // warp-collective: every lane loads
        const int n = n0 + c;
        if (valid && n < g.cout) {
          const int cnt = min(16, g.cout - n);
          if (bias != nullptr) {
            if (cnt == 16 && (reinterpret_cast<uintptr_t>(bias + n) & 15) == 0) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 q = __ldg(reinterpret_cast<const float4*>(bias + n) + i);
                v[4 * i] += q.x;
                v[4 * i + 1] += q.y;
                v[4 * i + 2] += q.z;
                v[4 * i + 3] += q.w;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (i < cnt) v[i] += __ldg(bias + n + i);
            }
          }
          if (g.res != nullptr) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += res_word(g, w, 16 * j + i);
          }
          store16(g, v, n, out_base + n);
        }
        if (STATS && n < g.cout)
          warp_stats16(v, valid, min(16, g.cout - n),
                       s_stats + ((static_cast<size_t>(warp - 2) * g.batch + b) * g.cout + n) * 3);
      }
    };
    if (STATS) {
      float* mine = s_stats + static_cast<size_t>(warp - 2) * g.batch * g.cout * 3;
      for (int e = lane; e < g.batch * g.cout * 3; e += 32) mine[e] = 0.f;
      __syncwarp();
    }
    for (int t = blockIdx.x; !EXACT && t < g.total_tiles && !*abort_flag; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      decode(t, n0, w0, h0, d0, b, phase);
      uint32_t ra[64], rb[64];
      issue(0, ra);
      if (!mbar_wait_bounded(&tmem_full[buf], static_cast<uint32_t>(lt >> 1) & 1u, kErrWaitAcc)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int k = 0; k < nblk; k += 2) {
        if (k + 1 < nblk) issue(k + 1, rb);
        finish(k, ra);
        if (k + 1 < nblk) {
          if (k + 2 < nblk) issue(k + 2, ra);
          finish(k + 1, rb);
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[buf]);
    }
    if (STATS) {
      // Every epilogue warp reaches this point (finished or aborted): merge the
      // four warps' moments in order and write this CTA's slot.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int et = threadIdx.x - 64;
      const int bc = g.batch * g.cout;
      for (int e = et; e < bc; e += 128) {
        float m[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          const float* a = s_stats + (static_cast<size_t>(wq) * bc + e) * 3;
          chan_merge(m, a[0], a[1], a[2]);
        }
        const int bb = e / g.cout, c = e - bb * g.cout;
        float* dst = g.stats + ((static_cast<size_t>(bb) * g.stats_slots + blockIdx.x) * g.cout + c) * 3;
        dst[0] = m[0];
        dst[1] = m[1];
        dst[2] = m[2];
      }
      if (blockIdx.x == 0) {  // slots past the grid hold nothing
        const int extra = g.stats_slots - static_cast<int>(gridDim.x);
        for (int e = et; e < g.batch * extra * g.cout; e += 128) {
          const int bb = e / (extra * g.cout), r = e - bb * extra * g.cout;
          float* dst = g.stats + (static_cast<size_t>(bb) * g.stats_slots * g.cout + gridDim.x * g.cout + r) * 3;
          dst[0] = 0.f;
          dst[1] = 0.f;
          dst[2] = 0.f;
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

template <int KC, int MT, int TW>
cudaError_t launch_v2_typed(const ConvMaps& maps, const ConvGeom& g, int grid, size_t smem, bool exact,
                            cudaStream_t stream) {
  // The statistics epilogue is a separate instantiation so the plain kernel keeps its registers;
  // TF32 operands are a third (the planner gives them no statistics), the fp32 split mode a fourth.
  if (g.operand_tf32 && g.stats != nullptr) return cudaErrorInvalidValue;
  if (exact && (MT != 1 || g.stats != nullptr || g.operand_tf32)) return cudaErrorInvalidValue;
  auto kern = exact ? conv3d_umma_v2_kernel<KC, MT, TW, false, false, MT == 1>
                    : g.operand_tf32 ? conv3d_umma_v2_kernel<KC, MT, TW, false, true, false>
                                     : (g.stats != nullptr ? conv3d_umma_v2_kernel<KC, MT, TW, true, false, false>
                                                           : conv3d_umma_v2_kernel<KC, MT, TW, false, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, grid, kThreadsV2, smem, stream, maps, g);
}

}  // namespace

// Shared-memory plan of the v2 kernel: the deepest pipeline (<= 6 stages) that
// fits one CTA per SM; 0 when fewer than 2 stages fit.
int conv_v2_stage_plan(int kc, int mt, int tw, int bn, size_t* smem_bytes, size_t stats_bytes, bool exact) {
  const V2Layout L(kc, mt, tw, bn, exact);
  const size_t extra = 1024 + 256 + stats_bytes;
  int stages = static_cast<int>((227 * 1024 - extra) / L.stage_bytes);
  if (stages > 6) stages = 6;
  if (stages < 2) return 0;
  *smem_bytes = static_cast<size_t>(stages) * L.stage_bytes + extra;
  return stages;
}

cudaError_t launch_conv3d_umma_v2(const ConvMaps& maps, const ConvGeom& g, int kc, int mt, int tw, int sms,
                                  size_t smem, bool exact, cudaStream_t stream) {
  if (g.total_tiles <= 0) return cudaErrorInvalidValue;
  const int grid = g.total_tiles < sms ? g.total_tiles : sms;
#define CTMR_V2(KC_, MT_, TW_) \
  if (kc == KC_ && mt == MT_ && tw == TW_) return launch_v2_typed<KC_, MT_, TW_>(maps, g, grid, smem, exact, stream);
  CTMR_V2(64, 2, 3) CTMR_V2(32, 2, 3) CTMR_V2(16, 2, 3)
  CTMR_V2(64, 1, 3) CTMR_V2(32, 1, 3) CTMR_V2(16, 1, 3)
  CTMR_V2(64, 2, 2) CTMR_V2(32, 2, 2) CTMR_V2(16, 2, 2)
  CTMR_V2(64, 1, 2) CTMR_V2(32, 1, 2) CTMR_V2(16, 1, 2)
  CTMR_V2(64, 2, 1) CTMR_V2(32, 2, 1) CTMR_V2(16, 2, 1)
  CTMR_V2(64, 1, 1) CTMR_V2(32, 1, 1) CTMR_V2(16, 1, 1)
#undef CTMR_V2
  return cudaErrorInvalidValue;
}

}  // namespace ctmr
