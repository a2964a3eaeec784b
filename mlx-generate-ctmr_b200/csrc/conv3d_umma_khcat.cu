// Persistent implicit-GEMM conv3d (3x3x3, padding 1, stride 1, 16-bit operands)
// for narrow outputs (<= 64 channels) with the three kh taps side by side in N.
//
// A tcgen05.mma with M = 128 costs a fixed ~67 cycles whatever its N below 128,
// so an N = 64 product runs at half the tensor-core rate. Here one MMA
// multiplies the activation tile by the weights of all three taps along h at
// once, B = [W(kh=0) | W(kh=1) | W(kh=2)] (N = 3 x C_out), and the epilogue adds
// the three column blocks with the right row shift:
//
//   y[h] = P0[h - 1] + P1[h] + P2[h + 1],   Pk[r] = sum_{kd, kw, c} x[r] w[kd, kh = k, kw, c]
//
// The M tile is 16 h x 8 w voxels of one depth with each 8-row swizzle atom
// holding 8 consecutive w of one h, so a shift by one h is a shift by one atom
// (8 TMEM lanes). A tile covers input rows h0 - 1 .. h0 + 14 and produces the
// 14 output rows h0 .. h0 + 13 (the first and last atom only feed neighbours).
// Stages walk (kd, kw) x channel blocks: one TMA box of the activations at the
// (kd, kw) offset and one box of the three kh taps' weights, shared by MT = 2
// depth tiles. The accumulator (2 x 3 x C_out fp32 columns) has one TMEM buffer;
// the eight epilogue warps (two per TMEM lane quarter, one per column half)
// read it out, combine the shifts (lane shuffles inside a warp, shared memory
// across quarters), release the accumulator, then add bias and residual and
// store while the next tile's MMAs run.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv3d_umma.cuh"
#include "epilogue.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

constexpr int kKhThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2..9 epilogue
constexpr int kKhRows = 14;      // output rows along h per tile
// Quarter-edge exchange: per (column half, buffer, TMEM quarter) the P0 rows of lanes 24..31 and
// the P2 rows of lanes 0..7, 16 columns each at a 20-float lane pitch (conflict-free float4s).
constexpr uint32_t kKhLanePitch = 20;
constexpr uint32_t kKhEdgeQuarter = 2u * 8u * kKhLanePitch;                // floats: [P0|P2][lane][col]
constexpr uint32_t kKhEdgeFloats = 2u * 2u * 4u * kKhEdgeQuarter;           // [half][buf][quarter]

__host__ __device__ constexpr uint32_t ru_kh(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct KhLayout {
  uint32_t a_m_bytes, a_bytes, b_bytes, stage_bytes;
  __host__ __device__ KhLayout(int kc, int bn, int mt) {
    a_m_bytes = 128u * static_cast<uint32_t>(kc) * 2u;
    a_bytes = static_cast<uint32_t>(mt) * a_m_bytes;
    b_bytes = ru_kh(3u * static_cast<uint32_t>(bn) * static_cast<uint32_t>(kc) * 2u, 1024);
    stage_bytes = a_bytes + b_bytes;
  }
};

// Issue one 16-column TMEM load of this warp's 32 lanes; completed by tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Ties 16 registers to this point of the program: their uses stay after the
// preceding tcgen05.wait::ld (both statements are volatile, so stay in order).
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}

// Barrier over `threads` threads that also returns whether `v` held on all of them.
__device__ __forceinline__ bool barrier_all(int id, int threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %2, 0;\n\t"
      "bar.red.and.pred p, %1, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(static_cast<uint32_t>(v)), "r"(threads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Accumulator buffers in the 512 TMEM columns: two (the epilogue of tile i overlaps the MMAs of
// tile i + 1) when 2 x MT x 3 x C_out columns fit, else one, released depth by depth.
__host__ __device__ constexpr int kh_buffers(int mt, int bn) { return 2 * mt * 3 * bn <= 512 ? 2 : 1; }

template <int KC, int MT>
__global__ void __launch_bounds__(kKhThreads, 1)
    conv3d_khcat_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvGeom g) {
  constexpr uint32_t kRowBytes = KC * 2;
  constexpr int kSteps = KC / 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(ru_kh(smem_u32(smem_raw), 1024) - smem_u32(smem_raw) +
                                             reinterpret_cast<uintptr_t>(smem_raw));
  const KhLayout L(KC, g.bn, MT);
  const int S = g.stages;
  uint8_t* edges = smem + static_cast<size_t>(S) * L.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(edges + kKhEdgeFloats * sizeof(float));
  uint64_t* empty = full + S;
  uint64_t* tmem_full = empty + S;      // [2]: accumulator buffer complete
  uint64_t* tmem_empty = tmem_full + 2;  // [2]: buffer (two buffers) or depth (one buffer) read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages_per_tile = 9 * g.kblocks;
  const int bn = g.bn;
  const uint32_t n3 = 3u * static_cast<uint32_t>(bn);
  const int nbuf = kh_buffers(MT, bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 256);
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
  griddep_wait();
  griddep_launch_dependents();

  // Tile t -> (w tile fastest, then h, d, batch item).
  auto decode = [&](int t, int& w0, int& h0, int& d0, int& b) {
    const int tw_i = t % g.tiles_w; t /= g.tiles_w;
    const int th_i = t % g.tiles_h; t /= g.tiles_h;
    const int td_i = t % g.tiles_d;
    b = t / g.tiles_d;
    w0 = tw_i * 8;
    h0 = th_i * kKhRows;
    d0 = td_i * MT;
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    tma_prefetch_desc(&maps.a[0]);
    tma_prefetch_desc(&maps.b);
    int it = 0;
    int issued = 0;
    const uint32_t stage_tx = L.a_bytes + n3 * KC * 2u;
    for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x) {
      int w0, h0, d0, b;
      decode(t, w0, h0, d0, b);
      for (int st = 0; st < stages_per_tile; ++st, ++it) {
        const int s = it % S;
        const uint32_t round = static_cast<uint32_t>(it / S);
        if (it >= S && !mbar_wait_bounded(&empty[s], (round - 1) & 1u, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        const int kdw = st / g.kblocks;
        const int c = (st - kdw * g.kblocks) * KC;
        const int kd = kdw / 3, kw = kdw - 3 * (kdw / 3);
        uint8_t* st_base = smem + static_cast<size_t>(s) * L.stage_bytes;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        // Activations (C, W, H, D, B): 8 w at the kw offset, 16 h from h0 - 1, MT depths at the kd offset.
        tma_load_5d(st_base, &maps.a[0], &full[s], c, w0 + kw - 1, h0 - 1, d0 + kd - 1, b);
        // Weights (c, o, kw, kh, kd): the three kh taps of (kd, kw) as N = 3 x C_out rows.
        tma_load_5d(st_base + L.a_bytes, &maps.b, &full[s], c, 0, kw, 0, kd);
        ++issued;
      }
    }
    for (int k = max(0, issued - S); k < issued; ++k) {
      if (!mbar_wait_bounded(&full[k % S], static_cast<uint32_t>(k / S) & 1u, kErrWaitDrain)) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(g.operand_bf16 != 0, 128, n3);
    int it = 0;
    int lt = 0;
    for (int t = blockIdx.x; t < g.total_tiles && !*abort_flag; t += gridDim.x, ++lt) {
      const int buf = nbuf == 2 ? (lt & 1) : 0;
      const uint32_t acc0 = tmem + static_cast<uint32_t>(buf * MT) * n3;
      for (int st = 0; st < stages_per_tile; ++st, ++it) {
        const int s = it % S;
        if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(it / S) & 1u, kErrWaitFull)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + static_cast<size_t>(s) * L.stage_bytes);
        const uint32_t b_base = a_base + L.a_bytes;
        bool stop = false;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          // The columns about to be overwritten must have been read out: with two buffers the
          // tile before last's buffer, with one the previous tile's depth m.
          const bool wait_rel = st == 0 && (nbuf == 2 ? (m == 0 && lt >= 2) : lt >= 1);
          if (wait_rel) {
            const int rel = nbuf == 2 ? buf : m;
            const uint32_t par = static_cast<uint32_t>(nbuf == 2 ? (lt >> 1) - 1 : lt - 1) & 1u;
            if (!mbar_wait_bounded(&tmem_empty[rel], par, kErrWaitAcc)) {
              stop = true;
              break;
            }
            tc_fence_after();
          }
#pragma unroll
          for (int k = 0; k < kSteps; ++k) {
            umma_f16(acc0 + static_cast<uint32_t>(m) * n3,
                     smem_desc_kmajor(a_base + static_cast<uint32_t>(m) * L.a_m_bytes + k * 32u, kRowBytes),
                     smem_desc_kmajor(b_base + k * 32u, kRowBytes), idesc, (st == 0 && k == 0) ? 0u : 1u);
          }
        }
        umma_commit(&empty[s]);
        if (stop) {
          *abort_flag = 1;
          break;
        }
      }
      umma_commit(&tmem_full[buf]);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes a warp may read: 32 x (warp id mod 4)
    const int half = ew >> 2;      // 16-column chunks j with j % 2 == half
    const int row = quarter * 32 + lane;
    const int atom = row >> 3, iw = row & 7;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int nchunks = bn >> 4;
    const uint32_t edge_base = smem_u32(edges);
    int lt = 0;
    int eit = 0;  // edge exchanges so far (uniform over the four warps of a half): picks the buffer
    // The eight epilogue warps take every decision together (the wait outcome is
    // voted on), so no warp leaves while another waits at a named barrier.
    for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++lt) {
      int w0, h0, d0, b;
      decode(t, w0, h0, d0, b);
      const int buf = nbuf == 2 ? (lt & 1) : 0;
      const bool ok = mbar_wait_bounded(&tmem_full[buf], static_cast<uint32_t>(nbuf == 2 ? lt >> 1 : lt) & 1u,
                                        kErrWaitAcc);
      if (!barrier_all(3, 256, ok && !*abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      float out[MT][2][16];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * jj + half;
          if (j >= nchunks) continue;  // uniform over the four warps of this half
          const uint32_t col = static_cast<uint32_t>(buf * MT + m) * n3 + static_cast<uint32_t>(j * 16);
          uint32_t r0[16], r1[16], r2[16];
          tmem_ld16_issue(lane_addr + col, r0);
          tmem_ld16_issue(lane_addr + col + static_cast<uint32_t>(bn), r1);
          tmem_ld16_issue(lane_addr + col + 2u * static_cast<uint32_t>(bn), r2);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
          reg_fence16(r2);
          // Quarter edges: P0 of lanes 24..31 feeds the next quarter's lanes 0..7,
          // P2 of lanes 0..7 the previous quarter's lanes 24..31.
          const int ebuf = eit++ & 1;
          const uint32_t eb = edge_base + static_cast<uint32_t>((half * 2 + ebuf) * 4) * kKhEdgeQuarter * 4u;
          const uint32_t own = eb + static_cast<uint32_t>(quarter) * kKhEdgeQuarter * 4u +
                               static_cast<uint32_t>(lane & 7) * kKhLanePitch * 4u;
          if (lane >= 24) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) sts128(own + i * 4u, r0[i], r0[i + 1], r0[i + 2], r0[i + 3]);
          }
          if (lane < 8) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              sts128(own + 8u * kKhLanePitch * 4u + i * 4u, r2[i], r2[i + 1], r2[i + 2], r2[i + 3]);
          }
          named_barrier(1 + half, 128);
          // Every lane reads both neighbours' edge rows (the same eight addresses per
          // quarter: broadcasts) and keeps what its own row needs.
          const uint32_t prev = eb + static_cast<uint32_t>(quarter > 0 ? quarter - 1 : 0) * kKhEdgeQuarter * 4u +
                                static_cast<uint32_t>(lane & 7) * kKhLanePitch * 4u;
          const uint32_t next = eb + static_cast<uint32_t>(quarter < 3 ? quarter + 1 : 3) * kKhEdgeQuarter * 4u +
                                8u * kKhLanePitch * 4u + static_cast<uint32_t>(lane & 7) * kKhLanePitch * 4u;
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 pv = lds128(prev + i * 4u);
            const float4 nv = lds128(next + i * 4u);
            const float pe[4] = {pv.x, pv.y, pv.z, pv.w};
            const float ne[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float p0 = __shfl_up_sync(0xffffffffu, __uint_as_float(r0[i + e]), 8);
              float p2 = __shfl_down_sync(0xffffffffu, __uint_as_float(r2[i + e]), 8);
              if (lane < 8) p0 = pe[e];
              if (lane >= 24) p2 = ne[e];
              out[m][jj][i + e] = (p0 + __uint_as_float(r1[i + e])) + p2;
            }
          }
        }
        // Depth m's columns are in registers (with one buffer the next tile may overwrite them now).
        if (nbuf == 1 || m == MT - 1) {
          tc_fence_before();
          mbar_arrive(&tmem_empty[nbuf == 2 ? buf : m]);
        }
      }

      const int oh = h0 + atom - 1, ow = w0 + iw;
      const float* bias = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const int od = d0 + m;
        const bool valid = atom >= 1 && atom <= kKhRows && oh < g.out_h && ow < g.out_w && od < g.out_d;
        if (!valid) continue;
        const long long vox = ((static_cast<long long>(b) * g.out_d + od) * g.out_h + oh) * g.out_w + ow;
        const long long out_base = vox * g.out_cstride + g.out_coff;
        long long res_base = 0;
        if (g.res != nullptr) {
          const int qd = g.res_up ? od >> 1 : od, qh = g.res_up ? oh >> 1 : oh, qw = g.res_up ? ow >> 1 : ow;
          res_base = (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride;
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = 2 * jj + half;
          const int n = j * 16;
          if (j >= nchunks || n >= g.cout) continue;
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = out[m][jj][i];
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

template <int KC, int MT>
cudaError_t launch_khcat_typed(const ConvMaps& maps, const ConvGeom& g, int grid, size_t smem, cudaStream_t stream) {
  auto kern = conv3d_khcat_kernel<KC, MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, grid, kKhThreads, smem, stream, maps, g);
}

}  // namespace

int conv_khcat_stage_plan(int kc, int bn, int mt, size_t* smem_bytes) {
  const KhLayout L(kc, bn, mt);
  const size_t extra = 1024 + kKhEdgeFloats * sizeof(float) + 256;
  int stages = static_cast<int>((227 * 1024 - extra) / L.stage_bytes);
  if (stages > 8) stages = 8;
  if (stages < 2) return 0;
  *smem_bytes = static_cast<size_t>(stages) * L.stage_bytes + extra;
  return stages;
}

int conv_khcat_rows() { return kKhRows; }

cudaError_t launch_conv3d_khcat(const ConvMaps& maps, const ConvGeom& g, int kc, int mt, int sms, size_t smem,
                                cudaStream_t stream) {
  if (g.total_tiles <= 0 || g.bn > 64 || g.bn % 16 != 0 || g.tmem_cols != 512) return cudaErrorInvalidValue;
  const int grid = g.total_tiles < sms ? g.total_tiles : sms;
#define CTMR_KH(KC_, MT_) \
  if (kc == KC_ && mt == MT_) return launch_khcat_typed<KC_, MT_>(maps, g, grid, smem, stream);
  CTMR_KH(64, 2) CTMR_KH(32, 2) CTMR_KH(16, 2) CTMR_KH(64, 1) CTMR_KH(32, 1) CTMR_KH(16, 1)
#undef CTMR_KH
  return cudaErrorInvalidValue;
}

}  // namespace ctmr
