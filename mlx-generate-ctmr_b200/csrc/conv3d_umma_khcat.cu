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
// The M tile is 16 h x 8 w voxels of one depth with h fastest (the TMA view is
// (C, H, W, D, B)): row r = 16 w + h, so the 16 h of one w sit in one half of a
// warp's 32 TMEM lanes and a shift by one h is a shift by one lane. A tile covers
// input rows h0 - 1 .. h0 + 14 and produces the 14 output rows h0 .. h0 + 13
// (rows h = 0 and 15 only feed their neighbours).
// Per (kd, channel block) one TMA box of the activations, 16 h x 10 w x MT depths,
// serves the three kw taps: the window of tap kw starts 16 rows (whole 8-row
// swizzle atoms) further on. Each (kd, kw, channel block) has its own box of the
// three kh taps' weights, shared by the MT = 2 depth tiles; activation and weight
// boxes stream through two rings (2 or 4 and up to 12 slots). The accumulator
// (2 x 3 x C_out fp32 columns) has one TMEM buffer; the eight epilogue warps (two
// per TMEM lane quarter, one per column half) read it out, combine the shifts
// with 16-wide lane shuffles and release it, then add bias and residual and
// store while the next tile's MMAs run (with 64 output channels through an
// 8-lane transpose, so that each warp store writes whole 128-byte lines).
// The FUSE variant (64-channel blocks) reads the fp32 input itself: four converter
// warps load each activation box's rows from the NDHWC source (16-byte loads, eight
// in flight per lane), apply the GroupNorm affine and SiLU, round to the operand
// type and store the rows into the 128-byte-swizzled ring slot, so the fp16 copy of
// the operand pass is never written or read. Rows outside the volume are the zero
// padding of the transformed input, as the TMA fill of the prepared copy gives.
// A CTA-pair variant (clusters of two, tcgen05.mma.cta_group::2 with M = 256) is at
// the end of the file; it runs only when CTMR_KHCAT_PAIR=1 selects it.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv3d_umma.cuh"
#include "epilogue.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

constexpr int kKhThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2..9 epilogue
// The variant that converts its own operand (FUSE) adds warps 10..13, which fill the activation
// ring from the fp32 source in place of the TMA activation boxes.
constexpr int kKhConvWarps = 4;
constexpr int kKhThreadsFused = kKhThreads + 32 * kKhConvWarps;
constexpr int kKhRows = 14;      // output rows along h per tile
constexpr int kKhBoxW = 10;      // w per activation box: 8 output columns and the kw halo
constexpr int kKhMaxBSlots = 12;  // weight ring slots at most

__host__ __device__ constexpr uint32_t ru_kh(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Shared-memory ring slots: activations (MT depth slabs of 16 h x 10 w rows of kc channels) and
// weights (3 x C_out rows of kc channels). Slots and depth slabs are multiples of 1024 bytes and
// the kw window offset (16 rows) is two swizzle atoms (8 rows x kc x 2 bytes each), so every MMA
// operand window starts on a swizzle-atom boundary.
// Small activation boxes (<= 24 KB: channel blocks of 32 or 16, or one depth per tile) serve
// only a few short MMA stages each, so their ring is deeper (4 slots) to keep loads in flight.
struct KhLayout {
  uint32_t a_m_bytes, a_bytes, kw_bytes, b_bytes;
  int a_slots;
  __host__ __device__ KhLayout(int kc, int bn, int mt) {
    kw_bytes = 16u * static_cast<uint32_t>(kc) * 2u;
    a_m_bytes = static_cast<uint32_t>(kKhBoxW) * kw_bytes;
    a_bytes = static_cast<uint32_t>(mt) * a_m_bytes;
    b_bytes = ru_kh(3u * static_cast<uint32_t>(bn) * static_cast<uint32_t>(kc) * 2u, 1024);
    a_slots = a_bytes <= 24u * 1024u ? 4 : 2;
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

// Transposes N x N float4s across each group of N lanes (gi = lane % N, N = 4 or 8): afterwards
// q[k] holds what lane k of the group had in q[gi]. log2(N) butterfly stages, each swapping the
// off-diagonal halves with the partner lane (gi ^ s).
template <int N>
__device__ __forceinline__ void transpose_f4(float4 (&q)[N], int gi) {
#pragma unroll
  for (int s = N / 2; s >= 1; s >>= 1) {
    const bool upper = (gi & s) != 0;
#pragma unroll
    for (int k = 0; k < N; ++k) {
      if (k & s) continue;
      const float4 send = upper ? q[k] : q[k | s];
      float4 recv;
      recv.x = __shfl_xor_sync(0xffffffffu, send.x, s);
      recv.y = __shfl_xor_sync(0xffffffffu, send.y, s);
      recv.z = __shfl_xor_sync(0xffffffffu, send.z, s);
      recv.w = __shfl_xor_sync(0xffffffffu, send.w, s);
      if (upper) q[k] = recv;
      else q[k | s] = recv;
    }
  }
}

// Reads the residual of 4 consecutive output channels n .. n + 3 (fp32 or bf16) as fp32;
// channels at or beyond C_out read as zero.
__device__ __forceinline__ float4 kh_load4(const ConvGeom& g, long long res_off, int n) {
  const int cnt = min(4, g.cout - n);
  float x[4] = {0.f, 0.f, 0.f, 0.f};
  if (g.res_bf16) {
    const uint16_t* r = static_cast<const uint16_t*>(g.res) + res_off;
    if (cnt == 4 && (reinterpret_cast<uintptr_t>(r) & 7) == 0) {
      const uint2 q = __ldcg(reinterpret_cast<const uint2*>(r));
      x[0] = bf16_to_f32(static_cast<uint16_t>(q.x & 0xFFFFu));
      x[1] = bf16_to_f32(static_cast<uint16_t>(q.x >> 16));
      x[2] = bf16_to_f32(static_cast<uint16_t>(q.y & 0xFFFFu));
      x[3] = bf16_to_f32(static_cast<uint16_t>(q.y >> 16));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < cnt) x[e] = bf16_to_f32(r[e]);
    }
  } else {
    const float* r = static_cast<const float*>(g.res) + res_off;
    if (cnt == 4 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) return __ldcg(reinterpret_cast<const float4*>(r));
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (e < cnt) x[e] = __ldcg(r + e);
  }
  return make_float4(x[0], x[1], x[2], x[3]);
}

// Stores 4 consecutive output channels n .. n + 3 in the output type; channels at or beyond
// C_out are skipped.
__device__ __forceinline__ void kh_store4(const ConvGeom& g, float4 v, int n, long long out_off) {
  const int cnt = min(4, g.cout - n);
  const float x[4] = {v.x, v.y, v.z, v.w};
  if (g.out_bf16) {
    uint16_t* o = static_cast<uint16_t*>(g.out) + out_off;
    if (cnt == 4 && (reinterpret_cast<uintptr_t>(o) & 7) == 0) {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (e < cnt) {
          __nv_bfloat16 h = __float2bfloat16_rn(x[e]);
          o[e] = *reinterpret_cast<uint16_t*>(&h);
        }
      }
    }
  } else {
    float* o = static_cast<float*>(g.out) + out_off;
    if (cnt == 4 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      *reinterpret_cast<float4*>(o) = v;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < cnt) o[e] = x[e];
    }
  }
}

// SiLU of the operand, the same expression as the operand pass's 16-bit path (hardware exponential
// and reciprocal), so that both routes give the same operand bits.
__device__ __forceinline__ float kh_silu(float t) { return __fdividef(t, 1.f + __expf(-t)); }

// One converter warp's share of an activation box: rows r = 8 i + 2 cw + (lane / 16) of the
// MT x 10 w x 16 h box (row r at byte r x 128 of the slot, its 16-byte chunks swizzled by r mod 8),
// each lane taking 4 channels (lane mod 16) of the 64-channel block starting at channel c0.
// Source voxel of row r: depth d0 + kd - 1 + r / 160, w w0 - 1 + (r mod 160) / 16, h h0 - 1 + r mod 16.
template <int MT>
__device__ __forceinline__ void kh_convert_box(const ConvGeom& g, uint32_t slot, int cw, int lane, int b, int dd,
                                               int h0, int w0, int c0) {
  constexpr int kRows = MT * kKhBoxW * 16;
  const int q = lane & 15;
  const int c = c0 + 4 * q;
  const bool in1 = c >= g.fuse_ch0;
  const float* src = in1 ? g.fuse_src1 + (c - g.fuse_ch0) : g.fuse_src0 + c;
  const long long cs = in1 ? g.fuse_cstride1 : g.fuse_cstride0;
  float sc[4] = {1.f, 1.f, 1.f, 1.f}, of[4] = {0.f, 0.f, 0.f, 0.f};
  const bool aff = g.fuse_affine != nullptr;
  if (aff) {
    const float4* a = reinterpret_cast<const float4*>(g.fuse_affine + (static_cast<long long>(b) * g.fuse_ctot + c) * 2);
    const float4 a0 = __ldg(a), a1 = __ldg(a + 1);
    sc[0] = a0.x, of[0] = a0.y, sc[1] = a0.z, of[1] = a0.w, sc[2] = a1.x, of[2] = a1.y, sc[3] = a1.z, of[3] = a1.w;
  }
  const bool silu = g.fuse_silu != 0;
  const int D = g.row_d, H = g.row_h, W = g.row_w;
  const uint32_t lane_byte = static_cast<uint32_t>(q & 1) << 3;
  const uint32_t chunk = static_cast<uint32_t>(q >> 1);
  const int r_first = 2 * cw + (lane >> 4);
#pragma unroll 1
  for (int r0 = 0; r0 < kRows; r0 += 64) {
    float4 v[8];
    uint32_t live = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = r0 + 8 * k + r_first;
      const int m = r >= kKhBoxW * 16 ? 1 : 0;
      const int rem = r - m * kKhBoxW * 16;
      const int d = dd + m, h = h0 - 1 + (rem & 15), w = w0 - 1 + (rem >> 4);
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < kRows && static_cast<unsigned>(d) < static_cast<unsigned>(D) &&
          static_cast<unsigned>(h) < static_cast<unsigned>(H) && static_cast<unsigned>(w) < static_cast<unsigned>(W)) {
        v[k] = __ldg(reinterpret_cast<const float4*>(
            src + (((static_cast<long long>(b) * D + d) * H + h) * W + w) * cs));
        live |= 1u << k;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = r0 + 8 * k + r_first;
      if (r >= kRows) continue;
      uint32_t lo = 0, hi = 0;  // zero padding outside the volume
      if (live & (1u << k)) {
        float x[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        if (aff) {
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = fmaf(x[e], sc[e], of[e]);
        }
        if (silu) {
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = kh_silu(x[e]);
        }
        if (g.operand_bf16) {
          lo = pack_bf16x2(x[0], x[1]);
          hi = pack_bf16x2(x[2], x[3]);
        } else {
          const __half2 p0 = __floats2half2_rn(x[0], x[1]);
          const __half2 p1 = __floats2half2_rn(x[2], x[3]);
          lo = *reinterpret_cast<const uint32_t*>(&p0);
          hi = *reinterpret_cast<const uint32_t*>(&p1);
        }
      }
      const uint32_t addr = slot + static_cast<uint32_t>(r) * 128u +
                            ((chunk ^ (static_cast<uint32_t>(r) & 7u)) << 4) + lane_byte;
      asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(lo), "r"(hi) : "memory");
    }
  }
}

// Accumulator buffers in the 512 TMEM columns: two (the epilogue of tile i overlaps the MMAs of
// tile i + 1) when 2 x MT x 3 x C_out columns fit, else one, released depth by depth.
__host__ __device__ constexpr int kh_buffers(int mt, int bn) { return 2 * mt * 3 * bn <= 512 ? 2 : 1; }

template <int KC, int MT, bool TF32, bool STATS, bool FUSE>
__global__ void __launch_bounds__(FUSE ? kKhThreadsFused : kKhThreads, 1)
    conv3d_khcat_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvGeom g) {
  static_assert(!FUSE || (KC == 64 && !TF32), "the converter warps fill 64-channel 16-bit rows");
  constexpr uint32_t kRowBytes = KC * 2;
  constexpr int kSteps = KC / 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(ru_kh(smem_u32(smem_raw), 1024) - smem_u32(smem_raw) +
                                             reinterpret_cast<uintptr_t>(smem_raw));
  const KhLayout L(KC, g.bn, MT);
  const int S = g.stages;  // weight ring slots
  const int SA = L.a_slots;  // activation ring slots
  uint8_t* b_ring = smem + static_cast<size_t>(SA) * L.a_bytes;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(b_ring + static_cast<size_t>(S) * L.b_bytes);
  uint64_t* a_empty = a_full + SA;
  uint64_t* full = a_empty + SA;  // weight ring
  uint64_t* empty = full + S;
  uint64_t* tmem_full = empty + S;      // [2]: accumulator buffer complete
  uint64_t* tmem_empty = tmem_full + 2;  // [2]: buffer (two buffers) or depth (one buffer) read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups_per_tile = 3 * g.kblocks;  // (kd, channel block) pairs, three kw taps each
  const int bn = g.bn;
  const uint32_t n3 = 3u * static_cast<uint32_t>(bn);
  const int nbuf = kh_buffers(MT, bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], FUSE ? kKhConvWarps : 1);  // the TMA box, or one arrival per converter warp
      mbar_init(&a_empty[s], 1);
    }
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
    if (!FUSE) tma_prefetch_desc(&maps.a[0]);
    tma_prefetch_desc(&maps.b);
    int ia = 0;  // activation boxes issued
    int ib = 0;  // weight boxes issued
    const uint32_t b_tx = n3 * KC * 2u;
    bool stop = false;
    for (int t = blockIdx.x; t < g.total_tiles && !stop && !*abort_flag; t += gridDim.x) {
      int w0, h0, d0, b;
      decode(t, w0, h0, d0, b);
      for (int gi = 0; gi < groups_per_tile && !stop; ++gi) {
        const int kd = gi / g.kblocks;
        const int c = (gi - kd * g.kblocks) * KC;
        if (!FUSE) {
          const int sa = ia % SA;
          if (ia >= SA &&
              !mbar_wait_bounded(&a_empty[sa], static_cast<uint32_t>(ia / SA - 1) & 1u, kErrWaitEmpty)) {
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&a_full[sa], L.a_bytes);
          // Activations (C, H, W, D, B): 16 h from h0 - 1, 10 w from w0 - 1 (the windows of all
          // three kw taps), MT depths at the kd offset.
          tma_load_5d(smem + static_cast<size_t>(sa) * L.a_bytes, &maps.a[0], &a_full[sa], c, h0 - 1, w0 - 1,
                      d0 + kd - 1, b);
          ++ia;
        }
        for (int kw = 0; kw < 3; ++kw) {
          const int s = ib % S;
          if (ib >= S && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(ib / S - 1) & 1u, kErrWaitEmpty)) {
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&full[s], b_tx);
          // Weights (c, o, kw, kh, kd): the three kh taps of (kd, kw) as N = 3 x C_out rows.
          tma_load_5d(b_ring + static_cast<size_t>(s) * L.b_bytes, &maps.b, &full[s], c, 0, kw, 0, kd);
          ++ib;
        }
      }
    }
    if (stop) *abort_flag = 1;
    // Every box in flight lands before the CTA exits (FUSE: weight boxes only, ia stays 0).
    for (int k = max(0, ia - SA); k < ia; ++k) {
      if (!mbar_wait_bounded(&a_full[k % SA], static_cast<uint32_t>(k / SA) & 1u, kErrWaitDrain)) break;
    }
    for (int k = max(0, ib - S); k < ib; ++k) {
      if (!mbar_wait_bounded(&full[k % S], static_cast<uint32_t>(k / S) & 1u, kErrWaitDrain)) break;
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(g.operand_bf16 != 0, 128, n3, TF32);
    int ia = 0;
    int ib = 0;
    int lt = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < g.total_tiles && !stop && !*abort_flag; t += gridDim.x, ++lt) {
      const int buf = nbuf == 2 ? (lt & 1) : 0;
      const uint32_t acc0 = tmem + static_cast<uint32_t>(buf * MT) * n3;
      for (int gi = 0; gi < groups_per_tile && !stop; ++gi) {
        const int sa = ia % SA;
        if (!mbar_wait_bounded(&a_full[sa], static_cast<uint32_t>(ia / SA) & 1u, kErrWaitFull)) {
          stop = true;
          break;
        }
        ++ia;
        const uint64_t a_desc0 = smem_desc_kmajor(smem_u32(smem + static_cast<size_t>(sa) * L.a_bytes), kRowBytes);
        for (int kw = 0; kw < 3 && !stop; ++kw) {
          const int s = ib % S;
          if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(ib / S) & 1u, kErrWaitFull)) {
            stop = true;
            break;
          }
          ++ib;
          tc_fence_after();
          const uint64_t b_desc = smem_desc_kmajor(smem_u32(b_ring + static_cast<size_t>(s) * L.b_bytes), kRowBytes);
          const bool first = gi == 0 && kw == 0;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            // The columns about to be overwritten must have been read out: with two buffers the
            // tile before last's buffer, with one the previous tile's depth m.
            const bool wait_rel = first && (nbuf == 2 ? (m == 0 && lt >= 2) : lt >= 1);
            if (wait_rel) {
              const int rel = nbuf == 2 ? buf : m;
              const uint32_t par = static_cast<uint32_t>(nbuf == 2 ? (lt >> 1) - 1 : lt - 1) & 1u;
              if (!mbar_wait_bounded(&tmem_empty[rel], par, kErrWaitAcc)) {
                stop = true;
                break;
              }
              tc_fence_after();
            }
            const uint64_t a_desc = desc_advance(a_desc0, static_cast<uint32_t>(m) * L.a_m_bytes +
                                                              static_cast<uint32_t>(kw) * L.kw_bytes);
            const uint32_t d_acc = acc0 + static_cast<uint32_t>(m) * n3;
#pragma unroll
            for (int k = 0; k < kSteps; ++k) {  // 32 bytes of K per MMA: +2 in the descriptors' address field
              umma<TF32>(d_acc, a_desc + 2u * k, b_desc + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
            }
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&a_empty[sa]);
      }
      if (stop) break;
      umma_commit(&tmem_full[buf]);
    }
    if (stop) *abort_flag = 1;
  } else if (FUSE && warp >= 10) {
    // ------------------------------------------------------------ operand converters
    // Same tile and (kd, channel block) order as the MMA issuer; each warp fills its rows of the
    // slot, makes its shared-memory stores visible to the tensor cores' async proxy and arrives.
    const int cw = warp - 10;
    int ia = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < g.total_tiles && !stop && !*abort_flag; t += gridDim.x) {
      int w0, h0, d0, b;
      decode(t, w0, h0, d0, b);
      for (int gi = 0; gi < groups_per_tile; ++gi) {
        const int kd = gi / g.kblocks;
        const int c = (gi - kd * g.kblocks) * KC;
        const int sa = ia % SA;
        if (ia >= SA &&
            !mbar_wait_bounded(&a_empty[sa], static_cast<uint32_t>(ia / SA - 1) & 1u, kErrWaitEmpty)) {
          stop = true;
          break;
        }
        kh_convert_box<MT>(g, smem_u32(smem + static_cast<size_t>(sa) * L.a_bytes), cw, lane, b, d0 + kd - 1, h0,
                           w0, c);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
        ++ia;
      }
    }
    if (stop) *abort_flag = 1;
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes a warp may read: 32 x (warp id mod 4)
    const int half = ew >> 2;      // which of the two 16-column chunk pairs this warp reads
    // Lane l of quarter q holds tile row h = l % 16 (0 and 15 are halo) of w = 2 q + l / 16.
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int nchunks = bn >> 4;
    // 64 output channels: half h reads chunks 2h, 2h + 1 (32 contiguous channels per lane), stored
    // through an 8-lane transpose. Fewer: chunks h, h + 2 (both halves busy), stored per voxel.
    const bool wide = nchunks == 4;
    // STATS (64 output columns only): each lane keeps, for its four output channels and the current
    // batch item (tiles come in batch order), the count of the voxels it stores and the sums of
    // (x - pivot) and (x - pivot)^2 around a pivot per channel (the first value it sees), with no
    // division per tile. At a batch change and at the end the lane turns them into (count, mean,
    // M2), the warp merges its four 8-lane groups by Chan's update and lanes 0..7 write the warp's
    // slot 4 x CTA + quarter. Batch items a warp never saw get zeros.
    float st_n = 0.f, st_p[4], st_s[4], st_q[4];
    bool st_have = false;
    int st_b = -1, st_next = 0;
    auto stats_reset = [&]() {
      st_n = 0.f;
      st_have = false;
#pragma unroll
      for (int e = 0; e < 4; ++e) st_p[e] = st_s[e] = st_q[e] = 0.f;
    };
    auto stats_zero = [&](int bb) {  // this warp's slot for batch item bb holds nothing
      if (lane < 8) {
        const int nc = 32 * half + 4 * lane;
        float* dst = g.stats + ((static_cast<size_t>(bb) * g.stats_slots + 4 * blockIdx.x + quarter) * g.cout) * 3;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (nc + e < g.cout) dst[(nc + e) * 3] = dst[(nc + e) * 3 + 1] = dst[(nc + e) * 3 + 2] = 0.f;
      }
    };
    auto stats_flush = [&]() {  // warp-collective: moments, merge the 8-lane groups, write slot of st_b
      float m[4][3];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float md = st_n > 0.f ? st_s[e] / st_n : 0.f;
        m[e][0] = st_n;
        m[e][1] = st_p[e] + md;
        m[e][2] = fmaxf(0.f, st_q[e] - st_s[e] * md);
      }
#pragma unroll
      for (int off = 8; off < 32; off <<= 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float on = __shfl_xor_sync(0xffffffffu, m[e][0], off);
          const float om = __shfl_xor_sync(0xffffffffu, m[e][1], off);
          const float o2 = __shfl_xor_sync(0xffffffffu, m[e][2], off);
          if (lane & off) {  // both partners merge (lower group, upper group): the same result
            float r[3] = {on, om, o2};
            chan_merge(r, m[e][0], m[e][1], m[e][2]);
            m[e][0] = r[0], m[e][1] = r[1], m[e][2] = r[2];
          } else {
            chan_merge(m[e], on, om, o2);
          }
        }
      }
      if (lane < 8) {
        const int nc = 32 * half + 4 * lane;
        float* dst = g.stats + ((static_cast<size_t>(st_b) * g.stats_slots + 4 * blockIdx.x + quarter) * g.cout) * 3;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (nc + e < g.cout) {
            dst[(nc + e) * 3] = m[e][0];
            dst[(nc + e) * 3 + 1] = m[e][1];
            dst[(nc + e) * 3 + 2] = m[e][2];
          }
      }
    };
    if (STATS) stats_reset();
    int lt = 0;
    // The eight epilogue warps take every decision together (the wait outcome is voted on).
    for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++lt) {
      int w0, h0, d0, b;
      decode(t, w0, h0, d0, b);
      if (STATS && b != st_b) {
        if (st_b >= 0) stats_flush();
        for (; st_next < b; ++st_next) stats_zero(st_next);
        st_b = b;
        st_next = b + 1;
        stats_reset();
      }
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
          const int j = wide ? 2 * half + jj : 2 * jj + half;
          if (j >= nchunks) {  // uniform over the four warps of this half
#pragma unroll
            for (int i = 0; i < 16; ++i) out[m][jj][i] = 0.f;
            continue;
          }
          const uint32_t col = static_cast<uint32_t>(buf * MT + m) * n3 + static_cast<uint32_t>(j * 16);
          uint32_t r0[16], r1[16], r2[16];
          tmem_ld16_issue(lane_addr + col, r0);
          tmem_ld16_issue(lane_addr + col + static_cast<uint32_t>(bn), r1);
          tmem_ld16_issue(lane_addr + col + 2u * static_cast<uint32_t>(bn), r2);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
          reg_fence16(r2);
          // y[h] = P0[h - 1] + P1[h] + P2[h + 1]: neighbouring h are neighbouring lanes of the
          // same 16-lane group (the group's end lanes are halo rows, whose sums are not stored).
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = __shfl_up_sync(0xffffffffu, __uint_as_float(r0[i]), 1, 16);
            const float p2 = __shfl_down_sync(0xffffffffu, __uint_as_float(r2[i]), 1, 16);
            out[m][jj][i] = (p0 + __uint_as_float(r1[i])) + p2;
          }
        }
        // Depth m's columns are in registers (with one buffer the next tile may overwrite them now).
        if (nbuf == 1 || m == MT - 1) {
          tc_fence_before();
          mbar_arrive(&tmem_empty[nbuf == 2 ? buf : m]);
        }
      }

      const float* bias_b = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
      if (wide) {
        // Each 8-lane group transposes its 32 channels (8 float4 per lane), so that store
        // instruction k writes lane k's voxel with the whole group: four voxels' 128-byte runs of
        // 32 channels per warp instruction instead of 32 scattered 16-byte pieces.
        const int gi = lane & 7, gbase = lane & ~7;
        const int n = 32 * half + 4 * gi;  // the four channels this lane stores
        float4 bq = make_float4(0.f, 0.f, 0.f, 0.f);
        if (bias_b != nullptr) {
          if (n + 4 <= g.cout && (reinterpret_cast<uintptr_t>(bias_b + n) & 15) == 0) {
            bq = __ldg(reinterpret_cast<const float4*>(bias_b + n));
          } else {
            float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (n + e < g.cout) t4[e] = __ldg(bias_b + n + e);
            bq = make_float4(t4[0], t4[1], t4[2], t4[3]);
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          // Before the transpose q[k] is channel group k of this lane's voxel; after it, channels
          // n .. n + 3 of voxel k of the group, so the bias goes in afterwards.
          float4 q[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float* s4 = &out[m][k >> 2][4 * (k & 3)];
            q[k] = make_float4(s4[0], s4[1], s4[2], s4[3]);
          }
          transpose_f4<8>(q, gi);
          const int od = d0 + m;
          if (od >= g.out_d) continue;
          long long vox[8];
          bool ok[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int src = gbase + k;  // the lane whose voxel instruction k stores
            const int sh = src & 15;
            const int oh = h0 + sh - 1, ow = w0 + 2 * quarter + (src >> 4);
            ok[k] = sh >= 1 && sh <= kKhRows && oh < g.out_h && ow < g.out_w;
            vox[k] = ((static_cast<long long>(b) * g.out_d + od) * g.out_h + oh) * g.out_w + ow;
            q[k].x += bq.x;
            q[k].y += bq.y;
            q[k].z += bq.z;
            q[k].w += bq.w;
          }
          if (g.res != nullptr) {
            // All eight residual reads go out before the first store. The residual is read through
            // L2 (ld.global.cg), not the read-only path: an in-place residual add (residual == output)
            // stays defined, each lane reading its addresses before it writes them.
            float4 rv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              rv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
              if (ok[k]) {
                const int src = gbase + k;
                const int oh = h0 + (src & 15) - 1, ow = w0 + 2 * quarter + (src >> 4);
                const int qd = g.res_up ? od >> 1 : od, qh = g.res_up ? oh >> 1 : oh, qw = g.res_up ? ow >> 1 : ow;
                const long long ro =
                    (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride + n;
                rv[k] = kh_load4(g, ro, n);
              }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              q[k].x += rv[k].x;
              q[k].y += rv[k].y;
              q[k].z += rv[k].z;
              q[k].w += rv[k].w;
            }
          }
          if (STATS) {  // shifted sums of this depth's (up to) eight stored voxels
            if (!st_have) {  // the first stored voxel of this batch item sets the pivots
#pragma unroll
              for (int k = 7; k >= 0; --k)
                if (ok[k]) st_p[0] = q[k].x, st_p[1] = q[k].y, st_p[2] = q[k].z, st_p[3] = q[k].w, st_have = true;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (!ok[k]) continue;
              const float dx = q[k].x - st_p[0], dy = q[k].y - st_p[1], dz = q[k].z - st_p[2], dw = q[k].w - st_p[3];
              st_s[0] += dx, st_s[1] += dy, st_s[2] += dz, st_s[3] += dw;
              st_q[0] = fmaf(dx, dx, st_q[0]), st_q[1] = fmaf(dy, dy, st_q[1]);
              st_q[2] = fmaf(dz, dz, st_q[2]), st_q[3] = fmaf(dw, dw, st_q[3]);
              st_n += 1.f;
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (ok[k]) kh_store4(g, q[k], n, vox[k] * g.out_cstride + g.out_coff + n);
        }
      } else {
        const int row = quarter * 32 + lane;
        const int oh = h0 + (row & 15) - 1, ow = w0 + (row >> 4);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int od = d0 + m;
          const bool valid = (row & 15) >= 1 && (row & 15) <= kKhRows && oh < g.out_h && ow < g.out_w && od < g.out_d;
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
            if (bias_b != nullptr) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (i < cnt) v[i] += __ldg(bias_b + n + i);
            }
            store_row16(g, v, n, out_base + n, res_base + n);
          }
        }
      }
    }
    if (STATS) {
      if (st_b >= 0) stats_flush();
      for (; st_next < g.batch; ++st_next) stats_zero(st_next);
      if (blockIdx.x == 0) {  // the slots of CTAs past the grid hold nothing
        const int first = 4 * static_cast<int>(gridDim.x), extra = g.stats_slots - first;
        for (int e = static_cast<int>(threadIdx.x) - 64; e < g.batch * extra * g.cout; e += 256) {
          const int bb = e / (extra * g.cout), r = e - bb * extra * g.cout;
          float* dst = g.stats + (static_cast<size_t>(bb) * g.stats_slots * g.cout + static_cast<size_t>(first) * g.cout + r) * 3;
          dst[0] = dst[1] = dst[2] = 0.f;
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

// ---------------------------------------------------------------- CTA-pair variant
// 64 -> 64 channels, 64-channel blocks, two depths per tile: the same tiling, but two CTAs of a
// cluster (one per SM) share every product. tcgen05.mma.cta_group::2 with M = 256 takes rows
// 0..127 from the first CTA's activation box (its tile) and rows 128..255 from the second's (the
// pair's other tile), and B's N = 192 rows half from each CTA: CTA r loads the three kh taps of
// output channels 32 r .. 32 r + 31, a (64 c, 32 o, 1, 3, 1) box of the weight view. So each SM
// streams half of every weight box (12 KB instead of 24 KB per (kd, kw)), reads half of B from
// shared memory per product, and one thread issues the products of both tiles. Each CTA's TMEM
// receives its own tile's 128 rows x 192 columns; column 96 h + 32 kh + (o - 32 h) holds P_kh
// of output channel o, h = o / 32. Both CTAs' copies of a stage count on the first CTA's
// barriers; the products' commits arrive on both CTAs' ring and accumulator barriers; each CTA's
// epilogue warps release a depth on the first CTA's barrier (16 warp arrivals).
constexpr int kPairKC = 64;
constexpr int kPairMT = 2;
constexpr int kPairBN = 64;
constexpr uint32_t kPairN = 3u * kPairBN;                         // accumulator columns per depth
constexpr uint32_t kPairKwBytes = 16u * kPairKC * 2u;             // 16 rows: one kw step
constexpr uint32_t kPairAmBytes = kKhBoxW * kPairKwBytes;         // one depth of the activation box
constexpr uint32_t kPairABytes = kPairMT * kPairAmBytes;          // 40 KB
constexpr uint32_t kPairBBytes = 3u * (kPairBN / 2) * kPairKC * 2u;  // 12 KB: this CTA's half of N
constexpr int kPairASlots = 2;
static_assert(kPairBBytes % 1024 == 0 && kPairABytes % 1024 == 0, "ring slots stay swizzle-atom aligned");
static_assert(kPairMT * kPairN <= 512, "both depths' accumulators fit one TMEM allocation");

__global__ void __launch_bounds__(kKhThreads, 1)
    conv3d_khcat_pair_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvGeom g) {
  constexpr uint32_t kRowBytes = kPairKC * 2;
  constexpr int kSteps = kPairKC / 16;
  constexpr int SA = kPairASlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(ru_kh(smem_u32(smem_raw), 1024) - smem_u32(smem_raw) +
                                             reinterpret_cast<uintptr_t>(smem_raw));
  const int S = g.stages;  // weight ring slots
  uint8_t* b_ring = smem + static_cast<size_t>(SA) * kPairABytes;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(b_ring + static_cast<size_t>(S) * kPairBBytes);
  uint64_t* a_empty = a_full + SA;
  uint64_t* full = a_empty + SA;  // weight ring
  uint64_t* empty = full + S;
  uint64_t* tmem_full = empty + S;       // [1]: the pair's accumulators complete
  uint64_t* tmem_empty = tmem_full + 2;  // [2]: depth m read out by both CTAs (first CTA's barrier)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the CTA whose thread issues the products
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int pair_tiles = (g.total_tiles + 1) >> 1;
  const int groups_per_tile = 3 * g.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 16);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before a copy, commit or arrive crosses the pair
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  // Pair tile pt holds tiles 2 pt (first CTA) and 2 pt + 1 (second); tile t -> (w tile fastest,
  // then h, d, batch item). With an odd tile count the last pair's second CTA computes a copy of
  // the last tile and stores nothing.
  auto decode = [&](int t, int& w0, int& h0, int& d0, int& b) {
    const int tw_i = t % g.tiles_w; t /= g.tiles_w;
    const int th_i = t % g.tiles_h; t /= g.tiles_h;
    const int td_i = t % g.tiles_d;
    b = t / g.tiles_d;
    w0 = tw_i * 8;
    h0 = th_i * kKhRows;
    d0 = td_i * kPairMT;
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    tma_prefetch_desc(&maps.a[0]);
    tma_prefetch_desc(&maps.b);
    const uint32_t a_full0 = cluster_addr(a_full, 0);
    const uint32_t full0 = cluster_addr(full, 0);
    int ia = 0;
    int ib = 0;
    bool stop = false;
    for (int pt = pair; pt < pair_tiles && !stop && !*abort_flag; pt += pairs) {
      int w0, h0, d0, b;
      decode(min(2 * pt + static_cast<int>(rank), g.total_tiles - 1), w0, h0, d0, b);
      for (int gi = 0; gi < groups_per_tile && !stop; ++gi) {
        const int kd = gi / g.kblocks;
        const int c = (gi - kd * g.kblocks) * kPairKC;
        const int sa = ia % SA;
        if (ia >= SA &&
            !mbar_wait_bounded(&a_empty[sa], static_cast<uint32_t>(ia / SA - 1) & 1u, kErrWaitEmpty)) {
          stop = true;
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(&a_full[sa], 2u * kPairABytes);
        tma_load_5d_pair(smem + static_cast<size_t>(sa) * kPairABytes, &maps.a[0], a_full0 + 8u * sa, c, h0 - 1,
                         w0 - 1, d0 + kd - 1, b);
        ++ia;
        for (int kw = 0; kw < 3; ++kw) {
          const int s = ib % S;
          if (ib >= S && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(ib / S - 1) & 1u, kErrWaitEmpty)) {
            stop = true;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2u * kPairBBytes);
          // Weights (c, o, kw, kh, kd): this CTA's 32 output channels, three kh taps.
          tma_load_5d_pair(b_ring + static_cast<size_t>(s) * kPairBBytes, &maps.b, full0 + 8u * s, c,
                           static_cast<int>(rank) * (kPairBN / 2), kw, 0, kd);
          ++ib;
        }
      }
    }
    if (stop) *abort_flag = 1;
    // The first CTA's barriers count both CTAs' bytes: every copy in flight lands before the
    // closing cluster barrier lets either CTA exit.
    if (rank == 0) {
      for (int k = max(0, ia - SA); k < ia; ++k) {
        if (!mbar_wait_bounded(&a_full[k % SA], static_cast<uint32_t>(k / SA) & 1u, kErrWaitDrain)) break;
      }
      for (int k = max(0, ib - S); k < ib; ++k) {
        if (!mbar_wait_bounded(&full[k % S], static_cast<uint32_t>(k / S) & 1u, kErrWaitDrain)) break;
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (first CTA)
    const uint32_t idesc = idesc_f16(g.operand_bf16 != 0, 256, kPairN);
    int ia = 0;
    int ib = 0;
    int lt = 0;
    bool stop = false;
    for (int pt = pair; pt < pair_tiles && !stop && !*abort_flag; pt += pairs, ++lt) {
      for (int gi = 0; gi < groups_per_tile && !stop; ++gi) {
        const int sa = ia % SA;
        if (!mbar_wait_bounded(&a_full[sa], static_cast<uint32_t>(ia / SA) & 1u, kErrWaitFull)) {
          stop = true;
          break;
        }
        ++ia;
        const uint64_t a_desc0 = smem_desc_kmajor(smem_u32(smem + static_cast<size_t>(sa) * kPairABytes), kRowBytes);
        for (int kw = 0; kw < 3 && !stop; ++kw) {
          const int s = ib % S;
          if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(ib / S) & 1u, kErrWaitFull)) {
            stop = true;
            break;
          }
          ++ib;
          tc_fence_after();
          const uint64_t b_desc = smem_desc_kmajor(smem_u32(b_ring + static_cast<size_t>(s) * kPairBBytes), kRowBytes);
          const bool first = gi == 0 && kw == 0;
#pragma unroll
          for (int m = 0; m < kPairMT; ++m) {
            // Depth m's columns must have been read out of both CTAs' TMEM (previous pair tile).
            if (first && lt >= 1) {
              if (!mbar_wait_bounded(&tmem_empty[m], static_cast<uint32_t>(lt - 1) & 1u, kErrWaitAcc)) {
                stop = true;
                break;
              }
              tc_fence_after();
            }
            const uint64_t a_desc =
                desc_advance(a_desc0, static_cast<uint32_t>(m) * kPairAmBytes + static_cast<uint32_t>(kw) * kPairKwBytes);
            const uint32_t d_acc = tmem + static_cast<uint32_t>(m) * kPairN;
#pragma unroll
            for (int k = 0; k < kSteps; ++k)
              umma_f16_pair(d_acc, a_desc + 2u * k, b_desc + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
          }
          umma_commit_pair(&empty[s]);
        }
        umma_commit_pair(&a_empty[sa]);
      }
      if (stop) break;
      umma_commit_pair(&tmem_full[0]);
    }
    if (stop) *abort_flag = 1;
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lanes a warp may read: 32 x (warp id mod 4)
    const int half = ew >> 2;      // output channels 32 half .. 32 half + 31
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t release0 = cluster_addr(tmem_empty, 0);
    const int gi = lane & 7, gbase = lane & ~7;
    const int n = 32 * half + 4 * gi;  // the four channels this lane stores after the transpose
    int lt = 0;
    for (int pt = pair; pt < pair_tiles; pt += pairs, ++lt) {
      const int t = 2 * pt + static_cast<int>(rank);
      const bool tile_ok = t < g.total_tiles;
      int w0, h0, d0, b;
      decode(min(t, g.total_tiles - 1), w0, h0, d0, b);
      const bool ok = mbar_wait_bounded(&tmem_full[0], static_cast<uint32_t>(lt) & 1u, kErrWaitAcc);
      if (!barrier_all(3, 256, ok && !*abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      float out[kPairMT][2][16];
#pragma unroll
      for (int m = 0; m < kPairMT; ++m) {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const uint32_t col = static_cast<uint32_t>(m) * kPairN + static_cast<uint32_t>(96 * half + 16 * jj);
          uint32_t r0[16], r1[16], r2[16];
          tmem_ld16_issue(lane_addr + col, r0);
          tmem_ld16_issue(lane_addr + col + 32u, r1);
          tmem_ld16_issue(lane_addr + col + 64u, r2);
          tmem_wait_ld();
          reg_fence16(r0);
          reg_fence16(r1);
          reg_fence16(r2);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = __shfl_up_sync(0xffffffffu, __uint_as_float(r0[i]), 1, 16);
            const float p2 = __shfl_down_sync(0xffffffffu, __uint_as_float(r2[i]), 1, 16);
            out[m][jj][i] = (p0 + __uint_as_float(r1[i])) + p2;
          }
        }
        // Depth m of this CTA's accumulator is in registers: one arrival per warp on the first
        // CTA's barrier, after every lane's TMEM loads.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(release0 + 8u * static_cast<uint32_t>(m));
      }

      const float* bias_b = g.bias != nullptr ? g.bias + static_cast<long long>(b) * g.bias_bstride : nullptr;
      float4 bq = make_float4(0.f, 0.f, 0.f, 0.f);
      if (bias_b != nullptr) {
        if (n + 4 <= g.cout && (reinterpret_cast<uintptr_t>(bias_b + n) & 15) == 0) {
          bq = __ldg(reinterpret_cast<const float4*>(bias_b + n));
        } else {
          float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (n + e < g.cout) t4[e] = __ldg(bias_b + n + e);
          bq = make_float4(t4[0], t4[1], t4[2], t4[3]);
        }
      }
#pragma unroll
      for (int m = 0; m < kPairMT; ++m) {
        float4 q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float* s4 = &out[m][k >> 2][4 * (k & 3)];
          q[k] = make_float4(s4[0], s4[1], s4[2], s4[3]);
        }
        transpose_f4<8>(q, gi);
        const int od = d0 + m;
        if (!tile_ok || od >= g.out_d) continue;
        long long vox[8];
        bool okk[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int src = gbase + k;
          const int sh = src & 15;
          const int oh = h0 + sh - 1, ow = w0 + 2 * quarter + (src >> 4);
          okk[k] = sh >= 1 && sh <= kKhRows && oh < g.out_h && ow < g.out_w;
          vox[k] = ((static_cast<long long>(b) * g.out_d + od) * g.out_h + oh) * g.out_w + ow;
          q[k].x += bq.x;
          q[k].y += bq.y;
          q[k].z += bq.z;
          q[k].w += bq.w;
        }
        if (g.res != nullptr) {
          float4 rv[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            rv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (okk[k]) {
              const int src = gbase + k;
              const int oh = h0 + (src & 15) - 1, ow = w0 + 2 * quarter + (src >> 4);
              const int qd = g.res_up ? od >> 1 : od, qh = g.res_up ? oh >> 1 : oh, qw = g.res_up ? ow >> 1 : ow;
              const long long ro =
                  (((static_cast<long long>(b) * g.res_d + qd) * g.res_h + qh) * g.res_w + qw) * g.res_cstride + n;
              rv[k] = kh_load4(g, ro, n);
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            q[k].x += rv[k].x;
            q[k].y += rv[k].y;
            q[k].z += rv[k].z;
            q[k].w += rv[k].w;
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (okk[k]) kh_store4(g, q[k], n, vox[k] * g.out_cstride + g.out_coff + n);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA exits while the other's products, copies or arrivals may reach it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <int KC, int MT>
cudaError_t launch_khcat_typed(const ConvMaps& maps, const ConvGeom& g, int grid, size_t smem, cudaStream_t stream) {
  // Epilogue statistics: 16-bit operands and 64 output columns only (the planner's condition).
  auto kern = g.stats != nullptr ? conv3d_khcat_kernel<KC, MT, false, true, false>
              : g.operand_tf32  ? conv3d_khcat_kernel<KC, MT, true, false, false>
                                : conv3d_khcat_kernel<KC, MT, false, false, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, grid, kKhThreads, smem, stream, maps, g);
}

template <int MT>
cudaError_t launch_khcat_fused_typed(const ConvMaps& maps, const ConvGeom& g, int grid, size_t smem,
                                     cudaStream_t stream) {
  auto kern = g.stats != nullptr ? conv3d_khcat_kernel<64, MT, false, true, true>
                                 : conv3d_khcat_kernel<64, MT, false, false, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, grid, kKhThreadsFused, smem, stream, maps, g);
}

}  // namespace

int conv_khcat_stage_plan(int kc, int bn, int mt, size_t* smem_bytes) {
  const KhLayout L(kc, bn, mt);
  const size_t extra = 1024 + 512;  // alignment slack, barriers
  const size_t fixed = extra + static_cast<size_t>(L.a_slots) * L.a_bytes;
  if (fixed >= 227 * 1024) return 0;
  int stages = static_cast<int>((227 * 1024 - fixed) / L.b_bytes);
  if (stages > kKhMaxBSlots) stages = kKhMaxBSlots;
  if (stages < 2) return 0;
  *smem_bytes = fixed + static_cast<size_t>(stages) * L.b_bytes;
  return stages;
}

int conv_khcat_rows() { return kKhRows; }

int conv_khcat_pair_stage_plan(size_t* smem_bytes) {
  const size_t fixed = 1024 + 512 + static_cast<size_t>(kPairASlots) * kPairABytes;
  int stages = static_cast<int>((227 * 1024 - fixed) / kPairBBytes);
  if (stages > kKhMaxBSlots) stages = kKhMaxBSlots;
  if (stages < 2) return 0;
  *smem_bytes = fixed + static_cast<size_t>(stages) * kPairBBytes;
  return stages;
}

// One cluster of two CTAs per SM pair, as many pairs as can be resident at once (queried once
// per device) or as there are pair tiles. cudaErrorNotSupported: no pair fits, use the one-SM kernel.
cudaError_t launch_conv3d_khcat_pair(const ConvMaps& maps, const ConvGeom& g, size_t smem, cudaStream_t stream) {
  if (g.total_tiles <= 0 || g.bn != kPairBN || g.kblocks < 1 || g.tmem_cols != 512 || g.operand_tf32)
    return cudaErrorInvalidValue;
  auto kern = conv3d_khcat_pair_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kKhThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  int clusters = dev >= 0 && dev < 64 ? cached[dev].load(std::memory_order_relaxed) : 0;
  if (clusters == 0) {
    cfg.gridDim = dim3(2 * (device_sm_count() / 2));
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
      (void)cudaGetLastError();
      clusters = -1;
    }
    if (dev >= 0 && dev < 64) cached[dev].store(clusters, std::memory_order_relaxed);
  }
  if (clusters < 1) return cudaErrorNotSupported;
  const int pair_tiles = (g.total_tiles + 1) / 2;
  cfg.gridDim = dim3(2 * (pair_tiles < clusters ? pair_tiles : clusters));
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, maps, g);
}

cudaError_t launch_conv3d_khcat(const ConvMaps& maps, const ConvGeom& g, int kc, int mt, int sms, size_t smem,
                                cudaStream_t stream) {
  if (g.total_tiles <= 0 || g.bn > 64 || g.bn % 16 != 0 || g.tmem_cols != 512) return cudaErrorInvalidValue;
  const int grid = g.total_tiles < sms ? g.total_tiles : sms;
  if (g.stats != nullptr && (g.bn != 64 || g.operand_tf32 || g.stats_slots < 4 * grid)) return cudaErrorInvalidValue;
  if (g.fuse_src0 != nullptr) {
    // The converter warps: 64-channel blocks of fp32 sources, 16-byte aligned 4-channel pieces.
    if (kc != 64 || g.operand_tf32 || g.fuse_ctot % 64 != 0 || g.fuse_ch0 % 64 != 0 || g.fuse_cstride0 % 4 != 0 ||
        (reinterpret_cast<uintptr_t>(g.fuse_src0) & 15) != 0 ||
        (g.fuse_ch0 < g.fuse_ctot && (g.fuse_src1 == nullptr || g.fuse_cstride1 % 4 != 0 ||
                                      (reinterpret_cast<uintptr_t>(g.fuse_src1) & 15) != 0)) ||
        (g.fuse_affine != nullptr && (reinterpret_cast<uintptr_t>(g.fuse_affine) & 15) != 0) ||
        g.kblocks * 64 != g.fuse_ctot)
      return cudaErrorInvalidValue;
    if (mt == 2) return launch_khcat_fused_typed<2>(maps, g, grid, smem, stream);
    if (mt == 1) return launch_khcat_fused_typed<1>(maps, g, grid, smem, stream);
    return cudaErrorInvalidValue;
  }
#define CTMR_KH(KC_, MT_) \
  if (kc == KC_ && mt == MT_) return launch_khcat_typed<KC_, MT_>(maps, g, grid, smem, stream);
  CTMR_KH(64, 2) CTMR_KH(32, 2) CTMR_KH(16, 2) CTMR_KH(64, 1) CTMR_KH(32, 1) CTMR_KH(16, 1)
#undef CTMR_KH
  return cudaErrorInvalidValue;
}

}  // namespace ctmr
