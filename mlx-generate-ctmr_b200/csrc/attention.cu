// Multi-head self-attention for head size 32 on the tensor cores: the
// `softmax(Q K^T * scale) V` of the MAISI UNet's spatial attention
// (`attention.py:92-160` -> `fast_fp32.self_attention_tokens`, `fast_fp32.py:352-396`,
// computed by the reference's `_flash_attention.flash_attention`,
// `_flash_attention.py:320-360`), as one flash-attention pass.
//
// Input: the fused Q/K/V projection (B, L, 3C) in fp16 or bf16, head h at
// columns h*32 (q), C + h*32 (k), 2C + h*32 (v); output (B, L, C) in the same
// type. One CTA per (128-query tile, head, batch item). Warp roles: a TMA
// producer (Q once, K/V tiles of 128 keys double-buffered), a single-thread
// tcgen05.mma issuer, and four softmax warps owning one query row per thread.
//
// Per key tile j: S = Q K_j^T (M = 128 queries, N = 128 keys, K = 32) lands in
// TMEM; the softmax threads read their row, track the running maximum m and
// sum l (base-2 exponentials of the scaled logits), write P_j = exp2(s - m_j)
// in the operand type to shared memory in the 128-byte-swizzled K-major layout
// (two 64-key chunks), and the issuer computes PV_j = P_j V_j (M = 128,
// N = 32, K = 128; V read MN-major: its 32 head channels are the contiguous N
// dimension) into one of two TMEM tiles. The output accumulator stays in the
// softmax threads' registers: while P_{j+1} is produced, PV_j is folded in as
// O = O * exp2(m_{j-1} - m_j) + PV_j, so the tensor core and the exponentials
// overlap. The last step divides by l and stores the row.
//
// At head size 32 the pass is bound by the exponentials (B x H x L^2 of them, 16 per clock
// per SM on the exponential unit), so a quarter of them (keys 24..31 of every 32) are
// computed on the FMA pipe instead: 2^x = 2^n * p(f) with x = n + f, n the nearest integer
// (Cody-Waite range reduction with the 1.5 * 2^23 rounding constant, f in [-1/2, 1/2]) and
// p a degree-3 polynomial fitted to 2^f on [-1/2, 1/2] for least maximum relative error
// (linear-programming minimax fit; max relative error 7.5e-5, below the fp16 P operand's
// half-ulp of 4.9e-4), 2^n added into the exponent field.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "attention.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace ctmr {
namespace {

constexpr int kAttnThreads = 192;      // warp 0 TMA, warp 1 MMA + TMEM, warps 2..5 softmax
constexpr int kRows = 128;             // queries per CTA, keys per tile
constexpr int kHead = 32;              // head size
constexpr uint32_t kTileBytes = kRows * kHead * 2;   // 8 KB: one Q, K or V tile (64-byte rows)
constexpr uint32_t kPBytes = kRows * kRows * 2;      // 32 KB: one P tile (two 64-key chunks)
constexpr uint32_t kTmemCols = 256;    // S: 128 columns, O tiles: 2 x 32

// smem: Q | K[2] | V[2] | P[2] | barriers
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + 2 * kTileBytes;
constexpr uint32_t kOffP = kOffV + 2 * kTileBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kPBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers + alignment slack

__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Waits for this thread's TMEM loads and ties the 32 registers to this point (their uses stay after it).
__device__ __forceinline__ void tmem_ld32_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
  asm volatile(""
               : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

// Shared-memory descriptor of an MN-major operand with 64-byte swizzling: 8-row
// groups along K are 8 x 64 B apart; the 32 MN elements of a row are one atom.
__device__ __forceinline__ uint64_t smem_desc_mn_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                        // LBO: one atom along MN (unused)
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;     // SBO: next 8 keys
  d |= 1ull << 46;                                             // descriptor version (sm_100)
  d |= 4ull << 61;                                             // 64-byte swizzle
  return d;
}

// 2^x on the exponential unit (flushes results below 2^-126 to zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA pipe: x = n + f (n nearest integer, |f| <= 1/2), 2^f by the degree-3
// minimax polynomial, n added to the exponent. x is clamped at -125 (2^-125 is zero in the P operand).
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;
__device__ __forceinline__ float poly_exp2(float x) {
  x = fmaxf(x, -125.f);
  const float j = x + 12582912.f;  // 1.5 * 2^23: the low mantissa bits of j hold round(x)
  const float f = x - (j - 12582912.f);
  float p = fmaf(kExp2C3, f, kExp2C2);
  p = fmaf(p, f, kExp2C1);
  p = fmaf(p, f, kExp2C0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two CTAs per SM (at most 170 registers per thread): while one waits on its tensor-core
// products the other's softmax warps keep the exponential unit busy.
template <bool BF16>
__global__ void __launch_bounds__(kAttnThreads, 2)
    attention_d32_kernel(const __grid_constant__ CUtensorMap map, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;
  uint64_t* s_free = bar + 6;
  uint64_t* p_full = bar + 7;    // [2]
  uint64_t* o_full = bar + 9;    // [2]
  uint64_t* o_free = bar + 11;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kRows, h = blockIdx.y, b = blockIdx.z;
  const int n_tiles = p.tokens / kRows;
  const int C = p.heads * kHead;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + 128;  // S columns [0, 128), O tiles [128, 192)
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    tma_prefetch_desc(&map);
    mbar_arrive_expect_tx(q_full, kTileBytes);
    tma_load_3d(smem + kOffQ, &map, q_full, h * kHead, q0, b);
    int j = 0;
    for (; j < n_tiles && !*abort_flag; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait_bounded(&kv_empty[s], static_cast<uint32_t>((j >> 1) - 1) & 1u, kErrWaitEmpty)) {
        *abort_flag = 1;
        break;
      }
      mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
      tma_load_3d(smem + kOffK + s * kTileBytes, &map, &kv_full[s], C + h * kHead, j * kRows, b);
      tma_load_3d(smem + kOffV + s * kTileBytes, &map, &kv_full[s], 2 * C + h * kHead, j * kRows, b);
    }
    // Drain: every issued load lands before the CTA can exit.
    mbar_wait_bounded(q_full, 0, kErrWaitDrain);
    for (int k = max(0, j - 2); k < j; ++k) mbar_wait_bounded(&kv_full[k & 1], static_cast<uint32_t>(k >> 1) & 1u, kErrWaitDrain);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t id_s = idesc_f16(BF16, kRows, kRows);                  // S = Q K^T, both K-major
    const uint32_t id_o = idesc_f16(BF16, kRows, kHead) | (1u << 16);     // O = P V, V MN-major
    const uint32_t a_q = smem_u32(smem + kOffQ);
    auto pv = [&](int i) -> bool {  // O tile (i & 1) = P_i V_i
      const int s = i & 1;
      if (!mbar_wait_bounded(&p_full[s], static_cast<uint32_t>(i >> 1) & 1u, kErrWaitFull)) return false;
      if (i >= 2 && !mbar_wait_bounded(&o_free[s], static_cast<uint32_t>((i >> 1) - 1) & 1u, kErrWaitAcc))
        return false;
      tc_fence_after();
      const uint32_t a_p = smem_u32(smem + kOffP + s * kPBytes);
      const uint32_t b_v = smem_u32(smem + kOffV + s * kTileBytes);
#pragma unroll
      for (int k = 0; k < kRows / 16; ++k) {  // 16 keys per MMA: chunk k / 4, 32 bytes apart in a row
        const uint32_t a_addr = a_p + static_cast<uint32_t>(k >> 2) * (kRows * 128u) + static_cast<uint32_t>(k & 3) * 32u;
        const uint32_t b_addr = b_v + static_cast<uint32_t>(k) * 1024u;  // 16 keys = two 8-key groups
        umma_f16(t_o + static_cast<uint32_t>(s) * kHead, smem_desc_kmajor(a_addr, 128), smem_desc_mn_sw64(b_addr),
                 id_o, k > 0 ? 1u : 0u);
      }
      umma_commit(&o_full[s]);
      umma_commit(&kv_empty[s]);  // K_i and V_i are no longer read
      return true;
    };
    bool ok = mbar_wait_bounded(q_full, 0, kErrWaitFull);
    for (int j = 0; ok && j < n_tiles && !*abort_flag; ++j) {
      const int s = j & 1;
      if (!mbar_wait_bounded(&kv_full[s], static_cast<uint32_t>(j >> 1) & 1u, kErrWaitFull)) { ok = false; break; }
      if (j >= 1 && !mbar_wait_bounded(s_free, static_cast<uint32_t>(j - 1) & 1u, kErrWaitAcc)) { ok = false; break; }
      tc_fence_after();
      const uint32_t b_k = smem_u32(smem + kOffK + s * kTileBytes);
#pragma unroll
      for (int k = 0; k < kHead / 16; ++k)
        umma_f16(t_s, smem_desc_kmajor(a_q + k * 32u, 64), smem_desc_kmajor(b_k + k * 32u, 64), id_s, k > 0 ? 1u : 0u);
      umma_commit(s_full);
      if (j >= 1 && !pv(j - 1)) { ok = false; break; }
    }
    if (ok && n_tiles > 0 && !pv(n_tiles - 1)) ok = false;
    if (!ok) *abort_flag = 1;
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax, one query row per thread
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const float scale = p.scale * 1.4426950408889634f;  // logits in base 2
    float m_prev = -INFINITY, m_cur = -INFINITY, l = 0.f;
    float acc[kHead];
#pragma unroll
    for (int i = 0; i < kHead; ++i) acc[i] = 0.f;
    bool ok = true;
    auto fold = [&](int i, float m_old, float m_new) -> bool {  // acc = acc * 2^(m_old - m_new) + PV_i
      const int s = i & 1;
      if (!mbar_wait_bounded(&o_full[s], static_cast<uint32_t>(i >> 1) & 1u, kErrWaitAcc)) return false;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32_issue(tmem + lane_addr + (t_o - tmem) + static_cast<uint32_t>(s) * kHead, r);
      tmem_ld32_wait(r);
      const float f = m_old == -INFINITY ? 0.f : fast_exp2(m_old - m_new);
#pragma unroll
      for (int c = 0; c < kHead; ++c) acc[c] = fmaf(acc[c], f, __uint_as_float(r[c]));
      tc_fence_before();
      mbar_arrive(&o_free[s]);
      return true;
    };
    for (int j = 0; j < n_tiles; ++j) {
      ok = mbar_wait_bounded(s_full, static_cast<uint32_t>(j) & 1u, kErrWaitAcc) && !*abort_flag;
      if (!ok) break;
      tc_fence_after();
      // Pass 1: the row maximum over the tile (two 32-column loads in flight per wait), in eight
      // independent running maxima so the comparisons do not form one serial chain.
      float mq[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) mq[q] = -INFINITY;
#pragma unroll
      for (int c = 0; c < kRows; c += 64) {
        uint32_t r[32], r2[32];
        tmem_ld32_issue(t_s + lane_addr + static_cast<uint32_t>(c), r);
        tmem_ld32_issue(t_s + lane_addr + static_cast<uint32_t>(c + 32), r2);
        tmem_ld32_wait(r);
        tmem_ld32_wait(r2);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          mq[i & 7] = fmaxf(mq[i & 7], fmaxf(__uint_as_float(r[i]), __uint_as_float(r2[i])));
      }
      const float mx = fmaxf(fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])),
                             fmaxf(fmaxf(mq[4], mq[5]), fmaxf(mq[6], mq[7])));
      const float m_new = fmaxf(m_cur, mx * scale);
      // Pass 2: P = 2^(s * scale - m_new) in the operand type, written swizzled.
      const int s = j & 1;
      uint8_t* prow = smem + kOffP + s * kPBytes + static_cast<size_t>(row) * 128;
      // The row sum in eight independent partial sums (no serial chain of 64 additions per chunk).
      float sq[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) sq[q] = 0.f;
#pragma unroll
      for (int c = 0; c < kRows; c += 32) {
        uint32_t r[32];
        tmem_ld32_issue(t_s + lane_addr + static_cast<uint32_t>(c), r);
        tmem_ld32_wait(r);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = fmaf(__uint_as_float(r[2 * i]), scale, -m_new);
          const float x1 = fmaf(__uint_as_float(r[2 * i + 1]), scale, -m_new);
          // Keys 24..31 of the 32 on the FMA pipe, the rest on the exponential unit.
          const float e0 = i >= 12 ? poly_exp2(x0) : fast_exp2(x0);
          const float e1 = i >= 12 ? poly_exp2(x1) : fast_exp2(x1);
          sq[i & 7] += e0 + e1;
          w[i] = pack2(e0, e1, BF16);
        }
        // Keys c .. c + 31: chunk c / 64, 16-byte units (c % 64) / 8 .. + 3, swizzled by row % 8.
        uint8_t* chunk = prow + static_cast<size_t>(c >> 6) * (kRows * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = (((c & 63) >> 3) + u) ^ (row & 7);
          *reinterpret_cast<uint4*>(chunk + unit * 16) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
        }
      }
      // S is read out: the next QK^T may overwrite it.
      tc_fence_before();
      mbar_arrive(s_free);
      // P_j is in shared memory: visible to the tensor core's async proxy, then published.
      fence_proxy_async_shared();
      mbar_arrive(&p_full[s]);
      const float sum = ((sq[0] + sq[1]) + (sq[2] + sq[3])) + ((sq[4] + sq[5]) + (sq[6] + sq[7]));
      l = (m_cur == -INFINITY ? 0.f : l * fast_exp2(m_cur - m_new)) + sum;
      // Fold PV_{j-1} (scale m_cur) while PV_j runs.
      if (j >= 1 && !fold(j - 1, m_prev, m_cur)) { ok = false; break; }
      m_prev = m_cur;
      m_cur = m_new;
    }
    if (ok && n_tiles > 0) ok = fold(n_tiles - 1, m_prev, m_cur);
    if (!ok) *abort_flag = 1;
    // Output row: acc / l.
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint32_t o[kHead / 2];
#pragma unroll
    for (int i = 0; i < kHead / 2; ++i) o[i] = pack2(acc[2 * i] * inv, acc[2 * i + 1] * inv, BF16);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) +
                                          (static_cast<long long>(b) * p.tokens + q0 + row) * C + h * kHead);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

size_t attention_d32_smem() { return kSmemBytes; }

cudaError_t launch_attention_d32(const CUtensorMap& map, const AttnParams& p, bool bf16, cudaStream_t stream) {
  if (p.tokens <= 0 || p.tokens % kRows != 0 || p.heads <= 0 || p.batch <= 0) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(p.tokens / kRows), static_cast<unsigned>(p.heads),
                  static_cast<unsigned>(p.batch));
  auto kern = bf16 ? attention_d32_kernel<true> : attention_d32_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
  if (e != cudaSuccess) return e;
  return launch_kernel(kern, grid, kAttnThreads, kSmemBytes, stream, map, p);
}

}  // namespace ctmr
