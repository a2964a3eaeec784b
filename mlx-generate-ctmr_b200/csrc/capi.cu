// The extern "C" boundary (include/ctmr_b200.h): argument validation, TMA
// descriptor encoding, tile planning and kernel dispatch. No call allocates
// device memory; every launch goes to the caller's stream.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ctmr_b200.h"
#include "conv3d_umma.cuh"
#include "groupnorm.cuh"
#include "conv3d_narrow.cuh"
#include "attention.cuh"
#include "conv3d_tiny.cuh"
#include "misc.cuh"
#include "pack.cuh"
#include "prepare.cuh"
#include "launch.cuh"

namespace ctmr {
int conv_stage_plan(int kc, int bn, bool exact, bool one_cta_per_sm, size_t* smem_bytes);
cudaError_t launch_conv3d_umma(const ConvMaps& maps, const ConvGeom& g, int kc, bool exact, size_t smem,
                               cudaStream_t stream);
int conv_v2_stage_plan(int kc, int mt, int tw, int bn, size_t* smem_bytes, size_t stats_bytes, bool exact);
cudaError_t launch_conv3d_umma_v2(const ConvMaps& maps, const ConvGeom& g, int kc, int mt, int tw, int sms,
                                  size_t smem, bool exact, cudaStream_t stream);
int conv_khcat_stage_plan(int kc, int bn, int mt, size_t* smem_bytes);
int conv_khcat_rows();
cudaError_t launch_conv3d_khcat(const ConvMaps& maps, const ConvGeom& g, int kc, int mt, int sms, size_t smem,
                                cudaStream_t stream);
int conv_khcat_pair_stage_plan(size_t* smem_bytes);
cudaError_t launch_conv3d_khcat_pair(const ConvMaps& maps, const ConvGeom& g, size_t smem, cudaStream_t stream);
extern __device__ unsigned int g_device_error;
}  // namespace ctmr

namespace {

thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CTMR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline long long round_up(long long v, long long a) { return (v + a - 1) / a * a; }
inline int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

CUtensorMapSwizzle swizzle_for(int kc) {
  return kc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : (kc == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// 5-D activation view (C, W, H, D, B) with byte strides for W/H/D/B.
int encode_act(CUtensorMap* map, const void* base, bool bf16, long long cpad, long long w, long long h, long long d,
               long long b, long long sw, long long sh, long long sd, long long sb, int kc, int tw, int th, int td) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CTMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(cpad), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(b)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(sw), static_cast<cuuint64_t>(sh), static_cast<cuuint64_t>(sd),
                           static_cast<cuuint64_t>(sb)};
  cuuint32_t box[5] = {static_cast<cuuint32_t>(kc), static_cast<cuuint32_t>(tw), static_cast<cuuint32_t>(th),
                       static_cast<cuuint32_t>(td), 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_for(kc), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTMR_ERR_INVALID, "activation tensor map rejected (CUresult %d)", int(r));
  return CTMR_OK;
}

int encode_weight(CUtensorMap* map, const void* base, bool bf16, long long cpad, long long opad, long long taps,
                  int kc, int bn) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CTMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cpad), static_cast<cuuint64_t>(opad),
                        static_cast<cuuint64_t>(taps)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cpad * 2), static_cast<cuuint64_t>(cpad * 2 * opad)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kc), static_cast<cuuint32_t>(bn), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_for(kc), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTMR_ERR_INVALID, "weight tensor map rejected (CUresult %d)", int(r));
  return CTMR_OK;
}

int encode_weight3(CUtensorMap* map, const void* base, bool bf16, long long cpad, long long opad, long long taps,
                   int kc, int bn, int box_taps) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CTMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cpad), static_cast<cuuint64_t>(opad),
                        static_cast<cuuint64_t>(taps)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cpad * 2), static_cast<cuuint64_t>(cpad * 2 * opad)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kc), static_cast<cuuint32_t>(bn), static_cast<cuuint32_t>(box_taps)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_for(kc), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTMR_ERR_INVALID, "weight tensor map rejected (CUresult %d)", int(r));
  return CTMR_OK;
}

// 5-D view (c, o, kw, kh, kd) of 3x3x3 packed weights [kd][kh][kw][O][C]: a box of
// (kc, box_o, 1, 3, 1) holds the three kh taps of one (kd, kw) as 3 x box_o rows (box_o = opad,
// or half of it for one CTA of a pair).
int encode_weight_kh(CUtensorMap* map, const void* base, bool bf16, long long cpad, long long opad, int kc,
                     long long box_o) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CTMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const long long tap = cpad * 2 * opad;
  cuuint64_t dims[5] = {static_cast<cuuint64_t>(cpad), static_cast<cuuint64_t>(opad), 3, 3, 3};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(cpad * 2), static_cast<cuuint64_t>(tap),
                           static_cast<cuuint64_t>(3 * tap), static_cast<cuuint64_t>(9 * tap)};
  cuuint32_t box[5] = {static_cast<cuuint32_t>(kc), static_cast<cuuint32_t>(box_o), 1, 3, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_for(kc), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTMR_ERR_INVALID, "weight tensor map rejected (CUresult %d)", int(r));
  return CTMR_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count() { return ctmr::device_sm_count(); }

constexpr long long kStatsMaxEntries = 512;  // batch x output channels with output statistics

int check_view(const ctmr_tensor& t, const char* name, bool required, bool labels_ok = false) {
  if (t.data == nullptr) {
    if (required) return fail(CTMR_ERR_INVALID, "%s is missing", name);
    return CTMR_OK;
  }
  if (t.dtype == CTMR_DTYPE_LABEL8) {
    if (!labels_ok) return fail(CTMR_ERR_INVALID, "%s cannot be a label volume", name);
    if (t.channels != 8 || t.cstride < 1) return fail(CTMR_ERR_INVALID, "%s label volume must be 8 channels", name);
    return CTMR_OK;
  }
  if (t.dtype != CTMR_DTYPE_F32 && t.dtype != CTMR_DTYPE_BF16) return fail(CTMR_ERR_INVALID, "%s dtype", name);
  if (t.channels <= 0 || t.cstride < t.channels) return fail(CTMR_ERR_INVALID, "%s channels/cstride", name);
  return CTMR_OK;
}

ctmr::PrepSource as_source(const ctmr_tensor& t) {
  ctmr::PrepSource s{};
  if (t.data != nullptr) {
    s.ptr = t.data;
    s.bf16 = t.dtype == CTMR_DTYPE_BF16 ? 1 : (t.dtype == CTMR_DTYPE_LABEL8 ? 2 : 0);
    s.channels = t.channels;
    s.cstride = t.cstride;
  }
  return s;
}

// Everything derived from a conv descriptor before any launch.
struct ConvPlan {
  int mode;
  int cin, cpad, opad, kc, bn, taps, phases;
  int in_d, in_h, in_w;     // grid the taps read (after trilinear / avgpool)
  int row_d, row_h, row_w;  // GEMM rows
  int out_d, out_h, out_w;
  bool exact, prepare, bf16, narrow;
  bool tf32;                // TF32 operands: fp32 rows, channel counts below in 16-bit units (2 per value)
  bool tiny;                // fp32 conv of <= 4 input channels: direct FMA kernel
  bool im2col;              // tiny-input 3x3x3 conv run as a 1x1x1 conv of its im2col rows
  int cin_raw, cpad_src;    // im2col: input channels and the packed weights' channel padding
  size_t prep_bytes;        // per plane
  size_t wrep_bytes;        // im2col: repacked weights, per plane
  bool gn_in;               // the call computes the input's GroupNorm itself
  bool gn_small;            // ... in the fused small-tensor operand kernel
  size_t gn_bytes;          // workspace for the affine [+ statistics partials] otherwise
  int gn_chunks;
  // per-tap kernel tiling and its split-K
  int tile_w, tile_h, tile_d, tiles_w, tiles_h, tiles_d, n_tiles, ksplit;
  size_t part_bytes;
  size_t workspace() const { return (prep_bytes + wrep_bytes) * (exact ? 2 : 1) + part_bytes + gn_bytes; }
  size_t gn_offset() const { return (prep_bytes + wrep_bytes) * (exact ? 2 : 1) + part_bytes; }
};

int plan_conv(const ctmr_conv3d_desc* d, ConvPlan* p) {
  if (d == nullptr) return fail(CTMR_ERR_INVALID, "null descriptor");
  if (d->batch <= 0 || d->depth <= 0 || d->height <= 0 || d->width <= 0)
    return fail(CTMR_ERR_INVALID, "grid must be positive");
  int st = check_view(d->x, "x", true, true);
  if (st) return st;
  if ((st = check_view(d->x2, "x2", false))) return st;
  if ((st = check_view(d->residual, "residual", false))) return st;
  if (d->x.dtype == CTMR_DTYPE_LABEL8 &&
      (d->x2.data != nullptr || d->trilinear || d->avgpool || d->upsample || d->stride != 1 || d->gn_groups > 0))
    return fail(CTMR_ERR_UNSUPPORTED, "a label volume input takes no x2, resampling, stride or in-call GroupNorm");
  if (d->precision != CTMR_PRECISION_FP32 && d->precision != CTMR_PRECISION_BF16 &&
      d->precision != CTMR_PRECISION_FP16 && d->precision != CTMR_PRECISION_TF32)
    return fail(CTMR_ERR_INVALID, "precision");
  if (d->out_channels <= 0) return fail(CTMR_ERR_INVALID, "out_channels");
  if (d->bias_row_stride != 0 && (d->bias_row_stride < d->out_channels || d->bias_row_stride > (1LL << 30)))
    return fail(CTMR_ERR_INVALID, "bias_row_stride %lld must be 0 or in [out_channels, 2^30]", d->bias_row_stride);
  if (d->weight == nullptr || (d->precision == CTMR_PRECISION_FP32 && d->weight_lo == nullptr))
    return fail(CTMR_ERR_INVALID, "packed weight missing");
  if (d->y == nullptr || (d->y_dtype != CTMR_DTYPE_F32 && d->y_dtype != CTMR_DTYPE_BF16))
    return fail(CTMR_ERR_INVALID, "output");
  if (d->y_coffset < 0 || d->y_cstride < d->y_coffset + d->out_channels)
    return fail(CTMR_ERR_INVALID, "output cstride %lld too small for offset %d + %d channels", d->y_cstride,
                d->y_coffset, d->out_channels);
  const int specials = (d->upsample != 0) + (d->trilinear != 0) + (d->avgpool != 0) + (d->stride == 2);
  if (specials > 1) return fail(CTMR_ERR_UNSUPPORTED, "upsample, trilinear, avgpool and stride 2 are exclusive");
  if (d->kernel_size == 1 && (d->upsample || d->stride != 1))
    return fail(CTMR_ERR_UNSUPPORTED, "1x1x1 convolutions support stride 1 only");
  if (d->kernel_size != 1 && d->kernel_size != 3) return fail(CTMR_ERR_UNSUPPORTED, "kernel_size must be 1 or 3");
  if (d->stride != 1 && d->stride != 2) return fail(CTMR_ERR_UNSUPPORTED, "stride must be 1 or 2");
  if (d->trilinear && (d->affine != nullptr || d->silu || d->gn_groups > 0))
    return fail(CTMR_ERR_UNSUPPORTED, "trilinear packing supports only a plain convolution");
  if (d->avgpool && (d->depth % 2 || d->height % 2 || d->width % 2))
    return fail(CTMR_ERR_INVALID, "average pooling needs even extents");
  if (d->stride == 2 && (d->depth < 2 || d->height < 2 || d->width < 2))
    return fail(CTMR_ERR_UNSUPPORTED, "stride-2 convolution needs extents >= 2");

  if (d->gn_groups < 0 || (d->gn_groups > 0 && d->affine != nullptr))
    return fail(CTMR_ERR_INVALID, "pass either an input affine or gn_groups, not both");
  p->exact = d->precision == CTMR_PRECISION_FP32;
  p->bf16 = d->precision == CTMR_PRECISION_BF16;
  p->tf32 = d->precision == CTMR_PRECISION_TF32;
  p->cin = d->x.channels + (d->x2.data ? d->x2.channels : 0);
  // Operand rows in 16-bit units: 16 values (one 32-byte MMA K step) or, for TF32, 8 fp32 values.
  p->cpad = p->tf32 ? 2 * static_cast<int>(round_up(p->cin, 8)) : static_cast<int>(round_up(p->cin, 16));
  p->opad = static_cast<int>(round_up(d->out_channels, 16));
  p->kc = p->cpad % 64 == 0 ? 64 : (p->cpad % 32 == 0 ? 32 : 16);
  p->bn = std::min(p->opad, 128);
  p->in_d = d->depth, p->in_h = d->height, p->in_w = d->width;
  if (d->trilinear) p->in_d *= 2, p->in_h *= 2, p->in_w *= 2;
  if (d->avgpool) p->in_d /= 2, p->in_h /= 2, p->in_w /= 2;
  p->phases = 1;
  if (d->upsample) {
    if (d->kernel_size != 3) return fail(CTMR_ERR_UNSUPPORTED, "upsample needs a 3x3x3 kernel");
    p->mode = ctmr::kModeUp2;
    p->taps = 8;
    p->phases = 8;
    p->row_d = p->in_d, p->row_h = p->in_h, p->row_w = p->in_w;
    p->out_d = 2 * p->in_d, p->out_h = 2 * p->in_h, p->out_w = 2 * p->in_w;
  } else if (d->kernel_size == 1) {
    p->mode = ctmr::kModeConv1;
    p->taps = 1;
    p->row_d = p->out_d = p->in_d, p->row_h = p->out_h = p->in_h, p->row_w = p->out_w = p->in_w;
  } else if (d->stride == 2) {
    p->mode = ctmr::kModeStride2;
    p->taps = 27;
    p->row_d = p->out_d = (p->in_d - 1) / 2 + 1;
    p->row_h = p->out_h = (p->in_h - 1) / 2 + 1;
    p->row_w = p->out_w = (p->in_w - 1) / 2 + 1;
  } else {
    p->mode = ctmr::kModeConv3;
    p->taps = 27;
    p->row_d = p->out_d = p->in_d, p->row_h = p->out_h = p->in_h, p->row_w = p->out_w = p->in_w;
  }
  // The raw input can be the MMA operand directly only in bf16 mode, with no
  // transform, 16-channel granularity and 16-byte aligned rows.
  const bool direct = p->bf16 && d->x2.data == nullptr && d->affine == nullptr && d->gn_groups == 0 && !d->silu &&
                      !d->trilinear &&
                      !d->avgpool && d->x.dtype == CTMR_DTYPE_BF16 && d->x.channels % 16 == 0 &&
                      d->x.cstride % 8 == 0 && aligned16(d->x.data);
  // Narrow outputs (<= 4 channels, e.g. the UNet / VAE output convolutions) with split-fp32
  // weights and an fp32 input run the direct fp32 kernel, which normalises while staging.
  p->narrow = p->exact && p->mode == ctmr::kModeConv3 && !d->trilinear && !d->avgpool && d->out_channels <= 4 &&
              d->x2.data == nullptr &&
              d->x.dtype == CTMR_DTYPE_F32 && (d->residual.data == nullptr || d->residual.dtype == CTMR_DTYPE_F32) &&
              d->y_dtype == CTMR_DTYPE_F32 && ctmr::narrow_conv_supported(p->cin, d->out_channels) &&
              getenv("CTMR_DISABLE_NARROW") == nullptr;
  // Inputs of at most 4 channels (the UNet / ControlNet / VAE conv_in on the 4-channel latent):
  // im2col rows of 27 * C columns instead of 27 taps of 16 mostly-zero channels.
  // In the fp32 mode they run a direct FMA kernel (108 products per output need no tensor cores).
  p->tiny = !p->narrow && p->exact && p->mode == ctmr::kModeConv3 && p->cin <= 4 && !d->trilinear && !d->avgpool &&
            d->x2.data == nullptr && d->x.dtype == CTMR_DTYPE_F32 &&
            (d->residual.data == nullptr || (d->residual.dtype == CTMR_DTYPE_F32 && !d->residual_upsampled)) &&
            d->y_dtype == CTMR_DTYPE_F32 && getenv("CTMR_DISABLE_TINY") == nullptr;
  p->im2col = !p->narrow && !p->tiny && !p->tf32 && p->mode == ctmr::kModeConv3 && p->cin <= 4 && !d->trilinear &&
              !d->avgpool && d->x2.data == nullptr && getenv("CTMR_DISABLE_IM2COL") == nullptr;
  p->cin_raw = p->cin;
  p->cpad_src = p->cpad;
  p->wrep_bytes = 0;
  if (p->im2col) {
    p->mode = ctmr::kModeConv1;
    p->taps = 1;
    p->cpad = static_cast<int>(round_up(27 * p->cin, 16));
    p->kc = p->cpad % 64 == 0 ? 64 : (p->cpad % 32 == 0 ? 32 : 16);
    p->wrep_bytes = static_cast<size_t>(round_up(static_cast<long long>(p->opad) * p->cpad * 2, 256));
  }
  p->prepare = (!direct || p->im2col) && !p->narrow && !p->tiny;
  p->prep_bytes = p->prepare ? static_cast<size_t>(round_up(static_cast<long long>(d->batch) * p->in_d * p->in_h *
                                                                p->in_w * p->cpad * 2,
                                                            256))
                             : 0;
  if (d->residual.data != nullptr) {
    if (d->residual.channels < d->out_channels)
      return fail(CTMR_ERR_INVALID, "residual has %d channels, output %d", d->residual.channels, d->out_channels);
  }
  // Per-tap kernel: a 128-voxel box over the GEMM rows, w fastest.
  p->tile_w = std::min(next_pow2(p->row_w), 128);
  p->tile_h = std::min(next_pow2(p->row_h), 128 / p->tile_w);
  p->tile_d = 128 / (p->tile_w * p->tile_h);
  p->tiles_w = (p->row_w + p->tile_w - 1) / p->tile_w;
  p->tiles_h = (p->row_h + p->tile_h - 1) / p->tile_h;
  p->tiles_d = (p->row_d + p->tile_d - 1) / p->tile_d;
  p->n_tiles = (p->opad + p->bn - 1) / p->bn;
  // Split K over the grid's z when the tiles alone cannot fill the GPU (the deep,
  // small grids): about 2 CTAs per SM, at least 4 K iterations per split.
  const long long ctas = static_cast<long long>(p->tiles_w) * p->tiles_h * p->tiles_d * d->batch * p->phases *
                         p->n_tiles;
  const int n_iter = p->taps * (p->cpad / p->kc);
  p->ksplit = 1;
  // Resident CTAs per SM of the per-tap kernel (its shared-memory plan; a TMEM
  // footprint above 256 columns forces one), so that the split grid is one wave.
  size_t smem_probe = 0;
  const int tcols = std::max(32, next_pow2(p->bn * (p->exact ? 3 : 1)));
  const int stages_probe = ctmr::conv_stage_plan(p->kc, p->bn, p->exact, tcols > 256, &smem_probe);
  const int per_sm = (stages_probe >= 2 && smem_probe + 1024 <= 114 * 1024) ? 2 : 1;
  const long long sms = sm_count();
  const long long wave = sms * per_sm;
  if (p->mode != ctmr::kModeUp2 && ctas < sms) {
    long long want = wave / ctas;  // whole splits per wave: no second, nearly empty wave
    want = std::min<long long>(want, n_iter / 4);
    if (want >= 2) p->ksplit = static_cast<int>(want);
  }
  p->part_bytes = p->ksplit > 1 ? static_cast<size_t>(p->ksplit) * d->batch * p->row_d * p->row_h * p->row_w *
                                      p->n_tiles * p->bn * sizeof(float)
                                : 0;
  p->part_bytes = static_cast<size_t>(round_up(static_cast<long long>(p->part_bytes), 256));
  if (p->narrow || p->tiny) p->part_bytes = 0;
  // GroupNorm of the input inside the call.
  p->gn_in = d->gn_groups > 0;
  p->gn_small = false;
  p->gn_bytes = 0;
  p->gn_chunks = 0;
  if (p->gn_in) {
    const long long voxels = static_cast<long long>(d->depth) * d->height * d->width;
    if (p->cin % d->gn_groups != 0) return fail(CTMR_ERR_INVALID, "gn_groups must divide the input channels");
    if (p->cin > 2048) return fail(CTMR_ERR_UNSUPPORTED, "group_norm supports at most 2048 channels");
    p->gn_small = p->prepare && !p->im2col && !p->tf32 && !d->trilinear && !d->avgpool &&
                  ctmr::gn_prepare_small_fits(voxels, p->cin, d->gn_groups) &&
                  getenv("CTMR_GN_FUSED") != nullptr;  // opt-in: slower in the MAISI UNet step (6.39 vs 6.26 ms)
    if (!p->gn_small) {
      p->gn_chunks = ctmr::gn_chunks_for(d->batch, voxels, p->cin);
      p->gn_bytes = static_cast<size_t>(round_up(static_cast<long long>(d->batch) * p->cin * 2 * 4, 256)) +
                    static_cast<size_t>(d->batch) * ctmr::gn_max_chunks(d->batch) * d->gn_groups * 3 * sizeof(float);
    }
  }
  return CTMR_OK;
}


// The persistent kernel's plan for a convolution, or false when it does not apply.
struct V2Plan {
  int kc, mt, tw, bn, stages;
  size_t smem, stats_bytes;
};

// Elements between the per-batch bias rows (0 for a per-channel bias).
int bias_row_stride(const ctmr_conv3d_desc* d) {
  if (!d->bias_per_batch) return 0;
  return static_cast<int>(d->bias_row_stride > 0 ? d->bias_row_stride : d->out_channels);
}

struct KhPlan {
  int kc, mt, stages;
  size_t smem;
};

// The kh-concatenated kernel: 16-bit stride-1 3x3x3 convolutions with at most 64
// output channels (three taps side by side fill an N = 3 x C_out MMA). With output
// statistics (four slots per CTA): 64 output columns and 16-bit operands only.
bool plan_khcat(const ConvPlan& p, const ctmr_conv3d_desc* d, bool with_stats, KhPlan* k) {
  if (p.exact || p.mode != ctmr::kModeConv3 || p.opad > 64 || (with_stats && (p.opad != 64 || p.tf32)) ||
      p.row_w < 8 || p.row_h < 8 || getenv("CTMR_DISABLE_KHCAT") != nullptr)
    return false;
  // Two depth tiles share each weight box (measured faster than one depth with two accumulator
  // buffers); CTMR_KHCAT_MT=1 selects the latter.
  const char* mt_env = getenv("CTMR_KHCAT_MT");
  k->mt = mt_env != nullptr && mt_env[0] == '1' ? 1 : 2;
  if (p.row_d < 2) k->mt = 1;
  for (int min_stages : {3, 2}) {
    for (int cand : {64, 32, 16}) {
      size_t sm_b = 0;
      const int st = p.cpad % cand ? 0 : ctmr::conv_khcat_stage_plan(cand, p.opad, k->mt, &sm_b);
      if (st >= min_stages) {
        k->kc = cand, k->smem = sm_b, k->stages = st;
        return true;
      }
    }
  }
  return false;
}

// Whether the kh-concatenated kernel converts its own operand (GroupNorm affine, SiLU and the
// 16-bit rounding in four converter warps) instead of the separate operand pass writing a 16-bit
// copy that the kernel then loads: CTMR_KHCAT_FUSE=1 / 0 forces it on / off.
constexpr bool kKhcatFuseDefault = false;
bool khcat_fuse_enabled() {
  const char* e = getenv("CTMR_KHCAT_FUSE");
  if (e != nullptr && e[0] != '\0') return e[0] == '1';
  return kKhcatFuseDefault;
}

// The fused route's conditions: a stride-1 3x3x3 conv in a 16-bit mode on the kh-concatenated
// kernel with 64-channel blocks, whose operand is a plain copy (optionally affine + SiLU) of fp32
// sources of whole 64-channel blocks with 16-byte aligned 4-channel pieces.
bool khcat_fusable(const ConvPlan& p, const ctmr_conv3d_desc* d, const KhPlan& kh, const float* affine) {
  if (!khcat_fuse_enabled() || kh.kc != 64 || !p.prepare || p.im2col || p.exact || p.tf32 || p.gn_small ||
      p.mode != ctmr::kModeConv3 || d->trilinear || d->avgpool || p.cin % 64 != 0 || p.cpad != p.cin)
    return false;
  if (d->x.dtype != CTMR_DTYPE_F32 || d->x.cstride % 4 != 0 || !aligned16(d->x.data)) return false;
  if (d->x2.data != nullptr && (d->x2.dtype != CTMR_DTYPE_F32 || d->x.channels % 64 != 0 ||
                                d->x2.cstride % 4 != 0 || !aligned16(d->x2.data)))
    return false;
  if (affine != nullptr && !aligned16(affine)) return false;
  // The converter warps read the sources while the epilogue writes the output: no overlap (the
  // operand pass would have read them in a launch of its own).
  const long long rows = static_cast<long long>(d->batch) * d->depth * d->height * d->width;
  const long long out_rows = static_cast<long long>(d->batch) * p.out_d * p.out_h * p.out_w;
  const size_t y_bytes = static_cast<size_t>(((out_rows - 1) * d->y_cstride + d->y_coffset + d->out_channels) *
                                             (d->y_dtype == CTMR_DTYPE_BF16 ? 2 : 4));
  const auto overlaps_y = [&](const ctmr_tensor& t) {
    const size_t t_bytes = static_cast<size_t>(((rows - 1) * t.cstride + t.channels) * 4);
    const uintptr_t a = reinterpret_cast<uintptr_t>(t.data), y = reinterpret_cast<uintptr_t>(d->y);
    return a < y + y_bytes && y < a + t_bytes;
  };
  if (overlaps_y(d->x) || (d->x2.data != nullptr && overlaps_y(d->x2))) return false;
  const long long total = static_cast<long long>((p.row_w + 7) / 8) *
                          ((p.row_h + ctmr::conv_khcat_rows() - 1) / ctmr::conv_khcat_rows()) *
                          ((p.row_d + kh.mt - 1) / kh.mt) * d->batch;
  return total > 0 && total < (1LL << 31);
}

bool plan_v2(const ConvPlan& p, const ctmr_conv3d_desc* d, bool with_stats, V2Plan* v) {
  if ((p.exact && with_stats) ||
      !(p.mode == ctmr::kModeConv3 || p.mode == ctmr::kModeUp2 || p.mode == ctmr::kModeConv1) || p.row_w < 16 ||
      p.row_h < 8 || getenv("CTMR_DISABLE_V2") != nullptr)
    return false;
  v->tw = p.mode == ctmr::kModeConv3 ? 3 : (p.mode == ctmr::kModeUp2 ? 2 : 1);
  // Two depth tiles share each weight box of a 3x3x3 or folded conv. A 1x1x1 conv into <= 64
  // channels has one short K walk and a short epilogue per tile, where one depth per tile drains
  // and refills faster (measured: 2 x 128 -> 64 at 64 x 64 x 32 54 -> 41 us, 1 x 128 -> 64 at
  // 96 x 256 x 128 549 -> 389 us; 1 x 256 -> 128 at 48 x 128 x 64 130 -> 135 us, so not above 64).
  v->mt = p.row_d >= 2 && !(p.mode == ctmr::kModeConv1 && p.opad <= 64) ? 2 : 1;
  // The fp32 split mode: one depth per tile, so that two hi chunk buffers and a double-buffered lo
  // accumulator (4 x bn columns) fit TMEM. On grids of fewer tiles than half the SMs the per-tap
  // kernel's split-K fills the GPU better (measured: 64 tiles 1.2-1.8x slower here, 128 tiles 1.3x faster).
  if (p.exact) {
    v->mt = 1;
    const long long tiles = static_cast<long long>((p.opad + std::min(p.opad, 128) - 1) / std::min(p.opad, 128)) *
                            ((p.row_w + 15) / 16) * ((p.row_h + 7) / 8) * p.row_d * d->batch * p.phases;
    if (2 * tiles < sm_count()) return false;
  }
  v->bn = std::min(p.opad, 128);
  v->stats_bytes = 0;
  if (with_stats) {
    if (p.tf32) return false;  // no TF32 instantiation with the statistics epilogue
    // Below 128 output channels the MMA work per tile is too short to hide the
    // statistics reduction in the epilogue; a separate pass is cheaper there.
    if (d->out_channels < 128) return false;
    // One (count, mean, M2) accumulator per epilogue warp for every (batch item, channel).
    if (static_cast<long long>(d->batch) * d->out_channels > kStatsMaxEntries) return false;
    v->stats_bytes = static_cast<size_t>(4) * d->batch * d->out_channels * 3 * sizeof(float);
  }
  // Largest channel block that fits a two-stage pipeline: fewer, larger stages
  // beat a deeper pipeline of small ones (each stage costs a barrier round trip;
  // measured 1104 -> 1228 TFLOP/s on 128 -> 128 channels with 64- instead of
  // 32-channel blocks at 2 instead of 5 stages).
  for (int min_stages : {2}) {
    for (int cand : {64, 32, 16}) {
      size_t sm_b = 0;
      const int st =
          p.cpad % cand ? 0 : ctmr::conv_v2_stage_plan(cand, v->mt, v->tw, v->bn, &sm_b, v->stats_bytes, p.exact);
      if (st >= min_stages) {
        v->kc = cand, v->smem = sm_b, v->stages = st;
        return true;
      }
    }
  }
  return false;
}
}  // namespace

namespace ctmr {
// Records `message` as this thread's ctmr_last_error() and returns `status`.
int set_last_error(int status, const char* message) { return fail(status, "%s", message); }
}  // namespace ctmr

extern "C" {

const char* ctmr_status_string(int status) {
  switch (status) {
    case CTMR_OK: return "ok";
    case CTMR_ERR_INVALID: return "invalid argument";
    case CTMR_ERR_UNSUPPORTED: return "unsupported configuration";
    case CTMR_ERR_WORKSPACE: return "workspace too small";
    case CTMR_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* ctmr_last_error(void) { return g_last_error; }

size_t ctmr_packed_weight_elems(int out_channels, int in_channels, int kernel_size, int upsample) {
  if (out_channels <= 0 || in_channels <= 0 || (kernel_size != 1 && kernel_size != 3)) return 0;
  const long long taps = upsample ? 64 : static_cast<long long>(kernel_size) * kernel_size * kernel_size;
  return static_cast<size_t>(taps * round_up(out_channels, 16) * round_up(in_channels, 16));
}

size_t ctmr_packed_weight_bytes(int out_channels, int in_channels, int kernel_size, int upsample, int precision) {
  if (precision == CTMR_PRECISION_TF32) {
    if (out_channels <= 0 || in_channels <= 0 || (kernel_size != 1 && kernel_size != 3)) return 0;
    const long long taps = upsample ? 64 : static_cast<long long>(kernel_size) * kernel_size * kernel_size;
    return static_cast<size_t>(taps * round_up(out_channels, 16) * round_up(in_channels, 8) * 4);
  }
  if (precision != CTMR_PRECISION_FP32 && precision != CTMR_PRECISION_BF16 && precision != CTMR_PRECISION_FP16)
    return 0;
  return 2 * ctmr_packed_weight_elems(out_channels, in_channels, kernel_size, upsample);
}

namespace {
int pack_weight_any(const float* weight, int out_channels, int in_channels, int kernel_size, int upsample,
                    int precision, void* packed, void* packed_lo, void* stream, int channels_last) {
  if (weight == nullptr || packed == nullptr) return fail(CTMR_ERR_INVALID, "null weight pointer");
  if (out_channels <= 0 || in_channels <= 0) return fail(CTMR_ERR_INVALID, "channel counts");
  if (kernel_size != 1 && kernel_size != 3) return fail(CTMR_ERR_UNSUPPORTED, "kernel_size must be 1 or 3");
  if (upsample && kernel_size != 3) return fail(CTMR_ERR_UNSUPPORTED, "upsample fold needs a 3x3x3 kernel");
  if (precision != CTMR_PRECISION_FP32 && precision != CTMR_PRECISION_BF16 && precision != CTMR_PRECISION_FP16 &&
      precision != CTMR_PRECISION_TF32)
    return fail(CTMR_ERR_INVALID, "precision");
  const bool split = precision == CTMR_PRECISION_FP32;
  if (split && packed_lo == nullptr) return fail(CTMR_ERR_INVALID, "lo plane missing");
  const bool tf32 = precision == CTMR_PRECISION_TF32;
  const int kind = split ? ctmr::kPackSplitF16
                         : (tf32 ? ctmr::kPackTF32 : (precision == CTMR_PRECISION_BF16 ? ctmr::kPackBF16 : ctmr::kPackF16));
  cudaError_t e = ctmr::launch_pack_weight(weight, out_channels, in_channels, kernel_size, upsample,
                                           static_cast<int>(round_up(out_channels, 16)),
                                           static_cast<int>(round_up(in_channels, tf32 ? 8 : 16)), kind, packed,
                                           packed_lo, static_cast<cudaStream_t>(stream), channels_last);
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "pack_weight launch");
}
}  // namespace

int ctmr_attention_d32(const void* qkv, int dtype, int batch, int tokens, int heads, float scale, void* out,
                       void* stream) {
  if (qkv == nullptr || out == nullptr) return fail(CTMR_ERR_INVALID, "null attention pointer");
  if (dtype != CTMR_DTYPE_BF16 && dtype != CTMR_DTYPE_F16) return fail(CTMR_ERR_INVALID, "attention dtype");
  if (batch <= 0 || heads <= 0 || tokens <= 0) return fail(CTMR_ERR_INVALID, "attention extents");
  if (tokens % 128 != 0) return fail(CTMR_ERR_UNSUPPORTED, "attention tokens must be a multiple of 128");
  if (!aligned16(qkv) || !aligned16(out)) return fail(CTMR_ERR_INVALID, "attention pointers must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(CTMR_ERR_INVALID, "attention scale must be positive");
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CTMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const long long c3 = 3LL * heads * 32;
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(c3), static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(c3 * 2), static_cast<cuuint64_t>(c3 * 2 * tokens)};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&map, dtype == CTMR_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   3, const_cast<void*>(qkv), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CTMR_ERR_INVALID, "attention tensor map rejected (CUresult %d)", int(r));
  ctmr::AttnParams p{};
  p.batch = batch, p.tokens = tokens, p.heads = heads, p.scale = scale, p.out = out;
  cudaError_t e = ctmr::launch_attention_d32(map, p, dtype == CTMR_DTYPE_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "attention launch");
}

int ctmr_pack_weight(const float* weight, int out_channels, int in_channels, int kernel_size, int upsample,
                     int precision, void* packed, void* packed_lo, void* stream) {
  return pack_weight_any(weight, out_channels, in_channels, kernel_size, upsample, precision, packed, packed_lo,
                         stream, 0);
}

int ctmr_pack_weight_channels_last(const float* weight, int out_channels, int in_channels, int kernel_size,
                                   int upsample, int precision, void* packed, void* packed_lo, void* stream) {
  return pack_weight_any(weight, out_channels, in_channels, kernel_size, upsample, precision, packed, packed_lo,
                         stream, 1);
}

size_t ctmr_conv3d_workspace_size(const ctmr_conv3d_desc* desc) {
  ConvPlan p{};
  if (plan_conv(desc, &p) != CTMR_OK) return 0;
  return p.workspace();
}

int ctmr_conv3d(const ctmr_conv3d_desc* d, void* workspace, size_t workspace_bytes, void* stream_ptr) {
  return ctmr_conv3d_stages(d, workspace, workspace_bytes, CTMR_CONV_PREPARE | CTMR_CONV_GEMM, stream_ptr);
}

int ctmr_conv3d_stages(const ctmr_conv3d_desc* d, void* workspace, size_t workspace_bytes, int stages,
                       void* stream_ptr) {
  if ((stages & ~(CTMR_CONV_PREPARE | CTMR_CONV_GEMM)) != 0 || stages == 0)
    return fail(CTMR_ERR_INVALID, "stages must combine CTMR_CONV_PREPARE and CTMR_CONV_GEMM");
  ConvPlan p{};
  int st = plan_conv(d, &p);
  if (st != CTMR_OK) return st;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const size_t need = p.workspace();
  if (need > workspace_bytes || (need > 0 && workspace == nullptr))
    return fail(CTMR_ERR_WORKSPACE, "conv3d needs %zu workspace bytes, got %zu", need, workspace_bytes);
  if (d->stats != nullptr && (p.narrow || p.tiny))
    return fail(CTMR_ERR_UNSUPPORTED, "output statistics need the persistent kernel (ctmr_conv3d_stats_slots)");
  // GroupNorm of the input inside the call: the statistics pass writes the affine
  // into the workspace (the fused small-tensor operand kernel needs none).
  const float* affine = d->affine;
  if (p.gn_in && !p.gn_small) {
    float* gn_affine = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.gn_offset());
    affine = gn_affine;
    if (stages & CTMR_CONV_PREPARE) {
      ctmr::GnParams gp{};
      gp.src[0] = as_source(d->x);
      gp.src[1] = as_source(d->x2);
      gp.batch = d->batch;
      gp.voxels = static_cast<long long>(d->depth) * d->height * d->width;
      gp.groups = d->gn_groups;
      gp.eps = d->gn_eps;
      gp.gamma = d->gn_gamma;
      gp.beta = d->gn_beta;
      gp.affine = gn_affine;
      gp.partials = gn_affine + round_up(static_cast<long long>(d->batch) * p.cin * 2, 64);
      gp.chunks = p.gn_chunks;
      cudaError_t e = ctmr::launch_group_norm_affine(gp, stream);
      if (e != cudaSuccess) return cuda_fail(e, "group_norm launch");
    }
  }

  if (p.narrow) {
    if (!(stages & CTMR_CONV_GEMM)) return CTMR_OK;
    ctmr::NarrowParams np{};
    np.x = d->x.data;
    np.x_cstride = d->x.cstride;
    np.vec4 = (d->x.cstride % 4 == 0) && (reinterpret_cast<uintptr_t>(d->x.data) % 16 == 0);
    np.batch = d->batch, np.d = d->depth, np.h = d->height, np.w = d->width;
    np.cin = p.cin, np.cout = d->out_channels;
    np.affine = affine;
    np.silu = d->silu;
    np.w_hi = static_cast<const __half*>(d->weight);
    np.w_lo = static_cast<const __half*>(d->weight_lo);
    np.opad = p.opad, np.cpad = p.cpad;
    np.bias = d->bias;
    np.bias_bstride = bias_row_stride(d);
    np.res = static_cast<const float*>(d->residual.data);
    np.res_cstride = d->residual.cstride;
    np.res_up = d->residual_upsampled;
    np.y = static_cast<float*>(d->y) + d->y_coffset;
    np.y_cstride = d->y_cstride;
    cudaError_t e = ctmr::launch_narrow_conv(np, stream);
    return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "narrow conv launch");
  }
  if (p.tiny) {
    if (!(stages & CTMR_CONV_GEMM)) return CTMR_OK;
    ctmr::TinyParams tp{};
    tp.x = d->x.data;
    tp.x_cstride = d->x.cstride;
    tp.vec4 = (d->x.cstride % 4 == 0) && (reinterpret_cast<uintptr_t>(d->x.data) % 16 == 0);
    tp.batch = d->batch, tp.d = d->depth, tp.h = d->height, tp.w = d->width;
    tp.cin = p.cin, tp.cout = d->out_channels;
    tp.affine = affine;
    tp.silu = d->silu;
    tp.w_hi = static_cast<const __half*>(d->weight);
    tp.w_lo = static_cast<const __half*>(d->weight_lo);
    tp.opad = p.opad, tp.cpad = p.cpad;
    tp.bias = d->bias;
    tp.bias_bstride = bias_row_stride(d);
    tp.res = static_cast<const float*>(d->residual.data);
    tp.res_cstride = d->residual.cstride;
    tp.y = static_cast<float*>(d->y) + d->y_coffset;
    tp.y_cstride = d->y_cstride;
    cudaError_t e = ctmr::launch_tiny_conv(tp, stream);
    return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "tiny-input conv launch");
  }

  // The kh-concatenated kernel's plan; with converter warps it reads the fp32 input itself and the
  // operand pass below is skipped (decided here, once its weight tensor map is known to encode).
  const bool with_stats = d->stats != nullptr;
  V2Plan v2{};
  KhPlan kh{};
  const bool kh_ok = plan_khcat(p, d, with_stats, &kh);
  ctmr::ConvMaps fuse_maps;
  bool fuse = false;
  if (kh_ok && khcat_fusable(p, d, kh, affine)) {
    std::memset(&fuse_maps, 0, sizeof(fuse_maps));
    fuse = encode_weight_kh(&fuse_maps.b, d->weight, p.bf16, p.cpad, p.opad, kh.kc, p.opad) == CTMR_OK;
  }

  // 1. Operand preparation (affine, SiLU, trilinear / avgpool, concat, cast or split).
  const void* a_hi = d->x.data;
  const void* a_lo = nullptr;
  long long a_cstride = d->x.cstride;
  if (p.prepare) {
    a_hi = workspace;
    a_lo = p.exact ? static_cast<uint8_t*>(workspace) + p.prep_bytes : nullptr;
    a_cstride = p.cpad;
  }
  // im2col: repacked weights after the prepared planes.
  const void* w_hi = d->weight;
  const void* w_lo = d->weight_lo;
  if (p.im2col) {
    uint8_t* wr = static_cast<uint8_t*>(workspace) + p.prep_bytes * (p.exact ? 2 : 1);
    w_hi = wr;
    w_lo = p.exact ? wr + p.wrep_bytes : nullptr;
  }
  if (p.im2col && (stages & CTMR_CONV_PREPARE)) {
    ctmr::PrepParams pp{};
    pp.src[0] = as_source(d->x);
    pp.batch = d->batch;
    pp.sd = pp.od = d->depth, pp.sh = pp.oh = d->height, pp.sw = pp.ow = d->width;
    pp.affine = affine;
    pp.silu = d->silu;
    pp.cpad = p.cpad;
    pp.out_cstride = p.cpad;
    pp.out_kind = p.exact ? ctmr::kPrepOutSplitF16 : (p.bf16 ? ctmr::kPrepOutBF16 : ctmr::kPrepOutF16);
    pp.out = workspace;
    pp.out_lo = p.exact ? static_cast<uint8_t*>(workspace) + p.prep_bytes : nullptr;
    cudaError_t e = ctmr::launch_im2col(pp, p.cin_raw, p.cpad, stream);
    if (e != cudaSuccess) return cuda_fail(e, "im2col launch");
    e = ctmr::launch_repack_im2col(d->weight, p.exact ? d->weight_lo : nullptr, p.opad, p.cpad_src, p.cin_raw,
                                   p.cpad, const_cast<void*>(w_hi), const_cast<void*>(w_lo), stream);
    if (e != cudaSuccess) return cuda_fail(e, "im2col weight repack launch");
  } else if (p.prepare && !fuse && (stages & CTMR_CONV_PREPARE)) {
    ctmr::PrepParams pp{};
    pp.src[0] = as_source(d->x);
    pp.src[1] = as_source(d->x2);
    pp.batch = d->batch;
    pp.sd = d->depth, pp.sh = d->height, pp.sw = d->width;
    pp.od = p.in_d, pp.oh = p.in_h, pp.ow = p.in_w;
    pp.mode = d->trilinear ? ctmr::kPrepTrilinear : (d->avgpool ? ctmr::kPrepAvgPool : ctmr::kPrepCopy);
    pp.affine = affine;
    pp.silu = d->silu;
    pp.cpad = p.tf32 ? p.cpad / 2 : p.cpad;  // in output elements (fp32 values for TF32)
    pp.out_cstride = pp.cpad;
    pp.out_kind = p.exact ? ctmr::kPrepOutSplitF16
                          : (p.tf32 ? ctmr::kPrepOutTF32 : (p.bf16 ? ctmr::kPrepOutBF16 : ctmr::kPrepOutF16));
    pp.out = workspace;
    pp.out_lo = p.exact ? static_cast<uint8_t*>(workspace) + p.prep_bytes : nullptr;
    cudaError_t e = p.gn_small ? ctmr::launch_gn_prepare_small(pp, d->gn_gamma, d->gn_beta, d->gn_groups, d->gn_eps,
                                                              stream)
                               : ctmr::launch_prepare(pp, stream);
    if (e != cudaSuccess) return cuda_fail(e, "prepare launch");
  }
  if (!(stages & CTMR_CONV_GEMM)) return CTMR_OK;

  // 2a. The persistent atom-shifted kernel for 16-bit stride-1 3x3x3, nearest-2x and 1x1x1 convolutions.
  if (with_stats && !(kh_ok ? d->stats_slots >= 4 * sm_count()
                            : d->stats_slots >= sm_count() && plan_v2(p, d, true, &v2)))
    return fail(CTMR_ERR_UNSUPPORTED, "output statistics need the persistent kernel (ctmr_conv3d_stats_slots)");
  if (kh_ok) {
    const int rows = ctmr::conv_khcat_rows(), md = kh.mt;
    ctmr::ConvGeom g{};
    g.batch = d->batch;
    g.row_d = p.row_d, g.row_h = p.row_h, g.row_w = p.row_w;
    g.tile_w = 8, g.tile_h = rows, g.tile_d = md;
    g.tiles_w = (p.row_w + 7) / 8;
    g.tiles_h = (p.row_h + rows - 1) / rows;
    g.tiles_d = (p.row_d + md - 1) / md;
    g.phases = 1;
    g.taps = 27;
    g.kblocks = p.cpad / kh.kc;
    g.mode = p.mode;
    g.bn = p.opad;
    g.cout = d->out_channels;
    g.stages = kh.stages;
    g.tmem_cols = 512;
    g.operand_bf16 = p.bf16 ? 1 : 0;
    g.operand_tf32 = p.tf32 ? 1 : 0;
    g.ksplit = 1;
    g.n_tiles = 1;
    g.stats = d->stats;
    g.stats_slots = d->stats_slots;
    const long long total = static_cast<long long>(g.tiles_w) * g.tiles_h * g.tiles_d * d->batch;
    if (total > 0 && total < (1LL << 31)) {
      g.total_tiles = static_cast<int>(total);
      g.bias = d->bias;
      g.bias_bstride = bias_row_stride(d);
      g.res = d->residual.data;
      g.res_bf16 = d->residual.dtype == CTMR_DTYPE_BF16;
      g.res_cstride = d->residual.cstride;
      g.res_up = d->residual_upsampled;
      g.res_d = d->residual_upsampled ? p.out_d / 2 : p.out_d;
      g.res_h = d->residual_upsampled ? p.out_h / 2 : p.out_h;
      g.res_w = d->residual_upsampled ? p.out_w / 2 : p.out_w;
      g.out = d->y;
      g.out_bf16 = d->y_dtype == CTMR_DTYPE_BF16;
      g.out_cstride = d->y_cstride;
      g.out_coff = d->y_coffset;
      g.out_d = p.out_d, g.out_h = p.out_h, g.out_w = p.out_w;
      if (fuse) {
        g.fuse_src0 = static_cast<const float*>(d->x.data);
        g.fuse_cstride0 = d->x.cstride;
        g.fuse_src1 = static_cast<const float*>(d->x2.data);
        g.fuse_cstride1 = d->x2.data != nullptr ? d->x2.cstride : 0;
        g.fuse_ch0 = d->x.channels;
        g.fuse_ctot = p.cin;
        g.fuse_affine = affine;
        g.fuse_silu = d->silu ? 1 : 0;
        cudaError_t e = ctmr::launch_conv3d_khcat(fuse_maps, g, kh.kc, kh.mt, sm_count(), kh.smem, stream);
        return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "conv3d kh-concatenated launch (converter warps)");
      }
      ctmr::ConvMaps maps;
      std::memset(&maps, 0, sizeof(maps));
      const long long rs = a_cstride * 2;
      const long long W = p.in_w, H = p.in_h, D = p.in_d;
      // H before W: the 16 h of one w are consecutive tile rows, so the kernel's shift by one h
      // is a shift by one TMEM lane and one by one w (the kw taps) 16 rows. Boxes of 10 w hold
      // the windows of all three kw taps.
      if (rs % 16 == 0 &&
          encode_act(&maps.a[0], a_hi, p.bf16, p.cpad, H, W, D, d->batch, W * rs, rs, H * W * rs, D * H * W * rs,
                     kh.kc, 16, 10, md) == CTMR_OK) {
        // CTMR_KHCAT_PAIR=1: 64 -> 64 channels in 64-channel blocks, two depths per tile, on the
        // CTA-pair kernel (each SM streams half of every weight box). Off by default: it measured
        // slower than the one-SM kernel (0.821 vs 0.763 ms on 1 x 64 x 96 x 256 x 128 -> 64).
        size_t smem_pair = 0;
        const char* pair_env = getenv("CTMR_KHCAT_PAIR");
        if (kh.kc == 64 && kh.mt == 2 && p.opad == 64 && !p.tf32 && !with_stats && g.total_tiles >= 2 &&
            pair_env != nullptr && pair_env[0] == '1') {
          const int st = ctmr::conv_khcat_pair_stage_plan(&smem_pair);
          ctmr::ConvMaps maps_pair = maps;
          if (st >= 2 && encode_weight_kh(&maps_pair.b, w_hi, p.bf16, p.cpad, p.opad, kh.kc, p.opad / 2) == CTMR_OK) {
            ctmr::ConvGeom gp = g;
            gp.stages = st;
            cudaError_t e = ctmr::launch_conv3d_khcat_pair(maps_pair, gp, smem_pair, stream);
            if (e == cudaSuccess) return CTMR_OK;
            if (e != cudaErrorNotSupported) return cuda_fail(e, "conv3d kh-concatenated pair launch");
          }
        }
        if (encode_weight_kh(&maps.b, w_hi, p.bf16, p.cpad, p.opad, kh.kc, p.opad) == CTMR_OK) {
          cudaError_t e = ctmr::launch_conv3d_khcat(maps, g, kh.kc, kh.mt, sm_count(), kh.smem, stream);
          return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "conv3d kh-concatenated launch");
        }
      }
      // A refused tensor map depends on this call's pointers and strides only: this call falls
      // through to the other kernels (none of which then keeps statistics for fewer than 128
      // output channels), later calls try again.
      if (with_stats && !plan_v2(p, d, true, &v2))
        return fail(CTMR_ERR_UNSUPPORTED, "output statistics: the kh-concatenated kernel's tensor maps were refused");
    }
  }
  if (plan_v2(p, d, with_stats, &v2)) {
    const int tw = v2.tw, mt = v2.mt, bn = v2.bn, kc = v2.kc, stages2 = v2.stages;
    const size_t smem2 = v2.smem;
    if (kc != 0) {
      ctmr::ConvGeom g{};
      g.batch = d->batch;
      g.row_d = p.row_d, g.row_h = p.row_h, g.row_w = p.row_w;
      g.tile_w = 16, g.tile_h = 8, g.tile_d = mt;
      g.tiles_w = (p.row_w + 15) / 16;
      g.tiles_h = (p.row_h + 7) / 8;
      g.tiles_d = (p.row_d + mt - 1) / mt;
      g.phases = p.phases;
      g.taps = p.taps;
      g.kblocks = p.cpad / kc;
      g.mode = p.mode;
      g.bn = bn;
      g.cout = d->out_channels;
      g.stages = stages2;
      g.tmem_cols = static_cast<uint32_t>(std::max(32, next_pow2(p.exact ? 4 * bn : 2 * mt * bn)));
      g.operand_bf16 = p.bf16 ? 1 : 0;
      g.operand_tf32 = p.tf32 ? 1 : 0;
      g.lo_scale = 1.0f / 2048.0f;
      g.ksplit = 1;
      g.n_tiles = (p.opad + bn - 1) / bn;
      const long long total = static_cast<long long>(g.n_tiles) * g.tiles_w * g.tiles_h * g.tiles_d * d->batch *
                              p.phases;
      if (total > 0 && total < (1LL << 31)) {
        g.total_tiles = static_cast<int>(total);
        g.bias = d->bias;
        g.bias_bstride = bias_row_stride(d);
        g.res = d->residual.data;
        g.res_bf16 = d->residual.dtype == CTMR_DTYPE_BF16;
        g.res_cstride = d->residual.cstride;
        g.res_up = d->residual_upsampled;
        g.res_d = d->residual_upsampled ? p.out_d / 2 : p.out_d;
        g.res_h = d->residual_upsampled ? p.out_h / 2 : p.out_h;
        g.res_w = d->residual_upsampled ? p.out_w / 2 : p.out_w;
        g.out = d->y;
        g.out_bf16 = d->y_dtype == CTMR_DTYPE_BF16;
        g.out_cstride = d->y_cstride;
        g.out_coff = d->y_coffset;
        g.out_d = p.out_d, g.out_h = p.out_h, g.out_w = p.out_w;
        g.stats = static_cast<float*>(d->stats);
        g.stats_slots = d->stats_slots;
        ctmr::ConvMaps maps;
        std::memset(&maps, 0, sizeof(maps));
        const long long rs = a_cstride * 2;
        const long long W = p.in_w, H = p.in_h, D = p.in_d;
        // H before W: an 8-row swizzle atom holds 8 consecutive h of one w.
        const long long wtaps = p.mode == ctmr::kModeUp2 ? 64 : (p.mode == ctmr::kModeConv1 ? 1 : 27);
        if (rs % 16 == 0 &&
            encode_act(&maps.a[0], a_hi, p.bf16, p.cpad, H, W, D, d->batch, W * rs, rs, H * W * rs, D * H * W * rs,
                       kc, 8, 16 + tw - 1, mt) == CTMR_OK &&
            encode_weight3(&maps.b, w_hi, p.bf16, p.cpad, p.opad, wtaps, kc, bn, tw) == CTMR_OK &&
            (!p.exact ||
             (encode_act(&maps.a_lo[0], a_lo, false, p.cpad, H, W, D, d->batch, W * rs, rs, H * W * rs,
                         D * H * W * rs, kc, 8, 16 + tw - 1, mt) == CTMR_OK &&
              encode_weight3(&maps.b_lo, w_lo, false, p.cpad, p.opad, wtaps, kc, bn, tw) == CTMR_OK))) {
          cudaError_t e = ctmr::launch_conv3d_umma_v2(maps, g, kc, mt, tw, sm_count(), smem2, p.exact, stream);
          return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "conv3d v2 launch");
        }
        // Refused for this call's pointers or strides: this call takes the per-tap kernel (which
        // cannot produce output statistics); later calls try again.
        if (with_stats) return fail(CTMR_ERR_UNSUPPORTED, "persistent kernel unavailable for output statistics");
      }
    }
  }

  // 2. Tile plan over the GEMM-row grid: a 128-voxel box, w fastest (planned in plan_conv).
  ctmr::ConvGeom g{};
  g.batch = d->batch;
  g.row_d = p.row_d, g.row_h = p.row_h, g.row_w = p.row_w;
  g.tile_w = p.tile_w, g.tile_h = p.tile_h, g.tile_d = p.tile_d;
  g.tiles_w = p.tiles_w, g.tiles_h = p.tiles_h, g.tiles_d = p.tiles_d;
  g.ksplit = p.ksplit;
  g.partial = p.ksplit > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                                      (p.prep_bytes + p.wrep_bytes) * (p.exact ? 2 : 1))
                           : nullptr;
  g.part_cstride = p.n_tiles * p.bn;
  g.phases = p.phases;
  g.taps = p.taps;
  g.kblocks = p.cpad / p.kc;
  g.mode = p.mode;
  g.bn = p.bn;
  g.cout = d->out_channels;
  // TMEM: one accumulator (bf16), or two alternating hi chunk buffers plus the lo accumulator (fp32).
  const int acc_cols = p.bn * (p.exact ? 3 : 1);
  g.tmem_cols = static_cast<uint32_t>(std::max(32, next_pow2(acc_cols)));
  g.chunk_iters = std::max(1, 32 / (p.kc / 16));
  size_t smem = 0;
  g.stages = ctmr::conv_stage_plan(p.kc, p.bn, p.exact, g.tmem_cols > 256, &smem);
  if (g.stages < 2) return fail(CTMR_ERR_UNSUPPORTED, "no pipeline fits shared memory");
  g.bias = d->bias;
  g.bias_bstride = bias_row_stride(d);
  g.res = d->residual.data;
  g.res_bf16 = d->residual.dtype == CTMR_DTYPE_BF16;
  g.res_cstride = d->residual.cstride;
  g.res_up = d->residual_upsampled;
  g.res_d = d->residual_upsampled ? p.out_d / 2 : p.out_d;
  g.res_h = d->residual_upsampled ? p.out_h / 2 : p.out_h;
  g.res_w = d->residual_upsampled ? p.out_w / 2 : p.out_w;
  g.out = d->y;
  g.out_bf16 = d->y_dtype == CTMR_DTYPE_BF16;
  g.out_cstride = d->y_cstride;
  g.out_coff = d->y_coffset;
  g.out_d = p.out_d, g.out_h = p.out_h, g.out_w = p.out_w;
  g.lo_scale = 1.0f / 2048.0f;
  g.operand_bf16 = p.bf16 ? 1 : 0;
    g.operand_tf32 = p.tf32 ? 1 : 0;

  // 3. TMA descriptors.
  ctmr::ConvMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const bool bf16 = p.bf16;
  const long long eb = 2;  // element bytes (bf16 / fp16)
  const long long rs = a_cstride * eb;
  if (rs % 16 != 0) return fail(CTMR_ERR_INVALID, "operand row pitch must be a multiple of 16 bytes");
  const long long W = p.in_w, H = p.in_h, D = p.in_d;
  const void* planes[2] = {a_hi, a_lo};
  for (int pl = 0; pl < (p.exact ? 2 : 1); ++pl) {
    CUtensorMap* dst = pl == 0 ? maps.a : maps.a_lo;
    if (p.mode == ctmr::kModeStride2) {
      for (int par = 0; par < 8; ++par) {
        const int pd = par >> 2, ph = (par >> 1) & 1, pw = par & 1;
        const uint8_t* base = static_cast<const uint8_t*>(planes[pl]) + ((pd * H + ph) * W + pw) * rs;
        st = encode_act(&dst[par], base, bf16, p.cpad, (W - pw + 1) / 2, (H - ph + 1) / 2, (D - pd + 1) / 2,
                        d->batch, 2 * rs, 2 * W * rs, 2 * H * W * rs, D * H * W * rs, p.kc, g.tile_w, g.tile_h,
                        g.tile_d);
        if (st) return st;
      }
    } else {
      st = encode_act(&dst[0], planes[pl], bf16, p.cpad, W, H, D, d->batch, rs, W * rs, H * W * rs, D * H * W * rs,
                      p.kc, g.tile_w, g.tile_h, g.tile_d);
      if (st) return st;
    }
  }
  const long long wtaps = p.mode == ctmr::kModeUp2 ? 64 : p.taps;
  st = encode_weight(&maps.b, w_hi, bf16, p.cpad, p.opad, wtaps, p.kc, p.bn);
  if (st) return st;
  if (p.exact) {
    st = encode_weight(&maps.b_lo, w_lo, bf16, p.cpad, p.opad, wtaps, p.kc, p.bn);
    if (st) return st;
  }

  cudaError_t e = ctmr::launch_conv3d_umma(maps, g, p.kc, p.exact, smem, stream);
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "conv3d launch");
}

size_t ctmr_group_norm_workspace_size(int batch, long long voxels, int groups) {
  if (batch <= 0 || voxels <= 0 || groups <= 0) return 0;
  return static_cast<size_t>(batch) * ctmr::gn_max_chunks(batch) * groups * 3 * sizeof(float);
}

int ctmr_group_norm_affine(ctmr_tensor x, ctmr_tensor x2, int batch, long long voxels, const float* gamma,
                           const float* beta, int groups, float eps, float* affine, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int st = check_view(x, "x", true);
  if (st) return st;
  if ((st = check_view(x2, "x2", false))) return st;
  const int ctot = x.channels + (x2.data ? x2.channels : 0);
  if (batch <= 0 || voxels <= 0) return fail(CTMR_ERR_INVALID, "group_norm extents");
  if (groups <= 0 || ctot % groups != 0) return fail(CTMR_ERR_INVALID, "group_norm channels must be divisible by num_groups");
  if (ctot > 2048) return fail(CTMR_ERR_UNSUPPORTED, "group_norm supports at most 2048 channels");
  if (affine == nullptr) return fail(CTMR_ERR_INVALID, "affine output missing");
  const size_t need = ctmr_group_norm_workspace_size(batch, voxels, groups);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(CTMR_ERR_WORKSPACE, "group_norm needs %zu workspace bytes, got %zu", need, workspace_bytes);
  ctmr::GnParams p{};
  p.src[0] = as_source(x);
  p.src[1] = as_source(x2);
  p.batch = batch;
  p.voxels = voxels;
  p.groups = groups;
  p.eps = eps;
  p.gamma = gamma;
  p.beta = beta;
  p.affine = affine;
  p.partials = static_cast<float*>(workspace);
  p.chunks = ctmr::gn_chunks_for(batch, voxels, ctot);
  cudaError_t e = ctmr::launch_group_norm_affine(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "group_norm launch");
}

int ctmr_group_norm_moments(ctmr_tensor x, ctmr_tensor x2, int batch, long long voxels, int groups, float* moments,
                            void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_view(x, "x", true);
  if (st) return st;
  if ((st = check_view(x2, "x2", false))) return st;
  const int ctot = x.channels + (x2.data ? x2.channels : 0);
  if (batch <= 0 || voxels <= 0) return fail(CTMR_ERR_INVALID, "group_norm extents");
  if (groups <= 0 || ctot % groups != 0) return fail(CTMR_ERR_INVALID, "group_norm channels must be divisible by num_groups");
  if (ctot > 2048) return fail(CTMR_ERR_UNSUPPORTED, "group_norm supports at most 2048 channels");
  if (moments == nullptr) return fail(CTMR_ERR_INVALID, "moments output missing");
  const size_t need = ctmr_group_norm_workspace_size(batch, voxels, groups);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(CTMR_ERR_WORKSPACE, "group_norm needs %zu workspace bytes, got %zu", need, workspace_bytes);
  ctmr::GnParams p{};
  p.src[0] = as_source(x);
  p.src[1] = as_source(x2);
  p.batch = batch;
  p.voxels = voxels;
  p.groups = groups;
  p.partials = static_cast<float*>(workspace);
  p.chunks = ctmr::gn_chunks_for(batch, voxels, ctot);
  cudaError_t e = ctmr::launch_group_norm_moments(p, moments, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "group_norm moments launch");
}

int ctmr_group_norm_affine_from_moments(const float* moments, int parts, int batch, int channels, const float* gamma,
                                        const float* beta, int groups, float eps, float* affine, void* stream) {
  if (moments == nullptr || affine == nullptr) return fail(CTMR_ERR_INVALID, "moments or affine missing");
  if (parts <= 0 || parts > 64 || batch <= 0) return fail(CTMR_ERR_INVALID, "moments parts / batch out of range");
  if (groups <= 0 || channels <= 0 || channels % groups != 0)
    return fail(CTMR_ERR_INVALID, "group_norm channels must be divisible by num_groups");
  ctmr::GnMomentsParams p{};
  p.moments = moments;
  p.parts = parts;
  p.batch = batch;
  p.channels = channels;
  p.groups = groups;
  p.eps = eps;
  p.gamma = gamma;
  p.beta = beta;
  p.affine = affine;
  cudaError_t e = ctmr::launch_group_norm_from_moments(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "group_norm from moments launch");
}

int ctmr_conv3d_stats_slots(const ctmr_conv3d_desc* d) {
  ConvPlan p{};
  if (d == nullptr || plan_conv(d, &p) != CTMR_OK) return 0;
  if (p.narrow || p.tiny) return 0;
  KhPlan kh{};
  if (plan_khcat(p, d, true, &kh)) return 4 * sm_count();  // one slot per epilogue lane quarter
  V2Plan v2{};
  if (!plan_v2(p, d, true, &v2)) return 0;
  return sm_count();
}

int ctmr_conv3d_launch_count(const ctmr_conv3d_desc* d) {
  ConvPlan p{};
  if (d == nullptr || plan_conv(d, &p) != CTMR_OK) return 0;
  const long long voxels = static_cast<long long>(d->depth) * d->height * d->width;
  int n = (p.gn_in && !p.gn_small) ? (ctmr::gn_direct_fits(voxels, p.cin, d->gn_groups) ? 1 : 2) : 0;
  if (p.narrow || p.tiny) return n + 1;
  V2Plan v2{};
  KhPlan kh{};
  const bool kh_ok = plan_khcat(p, d, d->stats != nullptr, &kh);
  // The fused route's affine is the caller's or, with the call's own GroupNorm, the workspace's
  // (256-byte aligned within it): only the caller's pointer can disqualify it here.
  const bool fused = kh_ok && khcat_fusable(p, d, kh, p.gn_in ? nullptr : d->affine);
  if (p.prepare && !fused) n += p.im2col ? 2 : 1;
  if (kh_ok || plan_v2(p, d, d->stats != nullptr, &v2)) return n + 1;
  return n + 1 + (p.ksplit > 1 ? 1 : 0);
}

int ctmr_group_norm_launch_count(long long voxels, int channels, int groups) {
  if (voxels < 0 || channels <= 0 || groups <= 0 || channels % groups != 0) return 0;
  return ctmr::gn_direct_fits(voxels, channels, groups) ? 1 : 2;
}

int ctmr_group_norm_affine_from_stats(const float* stats_a, int channels_a, const float* stats_b, int channels_b,
                                      int slots, int batch, const float* gamma, const float* beta, int groups,
                                      float eps, float* affine, void* stream) {
  if (stats_a == nullptr || channels_a <= 0 || (channels_b > 0 && stats_b == nullptr) || channels_b < 0)
    return fail(CTMR_ERR_INVALID, "group_norm statistics missing");
  if (slots <= 0 || batch <= 0) return fail(CTMR_ERR_INVALID, "group_norm statistics extents");
  const int ctot = channels_a + channels_b;
  if (groups <= 0 || ctot % groups != 0) return fail(CTMR_ERR_INVALID, "group_norm channels must be divisible by num_groups");
  if (affine == nullptr) return fail(CTMR_ERR_INVALID, "affine output missing");
  ctmr::GnStatsParams p{};
  p.stats[0] = stats_a;
  p.stats[1] = channels_b > 0 ? stats_b : nullptr;
  p.channels[0] = channels_a;
  p.channels[1] = channels_b;
  p.slots = slots;
  p.batch = batch;
  p.groups = groups;
  p.eps = eps;
  p.gamma = gamma;
  p.beta = beta;
  p.affine = affine;
  cudaError_t e = ctmr::launch_group_norm_from_stats(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "group_norm from statistics launch");
}

int ctmr_transform(const ctmr_transform_desc* d, void* stream) {
  if (d == nullptr) return fail(CTMR_ERR_INVALID, "null descriptor");
  int st = check_view(d->x, "x", true);
  if (st) return st;
  if ((st = check_view(d->x2, "x2", false))) return st;
  if (d->batch <= 0 || d->depth <= 0 || d->height <= 0 || d->width <= 0)
    return fail(CTMR_ERR_INVALID, "grid must be positive");
  if (d->y == nullptr ||
      (d->y_dtype != CTMR_DTYPE_F32 && d->y_dtype != CTMR_DTYPE_BF16 && d->y_dtype != CTMR_DTYPE_F16))
    return fail(CTMR_ERR_INVALID, "output");
  const int ctot = d->x.channels + (d->x2.data ? d->x2.channels : 0);
  if (d->y_channels < ctot || d->y_cstride < d->y_channels) return fail(CTMR_ERR_INVALID, "output channels");
  if (d->mode == CTMR_TRANSFORM_TRILINEAR && (d->affine != nullptr || d->silu))
    return fail(CTMR_ERR_UNSUPPORTED, "trilinear upsampling takes no affine/silu");
  if (d->mode == CTMR_TRANSFORM_AVGPOOL && (d->depth % 2 || d->height % 2 || d->width % 2))
    return fail(CTMR_ERR_INVALID, "average pooling needs even extents");
  ctmr::PrepParams pp{};
  pp.src[0] = as_source(d->x);
  pp.src[1] = as_source(d->x2);
  pp.batch = d->batch;
  pp.sd = d->depth, pp.sh = d->height, pp.sw = d->width;
  pp.od = d->depth, pp.oh = d->height, pp.ow = d->width;
  if (d->mode == CTMR_TRANSFORM_TRILINEAR) {
    pp.mode = ctmr::kPrepTrilinear;
    pp.od *= 2, pp.oh *= 2, pp.ow *= 2;
  } else if (d->mode == CTMR_TRANSFORM_AVGPOOL) {
    pp.mode = ctmr::kPrepAvgPool;
    pp.od /= 2, pp.oh /= 2, pp.ow /= 2;
  } else if (d->mode == CTMR_TRANSFORM_COPY) {
    pp.mode = ctmr::kPrepCopy;
  } else {
    return fail(CTMR_ERR_INVALID, "transform mode");
  }
  pp.affine = d->affine;
  pp.silu = d->silu;
  pp.cpad = d->y_channels;
  pp.out_cstride = d->y_cstride;
  pp.out_kind = d->y_dtype == CTMR_DTYPE_BF16 ? ctmr::kPrepOutBF16
                : (d->y_dtype == CTMR_DTYPE_F16 ? ctmr::kPrepOutF16 : ctmr::kPrepOutF32);
  pp.out = d->y;
  cudaError_t e = ctmr::launch_prepare(pp, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "transform launch");
}

int ctmr_ncdhw_to_ndhwc(const void* x, int x_dtype, void* y, int y_dtype, int batch, int channels, long long voxels,
                        void* stream) {
  if (x == nullptr || y == nullptr || batch <= 0 || channels <= 0 || voxels <= 0 || voxels > 0x7FFFFFFF)
    return fail(CTMR_ERR_INVALID, "layout arguments");
  cudaError_t e = ctmr::launch_transpose_cs(x, x_dtype == CTMR_DTYPE_BF16, y, y_dtype == CTMR_DTYPE_BF16, batch,
                                            channels, static_cast<int>(voxels), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "layout launch");
}

int ctmr_ndhwc_to_ncdhw(const void* x, int x_dtype, void* y, int y_dtype, int batch, int channels, long long voxels,
                        void* stream) {
  if (x == nullptr || y == nullptr || batch <= 0 || channels <= 0 || voxels <= 0 || voxels > 0x7FFFFFFF)
    return fail(CTMR_ERR_INVALID, "layout arguments");
  cudaError_t e = ctmr::launch_transpose_cs(x, x_dtype == CTMR_DTYPE_BF16, y, y_dtype == CTMR_DTYPE_BF16, batch,
                                            static_cast<int>(voxels), channels, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "layout launch");
}

int ctmr_window_accumulate(ctmr_tensor pred, int batch, int wd, int wh, int ww, int z0, int y0, int x0, int od,
                           int oh, int ow, const float* gz, const float* gy, const float* gx, int scale,
                           float floor_value, float* acc, float* wsum, void* stream) {
  int st = check_view(pred, "pred", true);
  if (st) return st;
  if (batch <= 0 || wd <= 0 || wh <= 0 || ww <= 0 || scale <= 0 || z0 < 0 || y0 < 0 || x0 < 0 || z0 + wd > od ||
      y0 + wh > oh || x0 + ww > ow)
    return fail(CTMR_ERR_INVALID, "window outside the output grid");
  if (gz == nullptr || gy == nullptr || gx == nullptr || acc == nullptr || wsum == nullptr)
    return fail(CTMR_ERR_INVALID, "window buffers");
  ctmr::WindowParams p{};
  p.pred = pred.data;
  p.pred_bf16 = pred.dtype == CTMR_DTYPE_BF16;
  p.pred_cstride = pred.cstride;
  p.batch = batch;
  p.channels = pred.channels;
  p.wd = wd, p.wh = wh, p.ww = ww;
  p.z0 = z0, p.y0 = y0, p.x0 = x0;
  p.od = od, p.oh = oh, p.ow = ow;
  p.gz = gz, p.gy = gy, p.gx = gx;
  p.scale = scale;
  p.floor_value = floor_value;
  p.acc = acc;
  p.wsum = wsum;
  cudaError_t e = ctmr::launch_window_accumulate(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "window launch");
}

int ctmr_window_finalize(const float* acc, const float* wsum, float* out, int batch, int channels, int od, int oh,
                         int ow, int cz0, int cy0, int cx0, int cd, int ch, int cw, void* stream) {
  if (acc == nullptr || wsum == nullptr || out == nullptr || batch <= 0 || channels <= 0 || cz0 < 0 || cy0 < 0 ||
      cx0 < 0 || cz0 + cd > od || cy0 + ch > oh || cx0 + cw > ow || cd <= 0 || ch <= 0 || cw <= 0)
    return fail(CTMR_ERR_INVALID, "window finalize arguments");
  cudaError_t e = ctmr::launch_window_finalize(acc, wsum, out, batch, channels, od, oh, ow, cz0, cy0, cx0, cd, ch, cw,
                                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "window finalize launch");
}

int ctmr_rflow_step(const float* z, const float* vel, long long n, float guidance, int guided, float dt,
                    const float* dt_device, float* out, void* stream) {
  if (z == nullptr || vel == nullptr || out == nullptr || n <= 0) return fail(CTMR_ERR_INVALID, "rflow arguments");
  cudaError_t e = ctmr::launch_rflow_step(z, vel, n, guidance, guided, dt, dt_device, out,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? CTMR_OK : cuda_fail(e, "rflow launch");
}

int ctmr_get_device_error(unsigned* bits, int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "synchronize");
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, ctmr::g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read device error");
  if (bits != nullptr) *bits = v;
  if (clear && v != 0) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(ctmr::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clear device error");
  }
  return CTMR_OK;
}

}  // extern "C"
