/*
 * ctmr_b200 — C ABI of the B200 (sm_100a) convolution stack that replaces the
 * reference's native path in mlx-generate-ctmr (v0.7.0):
 *   implicit-GEMM Conv3d (3x3x3 pad 1 / 1x1x1, stride 1 / 2, nearest-2x and
 *   trilinear-2x inputs) with the group-norm affine, SiLU, 2x average pool and
 *   a two-tensor channel concat fused into its input preparation, and the bias
 *   (per channel or per batch item) and residual add fused into its epilogue,
 *   plus the GroupNorm statistics that feed it.
 *
 * Conventions
 *   - Activations are channels-last (NDHWC): voxel rows of `channels` values,
 *     `cstride` elements apart (a view into a wider row is allowed). The
 *     reference's Python surface is NCDHW; torch's channels_last_3d storage of
 *     an NCDHW tensor is exactly this layout.
 *   - Weights use the Torch layout (O, C, k, k, k), fp32, and are packed once
 *     with ctmr_pack_weight.
 *   - Every call is asynchronous on `stream` (a cudaStream_t, NULL = legacy
 *     default stream) and returns a status code; nothing throws across the ABI.
 *   - No call allocates device memory: the caller passes workspace buffers
 *     whose sizes the *_workspace_size functions return.
 *   - All device-side waits are bounded; a kernel that gives up sets a bit in
 *     the library's device error word (ctmr_get_device_error) instead of hanging.
 */
#ifndef CTMR_B200_H
#define CTMR_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define CTMR_API __attribute__((visibility("default")))
#else
#define CTMR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. CTMR_ERR_INVALID corresponds to the reference's ValueError
 * for shape/dtype mismatches (`_nax_conv.py:523-526, 537-541, 559-560`). */
enum {
  CTMR_OK = 0,
  CTMR_ERR_INVALID = 1,
  CTMR_ERR_UNSUPPORTED = 2,
  CTMR_ERR_WORKSPACE = 3,
  CTMR_ERR_CUDA = 4
};

enum {
  CTMR_DTYPE_F32 = 0,
  CTMR_DTYPE_BF16 = 1,
  CTMR_DTYPE_F16 = 2,    /* ctmr_transform outputs only */
  /* Conv input `x` only: one int16 label id per voxel (cstride elements apart), read as 8
   * channels, channel k = bit k of the id (0.0 or 1.0): the ControlNet condition of
   * `condition.binarize_labels_ncdhw` (`condition.py:20-43`) formed in the operand pass.
   * channels must be 8; no x2, resampling or in-call GroupNorm. */
  CTMR_DTYPE_LABEL8 = 3
};

/* CTMR_PRECISION_FP32: fp32 operands carried as fp16 hi/lo pairs, three
 *   tensor-core products per step, fp32 accumulation (~2^-22 relative product
 *   error; needs |value| < 65504), the reference's "exact" mode
 *   (`_nax_conv.py:27-35`).
 * CTMR_PRECISION_BF16: bf16 operands, fp32 accumulation.
 * CTMR_PRECISION_FP16: fp16 operands (needs |value| < 65504), fp32 accumulation;
 *   the same tensor-core rate as bf16 with 3 more mantissa bits.
 * CTMR_PRECISION_TF32: operands rounded to TF32 (fp32 range, 10 mantissa bits,
 *   stored as fp32), fp32 accumulation, at half the 16-bit tensor-core rate: the
 *   TF32-input mode beside the reference's exact mode. */
enum { CTMR_PRECISION_FP32 = 0, CTMR_PRECISION_BF16 = 1, CTMR_PRECISION_FP16 = 2, CTMR_PRECISION_TF32 = 3 };

/* An NDHWC activation view. data == NULL means "absent". */
typedef struct ctmr_tensor {
  const void* data;
  int dtype;            /* CTMR_DTYPE_* */
  int channels;
  long long cstride;    /* elements between consecutive voxel rows, >= channels */
} ctmr_tensor;

/* One convolution: y = conv(prepare(x ++ x2)) + bias (+ residual).
 * Replaces `nax_conv3d(x, packed, bias, *, affine, silu, stride, upsample,
 * trilinear, residual, mx)` (`_nax_conv.py:475-487`) together with the 1x1x1
 * route of `fast_fp32.pointwise_conv_ncdhw` (`fast_fp32.py:121-130`) and the
 * pooled conv1 of `fast_fp32.residual_block_ncdhw` (`fast_fp32.py:250-265`). */
typedef struct ctmr_conv3d_desc {
  int batch, depth, height, width; /* grid of x (and x2) */
  ctmr_tensor x;
  ctmr_tensor x2;                  /* optional second input, concatenated after x's channels */
  int out_channels;
  int kernel_size;                 /* 3 (padding 1) or 1 */
  int stride;                      /* 1, or 2 with kernel_size 3 */
  int upsample;                    /* convolve the nearest-2x upsampling of x (weights packed with upsample=1) */
  int trilinear;                   /* convolve the half-pixel trilinear-2x upsampling of x */
  int avgpool;                     /* convolve the 2x2x2 mean of silu?(affine?(x)) */
  int precision;                   /* CTMR_PRECISION_* */
  const void* weight;              /* ctmr_pack_weight output (bf16 / fp16, or the fp16 hi plane) */
  const void* weight_lo;           /* fp16 lo plane for CTMR_PRECISION_FP32 */
  const float* affine;             /* (batch, C, 2) (scale, offset) pairs, or NULL */
  int silu;                        /* apply SiLU after the affine */
  const float* bias;               /* (out_channels) or (batch, out_channels), or NULL */
  int bias_per_batch;
  ctmr_tensor residual;            /* optional, on the output grid (half grid if residual_upsampled) */
  int residual_upsampled;          /* residual is nearest-2x upsampled on the fly */
  void* y;                         /* NDHWC output on the output grid */
  int y_dtype;
  long long y_cstride;
  int y_coffset;                   /* first channel written in each output row */
  /* Optional GroupNorm statistics of the output, for ctmr_group_norm_affine_from_stats:
   * float[batch][stats_slots][out_channels][3] moments (count, mean, M2) per
   * (batch item, slot, channel). stats_slots must be ctmr_conv3d_stats_slots(desc)
   * (> 0). Null: none. */
  float* stats;
  int stats_slots;
  /* Optional GroupNorm of the input computed inside the call (instead of passing
   * `affine`): gamma/beta per input channel (NULL: 1/0), gn_groups > 0 groups over
   * x ++ x2, gn_eps. The statistics are those of ctmr_group_norm_affine, reduced by
   * the call before its operand pass (with CTMR_GN_FUSED=1 in the environment, small
   * tensors use one kernel that reduces them and writes the operand). `affine` must
   * be NULL. */
  const float* gn_gamma;
  const float* gn_beta;
  int gn_groups;
  float gn_eps;
  /* Elements between consecutive batch items' rows of a per-batch bias (0: out_channels,
   * i.e. a dense (batch, out_channels) array; otherwise >= out_channels, e.g. a column
   * slice of a wider (batch, N) table). */
  long long bias_row_stride;
} ctmr_conv3d_desc;

/* Packed-weight element count per plane for a Torch (O, C, k, k, k) weight:
 * taps x round16(O) x round16(C), taps = k^3, or 64 with upsample.
 * Replaces the shapes of `pack_weight` / `pack_upsample_weight` (`_nax_conv.py:391-445`). */
CTMR_API size_t ctmr_packed_weight_elems(int out_channels, int in_channels, int kernel_size, int upsample);

/* Bytes of one packed-weight plane in `precision`: 2 x ctmr_packed_weight_elems in the 16-bit
 * and split modes; for CTMR_PRECISION_TF32, taps x round16(O) x round8(C) fp32 values. The
 * size counterpart of `pack_weight` (`_nax_conv.py:391-404`) per precision; 0 when invalid. */
CTMR_API size_t ctmr_packed_weight_bytes(int out_channels, int in_channels, int kernel_size, int upsample,
                                         int precision);

/* Pack an fp32 Torch-layout weight (device pointer). bf16 for CTMR_PRECISION_BF16,
 * fp16 for CTMR_PRECISION_FP16, TF32-rounded fp32 for CTMR_PRECISION_TF32 (packed_lo
 * unused), fp16 hi/lo planes for CTMR_PRECISION_FP32.
 * Replaces `pack_weight` (`_nax_conv.py:391-404`) and, with upsample = 1,
 * `pack_upsample_weight` (`_nax_conv.py:407-445`). */
CTMR_API int ctmr_pack_weight(const float* weight, int out_channels, int in_channels, int kernel_size, int upsample,
                     int precision, void* packed, void* packed_lo, void* stream);

/* ctmr_pack_weight for a weight stored channels-last, (O, k, k, k, C) (device pointer): the
 * layout of released safetensors checkpoints, which the reference transposes to Torch
 * layout on load (`weights.py:152-156`, LAYOUT_CONV3D_W); packed here without that copy.
 * Same packed result, bit for bit. */
CTMR_API int ctmr_pack_weight_channels_last(const float* weight, int out_channels, int in_channels,
                     int kernel_size, int upsample, int precision, void* packed, void* packed_lo,
                     void* stream);

/* Multi-head self-attention with head size 32, out = softmax(Q K^T * scale) V per head, on
 * the tensor cores in one flash-attention pass. `qkv` is the fused projection (batch, tokens,
 * 3 * heads * 32) of 16-bit values (dtype CTMR_DTYPE_BF16, or CTMR_DTYPE_F16 for fp16),
 * contiguous, head h at columns h*32 (q), C + h*32 (k), 2C + h*32 (v); `out` is
 * (batch, tokens, heads * 32) of the same type. tokens must be a multiple of 128.
 * Replaces `_flash_attention.flash_attention` (`_flash_attention.py:320-360`) as called by
 * `fast_fp32.self_attention_tokens` (`fast_fp32.py:352-396`). */
CTMR_API int ctmr_attention_d32(const void* qkv, int dtype, int batch, int tokens, int heads, float scale, void* out,
                       void* stream);

/* Workspace bytes ctmr_conv3d needs for this descriptor (the prepared operand). */
CTMR_API size_t ctmr_conv3d_workspace_size(const ctmr_conv3d_desc* desc);

/* Replaces `nax_conv3d` (`_nax_conv.py:475-684`): operand preparation (when
 * needed) followed by the implicit-GEMM kernel. */
CTMR_API int ctmr_conv3d(const ctmr_conv3d_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* The two launches of ctmr_conv3d separately, as the reference's pack and
 * GEMM kernels are (`_nax_conv.py:583-646`): stages = CTMR_CONV_PREPARE,
 * CTMR_CONV_GEMM or both. The GEMM stage reads the operand a previous
 * PREPARE stage left in the same workspace. */
enum { CTMR_CONV_PREPARE = 1, CTMR_CONV_GEMM = 2 };
CTMR_API int ctmr_conv3d_stages(const ctmr_conv3d_desc* desc, void* workspace, size_t workspace_bytes, int stages,
                                void* stream);

/* The convolution of ctmr_conv3d for callers that cannot allocate device
 * memory. (No counterpart in the reference: its MLX runtime allocates every
 * buffer itself.) Plugins living inside another framework's memory pool and
 * real-time or safety-constrained callers whose allocations are all made up
 * front cannot call cudaMalloc for the workspace ctmr_conv3d needs; this
 * variant takes that scratch from one static device
 * array of CTMR_CONV3D_NOALLOC_SCRATCH_BYTES that every GPU loading the
 * library holds until exit, and allocates nothing.
 *   - Inputs and outputs are passed exactly as for ctmr_conv3d.
 *   - Convolutions whose prepared operand (ctmr_conv3d_workspace_size) exceeds
 *     the scratch are rejected with CTMR_ERR_WORKSPACE, nothing launched.
 *   - The first call on a device looks up the array's address on that device
 *     (cudaGetSymbolAddress); make it before any stream capture.
 *   - All calls share the array and it keeps the last call's contents; nothing
 *     in it needs to start at zero. Calls whose kernels overlap on the GPU
 *     (unordered streams) race on it and must not be issued. */
#define CTMR_CONV3D_NOALLOC_SCRATCH_BYTES (32u << 20)
CTMR_API int ctmr_conv3d_noalloc(const ctmr_conv3d_desc* desc, void* stream);

/* Workspace bytes for ctmr_group_norm_affine. */
CTMR_API size_t ctmr_group_norm_workspace_size(int batch, long long voxels, int groups);

/* GroupNorm statistics of (x ++ x2) over each (batch item, group) ->
 * affine[b][c] = (gamma[c] * rstd, beta[c] - mean * gamma[c] * rstd), fp32.
 * Replaces `medmlx_core.group_norm.group_norm_affine` (called at `fast_fp32.py:183-189`;
 * layout (B*C*2) consumed at `_nax_conv.py:174-176`). gamma/beta may be NULL (1/0). */
CTMR_API int ctmr_group_norm_affine(ctmr_tensor x, ctmr_tensor x2, int batch, long long voxels, const float* gamma,
                           const float* beta, int groups, float eps, float* affine, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The GroupNorm statistics of ctmr_group_norm_affine stopped before the affine: the merged
 * (count, mean, M2) of each (batch item, group) of (x ++ x2), float moments[batch][groups][3].
 * Same workspace as ctmr_group_norm_affine. For a tensor split across devices (depth shards
 * of one volume, each holding `voxels` of it): each part computes its moments, the parts
 * exchange them, and ctmr_group_norm_affine_from_moments forms the affine of the whole
 * tensor. The reference normalises whole tensors only (`fast_fp32.py:183-189`); this is the
 * same statistic, split at the boundary between the two kernels of its computation. */
CTMR_API int ctmr_group_norm_moments(ctmr_tensor x, ctmr_tensor x2, int batch, long long voxels, int groups,
                                     float* moments, void* workspace, size_t workspace_bytes, void* stream);

/* The affine of group_norm_affine (`fast_fp32.py:183-189`) from the moments of `parts` parts
 * of one tensor, float moments[parts][batch][groups][3] (1 <= parts <= 64), merged in part
 * order in double precision, so every caller holding the same moments gets the same affine. */
CTMR_API int ctmr_group_norm_affine_from_moments(const float* moments, int parts, int batch, int channels,
                                                 const float* gamma, const float* beta, int groups, float eps,
                                                 float* affine, void* stream);

/* Kernel launches one ctmr_conv3d call with this descriptor issues (instrumentation;
 * no reference counterpart), or 0 for an invalid descriptor. */
CTMR_API int ctmr_conv3d_launch_count(const ctmr_conv3d_desc* desc);

/* Kernel launches one ctmr_group_norm_affine call over `voxels` voxels per batch item and
 * `channels` channels in `groups` groups issues for dense, 16-byte aligned fp32 sources: 1 for
 * small groups (one block per group and batch item computes the affine directly), 2 otherwise
 * (partials, then the merge); 0 for invalid extents. Instrumentation; no reference counterpart. */
CTMR_API int ctmr_group_norm_launch_count(long long voxels, int channels, int groups);

/* Statistics slots a convolution writes when desc->stats is set, or 0 when this
 * convolution does not produce them. The kh-concatenated persistent kernel (16-bit
 * operands, stride-1 3x3x3, 64 padded output channels) writes four per SM, one per
 * epilogue lane quarter of each CTA; the atom-shifted persistent kernel (at least 128
 * output channels, batch x out_channels <= 512) one per SM; other routes none. Has no
 * reference counterpart: the reference recomputes the statistics from the tensor. */
CTMR_API int ctmr_conv3d_stats_slots(const ctmr_conv3d_desc* desc);

/* The affine of ctmr_group_norm_affine from convolution output statistics instead
 * of a pass over the tensor: stats_a (channels_a) ++ stats_b (channels_b, may be
 * NULL with channels_b 0) in the ctmr_conv3d_desc.stats layout, each with `slots`
 * slots. Same result definition as `group_norm_affine` (`fast_fp32.py:183-189`);
 * the moments are merged in double precision in a fixed order. */
CTMR_API int ctmr_group_norm_affine_from_stats(const float* stats_a, int channels_a, const float* stats_b,
                                               int channels_b, int slots, int batch, const float* gamma,
                                               const float* beta, int groups, float eps, float* affine,
                                               void* stream);

enum { CTMR_TRANSFORM_COPY = 0, CTMR_TRANSFORM_TRILINEAR = 1, CTMR_TRANSFORM_AVGPOOL = 2 };

/* y = mode(silu?(affine?(x ++ x2))) materialised as fp32 or bf16 NDHWC, channels
 * past the input zero-filled up to y_channels. Replaces the materialising ops of
 * the operator surface: `fast_fp32.group_norm_ncdhw` (`fast_fp32.py:102-118`),
 * `silu`, `avg_pool3d_ncdhw` and `upsample_trilinear_ncdhw` (`source_vae.py:95-111`). */
typedef struct ctmr_transform_desc {
  int batch, depth, height, width; /* grid of x */
  ctmr_tensor x;
  ctmr_tensor x2;
  int mode;                        /* CTMR_TRANSFORM_* */
  const float* affine;
  int silu;
  void* y;
  int y_dtype;
  int y_channels;
  long long y_cstride;
} ctmr_transform_desc;

CTMR_API int ctmr_transform(const ctmr_transform_desc* desc, void* stream);

/* (B, C, S) <-> (B, S, C) layout change (NCDHW <-> NDHWC), fp32/bf16 in and out. */
CTMR_API int ctmr_ncdhw_to_ndhwc(const void* x, int x_dtype, void* y, int y_dtype, int batch, int channels,
                        long long voxels, void* stream);
CTMR_API int ctmr_ndhwc_to_ncdhw(const void* x, int x_dtype, void* y, int y_dtype, int batch, int channels,
                        long long voxels, void* stream);

/* Sliding-window blend (`decode.py:115-184`): acc += pred * w, wsum += w over one
 * window at (z0, y0, x0) of the output grid, w = max(gz[z/scale] gy[y/scale] gx[x/scale], floor). */
CTMR_API int ctmr_window_accumulate(ctmr_tensor pred, int batch, int wd, int wh, int ww, int z0, int y0, int x0,
                           int od, int oh, int ow, const float* gz, const float* gy, const float* gx, int scale,
                           float floor_value, float* acc, float* wsum, void* stream);

/* out (NCDHW, B x C x cd x ch x cw) = acc / wsum over the crop at (cz0, cy0, cx0). */
CTMR_API int ctmr_window_finalize(const float* acc, const float* wsum, float* out, int batch, int channels, int od, int oh,
                         int ow, int cz0, int cy0, int cx0, int cd, int ch, int cw, void* stream);

/* Guided Euler step of the rectified-flow sampler (`image.py:163-175`, `rflow.py:101-121`):
 * v = vel[n:] + guidance * (vel[:n] - vel[n:]) when guided, else vel[:n]; out = z + v * dt.
 * When dt_device is not NULL the step reads dt from that device scalar instead
 * (so one captured CUDA graph serves every step). out may alias z. */
CTMR_API int ctmr_rflow_step(const float* z, const float* vel, long long n, float guidance, int guided, float dt,
                             const float* dt_device, float* out, void* stream);

/* Device error word (bit set when a bounded wait gave up); optionally cleared.
 * Synchronises the current device. */
CTMR_API int ctmr_get_device_error(unsigned* bits, int clear);

CTMR_API const char* ctmr_status_string(int status);

/* Human-readable reason of the last failed call on this thread. */
CTMR_API const char* ctmr_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* CTMR_B200_H */
