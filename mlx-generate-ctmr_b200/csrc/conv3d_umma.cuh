// Device-side descriptors shared by the implicit-GEMM convolution kernel and
// its host launcher.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace ctmr {

enum ConvMode : int {
  kModeConv3 = 0,  // 3x3x3, padding 1, stride 1: 27 taps
  kModeConv1 = 1,  // 1x1x1: one tap
  kModeUp2 = 2,    // nearest-2x-upsample fold: 8 parities x 8 taps of 2x2x2 over the source grid
  kModeStride2 = 3 // 3x3x3, padding 1, stride 2: 27 taps over 8 parity views of the input
};

// TMA descriptors. `a` holds the activation view (one, or eight parity views
// for stride 2); `a_lo`/`b_lo` are the fp16 lo planes of the split-fp32 mode.
struct ConvMaps {
  CUtensorMap a[8];
  CUtensorMap a_lo[8];
  CUtensorMap b;
  CUtensorMap b_lo;
};

struct ConvGeom {
  int batch;
  int row_d, row_h, row_w;      // GEMM-row grid: output voxels (source voxels for kModeUp2)
  int tile_w, tile_h, tile_d;   // M-tile box (tile_w * tile_h * tile_d == 128)
  int tiles_w, tiles_h, tiles_d;
  int phases;                   // 8 for kModeUp2, else 1
  int taps;                     // taps per phase
  int kblocks;                  // padded input channels / KC
  int mode;
  int bn;                       // N tile (multiple of 16, <= 256)
  int cout;                     // real output channels
  int stages;
  uint32_t tmem_cols;
  int chunk_iters;              // EXACT: K iterations per promoted accumulator chunk
  int operand_bf16;             // single-plane modes: 1 bf16 operands, 0 fp16 operands
  int operand_tf32;             // single-plane mode with TF32 operands (fp32 rows; kind::tf32 MMAs)
  int n_tiles;                  // persistent kernel: N tiles per M tile
  int total_tiles;              // persistent kernel: all (M tile, N tile) pairs
  int ksplit;                   // per-tap kernel: K iterations split over grid.z (fp32 partial planes)
  float* partial;               // [ksplit][batch][row_d][row_h][row_w][part_cstride] when ksplit > 1
  int part_cstride;
  // epilogue
  const float* bias;            // may be null
  int bias_bstride;             // 0 (per channel) or cout (per batch item)
  const void* res;              // may be null
  int res_bf16;
  long long res_cstride;
  int res_up;                   // residual on the half-resolution grid, nearest-upsampled
  int res_d, res_h, res_w;
  void* out;
  int out_bf16;
  long long out_cstride;
  int out_coff;
  int out_d, out_h, out_w;
  float lo_scale;               // 2^-11: weight of the hi*lo + lo*hi accumulator
  // GroupNorm statistics of the output (persistent kernel): per (batch item, CTA
  // slot, channel) moments (count, mean, M2) as float[batch][stats_slots][cout][3].
  float* stats;                 // null: not requested
  int stats_slots;              // slots in the buffer (>= the grid; the rest are zeroed)
  // kh-concatenated kernel with its own operand conversion (no separate operand pass): the fp32
  // NDHWC source(s) on the row grid, channels [0, ch0) from src0 and [ch0, ctot) from src1, each
  // value taken through silu?(v * scale[b, c] + offset[b, c]) and rounded to the operand type.
  const float* fuse_src0;
  const float* fuse_src1;
  long long fuse_cstride0, fuse_cstride1;
  int fuse_ch0, fuse_ctot;
  const float* fuse_affine;     // [batch][ctot][2] (scale, offset) or null
  int fuse_silu;
};

}  // namespace ctmr
