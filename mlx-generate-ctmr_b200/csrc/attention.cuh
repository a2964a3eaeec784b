// Head-size-32 self-attention on the tensor cores (see attention.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace ctmr {

struct AttnParams {
  int batch, tokens, heads;  // tokens: a multiple of 128
  float scale;               // logit scale (1 / sqrt(32) for the MAISI attention)
  void* out;                 // (batch, tokens, heads * 32), the input's 16-bit type
};

size_t attention_d32_smem();
// `map`: the (3C, tokens, batch) view of the fused Q/K/V projection, box (32, 128, 1), 64-byte swizzle.
cudaError_t launch_attention_d32(const CUtensorMap& map, const AttnParams& p, bool bf16, cudaStream_t stream);

}  // namespace ctmr
