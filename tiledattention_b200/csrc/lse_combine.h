// Internal interface of the split-KV log-sum-exp merge kernel (lse_combine.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ta {

struct CombineParams {
  const float* o_part;    // [n_split][B*H][S][D] fp32, contiguous; D a multiple of 8 <= 256
  const float* lse_part;  // [n_split][B*H*S] fp32
  void* o;                // output [B,H,S,D] with the strides below
  float* lse;             // optional [B*H*S]
  int64_t o_sb, o_sh, o_ss;
  int n_split, BH, H, S;
  int D;  // head dim (set by launch_lse_combine)
};

// out_kind: 0 float16, 1 bfloat16, 2 float32.
cudaError_t launch_lse_combine(const CombineParams& p, int D, int out_kind, cudaStream_t stream);

}  // namespace ta
