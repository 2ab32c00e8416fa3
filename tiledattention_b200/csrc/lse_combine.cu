// Log-sum-exp merge of the key slices of a split-KV forward (HBM-bound, one pass).
//
// Slice s of a query row holds o_s = (sum_{c in s} p_c v_c) / l_s and
// lse_s = m_s + log l_s (natural log) over its own keys. The full-row result is
//   lse = log sum_s exp(lse_s),   o = sum_s exp(lse_s - lse) * o_s,
// with slices that saw no valid key (lse_s = -inf) contributing nothing, and a row with
// no valid key at all giving o = 0, lse = -inf. This is the same online-softmax
// rescaling the reference applies across key tiles (flash_fwd.py:426-436), applied
// across slices instead.
//
// Layout: o_part fp32 [n_split][B][H][S][D] contiguous (D a multiple of 8 up to 256), lse_part fp32 [n_split][B*H*S];
// output o [B,H,S,D] with element strides (f16 / bf16 / f32), optional lse [B*H*S].
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lse_combine.h"

namespace ta {

// DT: the head dim, or 0 for a head dim known at run time only (p.D, a multiple of 8 up to
// 256: four columns per thread, rows of D/4 threads packed into the 256-thread block).
template <int DT, int OUT>  // OUT: 0 f16, 1 bf16, 2 f32
__global__ void __launch_bounds__(256) lse_combine_kernel(CombineParams p) {
  const int D = DT > 0 ? DT : p.D;
  const int kThreadsPerRow = D / 4;
  const int kRowsPerBlock = 256 / kThreadsPerRow;
  if (threadIdx.x >= kRowsPerBlock * kThreadsPerRow) return;
  const int64_t rows = static_cast<int64_t>(p.BH) * p.S;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + threadIdx.x / kThreadsPerRow;
  const int d0 = (threadIdx.x % kThreadsPerRow) * 4;
  if (row >= rows) return;
  const int64_t split_rows = rows;
  float m = -INFINITY;
  for (int s = 0; s < p.n_split; ++s) m = fmaxf(m, p.lse_part[s * split_rows + row]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (m != -INFINITY) {
    for (int s = 0; s < p.n_split; ++s) {
      const float ls = p.lse_part[s * split_rows + row];
      if (ls == -INFINITY) continue;
      const float w = __expf(ls - m);
      const float4 v = *reinterpret_cast<const float4*>(p.o_part + (s * split_rows + row) * D + d0);
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
      wsum += w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  acc.x *= inv;
  acc.y *= inv;
  acc.z *= inv;
  acc.w *= inv;
  const int bh = static_cast<int>(row / p.S);
  const int srow = static_cast<int>(row % p.S);
  const int b = bh / p.H, h = bh % p.H;
  const int64_t off = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh +
                      static_cast<int64_t>(srow) * p.o_ss + d0;
  if constexpr (OUT == 2) {
    *reinterpret_cast<float4*>(static_cast<float*>(p.o) + off) = acc;
  } else if constexpr (OUT == 1) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 w2 = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.o) + off) = w2;
  } else {
    __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
    uint2 w2 = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    *reinterpret_cast<uint2*>(static_cast<__half*>(p.o) + off) = w2;
  }
  if (p.lse != nullptr && d0 == 0) p.lse[row] = wsum > 0.f ? m + __logf(wsum) : -INFINITY;
}

cudaError_t launch_lse_combine(const CombineParams& p, int D, int out_kind, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.BH) * p.S;
  if (rows == 0) return cudaSuccess;
  const int rows_per_block = 256 / (D / 4);
  const int64_t grid = (rows + rows_per_block - 1) / rows_per_block;
  if (grid > 0x7fffffffll) return cudaErrorInvalidValue;
  CombineParams q = p;
  q.D = D;
#define TA_COMB(DD, OO) \
  if ((DD == 0 || D == DD) && out_kind == OO) { lse_combine_kernel<DD, OO><<<static_cast<int>(grid), 256, 0, stream>>>(q); return cudaGetLastError(); }
  TA_COMB(64, 0) TA_COMB(64, 1) TA_COMB(64, 2) TA_COMB(128, 0) TA_COMB(128, 1) TA_COMB(128, 2)
  TA_COMB(256, 0) TA_COMB(256, 1) TA_COMB(256, 2)
  if (D >= 8 && D <= 256 && D % 8 == 0) {
    TA_COMB(0, 0) TA_COMB(0, 1) TA_COMB(0, 2)
  }
#undef TA_COMB
  return cudaErrorInvalidValue;
}

}  // namespace ta
