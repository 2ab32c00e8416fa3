// Device helpers shared by the SDPA forward kernels (sdpa_fwd_sm100*.cu).
#pragma once

#include <stdint.h>

#include "sdpa_fwd_sm100.h"
#include "sm100_ptx.cuh"

namespace ta {
namespace common {

// Records a failed bounded wait: sets the CTA's abort flag (every other wait of the CTA then
// gives up) and ORs `code` into the caller's device status word.
__device__ __forceinline__ void report(const FwdParams& p, uint32_t code, volatile int* abort_flag) {
  *abort_flag = 1;
  if (p.status) atomicOr(p.status, code);
}

// Two fp32 values -> one 32-bit word of two 16-bit values, `lo` in the low half.
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// acc_lo += low 16-bit value of w, acc_hi += high one (fp32 accumulation of bf16/fp16).
template <bool BF16>
__device__ __forceinline__ void add_packed16_to_f32(uint32_t w, float& acc_lo, float& acc_hi) {
  if constexpr (BF16)
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.bf16 %0, lo, %0;\n\tadd.rn.f32.bf16 %1, hi, %1;\n\t}"
        : "+f"(acc_lo), "+f"(acc_hi) : "r"(w));
  else
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.f16 %0, lo, %0;\n\tadd.rn.f32.f16 %1, hi, %1;\n\t}"
        : "+f"(acc_lo), "+f"(acc_hi) : "r"(w));
}

// One work item of the persistent kernels: key slice, (b, h) pair, first query row and the
// item's key-tile count.
struct Item {
  int split, bh, b, h, q_row0, kv_lo, kv_hi, n_kv;
};

__host__ __device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }

// Item order: key slice, then groups of group_bh (b,h) pairs whose K/V fit in L2 together;
// inside a group the longest causal query blocks (of kRows rows) of all its pairs come
// first, pairs interleaved, so the dynamic scheduler ends each group, and the launch, on
// short items. Host-callable too, so the order is checked on the CPU
// (tests/native/decode_item_check.cu).
template <bool CAUSAL, int kRows, int kKeysPerTile>
__host__ __device__ __forceinline__ Item decode_item(const FwdParams& p, int item) {
  Item it;
  const int per_split = p.BH * p.n_qblk;
  it.split = item / per_split;
  const int rem = item - it.split * per_split;
  const int group = rem / (p.group_bh * p.n_qblk);
  const int within = rem - group * (p.group_bh * p.n_qblk);
  const int gsize = imin(p.group_bh, p.BH - group * p.group_bh);
  const int qblk = p.n_qblk - 1 - within / gsize;
  it.bh = group * p.group_bh + within % gsize;
  it.b = it.bh / p.H;
  it.h = it.bh % p.H;
  it.q_row0 = qblk * kRows;
  // keys [kv_lo, kv_hi) take part (the whole range, or one slice for split-KV)
  it.kv_lo = imin(p.kv_end, p.kv_begin + it.split * p.split_len);
  it.kv_hi = imin(p.kv_end, it.kv_lo + p.split_len);
  const int kv_rows = CAUSAL ? imin(it.kv_hi, it.q_row0 + kRows) : it.kv_hi;
  it.n_kv = kv_rows > it.kv_lo ? (kv_rows - it.kv_lo + kKeysPerTile - 1) / kKeysPerTile : 0;
  return it;
}

}  // namespace common
}  // namespace ta
