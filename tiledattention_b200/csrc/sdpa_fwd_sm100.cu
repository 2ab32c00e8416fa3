// SDPA forward for B200 (sm_100a), head dims 64 and 128: persistent CTAs, TMA + mbarrier
// pipeline, tcgen05 MMAs with accumulators in tensor memory, warp-specialised online softmax.
//
// Algorithm (same maths as the reference cuTile kernel,
// src/tiledattention/kernels/flash_fwd.py:374-446 of thisistaimur/TiledAttention):
//   for each query row r:  m = -inf, l = 0, acc = 0
//   for each key tile:     s = q_r . k_c * scale, masked to -inf where c >= S or
//                          (causal and c > r)                    (flash_fwd.py:400-423)
//                          m' = max(m, max_c s); alpha = exp(m - m')
//                          p = exp(s - m'); l = l*alpha + sum p; acc = acc*alpha + p v
//   o_r = acc / l                                               (flash_fwd.py:438-444)
// Here every query row runs TWO such recurrences, one over the first 64 keys of every
// 128-key tile ("half a") and one over the last 64 ("half b"), each with its own m, l and
// accumulator; the epilogue merges them exactly:
//   m = max(m_a, m_b), l = l_a 2^(m_a-m) + l_b 2^(m_b-m),
//   o = (acc_a 2^(m_a-m) + acc_b 2^(m_b-m)) / l.
// (The same log-sum-exp combination the reference applies across key tiles,
// flash_fwd.py:426-436, applied across the two key halves.) This lets the two softmax
// warpgroups run without exchanging row maxima on every tile.
// Differences in precision, all towards the fp32 oracle: scores and P.V products are
// accumulated in fp32 tensor memory (the cuTile kernel rounds each tile product to
// the input dtype), and the exponent is evaluated as exp2 with log2(e) folded into
// the scale. The running max is rescaled lazily: an accumulator is only rescaled
// when its max grows by more than 2^8, which is exact after the final division by l.
//
// Work: one item = one (key slice, batch*head pair, 128-row query block). The grid has at
// most one CTA per SM; each CTA takes items from a global counter until they run out, in
// groups of (b,h) pairs whose K/V fit in L2, longest causal blocks of a group first.
// Consecutive items of a CTA overlap: while the epilogue warps write the output of item i,
// the softmax warps already work on item i+1, whose Q and first K tiles the producer loaded
// and whose first scores the QK^T issuer computed during item i's last tiles.
//
// CTA organisation (512 threads, one CTA per SM: all 512 TMEM columns):
//   warps 0-3   softmax of key columns 0-63 of every score tile (half a), accumulator O_a
//   warps 4-7   softmax of key columns 64-127 (half b), accumulator O_b; in both, thread
//               lane i of warp w owns query row 32*(w%4) + i of the item (its TMEM lane);
//               at the end of an item each half hands its (m, l) to the epilogue
//   warp  8     scheduler + TMA producer: per item Q, then K_0 .. K_{NB-1}, V_j, K_{j+NB}
//   warp  9     TMEM allocator and P.V issuer (one elected thread)
//   warp 10     QK^T issuer (one elected thread)
//   warp 11     idle (completes the third warpgroup for the register split)
//   warps 12-15 epilogue: merges O_a and O_b, normalises, stages the tile for one TMA store
// Tensor memory: NB score buffers of 128 columns (NB = 3 at D=64, 2 at D=128), then
// O_a and O_b (D columns each). The g-th score tile a CTA processes (counted over all its
// items) lives in buffer g%NB; each half's P (16-bit, two per column) overwrites the first
// 32 of that half's own 64 score columns (half a: columns 0-31, half b: 64-95), so neither
// half writes columns the other still reads, and feeds the P.V MMAs from tensor memory.
// The two issuers are not ordered with each other, so S_g is issued only after PV_{g-NB}
// (which reads the buffer's P) has completed.
// An accumulator rescale for a grown max (rare, lazy) happens in its warpgroup after P is
// stored and after the previous tile's PV completed, before the new P is published.
//
// Every wait is bounded (shared abort flag + global-timer timeout); on expiry the
// kernel records TA_DEVSTAT_* bits in the status word, drains its own in-flight TMA
// copies and MMAs, frees tensor memory and returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "sdpa_common.cuh"
#include "sm100_ptx.cuh"
#include "sdpa_fwd_sm100.h"
#include "tiledattention_b200.h"

namespace ta {

using common::add_packed16_to_f32;
using common::Item;
using common::pack2;
using common::report;

constexpr int kRowsPerTile = 128;  // query rows per item (= TMEM lanes)
constexpr int kKeysPerTile = 128;  // keys per K/V tile
constexpr int kKeysPerHalf = 64;   // keys of one half (one softmax warpgroup)
constexpr int kThreads = 512;
// Register split: the kernel is built for kLaunchRegs per thread (launch bounds 512 x 1);
// after start-up the producer/MMA warpgroup and the epilogue warpgroup give registers back
// (setmaxnreg.dec to kSideRegs / kEpilogueRegs) and the two softmax warpgroups take them
// (setmaxnreg.inc to kSoftmaxRegs). The sum equals the launch allocation, so the increase
// always fits; the host refuses to launch a build whose register count differs from
// kLaunchRegs.
constexpr int kLaunchRegs = 128;
#ifndef TA_SOFTMAX_REGS
#define TA_SOFTMAX_REGS 184
#define TA_EPILOGUE_REGS 72
#define TA_SIDE_REGS 72
#endif
constexpr int kSoftmaxRegs = TA_SOFTMAX_REGS;
constexpr int kEpilogueRegs = TA_EPILOGUE_REGS;
constexpr int kSideRegs = TA_SIDE_REGS;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kEpilogueRegs + 128 * kSideRegs ==
                  kThreads * kLaunchRegs,
              "register split must match the launch allocation");
constexpr int kProducerWarp = 8;
constexpr int kPvWarp = 9;
constexpr int kQkWarp = 10;
constexpr int kEpilogueWarp0 = 12;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr int kSumChains = 4;  // independent row-sum accumulators (short dependency chains)
constexpr uint64_t kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait
// Item-broadcast consumers: the two issuer threads and lane 0 of each softmax and epilogue
// warp.
constexpr int kItemConsumers = 2 + 8 + 4;
constexpr int kNoItem = -1;  // Item::split of "no item left"

// Every kPolyEvery-th element pair computes exp2 on the FMA pipe instead of the MUFU
// (0: never). Worth it only where the MUFU is the limit and the MMA work is small (D=64):
// measured on B200, every 3rd pair is fastest without a mask, every 5th with the causal mask
// (whose diagonal tiles add FMA-pipe masking work); at D=128 it does not pay.
template <int D, bool CAUSAL>
__host__ __device__ constexpr int poly_every() {
#if defined(TA_POLY_EVERY_D64) && defined(TA_POLY_EVERY_D128)
  return D == 64 ? TA_POLY_EVERY_D64 : TA_POLY_EVERY_D128;
#else
  return D == 64 ? (CAUSAL ? 5 : 3) : 0;
#endif
}

// Suspend-time hint (ns) of the kernel's barrier waits (0: none). With it, the warps that wait
// for most of an item (epilogue, producer, issuers) poll less and leave more issue slots to
// the softmax warps on their sub-partitions. Measured on B200 (100 us): +3.7 % at D=64
// non-causal, +0.4 % causal; -0.5 % at D=128, where it stays off.
template <int D>
__host__ __device__ constexpr uint32_t wait_hint_ns() {
#ifdef TA_WAIT_HINT_NS_D64
  return D == 64 ? TA_WAIT_HINT_NS_D64 : 0u;
#else
  return D == 64 ? 100000u : 0u;
#endif
}

template <int D>
struct Layout {
  static_assert(D == 64 || D == 128, "this kernel serves head dims 64 and 128");
  static constexpr int kSBufs = D == 64 ? 3 : 2;  // score buffers (128 TMEM columns each)
  static constexpr int kOCol = kSBufs * 128;       // O_a at kOCol, O_b at kOCol + D
  static_assert(kOCol + 2 * D <= 512, "tensor memory columns");
  static constexpr int kTileBytes = kRowsPerTile * D * 2;  // 128 rows x D x 16-bit
  static constexpr int kChunks = D / 64;                   // 128-byte swizzle atoms per row
  // Separate rings for K tiles (QK^T issuer) and V tiles (P.V issuer).
  static constexpr int kKStages = (D == 64) ? 4 : 2;
  static constexpr int kVStages = (D == 64) ? 4 : 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kTileBytes;
  static constexpr int kVOff = kKOff + kKStages * kTileBytes;
  // Output tile staged for the TMA store (16-bit output, same swizzled layout as Q).
  static constexpr int kStageOff = kVOff + kVStages * kTileBytes;
  static constexpr int kRedOff = kStageOff + kTileBytes;  // epilogue (m, l) exchange
  static constexpr int kRedBytes = 2 * 4 * kRowsPerTile * 4;       // [item%2][m|l][half][row]
  static constexpr int kBarOff = kRedOff + kRedBytes;
  static constexpr int kBytes = kBarOff + 512;
  static constexpr int kDynSmem = kBytes + 1024;  // slack for 1024-byte alignment
  static_assert(kDynSmem <= 227 * 1024, "shared memory");
};

struct Barriers {
  uint64_t q_full, q_empty;  // Q of the current item loaded / no longer read by QK^T
  uint64_t s_full[3];        // [g % NB]: score tile g complete
  uint64_t p_full[3];        // [g % NB]: both halves of P_g stored (8 softmax warps)
  uint64_t pv_done[4];       // [g % 4]: PV_g (both halves) completed
  uint64_t o_final;          // all PV of the current item completed
  uint64_t o_empty;          // the epilogue finished reading O_a, O_b (4 epilogue warps)
  uint64_t ml_full[2];       // [item % 2]: both halves' (m, l) of the item written (8 warps)
  uint64_t ml_empty[2];      // [item % 2]: the epilogue read them (4 warps)
  uint64_t stage_free;       // the previous output tile's TMA store read the staging buffer
  uint64_t staged;           // output tile written to the staging buffer (4 warps)
  uint64_t item_full[2], item_empty[2];
  uint64_t drain;            // both issuers' MMAs completed (2 commits)
  uint64_t never;            // self-test only: a barrier nothing arrives on
  uint64_t k_full[4], k_empty[4];
  uint64_t v_full[4], v_empty[4];
  int item[2][8];            // published items, decoded (an Item; split < 0: no item)
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 512, "barrier block");

#ifdef TA_TRACE
// Experiment builds only: clock64 of event `ev` (< 16) of tile j (< 32) of the first
// item of the first 64 blocks, for timeline analysis.
__device__ __forceinline__ void trace_ev(const FwdParams& p, int item_no, int j, int ev) {
  if (p.trace && item_no == 0 && blockIdx.x < 64 && j < 24) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    p.trace[(blockIdx.x * 32 + j) * 16 + ev] = c;
  }
}
#define TRACE(ic, j, ev) trace_ev(p, (ic), (j), (ev))
// Item-level events of the first 8 items: row 24 + ic of the block's trace area.
__device__ __forceinline__ void trace_item(const FwdParams& p, int ic, int ev) {
  if (p.trace && ic < 8 && blockIdx.x < 64) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    p.trace[(blockIdx.x * 32 + 24 + ic) * 16 + ev] = c;
  }
}
#define TRACE_ITEM(ic, ev) trace_item(p, (ic), (ev))
#else
#define TRACE(ic, j, ev)
#define TRACE_ITEM(ic, ev)
#endif

// OUT_F32: write o as fp32 (the normalised partial output of one key slice) instead of
// the input dtype. Items: n_split x B*H x n_qblk; slice s covers keys
// [kv_begin + s*split_len, min(kv_end, kv_begin + (s+1)*split_len)).
// S = Q K^T for one 128x128 score tile: D/16 MMAs of K=16. Q and K tiles are K-major,
// 128-byte swizzled, in chunks of 64 columns (16 KB per chunk of 128 rows); step kk reads
// columns 16kk..16kk+15: chunk kk/4, 32 bytes into the swizzle atom per kk%4.
template <int D, int kk = 0>
__device__ __forceinline__ void qk_mmas(uint32_t d_tmem, uint64_t qd, uint64_t kd, uint32_t idesc) {
  if constexpr (kk < D / 16) {
    constexpr uint32_t off = ((kk >> 2) * (kRowsPerTile * 128) + (kk & 3) * 32) >> 4;
    mma_ss_imm<off, off, (kk > 0 ? 1u : 0u)>(d_tmem, qd, kd, idesc);
    qk_mmas<D, kk + 1>(d_tmem, qd, kd, idesc);
  }
}

// O_hh (+)= P_hh V_hh: the 64 keys of half hh in 4 MMAs of K=16. P comes from tensor memory
// (16-bit pairs, 8 columns per 16 keys); V is MN-major, 128-byte swizzled (16 key rows =
// 2 KB). `acc` is the accumulate flag of the half's first MMA.
template <int HH, int k4 = 0>
__device__ __forceinline__ void pv_half_mmas(uint32_t d_tmem, uint32_t a_tmem, uint64_t vd,
                                             uint32_t idesc, uint32_t acc) {
  if constexpr (k4 < kKeysPerHalf / 16) {
    constexpr uint32_t off = ((HH * (kKeysPerHalf / 16) + k4) * 16 * 128) >> 4;
    if constexpr (k4 == 0)
      mma_ts_imm_acc<0, off>(d_tmem, a_tmem, vd, idesc, acc);
    else
      mma_ts_imm<k4 * 8, off, 1u>(d_tmem, a_tmem, vd, idesc);
    pv_half_mmas<HH, k4 + 1>(d_tmem, a_tmem, vd, idesc, acc);
  }
}

template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    sdpa_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v,
                    const __grid_constant__ CUtensorMap tmap_o, const FwdParams p) {
  using L = Layout<D>;
  constexpr int NB = L::kSBufs;
  constexpr int kPolyEvery = poly_every<D, CAUSAL>();
  constexpr uint32_t kWaitHint = wait_hint_ns<D>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = smem + L::kQOff;
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);  // [item%2][m|l][half][128]
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bars->abort_flag;
  const uint64_t kTimeoutNs = p.timeout_ns ? p.timeout_ns : kDefaultTimeoutNs;
  const int n_items = p.n_split * p.BH * p.n_qblk;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < NB; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 8);  // one arrival per softmax warp
    }
    for (int i = 0; i < 4; ++i) mbar_init(&bars->pv_done[i], 1);
    mbar_init(&bars->o_final, 1);
    // Barriers the softmax warps signal take one arrival per warp after a warp sync (256
    // per-thread arrivals on one barrier are 256 serialised shared-memory atomics).
    mbar_init(&bars->o_empty, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->ml_full[i], 8);
      mbar_init(&bars->ml_empty[i], 4);
    }
    mbar_init(&bars->stage_free, 1);
    mbar_init(&bars->staged, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->item_full[i], 1);
      mbar_init(&bars->item_empty[i], kItemConsumers);
    }
    mbar_init(&bars->drain, 2);
    mbar_init(&bars->never, 1);
    for (int s = 0; s < L::kKStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < L::kVStages; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    if (!OUT_F32) prefetch_tmap(&tmap_o);
  }
  if (warp == kPvWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Item ic of this CTA, as published by the scheduler (kNoItem: none left, or the
  // scheduler stopped). Every consumer releases the slot after reading it: the issuer
  // threads themselves, the softmax warps through lane 0.
  auto next_item = [&](int ic, bool warp_release, Item& w) -> bool {
    const int slot = ic & 1;
    bool got = mbar_wait_bounded<kWaitHint>(&bars->item_full[slot], (ic >> 1) & 1, abort_flag, kTimeoutNs);
    if (warp_release) got = __all_sync(0xffffffffu, got);
    if (got) {
      const int* v = bars->item[slot];
      w = Item{v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]};
    }
    if (warp_release) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->item_empty[slot]);
    } else {
      mbar_arrive(&bars->item_empty[slot]);
    }
    return got && w.split >= 0;
  };

  // Each role branch starts with its warpgroup's setmaxnreg so that the register limit
  // ptxas applies to the code after it is the one of that branch.
  if (warp >= kEpilogueWarp0) {
    regs_dec<kEpilogueRegs>();
    // ------------------------------------------------------------ epilogue (warps 12-15)
    // Per item: merge the two halves' accumulators exactly,
    //   m = max(m_a, m_b), l = l_a 2^(m_a-m) + l_b 2^(m_b-m),
    //   o = (O_a 2^(m_a-m) + O_b 2^(m_b-m)) / l,
    // convert, stage in shared memory and write with one TMA store (fp32 partials: direct
    // stores), while the softmax warps already work on the next item. Thread lane i of warp
    // w owns query row 32*(w%4) + i (its TMEM lane), all D output columns.
    const int quarter = warp & 3;
    const int r_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const bool leader = warp == kEpilogueWarp0 && lane == 0;  // issues the TMA stores
    bool ok = true;
    for (int ic = 0; ok; ++ic) {
      Item w;
      if (!next_item(ic, true, w)) break;
      const int slot = ic & 1;
      const int row = w.q_row0 + r_in_tile;
      if (!OUT_F32) {
        // The previous item's TMA store must have read the staging buffer.
        if (leader) {
          bulk_wait_group_read0();
          mbar_arrive(&bars->stage_free);
        }
        ok = mbar_wait_bounded<kWaitHint>(&bars->stage_free, ic & 1, abort_flag, kTimeoutNs);
      }
      if (ok) ok = mbar_wait_bounded<kWaitHint>(&bars->ml_full[slot], (ic >> 1) & 1, abort_flag, kTimeoutNs);
      if (ok) ok = mbar_wait_bounded<kWaitHint>(&bars->o_final, ic & 1, abort_flag, kTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float* red_i = red + slot * (4 * kRowsPerTile);
      const float m_a = red_i[r_in_tile], m_b = red_i[kRowsPerTile + r_in_tile];
      const float l_a = red_i[2 * kRowsPerTile + r_in_tile];
      const float l_b = red_i[3 * kRowsPerTile + r_in_tile];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ml_empty[slot]);
      const float m = fmaxf(m_a, m_b);
      // A half that saw no valid key has m = -inf: weight 0.
      const float w_a = m_a == -INFINITY ? 0.f : ex2_approx(m_a - m);
      const float w_b = m_b == -INFINITY ? 0.f : ex2_approx(m_b - m);
      const float l_tot = l_a * w_a + l_b * w_b;
      // Rows without any valid key (only with a key slice) get o = 0 and lse = -inf.
      const float inv_l = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float f_a = w_a * inv_l, f_b = w_b * inv_l;
      const bool in_range = row < p.S;
      const uint32_t t_oa = tmem + lane_bits + L::kOCol;
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t oa[16], ob[16];
        if (w.n_kv > 0) {
          tmem_ld16(t_oa + c * 16, oa);
          tmem_ld16(t_oa + D + c * 16, ob);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) oa[i] = ob[i] = 0u;
        }
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          v[i] = __uint_as_float(oa[i]) * f_a + __uint_as_float(ob[i]) * f_b;
        if constexpr (OUT_F32) {
          if (in_range) {
            float4* dst = reinterpret_cast<float4*>(
                reinterpret_cast<uint8_t*>(p.o) +
                4 * (static_cast<int64_t>(w.split) * p.o_split_stride +
                     static_cast<int64_t>(w.b) * p.o_sb + static_cast<int64_t>(w.h) * p.o_sh +
                     static_cast<int64_t>(row) * p.o_ss + c * 16));
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (c * 16 + 4 * i < p.d_out)  // columns beyond the true head dim
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        } else {
          // 16 output columns = two 16-byte units of the 128-byte-swizzled staging row (the
          // layout the tensor map's SWIZZLE_128B expects: unit u of row r at
          // r*128 + ((u ^ (r % 8)) * 16) within its 64-column chunk).
          const int col = c * 16;
          uint8_t* chunk = smem + L::kStageOff + (col / 64) * (kRowsPerTile * 128);
          const int u0 = (col % 64) / 8;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint4 val = make_uint4(pack2<BF16>(v[8 * i], v[8 * i + 1]),
                                         pack2<BF16>(v[8 * i + 2], v[8 * i + 3]),
                                         pack2<BF16>(v[8 * i + 4], v[8 * i + 5]),
                                         pack2<BF16>(v[8 * i + 6], v[8 * i + 7]));
            *reinterpret_cast<uint4*>(chunk + r_in_tile * 128 +
                                      (((u0 + i) ^ (r_in_tile & 7)) * 16)) = val;
          }
        }
      }
      // O may now be overwritten by the next item's first P.V.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_empty);
      if (!OUT_F32) {
        // Hand the staged tile to the TMA store (issued by the leader once all 4 warps wrote
        // their part; rows beyond S are clipped by the tensor map).
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->staged);
        if (leader) {
          if (mbar_wait_bounded<kWaitHint>(&bars->staged, ic & 1, abort_flag, kTimeoutNs)) {
#pragma unroll
            for (int c = 0; c < L::kChunks; ++c)
              tma_store_4d(&tmap_o, smem + L::kStageOff + c * (kRowsPerTile * 128), c * 64,
                           w.q_row0, w.h, w.b);
            bulk_commit_group();
          } else {
            ok = false;
          }
        }
      }
      if (leader) TRACE_ITEM(ic, 3);
      if (p.lse != nullptr && in_range)
        p.lse[static_cast<int64_t>(w.split) * p.BH * p.S + static_cast<int64_t>(w.bh) * p.S + row] =
            l_tot > 0.f ? (m + __log2f(l_tot)) * 0.69314718055994531f : -INFINITY;
      ok = __all_sync(0xffffffffu, ok);
    }
    // Stores must have completed before the CTA exits.
    if (!OUT_F32 && leader) bulk_wait_group0();
    if (!ok && lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_EPILOG, abort_flag);
  } else if (warp >= 8) {
  regs_dec<kSideRegs>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ scheduler + TMA producer
    if (lane == 0) {
      int k_it = 0, v_it = 0, ic = 0;
      bool ok = true;
      auto load = [&](bool is_v, int key0, int h, int b) {
        int& it = is_v ? v_it : k_it;
        const int n_st = is_v ? L::kVStages : L::kKStages;
        const int st = it % n_st;
        const uint32_t ph = (it / n_st) & 1;
        uint64_t* empty = is_v ? &bars->v_empty[st] : &bars->k_empty[st];
        uint64_t* full = is_v ? &bars->v_full[st] : &bars->k_full[st];
        if (!mbar_wait_bounded<kWaitHint>(empty, ph ^ 1, abort_flag, kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          ok = false;
          return;
        }
        mbar_arrive_expect_tx(full, L::kTileBytes);
        uint8_t* dst = smem + (is_v ? L::kVOff : L::kKOff) + st * L::kTileBytes;
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(dst + c * (kKeysPerTile * 128), is_v ? &tmap_v : &tmap_k, full, c * 64,
                      key0, h, b);
        ++it;
      };
      for (; ok; ++ic) {
        // Publish the next item (or kNoItem) once its slot was released.
        const int slot = ic & 1;
        if (!mbar_wait_bounded<kWaitHint>(&bars->item_empty[slot], ((ic >> 1) & 1) ^ 1, abort_flag,
                               kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          break;
        }
        TRACE_ITEM(ic, 4);
        const int item = static_cast<int>(atomicAdd(&p.sched[0], 1u));
        TRACE_ITEM(ic, 5);
        Item w;
        if (item < n_items) w = common::decode_item<CAUSAL, kRowsPerTile, kKeysPerTile>(p, item);
        else w.split = kNoItem;
        int* pub = bars->item[slot];
        pub[0] = w.split; pub[1] = w.bh; pub[2] = w.b; pub[3] = w.h;
        pub[4] = w.q_row0; pub[5] = w.kv_lo; pub[6] = w.kv_hi; pub[7] = w.n_kv;
        mbar_arrive(&bars->item_full[slot]);
        if (w.split < 0) break;
        // Q: the previous item's QK^T MMAs must be done with the buffer.
        if (!mbar_wait_bounded<kWaitHint>(&bars->q_empty, (ic & 1) ^ 1, abort_flag, kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          break;
        }
        TRACE_ITEM(ic, 6);
        mbar_arrive_expect_tx(&bars->q_full, L::kTileBytes);
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(q_smem + c * (kRowsPerTile * 128), &tmap_q, &bars->q_full, c * 64,
                      w.q_row0, w.h, w.b);
        for (int jj = 0; ok && jj < min(NB, w.n_kv); ++jj)
          load(false, w.kv_lo + jj * kKeysPerTile, w.h, w.b);
        for (int j = 0; ok && j < w.n_kv; ++j) {
          load(true, w.kv_lo + j * kKeysPerTile, w.h, w.b);
          if (ok && j + NB < w.n_kv) load(false, w.kv_lo + (j + NB) * kKeysPerTile, w.h, w.b);
        }
      }
      // Drain: every copy this thread issued must land before the CTA may exit.
      volatile int no_abort = 0;
      bool drained = true;
      if (ic > 0)
        drained &= mbar_wait_bounded<kWaitHint>(&bars->q_full, (ic - 1) & 1, &no_abort, kTimeoutNs);
      for (int i = max(0, k_it - L::kKStages); i < k_it; ++i)
        drained &= mbar_wait_bounded<kWaitHint>(&bars->k_full[i % L::kKStages], (i / L::kKStages) & 1,
                                     &no_abort, kTimeoutNs);
      for (int i = max(0, v_it - L::kVStages); i < v_it; ++i)
        drained &= mbar_wait_bounded<kWaitHint>(&bars->v_full[i % L::kVStages], (i / L::kVStages) & 1,
                                     &no_abort, kTimeoutNs);
      if (!drained && p.status) atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else if (warp == kPvWarp) {
    // ------------------------------------------------------------ P.V issuer
    if (lane == 0) {
      constexpr uint32_t kIdescPV = idesc_f16(kRowsPerTile, D, BF16, false, true);
      const uint64_t v_desc = sdesc_sw128(smem_u32(smem + L::kVOff), kKeysPerTile * 128, 1024);
      bool ok = true;
      // Self-test of the failure path: wait on a barrier nothing arrives on, so the wait
      // runs out, the kernel records the timeout and every role returns.
      if (p.selftest_stall) ok = mbar_wait_bounded<kWaitHint>(&bars->never, 0, abort_flag, kTimeoutNs);
      int g = 0, v_it = 0;
      for (int ic = 0; ok; ++ic) {
        Item w;
        if (!next_item(ic, false, w)) break;
        // The previous item's epilogue must have read O before PV_0 overwrites it (and
        // before o_final of this item, so o_final never completes twice unobserved).
        if (ic > 0) {
          ok = mbar_wait_bounded<kWaitHint>(&bars->o_empty, (ic - 1) & 1, abort_flag, kTimeoutNs);
          if (!ok) break;
        }
        for (int j = 0; ok && j < w.n_kv; ++j, ++g) {
          const int buf = g % NB;
          const int st = v_it % L::kVStages;
          ok = mbar_wait_bounded<kWaitHint>(&bars->v_full[st], (v_it / L::kVStages) & 1, abort_flag,
                                 kTimeoutNs);
          if (!ok) break;
          // One barrier per buffer: a warpgroup may run up to NB-1 tiles ahead of the
          // other, never NB (S_{g+NB} needs PV_g), so no phase completes unobserved.
          ok = mbar_wait_bounded<kWaitHint>(&bars->p_full[buf], (g / NB) & 1, abort_flag, kTimeoutNs);
          if (!ok) break;
          TRACE(ic, j, 8);
          tc_fence_after();
          const uint64_t vd = v_desc + static_cast<uint64_t>((st * L::kTileBytes) >> 4);
          // P_g[:, keys 64*hh .. 64*hh+63] . V[those keys] into O_hh (offsets as immediates:
          // the issuer runs on few registers).
          const uint32_t acc = j > 0 ? 1u : 0u;
          pv_half_mmas<0>(tmem + L::kOCol, tmem + buf * 128, vd, kIdescPV, acc);
          pv_half_mmas<1>(tmem + L::kOCol + D, tmem + buf * 128 + kKeysPerHalf, vd, kIdescPV, acc);
          mma_commit(&bars->pv_done[g & 3]);
          mma_commit(&bars->v_empty[st]);
          ++v_it;
          TRACE(ic, j, 9);
        }
        if (!ok) break;
        mma_commit(&bars->o_final);
      }
      if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
      mma_commit(&bars->drain);
    }
    __syncwarp();
  } else if (warp == kQkWarp) {
    // ------------------------------------------------------------ QK^T issuer
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_f16(kRowsPerTile, kKeysPerTile, BF16, false, false);
      // Descriptors are built once; per K step only the start-address field (low bits)
      // advances, by a compile-time constant, so issuing an MMA costs a 64-bit add.
      const uint64_t q_desc = sdesc_sw128(smem_u32(q_smem), 16, 1024);
      const uint64_t k_desc = sdesc_sw128(smem_u32(smem + L::kKOff), 16, 1024);
      bool ok = true;
      int g = 0, k_it = 0;
      for (int ic = 0; ok; ++ic) {
        Item w;
        if (!next_item(ic, false, w)) break;
        ok = mbar_wait_bounded<kWaitHint>(&bars->q_full, ic & 1, abort_flag, kTimeoutNs);
        for (int t = 0; ok && t < w.n_kv; ++t, ++g) {
          const int buf = g % NB;
          // S_g overwrites P_{g-NB}: wait until PV_{g-NB} completed. Barrier (g-NB)%4
          // completes next for PV_{g-NB+4}, which needs S_{g-NB+4} (not issued yet), so
          // the phase test is unambiguous.
          if (g >= NB) {
            ok = mbar_wait_bounded<kWaitHint>(&bars->pv_done[(g - NB) & 3], ((g - NB) >> 2) & 1,
                                   abort_flag, kTimeoutNs);
            if (!ok) break;
          }
          const int st = k_it % L::kKStages;
          ok = mbar_wait_bounded<kWaitHint>(&bars->k_full[st], (k_it / L::kKStages) & 1, abort_flag,
                                 kTimeoutNs);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kd = k_desc + static_cast<uint64_t>((st * L::kTileBytes) >> 4);
          qk_mmas<D>(tmem + buf * 128, q_desc, kd, kIdescQK);
          mma_commit(&bars->s_full[buf]);
          mma_commit(&bars->k_empty[st]);
          ++k_it;
          TRACE(ic, t, 10);
          if (t == 0) TRACE_ITEM(ic, 7);
        }
        if (!ok) break;
        mma_commit(&bars->q_empty);  // all QK^T MMAs of this item have read Q
      }
      if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
      mma_commit(&bars->drain);
    }
    __syncwarp();
  }
  // Drain: all MMAs of both issuers complete before tensor memory is freed.
  if (warp == kPvWarp && lane == 0) {
    volatile int no_abort = 0;
    if (!mbar_wait_bounded<kWaitHint>(&bars->drain, 0, &no_abort, kTimeoutNs) && p.status)
      atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
  }
  __syncwarp();
  } else {
    regs_inc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax + epilogue
    const int half = warp >> 2;           // key columns [64*half, 64*half + 64) of each tile
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int r_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_acc = tmem + lane_bits + L::kOCol + half * D;  // this half's O
    const float sl = p.scale_log2;
    bool ok = true;
    int g = 0;
    for (int ic = 0; ok; ++ic) {
      if (threadIdx.x == 0) TRACE_ITEM(ic, 8);
      Item w;
      const bool have = next_item(ic, true, w);
      if (threadIdx.x == 0) TRACE_ITEM(ic, 9);
      if (!have) break;
      const int row = w.q_row0 + r_in_tile;
      if (threadIdx.x == 0) TRACE_ITEM(ic, 0);
      float m_run = -INFINITY;  // running max of this half, in log2 units (score*scale*log2 e)
      float l_run = 0.f;        // running row sum of this half
      for (int j = 0; j < w.n_kv; ++j, ++g) {
        const int buf = g % NB;
        const uint32_t t_s = tmem + lane_bits + buf * 128;
        ok = mbar_wait_bounded<kWaitHint>(&bars->s_full[buf], (g / NB) & 1, abort_flag, kTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (threadIdx.x % 128 == 0) TRACE(ic, j, 0 + 4 * half);
        if (threadIdx.x == 0 && j == 0) TRACE_ITEM(ic, 1);
        uint32_t s0[32], s1[32];
        tmem_ld64(t_s + half * kKeysPerHalf, s0, s1);  // one load: 2-5 % faster than two x32
        tmem_wait_ld();
        reg_fence32(s0);
        reg_fence32(s1);
        const int c0 = w.kv_lo + j * kKeysPerTile + half * kKeysPerHalf;  // key of element 0
        const bool need_mask =
            (c0 + kKeysPerHalf > w.kv_hi) || (CAUSAL && c0 + kKeysPerHalf - 1 > w.q_row0);
        if (need_mask) {
          int lim = w.kv_hi - c0;
          if (CAUSAL) lim = min(lim, row - c0 + 1);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i >= lim) s0[i] = __float_as_uint(-INFINITY);
            if (32 + i >= lim) s1[i] = __float_as_uint(-INFINITY);
          }
        }
        // Row max over this half's 64 scores: four chains of 3-input max.
        float mx0 = fmaxf(__uint_as_float(s0[0]), __uint_as_float(s0[1]));
        float mx1 = fmaxf(__uint_as_float(s0[2]), __uint_as_float(s0[3]));
        float mx2 = fmaxf(__uint_as_float(s1[0]), __uint_as_float(s1[1]));
        float mx3 = fmaxf(__uint_as_float(s1[2]), __uint_as_float(s1[3]));
#pragma unroll
        for (int i = 4; i < 32; i += 4) {
          mx0 = fmax3(mx0, __uint_as_float(s0[i]), __uint_as_float(s0[i + 1]));
          mx1 = fmax3(mx1, __uint_as_float(s0[i + 2]), __uint_as_float(s0[i + 3]));
          mx2 = fmax3(mx2, __uint_as_float(s1[i]), __uint_as_float(s1[i + 1]));
          mx3 = fmax3(mx3, __uint_as_float(s1[i + 2]), __uint_as_float(s1[i + 3]));
        }
        const float m_cand = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl;
        if (threadIdx.x % 128 == 0) TRACE(ic, j, 1 + 4 * half);
        float alpha = 1.f;
        bool rescale = false;  // warp-uniform: this warp's O rows need alpha applied
        if (j == 0) {
          m_run = m_cand;
        } else {
          const bool grow = m_cand > m_run + kRescaleThreshold;
          rescale = __any_sync(0xffffffffu, grow);
          if (grow) {
            alpha = ex2_approx(m_run - m_cand);  // 0 while m_run is -inf
            l_run *= alpha;
            m_run = m_cand;
          }
        }
        // p = 2^(s*scale*log2e - m): packed FMA, then exp2 on the MUFU (every
        // kPolyEvery-th pair on the FMA pipe where enabled).
        // A row with no valid key yet in this half (m = -inf) uses 0 as the subtrahend, so
        // its weights are exactly 0 (2^-125 on the FMA path) instead of NaN.
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const uint64_t sl2 = f2_pack(sl, sl);
        const uint64_t negm2 = f2_pack(-m_use, -m_use);
        float acc_lo[kSumChains], acc_hi[kSumChains];
#pragma unroll
        for (int c = 0; c < kSumChains; ++c) acc_lo[c] = acc_hi[c] = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t* src = i < 16 ? s0 : s1;
          const int e = 2 * (i & 15);
          float p0, p1;
          const uint64_t x2 =
              f2_fma(f2_pack(__uint_as_float(src[e]), __uint_as_float(src[e + 1])), sl2, negm2);
          if (kPolyEvery > 0 && (i % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
            f2_unpack(exp2_poly_x2(x2), p0, p1);
          } else {
            float x0, x1;
            f2_unpack(x2, x0, x1);
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          pk[i] = pack2<BF16>(p0, p1);
          // Row sum of the rounded weights the P.V MMA sees, so the output is an exact
          // convex combination of V rows with those weights (summing the fp32 weights is
          // 3-10 % faster but differs by up to 2^-9 relative, which the sigma=4 parity
          // cases expose when one weight dominates a row).
          add_packed16_to_f32<BF16>(pk[i], acc_lo[i % kSumChains], acc_hi[i % kSumChains]);
        }
        // P of this half's 64 keys: 32 columns of 16-bit pairs over the first half of this
        // half's own score columns. Waited for at once: the store may read its source
        // registers asynchronously.
        tmem_st32(t_s + half * kKeysPerHalf, pk);
        tmem_wait_st();
        {
          float tot = 0.f;
#pragma unroll
          for (int c = 0; c < kSumChains; ++c) tot += acc_lo[c] + acc_hi[c];
          l_run += tot;
        }
        if (rescale) {
          // O_half must hold exactly the PV of this item's tiles before j when scaled: wait
          // for PV_{g-1}. Barrier (g-1)%4 completes next for PV_{g+3}, which needs this
          // warpgroup's P_{g+3}; PV_{g-5} completed before S_g could be issued (S_g waits
          // for PV_{g-NB}, NB <= 3). So the phase test is unambiguous.
          bool done = mbar_wait_bounded<kWaitHint>(&bars->pv_done[(g - 1) & 3], ((g - 1) >> 2) & 1,
                                        abort_flag, kTimeoutNs);
          done = __all_sync(0xffffffffu, done);
          if (!done) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t alpha2 = f2_pack(alpha, alpha);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_acc + c * 32, o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float a0, a1;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), alpha2),
                        a0, a1);
              o[i] = __float_as_uint(a0);
              o[i + 1] = __float_as_uint(a1);
            }
            tmem_st32(t_acc + c * 32, o);
            tmem_wait_st();
          }
        }
        tc_fence_before();
        if (threadIdx.x % 128 == 0) TRACE(ic, j, 2 + 4 * half);
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[buf]);
      }
      if (!ok) break;
      // ---- end of the item: hand (m, l) of this half to the epilogue warpgroup through the
      // slot of the item's parity and go on with the next item at once.
      const int slot = ic & 1;
      ok = mbar_wait_bounded<kWaitHint>(&bars->ml_empty[slot], ((ic >> 1) & 1) ^ 1, abort_flag, kTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      float* red_i = red + slot * (4 * kRowsPerTile);
      red_i[half * kRowsPerTile + r_in_tile] = m_run;
      red_i[2 * kRowsPerTile + half * kRowsPerTile + r_in_tile] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ml_full[slot]);
      if (threadIdx.x == 0) TRACE_ITEM(ic, 2);
    }
    if (!ok && lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_SOFTMAX, abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kPvWarp) tmem_dealloc(tmem, kTmemCols);
  // The last CTA to finish resets the scheduler slot for the next launch that uses it.
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&p.sched[1], 1u) == gridDim.x - 1) {
      atomicExch(&p.sched[0], 0u);
      atomicExch(&p.sched[1], 0u);
    }
  }
}

template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
static cudaError_t launch_variant(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                  const CUtensorMap& o, const FwdParams& p, int grid,
                                  cudaStream_t stream) {
  auto kern = sdpa_fwd_kernel<D, BF16, CAUSAL, OUT_F32>;
  constexpr int smem = Layout<D>::kDynSmem;
  static int configured_mask = 0;  // one bit per device ordinal (< 32)
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 32 || !(__atomic_load_n(&configured_mask, __ATOMIC_ACQUIRE) & (1 << dev))) {
    // setmaxnreg.inc would wait forever if the block were launched with fewer
    // registers than the split assumes: check the built register count first.
    cudaFuncAttributes attr;
    err = cudaFuncGetAttributes(&attr, kern);
    if (err != cudaSuccess) return err;
    if (attr.numRegs != kLaunchRegs) return cudaErrorInvalidKernelImage;
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    if (dev < 32) __atomic_fetch_or(&configured_mask, 1 << dev, __ATOMIC_ACQ_REL);
  }
  kern<<<grid, kThreads, smem, stream>>>(q, k, v, o, p);
  return cudaGetLastError();
}

namespace {

// Scheduler slots: {next item, CTAs finished} per launch, in device memory that belongs to
// the loaded library (no allocation per call). Launches take slots round-robin; the last
// CTA of a launch resets its slot, so a slot is clean again long before it comes round
// (kSchedSlots launches later).
constexpr int kSchedSlots = 1024;
__device__ unsigned int g_sched[kSchedSlots][2];
constexpr int kMaxDevices = 64;
std::atomic<unsigned int> g_sched_next[kMaxDevices];
std::atomic<unsigned int*> g_sched_base[kMaxDevices];
std::atomic<int> g_sm_count[kMaxDevices];

}  // namespace

cudaError_t launch_sdpa_fwd(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                            const CUtensorMap& o, const FwdParams& p_in,
                            int D, bool bf16, bool causal, bool out_f32, KernelKind kind,
                            cudaStream_t stream) {
  if (kind == kSharedKv)
    return launch_sdpa_fwd_shared_kv(q, k, v, p_in, D, bf16, causal, out_f32, stream);
  const long long items = static_cast<long long>(p_in.n_split) * p_in.BH * p_in.n_qblk;
  if (items == 0) return cudaSuccess;
  if (items > 0x7fffffffll) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int sms = g_sm_count[dev].load(std::memory_order_acquire);
  if (sms == 0) {
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    void* base = nullptr;
    err = cudaGetSymbolAddress(&base, g_sched);
    if (err != cudaSuccess) return err;
    g_sched_base[dev].store(static_cast<unsigned int*>(base), std::memory_order_relaxed);
    g_sm_count[dev].store(sms, std::memory_order_release);
  }
  FwdParams p = p_in;
  // (b,h) pairs per scheduling group: as many as have K and V (S x D x 16-bit each) within
  // 48 MB, a good part of the 126 MB L2, so their re-reads stay on chip.
#ifndef TA_SCHED_GROUP_MB
#define TA_SCHED_GROUP_MB 48
#endif
  const long long kv_bytes = 4ll * p.S * D;
  const long long group = (static_cast<long long>(TA_SCHED_GROUP_MB) << 20) / (kv_bytes > 0 ? kv_bytes : 1);
  p.group_bh = static_cast<int>(group < 1 ? 1 : (group > p.BH ? p.BH : group));
  const unsigned int slot = g_sched_next[dev].fetch_add(1, std::memory_order_relaxed) % kSchedSlots;
  p.sched = g_sched_base[dev].load(std::memory_order_relaxed) + 2 * slot;
  const int grid = static_cast<int>(items < sms ? items : sms);
#define TA_DISPATCH(DD, BB, CC, FF)                                               \
  if (D == DD && bf16 == BB && causal == CC && out_f32 == FF)                     \
    return launch_variant<DD, BB, CC, FF>(q, k, v, o, p, grid, stream);
#define TA_DISPATCH2(DD, BB, CC) TA_DISPATCH(DD, BB, CC, false) TA_DISPATCH(DD, BB, CC, true)
  TA_DISPATCH2(64, false, false)
  TA_DISPATCH2(64, false, true)
  TA_DISPATCH2(64, true, false)
  TA_DISPATCH2(64, true, true)
  TA_DISPATCH2(128, false, false)
  TA_DISPATCH2(128, false, true)
  TA_DISPATCH2(128, true, false)
  TA_DISPATCH2(128, true, true)
#undef TA_DISPATCH2
#undef TA_DISPATCH
  return cudaErrorInvalidValue;
}

namespace {
std::atomic<int> g_forced_kernel{kAuto};
}  // namespace

void force_kernel(int kind) {
  g_forced_kernel.store(kind == kPersistent || kind == kSharedKv ? kind : kAuto,
                        std::memory_order_relaxed);
}

KernelKind select_kernel(int D, int S, bool causal, long long bh) {
  const int forced = g_forced_kernel.load(std::memory_order_relaxed);
  if (forced == kSharedKv && (D == 128 || D == 256)) return kSharedKv;
  if (forced == kPersistent && (D == 64 || D == 128)) return kPersistent;
  if (uses_shared_kv(D, S, causal, bh)) return kSharedKv;
  return kPersistent;
}

int rows_per_item(KernelKind kind, int D) {
  if (kind == kSharedKv) return rows_per_cta_shared_kv(D);
  return kRowsPerTile;
}

}  // namespace ta
