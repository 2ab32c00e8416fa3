// SDPA forward for B200 (sm_100a), head dims 64 and 128: persistent CTAs over 256-row work
// items, two 128-row query tiles per item whose softmax warpgroups take turns ("ping-pong")
// on one K/V stream, a separate epilogue warpgroup, TMA + mbarrier pipelines and tcgen05
// MMAs with accumulators in tensor memory.
//
// Algorithm (same maths as the reference cuTile kernel,
// src/tiledattention/kernels/flash_fwd.py:374-446 of thisistaimur/TiledAttention):
//   for each query row r:  m = -inf, l = 0, acc = 0
//   for each key tile:     s = q_r . k_c * scale, masked to -inf where c >= S or
//                          (causal and c > r)                    (flash_fwd.py:400-423)
//                          m' = max(m, max_c s); alpha = exp(m - m')
//                          p = exp(s - m'); l = l*alpha + sum p; acc = acc*alpha + p v
//   o_r = acc / l                                               (flash_fwd.py:438-444)
// Differences in precision, all towards the fp32 oracle: scores and P.V products are
// accumulated in fp32 tensor memory (the cuTile kernel rounds each tile product to the
// input dtype), and the exponent is evaluated as exp2 with log2(e) folded into the scale.
// The running max is rescaled lazily: an accumulator is only rescaled when its max grows
// by more than 2^8, which is exact after the final division by l. The row sum adds the
// 16-bit rounded weights the P.V MMA sees, so each output row is an exact convex
// combination of V rows with those weights.
//
// Why two query tiles. Per 128-key tile a 128-row query tile needs QK^T and P.V (8 MMAs of
// 128x128x16 each at D=128) and 128x128 exp2 on the MUFU (16 per clock per SM), and the two
// are dependent: the softmax of S_j needs S_j, P_j feeds P.V_j, and S_{j+1} may only
// overwrite S_j's tensor memory once P.V_j has read P_j. With two tiles A and B sharing each
// K/V tile, one MMA thread per tile issues P.V_t(j) then QK^T_t(j+1) (in order, so the
// buffer reuse is safe), the tensor core works on one tile while the other tile's softmax
// runs, and the two softmax warpgroups take turns on the MUFU (an mbarrier pair), each
// running its exponentials alone. Per item the K/V tiles are loaded once for 256 query rows.
// P is published in two halves of 64 keys, so the first half's P.V MMAs run while the
// softmax computes the second half.
//
// Work: one item = one (key slice, batch*head pair, 256-row query block). The grid has at
// most one CTA per SM; items come from a global counter, in groups of (b,h) pairs whose K/V
// fit in L2, longest causal blocks of a group first. Consecutive items overlap: each MMA
// thread issues the next item's first QK^T right behind the current item's last P.V, and
// the epilogue of item i runs while the softmax warps work on item i+1.
//
// CTA organisation (512 threads, one CTA per SM, all 512 tensor-memory columns):
//   warps 0-3   softmax of query tile A (rows q0 .. q0+127 of the item); thread lane i of
//               warp w owns row 32*(w%4)+i, its TMEM lane
//   warps 4-7   softmax of query tile B (rows q0+128 .. q0+255)
//   warps 8-11  epilogue: o = acc / l for both tiles, 16-bit (or fp32 partial) stores, lse
//   warp  12    scheduler: takes items from the global counter, publishes them decoded, and
//               loads their Q tiles (TMA) after an L2 prefetch issued as early as it can
//   warp  13    tensor-memory allocator and MMA issuer of tile A (one elected thread)
//   warp  14    K/V producer (TMA), one ring for K and V tiles in consumption order
//   warp  15    MMA issuer of tile B
// Tensor memory: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [256+D,256+2D). P_t
// (16-bit, two per column) overwrites the first 64 columns of S_t, which the softmax has
// read into registers by then, and feeds the P.V MMA from tensor memory.
//
// Every wait is bounded (shared abort flag + global-timer timeout); on expiry the kernel
// records TA_DEVSTAT_* bits in the status word, drains its own in-flight TMA copies and
// MMAs, frees tensor memory and returns.

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
namespace pingpong {

using common::add_packed16_to_f32;
using common::Item;
using common::pack2;
using common::report;

constexpr int kRowsPerTile = 128;  // query rows per tile (= TMEM lanes)
constexpr int kTiles = 2;          // query tiles per item
constexpr int kRowsPerItem = kRowsPerTile * kTiles;
constexpr int kKeysPerTile = 128;  // keys per K/V tile
constexpr int kThreads = 512;
// Register split: launch bounds 512 x 1 give 128 registers per thread; after start-up the
// epilogue warpgroup drops to kEpilogueRegs, the producer/MMA/scheduler warpgroup to
// kSideRegs, and the two softmax warpgroups rise to kSoftmaxRegs. The sum equals the launch
// allocation, so every setmaxnreg.inc can be satisfied; the host refuses to launch a build
// whose register count differs from kLaunchRegs.
constexpr int kLaunchRegs = 128;
#ifndef TA_PP_SOFTMAX_REGS
#define TA_PP_SOFTMAX_REGS 192
#define TA_PP_EPILOGUE_REGS 72
#define TA_PP_SIDE_REGS 56
#endif
constexpr int kSoftmaxRegs = TA_PP_SOFTMAX_REGS;
constexpr int kEpilogueRegs = TA_PP_EPILOGUE_REGS;
constexpr int kSideRegs = TA_PP_SIDE_REGS;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kEpilogueRegs + 128 * kSideRegs ==
                  kThreads * kLaunchRegs,
              "register split must match the launch allocation");
constexpr int kEpilogueWarp0 = 8;
constexpr int kSchedWarp = 12;  // scheduler + Q producer (first warp of the side warpgroup)
constexpr int kMmaWarpA = 13;   // MMA issuer of query tile A, tensor-memory allocator
constexpr int kKvWarp = 14;     // K/V producer
constexpr int kMmaWarpB = 15;   // MMA issuer of query tile B
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kSumChains = 4;              // independent row-sum accumulators
constexpr uint64_t kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr int kItemSlots = 4;
// Item consumers: K/V producer, the two MMA threads, lane 0 of each softmax and epilogue
// warp (the scheduler keeps its own copy).
constexpr int kItemConsumers = 3 + 8 + 4;
constexpr int kNoItem = -1;

// Every kPolyEvery-th element pair computes exp2 on the FMA pipe instead of the MUFU (0:
// never), to take load off the MUFU where it is the limit.
template <int D>
__host__ __device__ constexpr int poly_every() {
#if defined(TA_PP_POLY_D64) && defined(TA_PP_POLY_D128)
  return D == 64 ? TA_PP_POLY_D64 : TA_PP_POLY_D128;
#else
  return D == 64 ? 4 : 0;
#endif
}

// How the softmax warps wait for their MUFU turn and their next score tile: 0 = suspending
// try_wait, 1 = polling test_wait, 2 = polling with a short nap between polls.
#ifndef TA_PP_SOFTMAX_WAIT
#define TA_PP_SOFTMAX_WAIT 0
#endif

template <int D>
struct Layout {
  static_assert(D == 64 || D == 128, "this kernel serves head dims 64 and 128");
  static constexpr int kTileBytes = kRowsPerTile * D * 2;  // 128 rows x D x 16-bit
  static constexpr int kChunks = D / 64;                   // 128-byte swizzle atoms per row
  static constexpr int kQStages = 2;                       // Q slot t holds query tile t
  static constexpr int kKvStages = (D == 64) ? 8 : 4;      // K and V tiles, one ring
  static constexpr int kOCol = 256;                        // O_A at 256, O_B at 256 + D
  static constexpr int kQOff = 0;
  static constexpr int kKvOff = kQOff + kQStages * kTileBytes;
  static constexpr int kRedOff = kKvOff + kKvStages * kTileBytes;
  static constexpr int kRedBytes = 2 * kTiles * 2 * kRowsPerTile * 4;  // [slot][tile][m|l][row]
  static constexpr int kBarOff = kRedOff + kRedBytes;
  static constexpr int kBytes = kBarOff + 1024;
  static constexpr int kDynSmem = kBytes + 1024;  // slack for 1024-byte alignment
  static_assert(kDynSmem <= 227 * 1024, "shared memory");
};

// Barriers that a whole warpgroup signals take one arrival per warp after a warp sync (128
// arrivals on one barrier are 128 serialised shared-memory atomics).
struct Barriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[8], kv_empty[8];
  uint64_t s_full[kTiles];         // score tile of query tile t complete (MMA commit)
  uint64_t p_half[kTiles];         // P of keys 0-63 of tile t stored, O rescaled (4 warps)
  uint64_t p_full[kTiles];         // P of keys 64-127 of tile t stored (4 warps)
  uint64_t o_full[kTiles];         // all P.V of the item's tile t completed (MMA commit)
  uint64_t o_empty[kTiles];        // the epilogue read O_t (4 warps)
  uint64_t ml_full[kTiles][2];     // softmax -> epilogue: (m, l) of the item (4 warps)
  uint64_t ml_empty[kTiles][2];    // the epilogue read them (4 warps)
  uint64_t exp_done[kTiles];       // softmax t finished the exponentials of a step (4 warps)
  uint64_t item_full[kItemSlots], item_empty[kItemSlots];
  uint64_t drain;                  // the MMA threads' last commits
  uint64_t never;                  // self-test only: a barrier nothing arrives on
  int item[kItemSlots][8];         // published items, decoded (split < 0: no item)
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 1024, "barrier block");

#ifdef TA_TRACE
// Experiment builds only: clock64 of event `ev` (< 16) of step j (< 32) of the first item of
// the first 64 blocks, for timeline analysis.
__device__ __forceinline__ void trace_ev(const FwdParams& p, int ic, int j, int ev) {
  if (p.trace && ic == 0 && blockIdx.x < 64 && j < 32) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    p.trace[(blockIdx.x * 32 + j) * 16 + ev] = c;
  }
}
#define TRACE(ic, j, ev) trace_ev(p, (ic), (j), (ev))
#else
#define TRACE(ic, j, ev)
#endif

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

// O (+)= P V over keys [16 kk, 16 kk1) of a 128-key tile: MMAs of K=16 keys. P comes from
// tensor memory (16-bit pairs, 8 columns per 16 keys); V is MN-major, 128-byte swizzled (16
// key rows = 2 KB). `acc` is the accumulate flag of the tile's first MMA (kk = 0).
template <int kk, int kk1>
__device__ __forceinline__ void pv_mmas(uint32_t d_tmem, uint32_t a_tmem, uint64_t vd,
                                        uint32_t idesc, uint32_t acc) {
  if constexpr (kk < kk1) {
    constexpr uint32_t off = (kk * 16 * 128) >> 4;
    if constexpr (kk == 0)
      mma_ts_imm_acc<0, off>(d_tmem, a_tmem, vd, idesc, acc);
    else
      mma_ts_imm<kk * 8, off, 1u>(d_tmem, a_tmem, vd, idesc);
    pv_mmas<kk + 1, kk1>(d_tmem, a_tmem, vd, idesc, acc);
  }
}

// How the MMA issuers wait for P: 0 = suspending try_wait, 1 = polling, 2 = polling with naps.
#ifndef TA_PP_ISSUER_WAIT
#define TA_PP_ISSUER_WAIT 0
#endif
__device__ __forceinline__ bool issuer_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                            uint64_t timeout_ns) {
#if TA_PP_ISSUER_WAIT == 1
  return mbar_wait_spin(bar, parity, abort_flag, timeout_ns);
#elif TA_PP_ISSUER_WAIT == 2
  return mbar_wait_spin(bar, parity, abort_flag, timeout_ns, 20);
#else
  return mbar_wait_bounded(bar, parity, abort_flag, timeout_ns);
#endif
}

__device__ __forceinline__ bool softmax_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             uint64_t timeout_ns) {
#if TA_PP_SOFTMAX_WAIT == 1
  return mbar_wait_spin(bar, parity, abort_flag, timeout_ns);
#elif TA_PP_SOFTMAX_WAIT == 2
  return mbar_wait_spin(bar, parity, abort_flag, timeout_ns, 32);
#else
  return mbar_wait_bounded(bar, parity, abort_flag, timeout_ns);
#endif
}

// OUT_F32: write o as fp32 (the normalised partial output of one key slice) instead of the
// input dtype. Items: n_split x B*H x n_qblk (blocks of 256 rows); slice s covers keys
// [kv_begin + s*split_len, min(kv_end, kv_begin + (s+1)*split_len)).
template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    sdpa_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const FwdParams p) {
  using L = Layout<D>;
  constexpr int kPolyEvery = poly_every<D>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bars->abort_flag;
  const uint64_t kTimeoutNs = p.timeout_ns ? p.timeout_ns : kDefaultTimeoutNs;
  const int n_items = p.n_split * p.BH * p.n_qblk;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], 1);
    }
    for (int s = 0; s < L::kKvStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], kTiles);  // both MMA threads release each entry
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_half[t], 4);
      mbar_init(&bars->p_full[t], 4);
      mbar_init(&bars->o_full[t], 1);
      mbar_init(&bars->o_empty[t], 4);
      for (int s = 0; s < 2; ++s) {
        mbar_init(&bars->ml_full[t][s], 4);
        mbar_init(&bars->ml_empty[t][s], 4);
      }
      mbar_init(&bars->exp_done[t], 4);
    }
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&bars->item_full[i], 1);
      mbar_init(&bars->item_empty[i], kItemConsumers);
    }
    mbar_init(&bars->drain, kTiles);
    mbar_init(&bars->never, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kSchedWarp && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  if (warp == kMmaWarpA) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Item ic of this CTA, as published by the scheduler (false: none left, or the scheduler
  // stopped). Every consumer releases the slot after reading it: single threads directly,
  // warps through lane 0.
  auto next_item = [&](int ic, bool warp_release, Item& w) -> bool {
    const int slot = ic % kItemSlots;
    bool got = mbar_wait_bounded(&bars->item_full[slot], (ic / kItemSlots) & 1, abort_flag,
                                 kTimeoutNs);
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
  if (warp >= kSchedWarp) {
    regs_dec<kSideRegs>();
    if (warp == kSchedWarp) {
      // ---------------------------------------------------------- scheduler + Q producer
      if (lane == 0) {
        int qph = 0;  // phase of the Q loads (one pair of Q tiles per item with key tiles)
        bool ok = true;
        for (int ic = 0; ok; ++ic) {
          const int slot = ic % kItemSlots;
          if (!mbar_wait_bounded(&bars->item_empty[slot], ((ic / kItemSlots) & 1) ^ 1,
                                 abort_flag, kTimeoutNs)) {
            if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
            break;
          }
          const int item = static_cast<int>(atomicAdd(&p.sched[0], 1u));
          Item w;
          if (item < n_items)
            w = common::decode_item<CAUSAL, kRowsPerItem, kKeysPerTile>(p, item);
          else
            w.split = kNoItem;
          int* pub = bars->item[slot];
          pub[0] = w.split; pub[1] = w.bh; pub[2] = w.b; pub[3] = w.h;
          pub[4] = w.q_row0; pub[5] = w.kv_lo; pub[6] = w.kv_hi; pub[7] = w.n_kv;
          mbar_arrive(&bars->item_full[slot]);
          if (w.split < 0) break;
          if (w.n_kv == 0) continue;  // no QK^T MMAs: no Q needed
          // Warm L2 with both tiles while the previous item's MMAs still hold the buffers.
          for (int t = 0; t < kTiles; ++t)
            for (int c = 0; c < L::kChunks; ++c)
              tma_prefetch_l2_4d(&tmap_q, c * 64, w.q_row0 + t * kRowsPerTile, w.h, w.b);
          // Q tile t of every item goes to Q slot t.
          for (int t = 0; t < kTiles; ++t) {
            if (!mbar_wait_bounded(&bars->q_empty[t], qph ^ 1, abort_flag, kTimeoutNs)) {
              if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->q_full[t], L::kTileBytes);
            uint8_t* dst = smem + L::kQOff + t * L::kTileBytes;
            for (int c = 0; c < L::kChunks; ++c)
              tma_load_4d(dst + c * (kRowsPerTile * 128), &tmap_q, &bars->q_full[t], c * 64,
                          w.q_row0 + t * kRowsPerTile, w.h, w.b);
          }
          if (ok) qph ^= 1;
        }
        // Drain: every copy this thread issued must land before the CTA may exit (the last
        // loads of each slot completed phase qph ^ 1; with no load, that wait passes).
        volatile int no_abort = 0;
        bool drained = true;
        if (ok)
          for (int t = 0; t < kTiles; ++t)
            drained &= mbar_wait_bounded(&bars->q_full[t], qph ^ 1, &no_abort, kTimeoutNs);
        if (!drained && p.status) atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
      }
      __syncwarp();
    } else if (warp == kKvWarp) {
      // ---------------------------------------------------------- K/V producer
      if (lane == 0) {
        int it = 0;  // ring entries loaded: K(0), V(0), K(1), V(1), ... of every item
        bool ok = true;
        for (int ic = 0; ok; ++ic) {
          Item w;
          if (!next_item(ic, false, w)) break;
          for (int e = 0; ok && e < 2 * w.n_kv; ++e, ++it) {
            const int st = it % L::kKvStages;
            if (!mbar_wait_bounded(&bars->kv_empty[st], ((it / L::kKvStages) & 1) ^ 1,
                                   abort_flag, kTimeoutNs)) {
              if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->kv_full[st], L::kTileBytes);
            const CUtensorMap* map = (e & 1) ? &tmap_v : &tmap_k;
            const int key0 = w.kv_lo + (e >> 1) * kKeysPerTile;
            uint8_t* dst = smem + L::kKvOff + st * L::kTileBytes;
            for (int c = 0; c < L::kChunks; ++c)
              tma_load_4d(dst + c * (kKeysPerTile * 128), map, &bars->kv_full[st], c * 64, key0,
                          w.h, w.b);
          }
        }
        volatile int no_abort = 0;
        bool drained = true;
        for (int i = max(0, it - L::kKvStages); i < it; ++i)
          drained &= mbar_wait_bounded(&bars->kv_full[i % L::kKvStages], (i / L::kKvStages) & 1,
                                       &no_abort, kTimeoutNs);
        if (!drained && p.status) atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
      }
      __syncwarp();
    } else {
      // ---------------------------------------------------------- MMA issuers (warps 13, 15)
      // One thread per query tile, each issuing its tile's MMAs in order: P.V_t(j) then
      // QK^T_t(j+1), so S_t(j+1) never overwrites P_t(j) before P.V_t(j) read it, and the
      // completion of S_t(j+1) implies that of P.V_t(j). The tensor pipe takes the two
      // threads' MMAs as they come; each thread waits only for its own tile's barriers, so
      // while one waits the other's MMAs keep the pipe busy (one thread issuing all MMAs and
      // waiting on all barriers was measured to be the bottleneck).
      const int t = warp == kMmaWarpB ? 1 : 0;
      if (lane == 0) {
        constexpr uint32_t kIdescQK = idesc_f16(kRowsPerTile, kKeysPerTile, BF16, false, false);
        constexpr uint32_t kIdescPV = idesc_f16(kRowsPerTile, D, BF16, false, true);
        // Descriptors are built once; per step only the start-address field (low bits)
        // advances, by immediates inside the MMA instructions.
        const uint64_t q_desc =
            sdesc_sw128(smem_u32(smem + L::kQOff + t * L::kTileBytes), 16, 1024);
        const uint64_t k_desc = sdesc_sw128(smem_u32(smem + L::kKvOff), 16, 1024);
        const uint64_t v_desc = sdesc_sw128(smem_u32(smem + L::kKvOff), kKeysPerTile * 128, 1024);
        const uint32_t s_tmem = tmem + t * 128;
        const uint32_t o_tmem = tmem + L::kOCol + t * D;
        int kv = 0;   // ring entries consumed
        int qph = 0;  // phase of the current item's Q load (items without key tiles load none)
        int g = 0;    // steps (key tiles) issued, over all items
        bool ok = true;
        // Self-test of the failure path: wait on a barrier nothing arrives on, so the wait
        // runs out, the kernel records the timeout and every role returns.
        if (p.selftest_stall) ok = mbar_wait_bounded(&bars->never, 0, abort_flag, kTimeoutNs);

        auto wait_kv = [&](int e) -> bool {
          return mbar_wait_bounded(&bars->kv_full[e % L::kKvStages], (e / L::kKvStages) & 1,
                                   abort_flag, kTimeoutNs);
        };
        // Key-tile count of item ic, or -1 when there is none.
        auto item_tiles = [&](int ic) -> int {
          Item w;
          return next_item(ic, false, w) ? w.n_kv : -1;
        };
        // QK^T against the K tile in ring entry e (waited for first), into S_t. ph >= 0: the
        // item's first QK^T, which waits for the Q load of phase ph; `last_qk`: the tile's
        // last QK^T of the item, which releases the Q slot. Releases the K entry.
        auto issue_qk = [&](int ph, int e, bool last_qk) -> bool {
          if (!wait_kv(e)) return false;
          if (ph >= 0 && !mbar_wait_bounded(&bars->q_full[t], ph, abort_flag, kTimeoutNs))
            return false;
          tc_fence_after();
          qk_mmas<D>(s_tmem, q_desc,
                     k_desc + static_cast<uint64_t>(((e % L::kKvStages) * L::kTileBytes) >> 4),
                     kIdescQK);
          mma_commit(&bars->s_full[t]);
          if (last_qk) mma_commit(&bars->q_empty[t]);
          mma_commit(&bars->kv_empty[e % L::kKvStages]);
          return true;
        };

        int ic = 0;
        int n = ok ? item_tiles(0) : -1;  // key tiles of the current item
        bool started = false;             // its first QK^T already issued
        while (ok && n >= 0) {
          if (n == 0) {
            // No key tile: no MMAs; the epilogue writes zeros. Keep the o_empty / o_full
            // phases in step with the item count.
            if (ic > 0)
              ok = mbar_wait_bounded(&bars->o_empty[t], (ic - 1) & 1, abort_flag, kTimeoutNs);
            if (!ok) break;
            mma_commit(&bars->o_full[t]);
            ++ic;
            n = item_tiles(ic);
            started = false;
            continue;
          }
          if (!started) {
            ok = issue_qk(qph, kv, n == 1);  // K(0)
            if (!ok) break;
            ++kv;
          }
          int n_next = -1;  // key tiles of the next item, once fetched
          for (int j = 0; ok && j < n; ++j, ++g) {
            const bool last = (j + 1 == n);
            const int e_v = kv;  // V(j); the ring entry after it is K(j+1) or the next K(0)
            TRACE(ic, j, 4 + 4 * t);
            ok = wait_kv(e_v);
            if (ok && j == 0 && ic > 0)  // the previous item's epilogue has read O_t
              ok = mbar_wait_bounded(&bars->o_empty[t], (ic - 1) & 1, abort_flag, kTimeoutNs);
            // P arrives in two halves (keys 0-63, 64-127): P.V of the first half runs while
            // the softmax computes the second. Polling waits: these are on the critical path.
            if (ok) ok = issuer_wait(&bars->p_half[t], g & 1, abort_flag, kTimeoutNs);
            if (!ok) break;
            TRACE(ic, j, 5 + 4 * t);
            tc_fence_after();
            const uint64_t vd =
                v_desc + static_cast<uint64_t>(((e_v % L::kKvStages) * L::kTileBytes) >> 4);
            pv_mmas<0, 4>(o_tmem, s_tmem, vd, kIdescPV, j > 0 ? 1u : 0u);
            ok = issuer_wait(&bars->p_full[t], g & 1, abort_flag, kTimeoutNs);
            if (!ok) break;
            tc_fence_after();
            pv_mmas<4, 8>(o_tmem, s_tmem, vd, kIdescPV, 1u);
            mma_commit(&bars->kv_empty[e_v % L::kKvStages]);
            TRACE(ic, j, 6 + 4 * t);
            if (last) {
              mma_commit(&bars->o_full[t]);
              n_next = item_tiles(ic + 1);
              // The next item's first QK^T right behind this P.V.
              if (n_next > 0) ok = issue_qk(qph ^ 1, e_v + 1, n_next == 1);
            } else {
              ok = issue_qk(-1, e_v + 1, j + 2 == n);
            }
            TRACE(ic, j, 7 + 4 * t);
            kv += (last && n_next <= 0) ? 1 : 2;
          }
          if (!ok) break;
          qph ^= 1;
          ++ic;
          n = n_next;
          started = n_next > 0;
        }
        if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
        // Drain: every MMA this thread issued completes before tensor memory is freed.
        mma_commit(&bars->drain);
      }
      __syncwarp();
      if (warp == kMmaWarpA && lane == 0) {
        volatile int no_abort = 0;
        if (!mbar_wait_bounded(&bars->drain, 0, &no_abort, kTimeoutNs) && p.status)
          atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
      }
      __syncwarp();
    }
  } else if (warp >= kEpilogueWarp0) {
    regs_dec<kEpilogueRegs>();
    // ------------------------------------------------------------ epilogue (warps 8-11)
    const int quarter = warp & 3;
    const int r_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    for (int ic = 0; ok; ++ic) {
      Item w;
      if (!next_item(ic, true, w)) break;
      const int slot = ic & 1;
      for (int t = 0; t < kTiles; ++t) {
        ok = mbar_wait_bounded(&bars->ml_full[t][slot], (ic >> 1) & 1, abort_flag, kTimeoutNs);
        if (ok) ok = mbar_wait_bounded(&bars->o_full[t], ic & 1, abort_flag, kTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float* red_t = red + (slot * kTiles + t) * (2 * kRowsPerTile);
        const float m = red_t[r_in_tile];
        const float l = red_t[kRowsPerTile + r_in_tile];
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ml_empty[t][slot]);
        // Rows without any valid key (only with a key slice) get o = 0 and lse = -inf.
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        const int row = w.q_row0 + t * kRowsPerTile + r_in_tile;
        const bool in_range = row < p.S;
        const uint32_t t_o = tmem + lane_bits + L::kOCol + t * D;
        constexpr int kOutBytes = OUT_F32 ? 4 : 2;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                        kOutBytes * (static_cast<int64_t>(w.split) * p.o_split_stride +
                                     static_cast<int64_t>(w.b) * p.o_sb +
                                     static_cast<int64_t>(w.h) * p.o_sh +
                                     static_cast<int64_t>(row) * p.o_ss);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          if (w.n_kv > 0) {
            tmem_ld32(t_o + c * 32, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
          if constexpr (OUT_F32) {
            if (in_range) {
              float4* dst = reinterpret_cast<float4*>(orow + c * 128);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (c * 32 + 4 * i < p.d_out)  // columns beyond the true head dim
                  dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l,
                                       __uint_as_float(o[4 * i + 1]) * inv_l,
                                       __uint_as_float(o[4 * i + 2]) * inv_l,
                                       __uint_as_float(o[4 * i + 3]) * inv_l);
            }
          } else {
            uint32_t pw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pw[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l,
                                  __uint_as_float(o[2 * i + 1]) * inv_l);
            if (in_range) {
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (c * 32 + 8 * i < p.d_out)  // columns beyond the true head dim
                  dst[i] = make_uint4(pw[4 * i], pw[4 * i + 1], pw[4 * i + 2], pw[4 * i + 3]);
            }
          }
        }
        // O_t may now be overwritten by the next item's first P.V.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->o_empty[t]);
        if (p.lse != nullptr && in_range)
          p.lse[static_cast<int64_t>(w.split) * p.BH * p.S + static_cast<int64_t>(w.bh) * p.S + row] =
              l > 0.f ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
      }
    }
    if (!ok && lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_EPILOG, abort_flag);
  } else {
    regs_inc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax (warps 0-7)
    const int t = warp >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int r_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_bits + t * 128;
    const uint32_t t_o = tmem + lane_bits + L::kOCol + t * D;
    const float sl = p.scale_log2;
    bool ok = true;
    int g = 0;
    for (int ic = 0; ok; ++ic) {
      Item w;
      if (!next_item(ic, true, w)) break;
      const int tile_row0 = w.q_row0 + t * kRowsPerTile;
      const int row = tile_row0 + r_in_tile;
      float m_run = -INFINITY;  // running max, log2 units (score * scale * log2 e)
      float l_run = 0.f;
      for (int j = 0; j < w.n_kv; ++j, ++g) {
        ok = softmax_wait(&bars->s_full[t], g & 1, abort_flag, kTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        if (r_in_tile == 0) TRACE(ic, j, 0 + 2 * t);
        tc_fence_after();
        uint32_t s[4][32];
        tmem_ld64(t_s, s[0], s[1]);
        tmem_ld64(t_s + 64, s[2], s[3]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) reg_fence32(s[q]);
        const int c0 = w.kv_lo + j * kKeysPerTile;  // key of column 0
        const bool need_mask =
            (c0 + kKeysPerTile > w.kv_hi) || (CAUSAL && c0 + kKeysPerTile - 1 > tile_row0);
        if (need_mask) {
          int lim = w.kv_hi - c0;
          if (CAUSAL) lim = min(lim, row - c0 + 1);
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (32 * q + i >= lim) s[q][i] = __float_as_uint(-INFINITY);
        }
        // Row max over 128 scores: eight independent chains of 3-input max.
        float mx[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          mx[2 * q] = fmaxf(__uint_as_float(s[q][0]), __uint_as_float(s[q][1]));
          mx[2 * q + 1] = fmaxf(__uint_as_float(s[q][16]), __uint_as_float(s[q][17]));
#pragma unroll
          for (int i = 2; i < 16; i += 2) {
            mx[2 * q] = fmax3(mx[2 * q], __uint_as_float(s[q][i]), __uint_as_float(s[q][i + 1]));
            mx[2 * q + 1] = fmax3(mx[2 * q + 1], __uint_as_float(s[q][16 + i]),
                                  __uint_as_float(s[q][17 + i]));
          }
        }
        const float m_cand =
            fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) * sl;
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
        // The two warpgroups take turns on the MUFU: A's exponentials of step g come after
        // B's of step g-1, B's of step g after A's of step g. Each then runs alone on the
        // MUFU while the tensor core works on the other tile (the two issuers alone would
        // let the tiles drift into lockstep). Loads and row maxima overlap the other's turn.
        if (t == 1 || g > 0) {
          const int phase = t == 0 ? ((g - 1) & 1) : (g & 1);
          ok = softmax_wait(&bars->exp_done[t ^ 1], phase, abort_flag, kTimeoutNs);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
        }
        if (r_in_tile == 0) TRACE(ic, j, 12 + t);
        // p = 2^(s*scale*log2e - m): packed FMA, then exp2 on the MUFU (every kPolyEvery-th
        // pair on the FMA pipe where enabled). A row with no valid key yet (m = -inf) uses 0
        // as the subtrahend, so its weights are exactly 0 instead of NaN.
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const uint64_t sl2 = f2_pack(sl, sl);
        const uint64_t negm2 = f2_pack(-m_use, -m_use);
        float acc_lo[kSumChains], acc_hi[kSumChains];
#pragma unroll
        for (int c = 0; c < kSumChains; ++c) acc_lo[c] = acc_hi[c] = 0.f;
        // Two halves of 64 keys; after the first, P of keys 0-63 is published (with O
        // rescaled first where the max grew), so the first P.V MMAs run during the second.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int q = 2 * h; q < 2 * h + 2; ++q) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float p0, p1;
              const uint64_t x2 = f2_fma(
                  f2_pack(__uint_as_float(s[q][2 * i]), __uint_as_float(s[q][2 * i + 1])), sl2, negm2);
              const int pair = q * 16 + i;
              if (kPolyEvery > 0 && (pair % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
                f2_unpack(exp2_poly_x2(x2), p0, p1);
              } else {
                float x0, x1;
                f2_unpack(x2, x0, x1);
                p0 = ex2_approx(x0);
                p1 = ex2_approx(x1);
              }
              pk[i] = pack2<BF16>(p0, p1);
              add_packed16_to_f32<BF16>(pk[i], acc_lo[i % kSumChains], acc_hi[i % kSumChains]);
            }
            // Keys 32q .. 32q+31 -> P columns 16q .. 16q+15 (two 16-bit weights per column).
            tmem_st16(t_s + 16 * q, pk);
          }
          if (h == 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->exp_done[t]);  // the MUFU is the other's
          }
          tmem_wait_st();
          if (h == 0 && rescale) {
            // O_t holds exactly the P.V of this item's tiles before j: S_t(j) was issued
            // after P.V_t(j-1) and its completion (s_full) implies that of every earlier MMA.
            const uint64_t alpha2 = f2_pack(alpha, alpha);
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(t_o + c * 32, o);
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
              tmem_st32(t_o + c * 32, o);
              tmem_wait_st();
            }
          }
          tc_fence_before();
          if (h == 1 && r_in_tile == 0) TRACE(ic, j, 1 + 2 * t);
          if (h == 1 && r_in_tile == 96) TRACE(ic, j, 14 + t);
          __syncwarp();
          if (lane == 0) mbar_arrive(h == 0 ? &bars->p_half[t] : &bars->p_full[t]);
        }
        {
          float tot = 0.f;
#pragma unroll
          for (int c = 0; c < kSumChains; ++c) tot += acc_lo[c] + acc_hi[c];
          l_run += tot;
        }
      }
      if (!ok) break;
      // Hand (m, l) of the item to the epilogue through slot ic & 1.
      const int slot = ic & 1;
      ok = mbar_wait_bounded(&bars->ml_empty[t][slot], ((ic >> 1) & 1) ^ 1, abort_flag, kTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      float* red_t = red + (slot * kTiles + t) * (2 * kRowsPerTile);
      red_t[r_in_tile] = m_run;
      red_t[kRowsPerTile + r_in_tile] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ml_full[t][slot]);
    }
    if (!ok && lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_SOFTMAX, abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarpA) tmem_dealloc(tmem, kTmemCols);
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
                                  const FwdParams& p, int grid, cudaStream_t stream) {
  auto kern = sdpa_fwd_kernel<D, BF16, CAUSAL, OUT_F32>;
  constexpr int smem = Layout<D>::kDynSmem;
  static int configured_mask = 0;  // one bit per device ordinal (< 32)
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 32 || !(__atomic_load_n(&configured_mask, __ATOMIC_ACQUIRE) & (1 << dev))) {
    // setmaxnreg.inc would wait forever if the block were launched with fewer registers
    // than the split assumes: check the built register count first.
    cudaFuncAttributes attr;
    err = cudaFuncGetAttributes(&attr, kern);
    if (err != cudaSuccess) return err;
    if (attr.numRegs != kLaunchRegs) return cudaErrorInvalidKernelImage;
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    if (dev < 32) __atomic_fetch_or(&configured_mask, 1 << dev, __ATOMIC_ACQ_REL);
  }
  kern<<<grid, kThreads, smem, stream>>>(q, k, v, p);
  return cudaGetLastError();
}

}  // namespace pingpong

cudaError_t launch_sdpa_fwd_pingpong(const CUtensorMap& q, const CUtensorMap& k,
                                     const CUtensorMap& v, const FwdParams& p, int grid, int D,
                                     bool bf16, bool causal, bool out_f32, cudaStream_t stream) {
#define TA_DISPATCH(DD, BB, CC, FF)                                               \
  if (D == DD && bf16 == BB && causal == CC && out_f32 == FF)                     \
    return pingpong::launch_variant<DD, BB, CC, FF>(q, k, v, p, grid, stream);
#define TA_DISPATCH4(DD)                                                          \
  TA_DISPATCH(DD, false, false, false) TA_DISPATCH(DD, false, false, true)        \
  TA_DISPATCH(DD, false, true, false) TA_DISPATCH(DD, false, true, true)          \
  TA_DISPATCH(DD, true, false, false) TA_DISPATCH(DD, true, false, true)          \
  TA_DISPATCH(DD, true, true, false) TA_DISPATCH(DD, true, true, true)
  TA_DISPATCH4(64)
  TA_DISPATCH4(128)
#undef TA_DISPATCH4
#undef TA_DISPATCH
  return cudaErrorInvalidValue;
}

}  // namespace ta
