// SDPA forward for B200 (sm_100a), head dim 128, on CTA pairs: the persistent split-halves
// design of sdpa_fwd_sm100.cu with every MMA issued once for two CTAs (tcgen05
// cta_group::2, M = 256: a work item is 256 query rows, 128 in each CTA of a 2-CTA
// cluster on neighbouring SMs).
//
// What the pair changes: a 128-key K tile is split by keys and a V tile by head-dim
// columns between the two CTAs (the MMA reads B's N extent half from each CTA), so each SM
// copies and reads half as much K/V through shared memory per tile. In the single-CTA
// kernel the QK^T MMA needs the full 128 B/clock of shared-memory bandwidth for its two
// operands and TMA writes compete with it; here each SM reads Q (its own 128 rows) and half
// of K. The even CTA of the pair (the leader) schedules items and issues the MMAs; both
// CTAs load their own operand halves (their copies count on the leader's barriers, no
// multicast loads), run the softmax of their own 128 rows and write their own output.
// MMA completion is signalled to both CTAs with one multicast tcgen05.commit.
//
// Maths, roles, tensor-memory layout and failure handling: as in sdpa_fwd_sm100.cu, per CTA.
// Cross-CTA waits are bounded mbarrier waits like all others; the only hardware barrier is
// the cluster barrier at start-up and exit, which every path reaches.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "sdpa_common.cuh"
#include "sm100_pair.cuh"
#include "sm100_ptx.cuh"
#include "sdpa_fwd_sm100.h"
#include "tiledattention_b200.h"

namespace ta {
namespace pair {

using common::add_packed16_to_f32;
using common::Item;
using common::pack2;
using common::report;

constexpr int kRowsPerTile = 128;  // query rows per CTA (= TMEM lanes)
constexpr int kRowsPerItem = 256;  // query rows per CTA pair
constexpr int kKeysPerTile = 128;  // keys per K/V tile
constexpr int kKeysPerHalf = 64;   // keys of one softmax half
constexpr int kThreads = 384;
constexpr int kLaunchRegs = 168;
#ifndef TA_SOFTMAX_REGS
#define TA_SOFTMAX_REGS 192
#define TA_SIDE_REGS 120
#endif
constexpr int kSoftmaxRegs = TA_SOFTMAX_REGS;
constexpr int kSideRegs = TA_SIDE_REGS;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kSideRegs == kThreads * kLaunchRegs,
              "register split must match the launch allocation");
constexpr int kProducerWarp = 8;
constexpr int kPvWarp = 9;
constexpr int kQkWarp = 10;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr int kSumChains = 4;
constexpr uint64_t kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait
// Item-broadcast consumers, counted on the leader's item_empty: leader (two issuers +
// 8 softmax warps) and peer (producer + 8 softmax warps).
constexpr int kItemConsumers = 10 + 9;
constexpr int kNoItem = -1;
constexpr uint16_t kBothCtas = 0x3;

template <int D>
struct Layout {
  static_assert(D == 128, "the CTA-pair kernel serves head dim 128");
  static constexpr int kSBufs = 2;
  static constexpr int kOCol = kSBufs * 128;
  static_assert(kOCol + 2 * D <= 512, "tensor memory columns");
  static constexpr int kQBytes = kRowsPerTile * D * 2;          // this CTA's 128 query rows
  static constexpr int kChunks = D / 64;                          // 128-byte swizzle atoms per row
  static constexpr int kKHalfBytes = (kKeysPerTile / 2) * D * 2;  // 64 keys x D
  static constexpr int kVHalfBytes = kKeysPerTile * (D / 2) * 2;  // 128 keys x D/2 columns
  static constexpr int kKStages = 4;
  static constexpr int kVStages = 4;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + kKStages * kKHalfBytes;
  static constexpr int kStageOff = kVOff + kVStages * kVHalfBytes;  // output staging
  static constexpr int kRedOff = kStageOff + kQBytes;
  static constexpr int kRedBytes = 2 * 4 * kRowsPerTile * 4;
  static constexpr int kBarOff = kRedOff + kRedBytes;
  static constexpr int kBytes = kBarOff + 512;
  static constexpr int kDynSmem = kBytes + 1024;
  static_assert(kDynSmem <= 227 * 1024, "shared memory");
};

struct Barriers {
  uint64_t q_full, q_empty;  // leader: both Q tiles loaded / both CTAs: Q no longer read
  uint64_t s_full[2];        // both: score tile in buffer complete
  uint64_t p_full[2];        // leader: P of both CTAs stored (16 warps)
  uint64_t pv_done[4];       // both: PV_g completed
  uint64_t o_final;          // both: all PV of the item completed
  uint64_t o_empty;          // leader: both CTAs' epilogues read O (16 warps)
  uint64_t ep;               // local (m, l) exchange of the two halves
  uint64_t staged;           // local output tile staged
  uint64_t item_full[2];     // both: item published into this CTA
  uint64_t item_empty[2];    // leader: every consumer of both CTAs read the slot
  uint64_t drain;            // leader: both issuers' MMAs completed
  uint64_t never;
  uint64_t k_full[4], k_empty[4];  // k_full/v_full on the leader count both CTAs' bytes
  uint64_t v_full[4], v_empty[4];
  int item[2][8];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 512, "barrier block");

#ifdef TA_TRACE
__device__ __forceinline__ void trace_ev(const FwdParams& p, int item_no, int j, int ev) {
  if (p.trace && item_no == 0 && blockIdx.x < 64 && j < 24) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    p.trace[(blockIdx.x * 32 + j) * 16 + ev] = c;
  }
}
#define TRACE(ic, j, ev) trace_ev(p, (ic), (j), (ev))
#else
#define TRACE(ic, j, ev)
#endif

template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    sdpa_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k64,
                         const __grid_constant__ CUtensorMap tmap_v,
                         const __grid_constant__ CUtensorMap tmap_o, const FwdParams p) {
  using L = Layout<D>;
  constexpr int NB = L::kSBufs;
  constexpr int kPolyEvery = 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = smem + L::kQOff;
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bars->abort_flag;
  const uint64_t kTimeoutNs = p.timeout_ns ? p.timeout_ns : kDefaultTimeoutNs;
  const int n_items = p.n_split * p.BH * p.n_qblk;
  const uint32_t rank = cluster_cta_rank();
  const bool leader = rank == 0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < NB; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 16);  // one arrival per softmax warp of both CTAs
    }
    for (int i = 0; i < 4; ++i) mbar_init(&bars->pv_done[i], 1);
    mbar_init(&bars->o_final, 1);
    mbar_init(&bars->o_empty, 16);
    mbar_init(&bars->ep, 2 * kRowsPerTile);
    mbar_init(&bars->staged, 2 * kRowsPerTile);
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
    prefetch_tmap(&tmap_k64);
    prefetch_tmap(&tmap_v);
    if (!OUT_F32) prefetch_tmap(&tmap_o);
  }
  if (warp == kPvWarp) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised before any remote arrival or copy reaches them.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Arrival on a barrier of the leader (local there, remote from the peer).
  auto arrive_leader = [&](uint64_t* bar) {
    if (leader) mbar_arrive(bar);
    else mbar_arrive_cluster(mapa_shared(bar, 0));
  };
  // One arrival per warp on a barrier of the leader, after every lane's preceding tensor-
  // memory operations (each lane waited for and fenced its own before calling this).
  // (p_full, o_empty: tensor-memory hand-offs, so the cheap remote arrive form suffices.)
  auto warp_arrive_leader = [&](uint64_t* bar) {
    __syncwarp();
    if (lane == 0) {
      if (leader) mbar_arrive(bar);
      else mbar_arrive_cluster_tc(mapa_shared(bar, 0));
    }
  };
  // Item ic of this CTA, as published by the leader's scheduler.
  auto next_item = [&](int ic, bool warp_release, Item& w) -> bool {
    const int slot = ic & 1;
    bool got = mbar_wait_cluster_bounded(&bars->item_full[slot], (ic >> 1) & 1, abort_flag,
                                         kTimeoutNs);
    if (warp_release) got = __all_sync(0xffffffffu, got);
    if (got) {
      const volatile int* v = bars->item[slot];
      w = Item{v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]};
    }
    if (warp_release) {
      __syncwarp();
      if (lane == 0) arrive_leader(&bars->item_empty[slot]);
    } else {
      arrive_leader(&bars->item_empty[slot]);
    }
    return got && w.split >= 0;
  };

  if (warp >= 8) {
  regs_dec<kSideRegs>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ scheduler + TMA producer
    // Both CTAs load their own Q rows, their key half of each K tile and their column half
    // of each V tile; the copies count on the leader's full barriers, for which the leader
    // alone expects the bytes of both CTAs.
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
        if (!mbar_wait_bounded(empty, ph ^ 1, abort_flag, kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          ok = false;
          return;
        }
        const int half_bytes = is_v ? L::kVHalfBytes : L::kKHalfBytes;
        if (leader) mbar_arrive_expect_tx(full, 2 * half_bytes);
        const uint32_t full_leader = mapa_shared(full, 0);
        if (is_v) {
          uint8_t* dst = smem + L::kVOff + st * L::kVHalfBytes;
          tma_load_4d_pair(dst, &tmap_v, full_leader, static_cast<int>(rank) * 64, key0, h, b);
        } else {
          uint8_t* dst = smem + L::kKOff + st * L::kKHalfBytes;
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d_pair(dst + c * ((kKeysPerTile / 2) * 128), &tmap_k64, full_leader, c * 64,
                             key0 + static_cast<int>(rank) * (kKeysPerTile / 2), h, b);
        }
        ++it;
      };
      for (; ok; ++ic) {
        const int slot = ic & 1;
        Item w;
        if (leader) {
          // Publish the next item (or kNoItem) to both CTAs once every consumer released
          // the slot; the peer's copy carries its own first query row.
          if (!mbar_wait_cluster_bounded(&bars->item_empty[slot], ((ic >> 1) & 1) ^ 1,
                                         abort_flag, kTimeoutNs)) {
            if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
            break;
          }
          const int item = static_cast<int>(atomicAdd(&p.sched[0], 1u));
          if (item < n_items) w = common::decode_item<CAUSAL, kRowsPerItem, kKeysPerTile>(p, item);
          else w.split = kNoItem;
          int* pub = bars->item[slot];
          const int vals[8] = {w.split, w.bh, w.b, w.h, w.q_row0, w.kv_lo, w.kv_hi, w.n_kv};
          for (int i = 0; i < 8; ++i) {
            pub[i] = vals[i];
            st_cluster_u32(mapa_shared(&pub[i], 1),
                           static_cast<uint32_t>(i == 4 ? vals[i] + kRowsPerTile : vals[i]));
          }
          mbar_arrive(&bars->item_full[slot]);
          mbar_arrive_cluster(mapa_shared(&bars->item_full[slot], 1));
          if (w.split < 0) break;
        } else {
          if (!next_item(ic, false, w)) break;
        }
        // Q: the previous item's QK^T MMAs must be done with this CTA's buffer.
        if (!mbar_wait_bounded(&bars->q_empty, (ic & 1) ^ 1, abort_flag, kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          break;
        }
        if (leader) mbar_arrive_expect_tx(&bars->q_full, 2 * L::kQBytes);
        const uint32_t q_full_leader = mapa_shared(&bars->q_full, 0);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d_pair(q_smem + c * (kRowsPerTile * 128), &tmap_q, q_full_leader, c * 64,
                           w.q_row0, w.h, w.b);
        for (int jj = 0; ok && jj < min(NB, w.n_kv); ++jj)
          load(false, w.kv_lo + jj * kKeysPerTile, w.h, w.b);
        for (int j = 0; ok && j < w.n_kv; ++j) {
          load(true, w.kv_lo + j * kKeysPerTile, w.h, w.b);
          if (ok && j + NB < w.n_kv) load(false, w.kv_lo + (j + NB) * kKeysPerTile, w.h, w.b);
        }
      }
      // Drain (leader): the full barriers count both CTAs' bytes, so waiting for the last
      // phases covers the peer's copies too (the peer stays alive until the cluster
      // barrier at exit).
      if (leader) {
        volatile int no_abort = 0;
        bool drained = true;
        if (ic > 0)
          drained &= mbar_wait_bounded(&bars->q_full, (ic - 1) & 1, &no_abort, kTimeoutNs);
        for (int i = max(0, k_it - L::kKStages); i < k_it; ++i)
          drained &= mbar_wait_bounded(&bars->k_full[i % L::kKStages], (i / L::kKStages) & 1,
                                       &no_abort, kTimeoutNs);
        for (int i = max(0, v_it - L::kVStages); i < v_it; ++i)
          drained &= mbar_wait_bounded(&bars->v_full[i % L::kVStages], (i / L::kVStages) & 1,
                                       &no_abort, kTimeoutNs);
        if (!drained && p.status) atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp == kPvWarp && leader) {
    // ------------------------------------------------------------ P.V issuer (leader)
    if (lane == 0) {
      constexpr uint32_t kIdescPV = idesc_f16(2 * kRowsPerTile, D, BF16, false, true);
      const uint64_t v_desc = sdesc_sw128(smem_u32(smem + L::kVOff), kKeysPerTile * 128, 1024);
      bool ok = true;
      if (p.selftest_stall) ok = mbar_wait_bounded(&bars->never, 0, abort_flag, kTimeoutNs);
      int g = 0, v_it = 0;
      for (int ic = 0; ok; ++ic) {
        Item w;
        if (!next_item(ic, false, w)) break;
        if (ic > 0) {
          ok = mbar_wait_cluster_bounded(&bars->o_empty, (ic - 1) & 1, abort_flag, kTimeoutNs);
          if (!ok) break;
        }
        for (int j = 0; ok && j < w.n_kv; ++j, ++g) {
          const int buf = g % NB;
          const int st = v_it % L::kVStages;
          ok = mbar_wait_bounded(&bars->v_full[st], (v_it / L::kVStages) & 1, abort_flag,
                                 kTimeoutNs);
          if (!ok) break;
          TRACE(ic, j, 11);
          ok = mbar_wait_cluster_bounded(&bars->p_full[buf], (g / NB) & 1, abort_flag,
                                         kTimeoutNs);
          if (!ok) break;
          TRACE(ic, j, 8);
          tc_fence_after();
          const uint64_t vd = v_desc + static_cast<uint64_t>((st * L::kVHalfBytes) >> 4);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t a_tmem = tmem + buf * 128 + hh * kKeysPerHalf;
            const uint32_t d_tmem = tmem + L::kOCol + hh * D;
#pragma unroll
            for (int k4 = 0; k4 < kKeysPerHalf / 16; ++k4) {
              const int kk = hh * (kKeysPerHalf / 16) + k4;
              mma_ts_pair(d_tmem, a_tmem + k4 * 8,
                          vd + static_cast<uint64_t>((kk * 16 * 128) >> 4), kIdescPV,
                          (j > 0 || k4 > 0) ? 1u : 0u);
            }
          }
          mma_commit_pair(&bars->pv_done[g & 3], kBothCtas);
          mma_commit_pair(&bars->v_empty[st], kBothCtas);
          ++v_it;
          TRACE(ic, j, 9);
        }
        if (!ok) break;
        mma_commit_pair(&bars->o_final, kBothCtas);
      }
      if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
      mma_commit_pair(&bars->drain, 0x1);
    }
    __syncwarp();
  } else if (warp == kQkWarp && leader) {
    // ------------------------------------------------------------ QK^T issuer (leader)
    if (lane == 0) {
      constexpr uint32_t kIdescQK =
          idesc_f16(2 * kRowsPerTile, kKeysPerTile, BF16, false, false);
      const uint64_t q_desc = sdesc_sw128(smem_u32(q_smem), 16, 1024);
      const uint64_t k_desc = sdesc_sw128(smem_u32(smem + L::kKOff), 16, 1024);
      bool ok = true;
      int g = 0, k_it = 0;
      for (int ic = 0; ok; ++ic) {
        Item w;
        if (!next_item(ic, false, w)) break;
        ok = mbar_wait_bounded(&bars->q_full, ic & 1, abort_flag, kTimeoutNs);
        for (int t = 0; ok && t < w.n_kv; ++t, ++g) {
          const int buf = g % NB;
          if (g >= NB) {
            ok = mbar_wait_bounded(&bars->pv_done[(g - NB) & 3], ((g - NB) >> 2) & 1,
                                   abort_flag, kTimeoutNs);
            if (!ok) break;
          }
          const int st = k_it % L::kKStages;
          ok = mbar_wait_bounded(&bars->k_full[st], (k_it / L::kKStages) & 1, abort_flag,
                                 kTimeoutNs);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kd = k_desc + static_cast<uint64_t>((st * L::kKHalfBytes) >> 4);
          const uint32_t d_tmem = tmem + buf * 128;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            constexpr int kAtomQ = kRowsPerTile * 128;        // 64-column chunk of Q
            constexpr int kAtomK = (kKeysPerTile / 2) * 128;  // 64-column chunk of a K half
            const uint64_t qo = static_cast<uint64_t>(((kk >> 2) * kAtomQ + (kk & 3) * 32) >> 4);
            const uint64_t ko = static_cast<uint64_t>(((kk >> 2) * kAtomK + (kk & 3) * 32) >> 4);
            mma_ss_pair(d_tmem, q_desc + qo, kd + ko, kIdescQK, kk > 0 ? 1u : 0u);
          }
          mma_commit_pair(&bars->s_full[buf], kBothCtas);
          mma_commit_pair(&bars->k_empty[st], kBothCtas);
          ++k_it;
          TRACE(ic, t, 10);
        }
        if (!ok) break;
        mma_commit_pair(&bars->q_empty, kBothCtas);
      }
      if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
      mma_commit_pair(&bars->drain, 0x1);
    }
    __syncwarp();
  }
  if (warp == kPvWarp && leader && lane == 0) {
    volatile int no_abort = 0;
    if (!mbar_wait_bounded(&bars->drain, 0, &no_abort, kTimeoutNs) && p.status)
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
      Item w;
      const bool have = next_item(ic, true, w);
      if (!have) break;
      const int row = w.q_row0 + r_in_tile;
      float m_run = -INFINITY;  // running max of this half, in log2 units (score*scale*log2 e)
      float l_run = 0.f;        // running row sum of this half
      for (int j = 0; j < w.n_kv; ++j, ++g) {
        const int buf = g % NB;
        const uint32_t t_s = tmem + lane_bits + buf * 128;
        ok = mbar_wait_bounded(&bars->s_full[buf], (g / NB) & 1, abort_flag, kTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (threadIdx.x % 128 == 0) TRACE(ic, j, 0 + 4 * half);
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
          bool done = mbar_wait_bounded(&bars->pv_done[(g - 1) & 3], ((g - 1) >> 2) & 1,
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
        if (threadIdx.x % 128 == 96) TRACE(ic, j, 3 + 4 * half);
        warp_arrive_leader(&bars->p_full[buf]);
      }
      if (!ok) break;
      // ---- epilogue of the item: merge the two halves. Exchange (m, l) with the partner
      // thread (same row, other warpgroup) through the slot of this item's parity, then
      // each warpgroup writes D/2 output columns from both accumulators.
      float* red_i = red + (ic & 1) * (4 * kRowsPerTile);
      red_i[half * kRowsPerTile + r_in_tile] = m_run;
      red_i[2 * kRowsPerTile + half * kRowsPerTile + r_in_tile] = l_run;
      // The thread that issues the output TMA store makes sure the previous item's store has
      // finished reading the staging buffer before anyone passes this exchange.
      if (!OUT_F32 && threadIdx.x == 0) bulk_wait_group_read0();
      mbar_arrive(&bars->ep);
      ok = mbar_wait_bounded(&bars->ep, ic & 1, abort_flag, kTimeoutNs);
      if (ok) ok = mbar_wait_bounded(&bars->o_final, ic & 1, abort_flag, kTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_EPILOG, abort_flag);
        break;
      }
      tc_fence_after();
      const float m_a = red_i[r_in_tile], m_b = red_i[kRowsPerTile + r_in_tile];
      const float l_a = red_i[2 * kRowsPerTile + r_in_tile];
      const float l_b = red_i[3 * kRowsPerTile + r_in_tile];
      const float m = fmaxf(m_a, m_b);
      // A half that saw no valid key has m = -inf: weight 0.
      const float w_a = m_a == -INFINITY ? 0.f : ex2_approx(m_a - m);
      const float w_b = m_b == -INFINITY ? 0.f : ex2_approx(m_b - m);
      const float l_tot = l_a * w_a + l_b * w_b;
      // Rows without any valid key (only with a key slice) get o = 0 and lse = -inf.
      const float inv_l = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float f_a = w_a * inv_l, f_b = w_b * inv_l;
      const bool in_range = row < p.S;
      const int col0 = half * (D / 2);  // output columns of this warpgroup
      const uint32_t t_oa = tmem + lane_bits + L::kOCol + col0;
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        uint32_t oa[32], ob[32];
        if (w.n_kv > 0) {
          tmem_ld32(t_oa + c * 32, oa);
          tmem_ld32(t_oa + D + c * 32, ob);
          tmem_wait_ld();
          reg_fence32(oa);
          reg_fence32(ob);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) oa[i] = ob[i] = 0u;
        }
        float* v = reinterpret_cast<float*>(oa);  // merged values, in place
#pragma unroll
        for (int i = 0; i < 32; ++i)
          v[i] = __uint_as_float(oa[i]) * f_a + __uint_as_float(ob[i]) * f_b;
        if constexpr (OUT_F32) {
          if (in_range) {
            float4* dst = reinterpret_cast<float4*>(
                reinterpret_cast<uint8_t*>(p.o) +
                4 * (static_cast<int64_t>(w.split) * p.o_split_stride +
                     static_cast<int64_t>(w.b) * p.o_sb + static_cast<int64_t>(w.h) * p.o_sh +
                     static_cast<int64_t>(row) * p.o_ss + col0 + c * 32));
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (col0 + c * 32 + 4 * i < p.d_out)  // columns beyond the true head dim
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        } else {
          // 32 output columns = four 16-byte units of the 128-byte-swizzled staging row
          // (the layout the tensor map's SWIZZLE_128B expects: unit u of row r at
          // r*128 + ((u ^ (r % 8)) * 16) within its 64-column chunk).
          const int col = col0 + c * 32;
          uint8_t* chunk = smem + L::kStageOff + (col / 64) * (kRowsPerTile * 128);
          const int u0 = (col % 64) / 8;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
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
      warp_arrive_leader(&bars->o_empty);
      if (!OUT_F32) {
        // Hand the staged tile to the TMA store (issued by thread 0 once all 256 threads
        // wrote their part; rows beyond S are clipped by the tensor map).
        fence_proxy_async_shared();
        mbar_arrive(&bars->staged);
        if (threadIdx.x == 0) {
          if (mbar_wait_bounded(&bars->staged, ic & 1, abort_flag, kTimeoutNs)) {
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
      if (half == 0 && p.lse != nullptr && in_range)
        p.lse[static_cast<int64_t>(w.split) * p.BH * p.S + static_cast<int64_t>(w.bh) * p.S + row] =
            l_tot > 0.f ? (m + __log2f(l_tot)) * 0.69314718055994531f : -INFINITY;
      ok = __all_sync(0xffffffffu, ok);
    }
    // Stores must have completed before the CTA exits.
    if (!OUT_F32 && threadIdx.x == 0) bulk_wait_group0();
    if (!ok && lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_SOFTMAX, abort_flag);
  }


  tc_fence_before();
  __syncthreads();
  // No CTA of the pair leaves (or frees tensor memory) while the other may still arrive on
  // its barriers or the leader's MMAs may still write its tensor memory.
  cluster_sync();
  tc_fence_after();
  if (warp == kPvWarp) tmem_dealloc_pair(tmem, kTmemCols);
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&p.sched[1], 1u) == gridDim.x - 1) {
      atomicExch(&p.sched[0], 0u);
      atomicExch(&p.sched[1], 0u);
    }
  }
}

namespace {

constexpr int kSchedSlots = 1024;
__device__ unsigned int g_sched[kSchedSlots][2];
constexpr int kMaxDevices = 64;
std::atomic<unsigned int> g_sched_next[kMaxDevices];
std::atomic<unsigned int*> g_sched_base[kMaxDevices];
std::atomic<int> g_max_pairs[kMaxDevices];

template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
cudaError_t launch_variant(const CUtensorMap& q, const CUtensorMap& k64, const CUtensorMap& v,
                           const CUtensorMap& o, const FwdParams& p, long long items,
                           int dev, cudaStream_t stream) {
  auto kern = sdpa_fwd_pair_kernel<D, BF16, CAUSAL, OUT_F32>;
  constexpr int smem = Layout<D>::kDynSmem;
  static int configured_mask = 0;
  cudaError_t err;
  if (dev >= 32 || !(__atomic_load_n(&configured_mask, __ATOMIC_ACQUIRE) & (1 << dev))) {
    cudaFuncAttributes attr;
    err = cudaFuncGetAttributes(&attr, kern);
    if (err != cudaSuccess) return err;
    if (attr.numRegs != kLaunchRegs) return cudaErrorInvalidKernelImage;
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    if (dev < 32) __atomic_fetch_or(&configured_mask, 1 << dev, __ATOMIC_ACQ_REL);
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_pairs = g_max_pairs[dev].load(std::memory_order_acquire);
  if (max_pairs == 0) {
    cfg.gridDim = dim3(2 * 74, 1, 1);
    int clusters = 0;
    err = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (err != cudaSuccess) return err;
    max_pairs = clusters > 0 ? clusters : 1;
    g_max_pairs[dev].store(max_pairs, std::memory_order_release);
  }
  const long long pairs = items < max_pairs ? items : max_pairs;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, q, k64, v, o, p);
}

}  // namespace
}  // namespace pair

cudaError_t launch_sdpa_fwd_pair(const CUtensorMap& q, const CUtensorMap& k64,
                                 const CUtensorMap& v, const CUtensorMap& o,
                                 const FwdParams& p_in, int D, bool bf16, bool causal,
                                 bool out_f32, cudaStream_t stream) {
  if (D != 128) return cudaErrorInvalidValue;
  const long long items = static_cast<long long>(p_in.n_split) * p_in.BH * p_in.n_qblk;
  if (items == 0) return cudaSuccess;
  if (items > 0x7fffffffll) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= pair::kMaxDevices) return cudaErrorInvalidDevice;
  unsigned int* base = pair::g_sched_base[dev].load(std::memory_order_acquire);
  if (base == nullptr) {
    void* b = nullptr;
    err = cudaGetSymbolAddress(&b, pair::g_sched);
    if (err != cudaSuccess) return err;
    base = static_cast<unsigned int*>(b);
    pair::g_sched_base[dev].store(base, std::memory_order_release);
  }
  FwdParams p = p_in;
  const unsigned int slot =
      pair::g_sched_next[dev].fetch_add(1, std::memory_order_relaxed) % pair::kSchedSlots;
  p.sched = base + 2 * slot;
  const long long kv_bytes = 4ll * p.S * D;
  const long long group = (48ll << 20) / (kv_bytes > 0 ? kv_bytes : 1);
  p.group_bh = static_cast<int>(group < 1 ? 1 : (group > p.BH ? p.BH : group));
#define TA_DISPATCH(BB, CC, FF)                                                    \
  if (bf16 == BB && causal == CC && out_f32 == FF)                                 \
    return pair::launch_variant<128, BB, CC, FF>(q, k64, v, o, p, items, dev, stream);
  TA_DISPATCH(false, false, false) TA_DISPATCH(false, false, true)
  TA_DISPATCH(false, true, false) TA_DISPATCH(false, true, true)
  TA_DISPATCH(true, false, false) TA_DISPATCH(true, false, true)
  TA_DISPATCH(true, true, false) TA_DISPATCH(true, true, true)
#undef TA_DISPATCH
  return cudaErrorInvalidValue;
}

}  // namespace ta
