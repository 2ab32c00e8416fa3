// SDPA forward for B200 (sm_100a) where query tiles share every K/V tile: head dim 256
// (also the padded target of head dims 129-255) and long head-dim-128 sequences. TMA +
// mbarrier pipeline, tcgen05 MMAs with accumulators in tensor memory, warp-specialised
// online softmax. At D=128 one CTA covers two 128-row query tiles (256 rows), so each K/V
// tile is loaded and written to shared memory once per 256 rows - half the per-SM copy
// traffic of the persistent one-tile kernel, which matters once sequences are long and the
// per-CTA start-up cost is amortised. At D=256 the accumulator alone takes 256 of the 512
// tensor-memory columns, so the CTA keeps one query tile.
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
// accumulated in fp32 tensor memory (the cuTile kernel rounds each tile product to
// the input dtype), and the exponent is evaluated as exp2 with log2(e) folded into
// the scale. The running max is rescaled lazily: the accumulator is only rescaled
// when the max grows by more than 2^8, which is exact after the final division by l.
//
// CTA organisation (one CTA per SM: 192 KB shared memory, all 512 TMEM columns):
//   one CTA = one (batch, head) pair x 256 query rows = two 128-row query tiles
//   warps 0-3  softmax + epilogue for query tile 0 (thread i owns TMEM lane / row i)
//   warps 4-7  softmax + epilogue for query tile 1
//   warp  8    TMA producer: Q tiles once, then K_0, V_0, K_1, V_1 ... through a ring
//   warp  9    TMEM allocator and single-thread tcgen05.mma issuer
//   warps 10-11 idle (complete the third warpgroup for the register split)
// Tensor memory: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D) columns;
// P_t (16-bit, two per column) overwrites the first 64 columns of S_t and feeds the
// P.V MMA straight from tensor memory.
// MMA issue order per key tile j (in-order tensor pipe):
//   PV0(j-1)... S0(j) S1(j) | PV0(j) S0(j+1) | PV1(j) S1(j+1) ...
// so that when S_t(j+1) is signalled complete, PV_t(j) has completed too and
// the softmax warps may rescale O_t without another barrier.
//
// Every wait is bounded (shared abort flag + global-timer timeout); on expiry the
// kernel records TA_DEVSTAT_* bits in the status word, drains its own in-flight TMA
// copies and MMAs, frees tensor memory and returns.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sdpa_common.cuh"
#include "sm100_ptx.cuh"
#include "sdpa_fwd_sm100.h"
#include "tiledattention_b200.h"

namespace ta {
namespace shared_kv {

using common::add_packed16_to_f32;
using common::pack2;
using common::report;

constexpr int kRowsPerTile = 128;  // query rows per tile (= TMEM lanes)
// Query tiles per CTA: two 128-row tiles up to D=128; one at D=256, where S (128) + O (256)
// tensor-memory columns per tile leave no room for a second tile.
template <int D>
constexpr int tiles_per_cta() { return D == 256 ? 1 : 2; }
constexpr int kKeysPerTile = 128;  // keys per K/V tile
constexpr int kThreads = 384;
// Register split: the kernel is built for kLaunchRegs per thread (launch bounds 384 x 1);
// after start-up the producer/MMA warpgroup gives registers back (setmaxnreg.dec to
// kSideRegs) and the two softmax warpgroups take them (setmaxnreg.inc to kSoftmaxRegs).
// 2*128*kSoftmaxRegs + 128*kSideRegs == 384*kLaunchRegs, so the increase always fits
// in the block's launch allocation; the host refuses to launch a build whose register
// count differs from kLaunchRegs.
constexpr int kLaunchRegs = 168;
#ifndef TA_SOFTMAX_REGS
#define TA_SOFTMAX_REGS 208
#define TA_SIDE_REGS 88
#endif
constexpr int kSoftmaxRegs = TA_SOFTMAX_REGS;
constexpr int kSideRegs = TA_SIDE_REGS;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kSideRegs == kThreads * kLaunchRegs,
              "register split must match the launch allocation");
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr int kSumChains = 4;  // independent row-sum accumulators (short dependency chains)
#ifndef TA_POLY_EVERY
#define TA_POLY_EVERY 0
#endif
constexpr int kPolyEvery = TA_POLY_EVERY;  // every kPolyEvery-th element pair: exp2 on the FMA pipe
constexpr uint64_t kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait

template <int D>
struct Layout {
  static constexpr int kTileBytes = kRowsPerTile * D * 2;  // 128 rows x D x 16-bit
  static constexpr int kChunks = D / 64;                   // 128-byte swizzle atoms per row
  static constexpr int kTiles = tiles_per_cta<D>();
  static constexpr int kRowsPerCta = kRowsPerTile * kTiles;
  static constexpr int kStages = (D == 64) ? 6 : (D == 128 ? 4 : 2);
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = kQOff + kTiles * kTileBytes;
  static constexpr int kBarOff = kKVOff + kStages * kTileBytes;
  static constexpr int kBytes = kBarOff + 256;
  static constexpr int kDynSmem = kBytes + 1024;  // slack for 1024-byte alignment
};

struct Barriers {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_final[2];
  uint64_t drain;
  uint64_t never;     // self-test only: a barrier nothing arrives on
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 256, "barrier block");

#ifdef TA_TRACE
// Experiment builds only: clock64 of event `ev` (< 16) of key tile j (< 32) in the
// first 64 blocks, for timeline analysis.
__device__ __forceinline__ void trace_ev(const FwdParams& p, int j, int ev) {
  if (p.trace && blockIdx.x < 64 && j < 32) {
    unsigned long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    p.trace[(blockIdx.x * 32 + j) * 16 + ev] = c;
  }
}
#define TRACE(j, ev) trace_ev(p, (j), (ev))
#else
#define TRACE(j, ev)
#endif

// OUT_F32: write o as fp32 (the normalised partial output of one key slice) instead of
// the input dtype. Grid = n_split x B*H x n_qblk; slice s covers keys
// [kv_begin + s*split_len, min(kv_end, kv_begin + (s+1)*split_len)).
template <int D, bool BF16, bool CAUSAL, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    sdpa_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const FwdParams p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = smem + L::kQOff;
  uint8_t* kv_smem = smem + L::kKVOff;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bars->abort_flag;
  const uint64_t kTimeoutNs = p.timeout_ns ? p.timeout_ns : kDefaultTimeoutNs;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Block -> (bh, query block). Consecutive blocks share a (b,h) so its K/V stays in L2;
  // inside a (b,h) the longest causal rows are issued first.
  const int per_split = p.BH * p.n_qblk;
  const int split = blockIdx.x / per_split;
  const int blk = blockIdx.x - split * per_split;
  const int bh = blk / p.n_qblk;
  const int qblk = p.n_qblk - 1 - (blk % p.n_qblk);
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int S = p.S;
  // keys [kv_lo, kv_hi) take part (the whole range, or one slice for split-KV)
  const int kv_lo = min(p.kv_end, p.kv_begin + split * p.split_len);
  const int kv_hi = min(p.kv_end, kv_lo + p.split_len);
  const int q_row0 = qblk * L::kRowsPerCta;
  const int kv_rows = CAUSAL ? min(kv_hi, q_row0 + L::kRowsPerCta) : kv_hi;
  const int n_kv = kv_rows > kv_lo ? (kv_rows - kv_lo + kKeysPerTile - 1) / kKeysPerTile : 0;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], kRowsPerTile);
      mbar_init(&bars->o_final[t], 1);
    }
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->never, 1);
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Each role branch starts with its warpgroup's setmaxnreg so that the register limit
  // ptxas applies to the code after it is the one of that branch.
  if (warp >= 8) {
  regs_dec<kSideRegs>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->q_full, L::kTiles * L::kTileBytes);
      for (int t = 0; t < L::kTiles; ++t)
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(q_smem + t * L::kTileBytes + c * (kRowsPerTile * 128), &tmap_q,
                      &bars->q_full, c * 64, q_row0 + t * kRowsPerTile, h, b);
      int issued = 0;
      for (int it = 0; it < 2 * n_kv; ++it) {
        const int st = it % L::kStages;
        const uint32_t ph = (it / L::kStages) & 1;
        if (!mbar_wait_bounded(&bars->kv_empty[st], ph ^ 1, abort_flag, kTimeoutNs)) {
          if (!*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_LOAD, abort_flag);
          break;
        }
        mbar_arrive_expect_tx(&bars->kv_full[st], L::kTileBytes);
        const CUtensorMap* map = (it & 1) ? &tmap_v : &tmap_k;
        const int key0 = kv_lo + (it >> 1) * kKeysPerTile;
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(kv_smem + st * L::kTileBytes + c * (kKeysPerTile * 128), map,
                      &bars->kv_full[st], c * 64, key0, h, b);
        issued = it + 1;
      }
      // Drain: every copy this thread issued must land before the CTA may exit.
      volatile int no_abort = 0;
      bool ok = mbar_wait_bounded(&bars->q_full, 0, &no_abort, kTimeoutNs);
      for (int it = max(0, issued - L::kStages); it < issued; ++it)
        ok &= mbar_wait_bounded(&bars->kv_full[it % L::kStages], (it / L::kStages) & 1,
                                &no_abort, kTimeoutNs);
      if (!ok && p.status) atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_f16(kRowsPerTile, kKeysPerTile, BF16, false, false);
      constexpr uint32_t kIdescPV = idesc_f16(kRowsPerTile, D, BF16, false, true);
      // Descriptors are built once; per K step only the start-address field (low bits)
      // advances, by a compile-time constant, so issuing an MMA costs a 64-bit add.
      const uint64_t q_desc = sdesc_sw128(smem_u32(q_smem), 16, 1024);
      const uint64_t kv_desc_k = sdesc_sw128(smem_u32(kv_smem), 16, 1024);
      const uint64_t kv_desc_v = sdesc_sw128(smem_u32(kv_smem), kKeysPerTile * 128, 1024);
      auto issue_qk = [&](int t, int st) {
        const uint64_t qd = q_desc + static_cast<uint64_t>((t * L::kTileBytes) >> 4);
        const uint64_t kd = kv_desc_k + static_cast<uint64_t>((st * L::kTileBytes) >> 4);
        const uint32_t d_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr int kAtom = kRowsPerTile * 128;
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kAtom + (kk & 3) * 32) >> 4);
          mma_ss(d_tmem, qd + off, kd + off, kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int st, bool acc) {
        const uint64_t vd = kv_desc_v + static_cast<uint64_t>((st * L::kTileBytes) >> 4);
        const uint32_t d_tmem = tmem + 256 + t * D;
        const uint32_t a_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < kKeysPerTile / 16; ++kk)
          mma_ts(d_tmem, a_tmem + kk * 8, vd + static_cast<uint64_t>((kk * 16 * 128) >> 4),
                 kIdescPV, (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = true;
      int it = 0;
      // Self-test of the failure path: wait on a barrier nothing arrives on, so the wait
      // runs out, the kernel records the timeout and every role returns.
      if (p.selftest_stall) ok = mbar_wait_bounded(&bars->never, 0, abort_flag, kTimeoutNs);
      if (ok && n_kv > 0) ok = mbar_wait_bounded(&bars->q_full, 0, abort_flag, kTimeoutNs);
      if (ok && n_kv > 0) {
        const int st = 0;
        ok = mbar_wait_bounded(&bars->kv_full[st], 0, abort_flag, kTimeoutNs);
        if (ok) {
          tc_fence_after();
          issue_qk(0, st);
          mma_commit(&bars->s_full[0]);
          if constexpr (L::kTiles == 2) {
            issue_qk(1, st);
            mma_commit(&bars->s_full[1]);
          }
          mma_commit(&bars->kv_empty[st]);
          it = 1;
        }
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st_v = it % L::kStages;
        ok = mbar_wait_bounded(&bars->kv_full[st_v], (it / L::kStages) & 1, abort_flag, kTimeoutNs);
        if (!ok) break;
        ++it;
        const bool more = (j + 1 < n_kv);
        const int st_k = it % L::kStages;
        // query tile 0
        ok = mbar_wait_bounded(&bars->p_full[0], j & 1, abort_flag, kTimeoutNs);
        if (!ok) break;
        TRACE(j, 8);
        tc_fence_after();
        issue_pv(0, st_v, j > 0);
        if (more) {
          ok = mbar_wait_bounded(&bars->kv_full[st_k], (it / L::kStages) & 1, abort_flag,
                                 kTimeoutNs);
          if (!ok) break;
          tc_fence_after();
          issue_qk(0, st_k);
          mma_commit(&bars->s_full[0]);
        } else {
          mma_commit(&bars->o_final[0]);
        }
        if constexpr (L::kTiles == 2) {
          // query tile 1
          TRACE(j, 9);
          ok = mbar_wait_bounded(&bars->p_full[1], j & 1, abort_flag, kTimeoutNs);
          if (!ok) break;
          TRACE(j, 10);
          tc_fence_after();
          issue_pv(1, st_v, j > 0);
          mma_commit(&bars->kv_empty[st_v]);
          if (more) {
            issue_qk(1, st_k);
            mma_commit(&bars->s_full[1]);
            mma_commit(&bars->kv_empty[st_k]);
            ++it;
          } else {
            mma_commit(&bars->o_final[1]);
          }
        } else {
          mma_commit(&bars->kv_empty[st_v]);
          if (more) {
            mma_commit(&bars->kv_empty[st_k]);
            ++it;
          }
        }
        TRACE(j, 11);
      }
      if (!ok && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_MMA, abort_flag);
      // Drain: all MMAs this thread issued complete before tensor memory is freed.
      mma_commit(&bars->drain);
      volatile int no_abort = 0;
      if (!mbar_wait_bounded(&bars->drain, 0, &no_abort, kTimeoutNs) && p.status)
        atomicOr(p.status, TA_DEVSTAT_TIMEOUT_DRAIN);
    }
    __syncwarp();
  }
  } else {
    regs_inc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;            // query tile of this warpgroup
    if (t < L::kTiles) {
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int r_in_tile = quarter * 32 + lane;
    const int tile_row0 = q_row0 + t * kRowsPerTile;
    const int row = tile_row0 + r_in_tile;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_bits + t * 128;
    const uint32_t t_o = tmem + lane_bits + 256 + t * D;
    const float sl = p.scale_log2;

    float m_run = -INFINITY;  // running max, in log2 units (score * scale * log2 e)
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait_bounded(&bars->s_full[t], j & 1, abort_flag, kTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      if (threadIdx.x % 128 == 0) TRACE(j, 0 + 4 * t);
      float s[kKeysPerTile];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(t_s + 0, r0);
        tmem_ld32(t_s + 32, r1);
        tmem_ld32(t_s + 64, r2);
        tmem_ld32(t_s + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
          s[64 + i] = __uint_as_float(r2[i]);
          s[96 + i] = __uint_as_float(r3[i]);
        }
      }
      if (threadIdx.x % 128 == 0) TRACE(j, 1 + 4 * t);
      const int c0 = kv_lo + j * kKeysPerTile;  // absolute index of the tile's first key
      const bool need_mask =
          (c0 + kKeysPerTile > kv_hi) || (CAUSAL && c0 + kKeysPerTile - 1 > tile_row0);
      if (need_mask) {
        int lim = kv_hi - c0;
        if (CAUSAL) lim = min(lim, row - c0 + 1);
#pragma unroll
        for (int i = 0; i < kKeysPerTile; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      // Row max: four independent chains of 3-input max.
      float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
      float mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
#pragma unroll
      for (int i = 8; i < kKeysPerTile; i += 8) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[i + 2], s[i + 3]);
        mx2 = fmax3(mx2, s[i + 4], s[i + 5]);
        mx3 = fmax3(mx3, s[i + 6], s[i + 7]);
      }
      const float m_cand = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl;
      if (j == 0) {
        m_run = m_cand;
      } else {
        const bool grow = m_cand > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, grow)) {
          float alpha = 1.f;
          if (grow) {
            alpha = ex2_approx(m_run - m_cand);  // 0 while m_run is -inf
            l_run *= alpha;
            m_run = m_cand;
          }
          const uint64_t alpha2 = f2_pack(alpha, alpha);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float a0, a1;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), alpha2),
                        a0, a1);
              o[i] = __float_as_uint(a0);
              o[i + 1] = __float_as_uint(a1);
            }
            tmem_st32(t_o + c * 32, o);
          }
        }
      }
      // p = 2^(s*scale*log2e - m): packed FMA, then exp2 on the MUFU (or, with
      // TA_POLY_EVERY > 0, every kPolyEvery-th pair on the FMA pipe).
      if (threadIdx.x % 128 == 0) TRACE(j, 2 + 4 * t);
      // A row with no valid key yet (m = -inf; only possible with a key slice) uses 0 as
      // the subtrahend, so its weights are exactly 0 instead of NaN.
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      const uint64_t sl2 = f2_pack(sl, sl);
      const uint64_t negm2 = f2_pack(-m_use, -m_use);
      float acc_lo[kSumChains], acc_hi[kSumChains];
#pragma unroll
      for (int c = 0; c < kSumChains; ++c) acc_lo[c] = acc_hi[c] = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int e = 64 * half + 2 * i;
          float p0, p1;
          const uint64_t x2 = f2_fma(f2_pack(s[e], s[e + 1]), sl2, negm2);
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
        tmem_st32(t_s + 32 * half, pk);
      }
      {
        float tot = 0.f;
#pragma unroll
        for (int c = 0; c < kSumChains; ++c) tot += acc_lo[c] + acc_hi[c];
        l_run += tot;
      }
      tmem_wait_st();
      tc_fence_before();
      if (threadIdx.x % 128 == 0) TRACE(j, 3 + 4 * t);
      mbar_arrive(&bars->p_full[t]);
    }
    if (!ok) {
      if (lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_SOFTMAX, abort_flag);
    } else {
      if (n_kv > 0) {
        ok = mbar_wait_bounded(&bars->o_final[t], 0, abort_flag, kTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (!ok) {
        if (lane == 0 && !*abort_flag) report(p, TA_DEVSTAT_TIMEOUT_EPILOG, abort_flag);
      } else {
        tc_fence_after();
        // Rows without any valid key (only with a key slice) get o = 0 and lse = -inf.
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
        const bool in_range = row < S;
        constexpr int kOutBytes = OUT_F32 ? 4 : 2;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                        kOutBytes * (static_cast<int64_t>(split) * p.o_split_stride +
                                     static_cast<int64_t>(b) * p.o_sb +
                                     static_cast<int64_t>(h) * p.o_sh +
                                     static_cast<int64_t>(row) * p.o_ss);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          if (n_kv > 0) {
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
                if (c * 32 + 4 * i < p.d_out)  // output columns beyond the true head dim
                  dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l, __uint_as_float(o[4 * i + 1]) * inv_l,
                                       __uint_as_float(o[4 * i + 2]) * inv_l, __uint_as_float(o[4 * i + 3]) * inv_l);
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
                if (c * 32 + 8 * i < p.d_out)  // output columns beyond the true head dim
                  dst[i] = make_uint4(pw[4 * i], pw[4 * i + 1], pw[4 * i + 2], pw[4 * i + 3]);
            }
          }
        }
        if (p.lse != nullptr && in_range)
          p.lse[static_cast<int64_t>(split) * p.BH * S + static_cast<int64_t>(bh) * S + row] =
              l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
      }
    }
    }  // t < kTiles
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
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
  kern<<<grid, kThreads, smem, stream>>>(q, k, v, p);
  return cudaGetLastError();
}

}  // namespace shared_kv

cudaError_t launch_sdpa_fwd_shared_kv(const CUtensorMap& q, const CUtensorMap& k,
                                      const CUtensorMap& v, const FwdParams& p, int D,
                                      bool bf16, bool causal, bool out_f32,
                                      cudaStream_t stream) {
  const long long grid = static_cast<long long>(p.n_split) * p.BH * p.n_qblk;
  if (grid == 0) return cudaSuccess;
  if (grid > 0x7fffffffll) return cudaErrorInvalidValue;
#define TA_DISPATCH(DD, BB, CC, FF)                                               \
  if (D == DD && bf16 == BB && causal == CC && out_f32 == FF)                     \
    return shared_kv::launch_variant<DD, BB, CC, FF>(q, k, v, p, static_cast<int>(grid), stream);
#define TA_DISPATCH4(DD)                                                          \
  TA_DISPATCH(DD, false, false, false) TA_DISPATCH(DD, false, false, true)        \
  TA_DISPATCH(DD, false, true, false) TA_DISPATCH(DD, false, true, true)          \
  TA_DISPATCH(DD, true, false, false) TA_DISPATCH(DD, true, false, true)          \
  TA_DISPATCH(DD, true, true, false) TA_DISPATCH(DD, true, true, true)
  TA_DISPATCH4(128)
  TA_DISPATCH4(256)
#undef TA_DISPATCH4
#undef TA_DISPATCH
  return cudaErrorInvalidValue;
}

int rows_per_cta_shared_kv(int D) {
  return D == 256 ? shared_kv::Layout<256>::kRowsPerCta : shared_kv::Layout<128>::kRowsPerCta;
}

}  // namespace ta
