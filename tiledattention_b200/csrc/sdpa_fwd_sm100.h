// Internal interface between the C ABI (capi.cu) and the sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ta {

struct FwdParams {
  void* o;                 // output base pointer, [B,H,S,D]
  float* lse;              // optional [B*H*S] natural-log log-sum-exp per row
  unsigned int* status;    // optional device status word (TA_DEVSTAT_* bits)
  int64_t o_sb, o_sh, o_ss;  // output element strides (dim stride is 1)
  int S, H, BH, n_qblk;
  int kv_begin, kv_end;    // keys [kv_begin, kv_end) take part (0, S for full attention)
  int n_split, split_len;  // key slices per launch (grid dim) and keys per slice
  int64_t o_split_stride;  // output element stride between slices (partial mode)
  float scale_log2;        // scale * log2(e)
  unsigned long long* trace;  // experiment builds (-DTA_TRACE) only: event clocks
  unsigned long long timeout_ns;  // limit of every in-kernel wait (0: 1 s)
  int selftest_stall;      // 1: the MMA warp waits on a barrier nothing arrives on
  unsigned int* sched;     // {next work item, CTAs finished} of this launch (set by the launcher)
  int group_bh;            // persistent kernel: (b,h) pairs per scheduling group (see decode)
  int d_out;               // head dim of the output (<= the kernel's; multiple of 8); the
                           // kernel writes only these columns
};

// Whether (D, S, causal) runs on the shared-K/V kernel (sdpa_fwd_sm100_shared_kv.cu): head
// dim 256 always; head dim 128 from kSharedKvMinSeq keys on (causal) or
// kSharedKvMinSeqNonCausal (non-causal), where the persistent one-tile kernel's lower
// start-up cost no longer outweighs loading each K/V tile once per 128 query rows instead of
// once per 256 (crossovers measured on B200).
#ifndef TA_SKV_MIN_SEQ
#define TA_SKV_MIN_SEQ 65536
#endif
#ifndef TA_SKV_MIN_SEQ_NONCAUSAL
#define TA_SKV_MIN_SEQ_NONCAUSAL 16384
#endif
constexpr int kSharedKvMinSeq = TA_SKV_MIN_SEQ;
constexpr int kSharedKvMinSeqNonCausal = TA_SKV_MIN_SEQ_NONCAUSAL;
inline bool uses_shared_kv(int D, int S, bool causal) {
  return D == 256 ||
         (D == 128 && S >= (causal ? kSharedKvMinSeq : kSharedKvMinSeqNonCausal));
}

// The forward kernels of this library.
//   kPersistent  one 128-row query tile per work item, two softmax warpgroups on the two
//                64-key halves of every score tile (sdpa_fwd_sm100.cu); head dims 64, 128
//   kSharedKv    non-persistent, query tiles of one CTA share every K/V tile
//                (sdpa_fwd_sm100_shared_kv.cu); head dims 128, 256
enum KernelKind { kAuto = 0, kPersistent = 1, kSharedKv = 3 };

// The kernel that serves (kernel head dim D, S, causal, B*H): the process-wide forced
// choice (ta_debug_set_kernel) where it serves D, else the measured default.
KernelKind select_kernel(int D, int S, bool causal, long long bh);
void force_kernel(int kind);

// Query rows one work item (CTA) of `kind` covers.
int rows_per_item(KernelKind kind, int D);


// The shared-K/V kernel, reached through launch_sdpa_fwd.
cudaError_t launch_sdpa_fwd_shared_kv(const CUtensorMap& q, const CUtensorMap& k,
                                      const CUtensorMap& v, const FwdParams& p, int D,
                                      bool bf16, bool causal, bool out_f32, cudaStream_t stream);
int rows_per_cta_shared_kv(int D);

// Launches the variant of `kind` for (D, dtype, causal) on `stream`. Tensor maps are 4-D
// (D, S, H, B) with a 64 x 128 box and 128-byte swizzle. `o` is a map of the output like
// q's (used by the persistent kernel for 16-bit output; ignored otherwise). p.n_qblk must
// count blocks of rows_per_item(kind, D) rows.
cudaError_t launch_sdpa_fwd(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                            const CUtensorMap& o, const FwdParams& p,
                            int D, bool bf16, bool causal, bool out_f32, KernelKind kind,
                            cudaStream_t stream);

}  // namespace ta
