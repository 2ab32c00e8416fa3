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

// Whether (D, S, causal, B*H) runs on the shared-K/V kernel (sdpa_fwd_sm100_shared_kv.cu):
// head dim 256 always; head dim 128 where loading each K/V tile once per 256 query rows
// instead of once per 128 outweighs the persistent one-tile kernel's scheduling and lower
// start-up cost. Crossovers measured on B200 over B*H in {8, 16, 64, 256} and S from 4096 to
// 65536 (both kernels within 3 % of each other near the lines):
//   non-causal  B*H * S^2 >= 2^34 (S 8192 from B*H 256, 16384 from 64, 32768 from 16,
//               65536 from 4);
//   causal      S >= 65536, or S >= 32768 with B*H >= 256.
inline bool uses_shared_kv(int D, int S, bool causal, long long bh) {
  if (D == 256) return true;
  if (D != 128) return false;
  const double s = static_cast<double>(S);
  if (!causal) return static_cast<double>(bh) * s * s >= 17179869184.0;  // 2^34
  return S >= 65536 || (S >= 32768 && bh >= 256);
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
