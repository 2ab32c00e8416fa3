// Exchange step of the multi-GPU split-KV forward, written over NVLink peer memory.
//
// Every GPU of a group attends all query rows to its own key slices and leaves its
// per-slice state (o fp32 [n_slices][B*H][S][D], lse fp32 [n_slices][B*H*S]) in a buffer
// that every peer has mapped (e.g. torch symmetric memory). Two kernels then finish the
// forward without any collective library in the data path:
//
//   ta_peer_barrier     one CTA; thread i stores the call's epoch into peer i's flag slot
//                       for this rank (release, system scope) and waits, with a time
//                       limit, until peer i's epoch appears in this rank's own slot i
//                       (acquire, system scope). On expiry it sets TA_DEVSTAT_PEER_TIMEOUT
//                       in the status word and returns, so the context stays usable.
//   ta_lse_merge_peers  rows [s_begin, s_end) of every (b,h): reads the states of every
//                       slice of every peer straight from their memory (plain 16-byte P2P
//                       loads, no multicast), merges them by log-sum-exp exactly like
//                       lse_combine, and stores the result to every destination given
//                       (this GPU's output for a reduce-scatter by rows, or all peers'
//                       outputs, which fuses the all-gather into the same pass).
//
// The merge reads the status word first; if the barrier before it timed out, it writes
// NaN instead of merging states that may not have arrived.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "capi_internal.h"
#include "tiledattention_b200.h"

namespace {

constexpr int kMaxPeers = TA_MAX_PEERS;
constexpr int kMaxSources = 16;

struct PeerMergeParams {
  const float* o_src[kMaxSources];
  const float* lse_src[kMaxSources];
  void* o_dst[kMaxPeers];
  float* lse_dst[kMaxPeers];
  const unsigned int* status;
  int64_t o_sb, o_sh, o_ss;
  int n_src, n_dst, BH, H, S, s_begin, s_end, out_rows, row_base;
  int D;  // head dim (set by launch_merge)
};

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct BarrierParams {
  unsigned int* flags[kMaxPeers];  // flags[i]: peer i's slot array (kMaxPeers words)
  unsigned int* status;
  unsigned long long timeout_ns;
  unsigned int epoch;
  int n_peers, rank;
};

__global__ void peer_barrier_kernel(BarrierParams p) {
  const int i = threadIdx.x;
  if (i >= p.n_peers) return;
  // Everything this GPU wrote before the barrier (the states) becomes visible to the
  // peers before they can observe the flag.
  __threadfence_system();
  store_release_sys(p.flags[i] + p.rank, p.epoch);
  const unsigned int* mine = p.flags[p.rank] + i;
  const uint64_t t0 = global_timer_ns();
  while (static_cast<int>(load_acquire_sys(mine) - p.epoch) < 0) {
    if (global_timer_ns() - t0 > p.timeout_ns) {
      if (p.status) atomicOr(p.status, TA_DEVSTAT_PEER_TIMEOUT);
      return;
    }
    __nanosleep(64);
  }
}

// DT: the head dim, or 0 for a head dim known at run time only (p.D, a multiple of 8 up to
// 256: four columns per thread, rows of D/4 threads packed into the 256-thread block).
template <int DT, int OUT>  // OUT: 0 f16, 1 bf16, 2 f32
__global__ void __launch_bounds__(256) lse_merge_peers_kernel(PeerMergeParams p) {
  const int D = DT > 0 ? DT : p.D;
  const int kThreadsPerRow = D / 4;
  const int kRowsPerBlock = 256 / kThreadsPerRow;
  if (threadIdx.x >= kRowsPerBlock * kThreadsPerRow) return;
  const int slice = p.s_end - p.s_begin;
  const int64_t rows = static_cast<int64_t>(p.BH) * slice;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + threadIdx.x / kThreadsPerRow;
  const int d0 = (threadIdx.x % kThreadsPerRow) * 4;
  if (r >= rows) return;
  const int bh = static_cast<int>(r / slice);
  const int s = p.s_begin + static_cast<int>(r % slice);
  const int64_t src_row = static_cast<int64_t>(bh) * p.S + s;
  const bool failed = p.status != nullptr && (*p.status & TA_DEVSTAT_PEER_TIMEOUT) != 0u;

  float ls[kMaxSources];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxSources; ++i) {
    ls[i] = (i < p.n_src && !failed) ? p.lse_src[i][src_row] : -INFINITY;
    m = fmaxf(m, ls[i]);
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (m != -INFINITY) {
#pragma unroll
    for (int i = 0; i < kMaxSources; ++i) {
      if (i >= p.n_src || ls[i] == -INFINITY) continue;
      const float w = __expf(ls[i] - m);
      const float4 v = *reinterpret_cast<const float4*>(p.o_src[i] + src_row * D + d0);
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
  float lse = wsum > 0.f ? m + __logf(wsum) : -INFINITY;
  if (failed) {
    acc = make_float4(NAN, NAN, NAN, NAN);
    lse = NAN;
  }
  const int b = bh / p.H, h = bh % p.H;
  const int64_t off = static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh +
                      static_cast<int64_t>(s - p.row_base) * p.o_ss + d0;
  uint2 packed;
  if constexpr (OUT == 1) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  } else if constexpr (OUT == 0) {
    __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
    packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  }
  const int64_t lse_off = static_cast<int64_t>(bh) * p.out_rows + (s - p.row_base);
#pragma unroll
  for (int j = 0; j < kMaxPeers; ++j) {
    if (j >= p.n_dst) break;
    if constexpr (OUT == 2) {
      *reinterpret_cast<float4*>(static_cast<float*>(p.o_dst[j]) + off) = acc;
    } else {
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.o_dst[j]) + off) = packed;
    }
    if (p.lse_dst[j] != nullptr && d0 == 0) p.lse_dst[j][lse_off] = lse;
  }
  // Stores into peers' memory are made visible system-wide before the barrier that follows
  // this kernel lets a peer read them.
  if (p.n_dst > 1) __threadfence_system();
}

cudaError_t launch_merge(const PeerMergeParams& p, int D, int out_kind, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.BH) * (p.s_end - p.s_begin);
  if (rows <= 0) return cudaSuccess;
  const int rows_per_block = 256 / (D / 4);
  const int64_t grid = (rows + rows_per_block - 1) / rows_per_block;
  if (grid > 0x7fffffffll) return cudaErrorInvalidValue;
PeerMergeParams q = p;
  q.D = D;
#define TA_MERGE(DD, OO)                                                                   \
  if ((DD == 0 || D == DD) && out_kind == OO) {                                           \
    lse_merge_peers_kernel<DD, OO><<<static_cast<int>(grid), 256, 0, stream>>>(q);        \
    return cudaGetLastError();                                                            \
  }
  TA_MERGE(64, 0) TA_MERGE(64, 1) TA_MERGE(64, 2) TA_MERGE(128, 0) TA_MERGE(128, 1)
  TA_MERGE(128, 2) TA_MERGE(256, 0) TA_MERGE(256, 1) TA_MERGE(256, 2)
  if (D >= 8 && D <= 256 && D % 8 == 0) {
    TA_MERGE(0, 0) TA_MERGE(0, 1) TA_MERGE(0, 2)
  }
#undef TA_MERGE
  return cudaErrorInvalidValue;
}

bool aligned16(const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

}  // namespace

extern "C" int ta_peer_barrier(unsigned int* const* flags, int n_peers, int rank,
                               unsigned int epoch, unsigned long long timeout_ns,
                               unsigned int* dev_status, void* stream) {
  TaNvtxRange nvtx_range("ta_peer_barrier");
  ta_capi_clear_error();
  if (!flags) return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "null flags array");
  if (n_peers < 1 || n_peers > kMaxPeers || rank < 0 || rank >= n_peers)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "n_peers must be in [1, 8] and 0 <= rank < n_peers");
  BarrierParams p{};
  for (int i = 0; i < n_peers; ++i) {
    if (!flags[i] || reinterpret_cast<uintptr_t>(flags[i]) % 4)
      return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "null or unaligned peer flag pointer");
    p.flags[i] = flags[i];
  }
  p.status = dev_status;
  p.timeout_ns = timeout_ns ? timeout_ns : 1000000000ull;
  p.epoch = epoch;
  p.n_peers = n_peers;
  p.rank = rank;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ta_capi_fail(TA_ERR_CUDA, "peer barrier launch failed");
  return TA_OK;
}

extern "C" int ta_lse_merge_peers(const void* const* o_src, const void* const* lse_src, int n_src,
                                  int B, int H, int S, int D, int s_begin, int s_end,
                                  void* const* o_dst, float* const* lse_dst, int n_dst,
                                  const int64_t* o_strides, int out_rows, int row_base,
                                  int out_dtype, const unsigned int* dev_status, void* stream) {
  TaNvtxRange nvtx_range("ta_lse_merge_peers");
  ta_capi_clear_error();
  if (!o_src || !lse_src || !o_dst || !o_strides)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n_src < 1 || n_src > kMaxSources || n_dst < 1 || n_dst > kMaxPeers)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "n_src must be in [1, 16] and n_dst in [1, 8]");
  if (B <= 0 || H <= 0 || S <= 0 || s_begin < 0 || s_end > S || s_begin > s_end ||
      row_base < 0 || row_base > s_begin || s_end - row_base > out_rows)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "bad sizes or row range");
  if (D < 8 || D > 256 || D % 8 != 0)
    return ta_capi_fail(TA_ERR_UNSUPPORTED_DIM, "head dim must be a multiple of 8 up to 256");
  if (out_dtype != TA_DTYPE_F16 && out_dtype != TA_DTYPE_BF16 && out_dtype != TA_DTYPE_F32)
    return ta_capi_fail(TA_ERR_UNSUPPORTED_DTYPE, "output dtype must be f16, bf16 or f32");
  const int64_t esz = out_dtype == TA_DTYPE_F32 ? 4 : 2;
  const int64_t vec = esz * 4;  // bytes one thread stores per row
  if (o_strides[3] != 1 || (o_strides[2] * esz) % vec || (o_strides[1] * esz) % vec ||
      (o_strides[0] * esz) % vec)
    return ta_capi_fail(TA_ERR_LAYOUT, "o: unit head-dim stride and aligned strides required");
  PeerMergeParams p{};
  for (int i = 0; i < n_src; ++i) {
    if (!o_src[i] || !lse_src[i] || !aligned16(o_src[i]))
      return ta_capi_fail(TA_ERR_LAYOUT, "null or unaligned source state pointer");
    p.o_src[i] = static_cast<const float*>(o_src[i]);
    p.lse_src[i] = static_cast<const float*>(lse_src[i]);
  }
  for (int j = 0; j < n_dst; ++j) {
    if (!o_dst[j] || reinterpret_cast<uintptr_t>(o_dst[j]) % vec)
      return ta_capi_fail(TA_ERR_LAYOUT, "null or unaligned destination pointer");
    p.o_dst[j] = o_dst[j];
    p.lse_dst[j] = lse_dst ? lse_dst[j] : nullptr;
  }
  p.status = dev_status;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.n_src = n_src;
  p.n_dst = n_dst;
  p.BH = B * H;
  p.H = H;
  p.S = S;
  p.s_begin = s_begin;
  p.s_end = s_end;
  p.out_rows = out_rows;
  p.row_base = row_base;
  const int kind = out_dtype == TA_DTYPE_F32 ? 2 : (out_dtype == TA_DTYPE_BF16 ? 1 : 0);
  const cudaError_t err = launch_merge(p, D, kind, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return ta_capi_fail(TA_ERR_CUDA, "peer merge launch failed");
  return TA_OK;
}
