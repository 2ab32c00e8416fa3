// Split-KV SDPA forward that allocates no device memory (ta_sdpa_fwd_split_noalloc).
//
// Who needs this: callers that must not call cudaMalloc from the code that runs attention.
// Examples are runtimes and plugins embedded in a host application that owns all device
// memory (the plugin is handed its inputs and outputs and nothing else), and latency-bound
// serving loops where an allocation could synchronise the device or fail under memory
// pressure at a bad moment. The split-KV path normally needs a temporary buffer for the
// per-slice partial results; here that buffer is a fixed array in device global memory
// that is part of the loaded library, so the call itself never allocates.
//
// Costs and limits of that choice:
//   - every GPU that loads the library reserves kScratchBytes (64 MiB) of global memory
//     for this array until the process exits, whether or not this entry point is used;
//   - one call needs n_split * B * H * S * (D + 1) * 4 bytes of it (D = the caller's head
//     dim, a multiple of 8 up to 256); larger problems are rejected with
//     TA_ERR_INVALID_ARGUMENT;
//   - all calls on a device share the one array, so calls whose work overlaps on the GPU
//     (different streams, or different host threads without ordering) race and corrupt
//     each other's results. Issue them on one stream, or order them. Each call overwrites
//     every scratch entry it later reads (every slice writes all of its rows, including
//     zeros / -inf for rows without keys), so nothing has to be cleared between calls;
//   - the first call on each device looks up the device address of the array
//     (cudaGetSymbolAddress) with that device current, and caches it. Make that first call
//     before any stream capture begins on the device.
#include <cuda_runtime.h>

#include <mutex>

#include "capi_internal.h"
#include "lse_combine.h"
#include "tiledattention_b200.h"

namespace {

constexpr size_t kScratchBytes = 64ull << 20;

// The scratch array. In host code its name is only a host-side stand-in for the symbol;
// kernels must be given the device address returned by cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_split_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return ta_capi_fail(TA_ERR_CUDA, "cudaGetDevice failed or device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_split_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return ta_capi_fail(TA_ERR_CUDA, "cudaGetSymbolAddress of the split-KV scratch failed");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return TA_OK;
}

}  // namespace

extern "C" int ta_sdpa_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o,
                                         float* lse, int B, int H, int S, int D,
                                         const int64_t* q_strides, const int64_t* k_strides,
                                         const int64_t* v_strides, const int64_t* o_strides,
                                         int dtype, int causal, float scale, int n_split,
                                         unsigned int* dev_status, void* stream) {
  TaNvtxRange nvtx_range("ta_sdpa_fwd_split_noalloc");
  ta_capi_clear_error();
  if (B <= 0 || H <= 0 || S <= 0 || n_split < 1)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "B, H, S, n_split must be positive");
  // The slice partials keep the caller's head dim (the forward writes only its columns).
  if (D < 8 || D > 256 || D % 8 != 0)
    return ta_capi_fail(TA_ERR_UNSUPPORTED_DIM, "head dim must be a multiple of 8 up to 256");
  const unsigned long long rows =
      static_cast<unsigned long long>(n_split) * B * H * static_cast<unsigned long long>(S);
  const unsigned long long o_bytes = rows * static_cast<unsigned long long>(D) * 4ull;
  const unsigned long long need = o_bytes + rows * 4ull;
  if (need > kScratchBytes)
    return ta_capi_fail(TA_ERR_INVALID_ARGUMENT,
                        "problem too large for the 64 MiB split-KV scratch array: "
                        "n_split*B*H*S*(D+1)*4 bytes must not exceed 67108864");
  if (!o || !o_strides) return ta_capi_fail(TA_ERR_INVALID_ARGUMENT, "null output pointer");
  if (o_strides[3] != 1 || reinterpret_cast<uintptr_t>(o) % 16 || (o_strides[2] * 2) % 8 ||
      (o_strides[1] * 2) % 8 || (o_strides[0] * 2) % 8)
    return ta_capi_fail(TA_ERR_LAYOUT, "o: unit head-dim stride, aligned base and strides required");
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  float* o_part = static_cast<float*>(scratch);
  float* lse_part = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + o_bytes);

  const int64_t part_strides[4] = {static_cast<int64_t>(H) * S * D, static_cast<int64_t>(S) * D, D,
                                   1};
  rc = run_forward(q, k, v, o_part, true, part_strides, static_cast<int64_t>(B) * H * S * D,
                   lse_part, B, H, S, D, q_strides, k_strides, v_strides, dtype, causal, scale,
                   0, S, n_split, dev_status, stream);
  if (rc) return rc;
  ta::CombineParams p{};
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.o = o;
  p.lse = lse;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.n_split = n_split;
  p.BH = B * H;
  p.H = H;
  p.S = S;
  const cudaError_t err =
      ta::launch_lse_combine(p, D, dtype == TA_DTYPE_BF16 ? 1 : 0, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return ta_capi_fail(TA_ERR_CUDA, "combine launch failed");
  return TA_OK;
}
