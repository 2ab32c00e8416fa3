// C ABI of tiledattention_b200: argument checks, TMA tensor-map encoding and the
// launch of the sm_100a SDPA forward kernel on the caller's stream.
//
// Replaces the reference host launcher run_flash_fwd
// (src/tiledattention/kernels/flash_fwd.py:821-973) and _launch_cutile_kernel
// (flash_fwd.py:786-818). The reference reshapes to [B*H,S,D] with .contiguous()
// and builds a K transpose view; here each operand is described by a 4-D TMA map
// (D, S, H, B) over the caller's own strides, so no copy or transpose is made.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "capi_internal.h"
#include "lse_combine.h"
#include "sdpa_fwd_sm100.h"
#include "tiledattention_b200.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D map over a [B,H,S,D] operand: dims (D, S, H, B), box 64 x 128 x 1 x 1,
// 128-byte swizzle, zero fill out of bounds (ragged sequence tail).
int make_map(CUtensorMap* map, const void* base, int B, int H, int S, int D,
             const int64_t* st, int dtype, const char* name, unsigned box_rows = 128) {
  auto enc = encode_fn();
  if (!enc) return fail(TA_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  const uint64_t esz = 2;
  if (st[3] != 1) return fail(TA_ERR_LAYOUT, "%s: head-dim stride must be 1 (got %lld)", name,
                              static_cast<long long>(st[3]));
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(TA_ERR_LAYOUT, "%s: base pointer not 16-byte aligned", name);
  const int64_t ext[3] = {S, H, B};
  const int64_t str[3] = {st[2], st[1], st[0]};
  cuuint64_t gdim[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t gstride[3];
  // A unit dimension's stride is never used to form an address; give it a legal value.
  uint64_t span = static_cast<uint64_t>(D) * esz;
  for (int i = 0; i < 3; ++i) {
    uint64_t s = static_cast<uint64_t>(str[i]) * esz;
    if (ext[i] == 1 || str[i] <= 0) {
      if (ext[i] != 1) return fail(TA_ERR_LAYOUT, "%s: non-positive stride", name);
      s = (span + 15) / 16 * 16;
    }
    if (s % 16) return fail(TA_ERR_LAYOUT, "%s: stride %d not a multiple of 16 bytes", name, i);
    gstride[i] = s;
    span = s * static_cast<uint64_t>(ext[i]);
  }
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype == TA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(base), gdim, gstride, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TA_ERR_LAYOUT, "%s: cuTensorMapEncodeTiled rejected the layout (CUresult %d)",
                name, static_cast<int>(r));
  return TA_OK;
}

int check_device() {
  static int cached[64];  // 0 unknown, 1 ok, 2 unsupported
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TA_ERR_CUDA, "cudaGetDevice failed");
  if (dev < 64 && cached[dev] == 1) return TA_OK;
  if (!ta_device_supported(dev))
    return fail(TA_ERR_DEVICE, "device %d is not a compute-capability 10.0 (B200) GPU", dev);
  if (dev < 64) cached[dev] = 1;
  return TA_OK;
}

#ifdef TA_TRACE
unsigned long long* g_trace = nullptr;
#endif
// Failure-path self-test settings (ta_debug_set_selftest); off by default.
std::atomic<int> g_selftest_stall{0};
std::atomic<unsigned long long> g_timeout_ns{0};
}  // namespace

int ta_capi_fail(int code, const char* msg) { return fail(code, "%s", msg); }

void ta_capi_clear_error() { g_last_error.clear(); }

extern "C" {

#ifdef TA_TRACE
// Experiment builds only (not part of the public header): device buffer for kernel
// event clocks, 64 blocks x 32 key tiles x 16 events of uint64.
void ta_debug_set_trace(void* dev_ptr) { g_trace = static_cast<unsigned long long*>(dev_ptr); }
#endif

int ta_abi_version(void) { return 100; }

void ta_debug_set_selftest(int stall, unsigned long long timeout_ns) {
  g_selftest_stall.store(stall ? 1 : 0);
  g_timeout_ns.store(timeout_ns);
}


const char* ta_last_error(void) { return g_last_error.c_str(); }

const char* ta_status_string(int status) {
  switch (status) {
    case TA_OK: return "ok";
    case TA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TA_ERR_UNSUPPORTED_DIM: return "unsupported head dim (supported: multiples of 8 up to 256)";
    case TA_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype (supported: float16, bfloat16)";
    case TA_ERR_LAYOUT: return "layout not expressible as a TMA tensor map";
    case TA_ERR_CUDA: return "CUDA runtime error";
    case TA_ERR_DRIVER: return "CUDA driver entry point error";
    case TA_ERR_DEVICE: return "unsupported device (requires compute capability 10.0)";
    default: return "unknown status";
  }
}

void ta_debug_set_kernel(int kind) { ta::force_kernel(kind); }

int ta_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

}  // extern "C"

// Shared body of the forward entry points: argument checks, tensor maps, launch.
int run_forward(const void* q, const void* k, const void* v, void* o, bool out_f32,
                       const int64_t* o_strides, int64_t o_split_stride, float* lse, int B,
                       int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, int dtype, int causal, float scale,
                       int kv_begin, int kv_end, int n_split, unsigned int* dev_status,
                       void* stream) {
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides)
    return fail(TA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || H <= 0 || S <= 0)
    return fail(TA_ERR_INVALID_ARGUMENT, "B, H, S must be positive (got %d, %d, %d)", B, H, S);
  // Kernel head dim: 64, 128 and 256 are native. Any other head dim that is a multiple of 8
  // (up to 256) runs on the next native kernel with tensor maps over its true extent: loads
  // zero-fill the missing columns (which add nothing to q.k and give zero output columns)
  // and the output is written for the true columns only (clipped TMA store, or predicated
  // 16-byte stores), so no padded copies are needed. Others: TA_ERR_UNSUPPORTED_DIM (the
  // caller pads).
  int kd = D;
  if (D != 64 && D != 128 && D != 256) {
    if (D < 8 || D > 256 || D % 8 != 0)
      return fail(TA_ERR_UNSUPPORTED_DIM,
                  "head dim %d: 64, 128, 256, or another multiple of 8 up to 256", D);
    kd = D <= 64 ? 64 : (D <= 128 ? 128 : 256);
  }
  if (dtype != TA_DTYPE_F16 && dtype != TA_DTYPE_BF16)
    return fail(TA_ERR_UNSUPPORTED_DTYPE, "dtype code %d", dtype);
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(TA_ERR_INVALID_ARGUMENT, "scale must be a positive finite number");
  if (kv_begin < 0 || kv_end > S || kv_begin > kv_end)
    return fail(TA_ERR_INVALID_ARGUMENT, "key range [%d, %d) outside [0, %d]", kv_begin, kv_end, S);
  if (n_split < 1 || n_split > 4096)
    return fail(TA_ERR_INVALID_ARGUMENT, "n_split must be in [1, 4096] (got %d)", n_split);
  const int64_t esz = out_f32 ? 4 : 2;
  if (o_strides[3] != 1) return fail(TA_ERR_LAYOUT, "o: head-dim stride must be 1");
  if (reinterpret_cast<uintptr_t>(o) % 16 || (o_strides[2] * esz) % 16 ||
      (o_strides[1] * esz) % 16 || (o_strides[0] * esz) % 16 || (o_split_stride * esz) % 16)
    return fail(TA_ERR_LAYOUT, "o: base / strides must be 16-byte aligned");
  if (static_cast<int64_t>(B) * H > (1ll << 24))
    return fail(TA_ERR_INVALID_ARGUMENT, "B*H too large");
  int rc = check_device();
  if (rc) return rc;

  CUtensorMap mq, mk, mv;
  if ((rc = make_map(&mq, q, B, H, S, D, q_strides, dtype, "q"))) return rc;
  if ((rc = make_map(&mk, k, B, H, S, D, k_strides, dtype, "k"))) return rc;
  if ((rc = make_map(&mv, v, B, H, S, D, v_strides, dtype, "v"))) return rc;
  const ta::KernelKind kind =
      ta::select_kernel(kd, S, causal != 0, static_cast<long long>(B) * H);
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  if (!out_f32 && kind == ta::kPersistent &&
      (rc = make_map(&mo, o, B, H, S, D, o_strides, dtype, "o")))
    return rc;

  ta::FwdParams p{};
  p.o = o;
  p.lse = lse;
  p.status = dev_status;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.o_split_stride = o_split_stride;
  p.d_out = D;
  p.S = S;
  p.H = H;
  p.BH = B * H;
  p.kv_begin = kv_begin;
  p.kv_end = kv_end;
  p.n_split = n_split;
  // Slices are whole 128-key tiles, so only the last one can be ragged.
  const int span = kv_end - kv_begin;
  p.split_len = ((span + n_split - 1) / n_split + 127) / 128 * 128;
  if (p.split_len == 0) p.split_len = 128;
  const int rows_per_item = ta::rows_per_item(kind, kd);
  p.n_qblk = (S + rows_per_item - 1) / rows_per_item;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
#ifdef TA_TRACE
  p.trace = g_trace;
#endif
  p.timeout_ns = g_timeout_ns.load();
  p.selftest_stall = g_selftest_stall.load();
  cudaError_t err = ta::launch_sdpa_fwd(mq, mk, mv, mo, p, kd, dtype == TA_DTYPE_BF16,
                                        causal != 0, out_f32, kind,
                                        static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess)
    return fail(TA_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(err));
  return TA_OK;
}

extern "C" {

int ta_sdpa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
                int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, const int64_t* o_strides, int dtype, int causal,
                float scale, unsigned int* dev_status, void* stream) {
  TaNvtxRange nvtx_range("ta_sdpa_fwd");
  g_last_error.clear();
  return run_forward(q, k, v, o, false, o_strides, 0, lse, B, H, S, D, q_strides, k_strides,
                     v_strides, dtype, causal, scale, 0, S, 1, dev_status, stream);
}

int ta_sdpa_fwd_partial(const void* q, const void* k, const void* v, float* o_part,
                        float* lse_part, int B, int H, int S, int D, const int64_t* q_strides,
                        const int64_t* k_strides, const int64_t* v_strides, int dtype,
                        int causal, float scale, int kv_begin, int kv_end, int n_split,
                        unsigned int* dev_status, void* stream) {
  TaNvtxRange nvtx_range("ta_sdpa_fwd_partial");
  g_last_error.clear();
  if (!lse_part) return fail(TA_ERR_INVALID_ARGUMENT, "lse_part must not be null");
  const int64_t st[4] = {static_cast<int64_t>(H) * S * D, static_cast<int64_t>(S) * D, D, 1};
  return run_forward(q, k, v, o_part, true, st, static_cast<int64_t>(B) * H * S * D, lse_part, B,
                     H, S, D, q_strides, k_strides, v_strides, dtype, causal, scale, kv_begin,
                     kv_end, n_split, dev_status, stream);
}

int ta_lse_combine(const float* o_part, const float* lse_part, int n_split, int B, int H, int S,
                   int D, void* o, const int64_t* o_strides, int out_dtype, float* lse,
                   void* stream) {
  TaNvtxRange nvtx_range("ta_lse_combine");
  g_last_error.clear();
  if (!o_part || !lse_part || !o || !o_strides)
    return fail(TA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (B <= 0 || H <= 0 || S <= 0 || n_split < 1)
    return fail(TA_ERR_INVALID_ARGUMENT, "B, H, S, n_split must be positive");
  if (D < 8 || D > 256 || D % 8 != 0)
    return fail(TA_ERR_UNSUPPORTED_DIM, "head dim %d is not a multiple of 8 up to 256", D);
  if (out_dtype != TA_DTYPE_F16 && out_dtype != TA_DTYPE_BF16 && out_dtype != TA_DTYPE_F32)
    return fail(TA_ERR_UNSUPPORTED_DTYPE, "output dtype code %d", out_dtype);
  const int64_t esz = out_dtype == TA_DTYPE_F32 ? 4 : 2;
  if (o_strides[3] != 1 || reinterpret_cast<uintptr_t>(o) % 16 ||
      reinterpret_cast<uintptr_t>(o_part) % 16 || (o_strides[2] * esz) % 8 ||
      (o_strides[1] * esz) % 8 || (o_strides[0] * esz) % 8)
    return fail(TA_ERR_LAYOUT, "o: unit head-dim stride, aligned base and strides required");
  int rc = check_device();
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
  const int kind = out_dtype == TA_DTYPE_F32 ? 2 : (out_dtype == TA_DTYPE_BF16 ? 1 : 0);
  cudaError_t err = ta::launch_lse_combine(p, D, kind, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess)
    return fail(TA_ERR_CUDA, "combine launch failed: %s", cudaGetErrorString(err));
  return TA_OK;
}

}  // extern "C"
