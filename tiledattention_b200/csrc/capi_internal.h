// Entry-point helpers shared between the C-ABI translation units (not part of the ABI).
#pragma once

#include <stdint.h>

#include <nvtx3/nvToolsExt.h>

// Argument checks, tensor maps and the launch of the SDPA forward kernel; out_f32 selects
// the fp32 (split-KV partial) output. Defined in capi.cu.
int run_forward(const void* q, const void* k, const void* v, void* o, bool out_f32,
                const int64_t* o_strides, int64_t o_split_stride, float* lse, int B, int H,
                int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, int dtype, int causal, float scale, int kv_begin,
                int kv_end, int n_split, unsigned int* dev_status, void* stream);

// Record an error message for ta_last_error() and return `code`.
int ta_capi_fail(int code, const char* msg);
void ta_capi_clear_error();

// NVTX range named after the entry point, open for the scope (host-side launch work, seen on
// the CPU row of nsys and by ncu --nvtx filters). Without a tool attached it costs a check.
struct TaNvtxRange {
  explicit TaNvtxRange(const char* name) { nvtxRangePushA(name); }
  ~TaNvtxRange() { nvtxRangePop(); }
  TaNvtxRange(const TaNvtxRange&) = delete;
  TaNvtxRange& operator=(const TaNvtxRange&) = delete;
};
