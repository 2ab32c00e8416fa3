// One-call host launcher for the common case of tiledattention_b200.sdpa: the reference's
// per-call Python path (src/tiledattention/sdpa.py:14-48 -> kernels/flash_fwd.py:821-973)
// costs ~35 us at S=512; this module does the checks, the output allocation, the stream
// lookup and the ta_sdpa_fwd call in one CPython call.
//
//   launch(q, k, v, causal: bool, scale: float, want_lse: bool) -> o | (o, lse) | None
//
// scale == -1.0 selects the default 1/sqrt(D). The device status word of each device is
// registered once with set_status(device_index, address); a device without one takes the
// full path (which creates and registers it).
//
// It returns None, having launched nothing, for every case it does not take: inputs the
// contract rejects, head dims outside {64, 128, 256} and multiples of 8 up to 256, strides a
// tensor map cannot describe, or any non-OK status from ta_sdpa_fwd (all of which are
// reported before a launch). The caller then runs the full Python path, which raises the
// reference's error for the case or copies / pads the inputs. ta_sdpa_fwd is bound once
// through set_entry(address) with the address of the symbol in the already-loaded native
// library, so the two share one copy of the library's state.
//
// The same module registers the torch operators of the reference's native-op slot
// (torch-ext/torch_binding.cpp:6-19: TORCH_LIBRARY + ops.impl(..., kCUDA, ...)) in C++:
//   tiledattention_b200::sdpa_fwd(Tensor q, Tensor k, Tensor v, bool causal, float scale)
//       -> Tensor
//   tiledattention_b200::sdpa_fwd_partial(Tensor q, Tensor k, Tensor v, bool causal,
//       float scale, int kv_begin, int kv_end, int n_split) -> (Tensor, Tensor)
// with CUDA kernels over the C ABI (copying strides a tensor map cannot describe, padding
// head dims that are not multiples of 8) and Meta kernels for shape propagation. Errors are
// raised with TORCH_CHECK, as the reference's op stub does (tiledattention.cu:13-33).
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <ATen/ops/constant_pad_nd.h>
#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>
#include <torch/library.h>

#include <tuple>

#include "tiledattention_b200.h"

#include <cmath>
#include <cstdint>

namespace {

using SdpaFwdFn = decltype(&ta_sdpa_fwd);
using SdpaPartialFn = decltype(&ta_sdpa_fwd_partial);
using LastErrorFn = decltype(&ta_last_error);

SdpaFwdFn g_entry = nullptr;
SdpaPartialFn g_partial = nullptr;
LastErrorFn g_last_error = nullptr;
constexpr int kMaxDevices = 64;
unsigned int* g_status[kMaxDevices] = {};
unsigned long long g_launches = 0;  // launches taken by this module (read by the tests)

constexpr int kDtypeF16 = TA_DTYPE_F16;
constexpr int kDtypeBf16 = TA_DTYPE_BF16;

// Tensor-map compatible: unit inner stride, 16-byte aligned base and outer strides.
bool tma_ok(const at::Tensor& t) {
  if (t.stride(3) != 1 || reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) return false;
  const int64_t esz = t.element_size();
  for (int d = 0; d < 3; ++d)
    if (t.size(d) > 1 && (t.stride(d) * esz) % 16) return false;
  return true;
}

PyObject* set_entry(PyObject*, PyObject* arg) {
  const unsigned long long addr = PyLong_AsUnsignedLongLong(arg);
  if (PyErr_Occurred()) return nullptr;
  g_entry = reinterpret_cast<SdpaFwdFn>(static_cast<uintptr_t>(addr));
  Py_RETURN_NONE;
}

// bind_ops(partial_address, last_error_address): the other entry points the torch
// operators call.
PyObject* bind_ops(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 2) {
    PyErr_SetString(PyExc_TypeError, "bind_ops(partial_address, last_error_address)");
    return nullptr;
  }
  const unsigned long long a = PyLong_AsUnsignedLongLong(args[0]);
  const unsigned long long b = PyLong_AsUnsignedLongLong(args[1]);
  if (PyErr_Occurred()) return nullptr;
  g_partial = reinterpret_cast<SdpaPartialFn>(static_cast<uintptr_t>(a));
  g_last_error = reinterpret_cast<LastErrorFn>(static_cast<uintptr_t>(b));
  Py_RETURN_NONE;
}

PyObject* set_status(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 2) {
    PyErr_SetString(PyExc_TypeError, "set_status(device_index, address)");
    return nullptr;
  }
  const long idx = PyLong_AsLong(args[0]);
  const unsigned long long addr = PyLong_AsUnsignedLongLong(args[1]);
  if (PyErr_Occurred()) return nullptr;
  if (idx < 0 || idx >= kMaxDevices) Py_RETURN_NONE;
  g_status[idx] = reinterpret_cast<unsigned int*>(static_cast<uintptr_t>(addr));
  Py_RETURN_NONE;
}

PyObject* launches(PyObject*, PyObject*) { return PyLong_FromUnsignedLongLong(g_launches); }

PyObject* launch(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 6 || g_entry == nullptr) Py_RETURN_NONE;
  for (int i = 0; i < 3; ++i)
    if (!THPVariable_Check(args[i])) Py_RETURN_NONE;
  if (!PyBool_Check(args[3]) || !PyFloat_Check(args[4]) || !PyBool_Check(args[5]))
    Py_RETURN_NONE;
  try {
    const at::Tensor& q = THPVariable_Unpack(args[0]);
    const at::Tensor& k = THPVariable_Unpack(args[1]);
    const at::Tensor& v = THPVariable_Unpack(args[2]);
    const bool causal = args[3] == Py_True;
    const bool want_lse = args[5] == Py_True;
    double scale = PyFloat_AS_DOUBLE(args[4]);
    if (scale != -1.0 && !(scale > 0.0)) Py_RETURN_NONE;

    if (q.dim() != 4 || !q.is_cuda() || !k.is_cuda() || !v.is_cuda()) Py_RETURN_NONE;
    if (q.sizes() != k.sizes() || q.sizes() != v.sizes()) Py_RETURN_NONE;
    const auto st = q.scalar_type();
    if (k.scalar_type() != st || v.scalar_type() != st) Py_RETURN_NONE;
    int dtype;
    if (st == at::kHalf)
      dtype = kDtypeF16;
    else if (st == at::kBFloat16)
      dtype = kDtypeBf16;
    else
      Py_RETURN_NONE;
    const c10::Device dev = q.device();
    if (k.device() != dev || v.device() != dev) Py_RETURN_NONE;
    const int dev_idx = dev.index();
    if (dev_idx < 0 || dev_idx >= kMaxDevices || g_status[dev_idx] == nullptr) Py_RETURN_NONE;
    if (q.requires_grad() || k.requires_grad() || v.requires_grad()) Py_RETURN_NONE;

    const int64_t B = q.size(0), H = q.size(1), S = q.size(2), D = q.size(3);
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0 || B * H > INT32_MAX || S > INT32_MAX)
      Py_RETURN_NONE;
    if (!(D == 64 || D == 128 || D == 256 || (D % 8 == 0 && D < 256))) Py_RETURN_NONE;
    if (!tma_ok(q) || !tma_ok(k) || !tma_ok(v)) Py_RETURN_NONE;
    if (scale == -1.0) scale = 1.0 / std::sqrt(static_cast<double>(D));

    c10::cuda::CUDAGuard guard(dev);
    at::Tensor o = at::empty({B, H, S, D}, q.options());
    at::Tensor lse;
    if (want_lse) lse = at::empty({B, H, S}, q.options().dtype(at::kFloat));
    const int64_t qs[4] = {q.stride(0), q.stride(1), q.stride(2), q.stride(3)};
    const int64_t ks[4] = {k.stride(0), k.stride(1), k.stride(2), k.stride(3)};
    const int64_t vs[4] = {v.stride(0), v.stride(1), v.stride(2), v.stride(3)};
    const int64_t os[4] = {o.stride(0), o.stride(1), o.stride(2), o.stride(3)};
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev_idx).stream();
    int rc;
    Py_BEGIN_ALLOW_THREADS
    rc = g_entry(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                 want_lse ? lse.data_ptr<float>() : nullptr, static_cast<int>(B),
                 static_cast<int>(H), static_cast<int>(S), static_cast<int>(D), qs, ks, vs, os,
                 dtype, causal ? 1 : 0, static_cast<float>(scale),
                 g_status[dev_idx], stream);
    Py_END_ALLOW_THREADS
    if (rc != 0) Py_RETURN_NONE;
    ++g_launches;
    if (!want_lse) return THPVariable_Wrap(std::move(o));
    PyObject* po = THPVariable_Wrap(std::move(o));
    if (po == nullptr) return nullptr;
    PyObject* pl = THPVariable_Wrap(std::move(lse));
    if (pl == nullptr) {
      Py_DECREF(po);
      return nullptr;
    }
    PyObject* tup = PyTuple_Pack(2, po, pl);
    Py_DECREF(po);
    Py_DECREF(pl);
    return tup;
  } catch (const std::exception&) {
    // Any ATen error (e.g. out of memory on the output): leave it to the full path, which
    // raises it through torch's own error translation.
    Py_RETURN_NONE;
  }
}


// ---------------------------------------------------------------- torch operators

const char* last_error() {
  const char* e = g_last_error ? g_last_error() : nullptr;
  return e && *e ? e : "native call failed";
}

// Inputs as the kernels take them: validated, head dim padded with zeros to the next native
// size unless it is a multiple of 8, strides a tensor map cannot describe copied.
struct Inputs {
  at::Tensor q, k, v;
  int64_t D, kd;
  int dtype;
};

Inputs prepare(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const char* op) {
  TORCH_CHECK(q.dim() == 4, op, ": q, k, v must be [B, H, S, D] tensors");
  TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(), op,
              ": q, k, v must have identical shapes");
  TORCH_CHECK(q.is_cuda() && k.device() == q.device() && v.device() == q.device(), op,
              ": q, k, v must be CUDA tensors on one device");
  const auto st = q.scalar_type();
  TORCH_CHECK(k.scalar_type() == st && v.scalar_type() == st, op,
              ": q, k, v must share one dtype");
  TORCH_CHECK(st == at::kHalf || st == at::kBFloat16, op,
              ": dtype must be torch.float16 or torch.bfloat16");
  Inputs in{q, k, v, q.size(3), 0, st == at::kBFloat16 ? kDtypeBf16 : kDtypeF16};
  TORCH_CHECK(in.D >= 1 && in.D <= 256, op, ": head dim ", in.D, " is not in [1, 256]");
  in.kd = in.D % 8 == 0 ? in.D : (in.D <= 64 ? 64 : (in.D <= 128 ? 128 : 256));
  at::Tensor* ts[3] = {&in.q, &in.k, &in.v};
  for (at::Tensor* t : ts) {
    if (in.kd != in.D) *t = at::constant_pad_nd(*t, {0, in.kd - in.D}, 0);
    if (!tma_ok(*t)) *t = t->contiguous();
  }
  return in;
}

unsigned int* status_of(const at::Tensor& t) {
  const int idx = t.device().index();
  return idx >= 0 && idx < kMaxDevices ? g_status[idx] : nullptr;
}

at::Tensor sdpa_fwd_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         bool causal, double scale) {
  TORCH_CHECK(scale > 0.0, "sdpa_fwd: scale must be positive");
  TORCH_CHECK(g_entry != nullptr, "sdpa_fwd: native library not bound");
  c10::cuda::CUDAGuard guard(q.device());
  if (q.numel() == 0) return at::empty(q.sizes(), q.options());
  Inputs in = prepare(q, k, v, "sdpa_fwd");
  const int64_t B = q.size(0), H = q.size(1), S = q.size(2);
  at::Tensor o = at::empty({B, H, S, in.kd}, q.options());
  const int64_t qs[4] = {in.q.stride(0), in.q.stride(1), in.q.stride(2), in.q.stride(3)};
  const int64_t ks[4] = {in.k.stride(0), in.k.stride(1), in.k.stride(2), in.k.stride(3)};
  const int64_t vs[4] = {in.v.stride(0), in.v.stride(1), in.v.stride(2), in.v.stride(3)};
  const int64_t os[4] = {o.stride(0), o.stride(1), o.stride(2), o.stride(3)};
  const int rc = g_entry(in.q.data_ptr(), in.k.data_ptr(), in.v.data_ptr(), o.data_ptr(), nullptr,
                         static_cast<int>(B), static_cast<int>(H), static_cast<int>(S),
                         static_cast<int>(in.kd), qs, ks, vs, os, in.dtype, causal ? 1 : 0,
                         static_cast<float>(scale), status_of(q),
                         c10::cuda::getCurrentCUDAStream(q.device().index()).stream());
  TORCH_CHECK(rc == TA_OK, "sdpa_fwd: ", last_error());
  return in.kd == in.D ? o : o.narrow(3, 0, in.D).contiguous();
}

std::tuple<at::Tensor, at::Tensor> sdpa_fwd_partial_cuda(const at::Tensor& q, const at::Tensor& k,
                                                         const at::Tensor& v, bool causal,
                                                         double scale, int64_t kv_begin,
                                                         int64_t kv_end, int64_t n_split) {
  TORCH_CHECK(scale > 0.0, "sdpa_fwd_partial: scale must be positive");
  TORCH_CHECK(n_split >= 1, "sdpa_fwd_partial: n_split must be at least 1");
  TORCH_CHECK(g_partial != nullptr, "sdpa_fwd_partial: native library not bound");
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t B = q.size(0), H = q.size(1), S = q.size(2);
  auto f32 = q.options().dtype(at::kFloat);
  if (q.numel() == 0)
    return {at::empty({n_split, B, H, S, q.size(3)}, f32), at::empty({n_split, B, H, S}, f32)};
  Inputs in = prepare(q, k, v, "sdpa_fwd_partial");
  at::Tensor o = at::empty({n_split, B, H, S, in.kd}, f32);
  at::Tensor lse = at::empty({n_split, B, H, S}, f32);
  const int64_t qs[4] = {in.q.stride(0), in.q.stride(1), in.q.stride(2), in.q.stride(3)};
  const int64_t ks[4] = {in.k.stride(0), in.k.stride(1), in.k.stride(2), in.k.stride(3)};
  const int64_t vs[4] = {in.v.stride(0), in.v.stride(1), in.v.stride(2), in.v.stride(3)};
  const int rc = g_partial(in.q.data_ptr(), in.k.data_ptr(), in.v.data_ptr(),
                           o.data_ptr<float>(), lse.data_ptr<float>(), static_cast<int>(B),
                           static_cast<int>(H), static_cast<int>(S), static_cast<int>(in.kd), qs,
                           ks, vs, in.dtype, causal ? 1 : 0, static_cast<float>(scale),
                           static_cast<int>(kv_begin), static_cast<int>(kv_end),
                           static_cast<int>(n_split), status_of(q),
                           c10::cuda::getCurrentCUDAStream(q.device().index()).stream());
  TORCH_CHECK(rc == TA_OK, "sdpa_fwd_partial: ", last_error());
  if (in.kd != in.D) o = o.narrow(4, 0, in.D).contiguous();
  return {o, lse};
}

at::Tensor sdpa_fwd_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, bool, double) {
  return at::empty(q.sizes(), q.options());
}

std::tuple<at::Tensor, at::Tensor> sdpa_fwd_partial_meta(const at::Tensor& q, const at::Tensor&,
                                                         const at::Tensor&, bool, double,
                                                         int64_t, int64_t, int64_t n_split) {
  auto f32 = q.options().dtype(at::kFloat);
  return {at::empty({n_split, q.size(0), q.size(1), q.size(2), q.size(3)}, f32),
          at::empty({n_split, q.size(0), q.size(1), q.size(2)}, f32)};
}

PyMethodDef kMethods[] = {
    {"set_entry", reinterpret_cast<PyCFunction>(set_entry), METH_O,
     "Bind ta_sdpa_fwd by its address in the loaded native library."},
    {"bind_ops", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(bind_ops)),
     METH_FASTCALL, "Bind the entry points the torch operators call."},
    {"set_status", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(set_status)),
     METH_FASTCALL, "Register the device status word of a device."},
    {"launches", reinterpret_cast<PyCFunction>(launches), METH_NOARGS,
     "Number of launches this module has made."},
    {"launch", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(launch)),
     METH_FASTCALL, "Checked single-call sdpa launch; None when the full path must run."},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_fast_launch", nullptr, -1, kMethods,
                       nullptr, nullptr, nullptr, nullptr};

}  // namespace

TORCH_LIBRARY(tiledattention_b200, m) {
  m.def("sdpa_fwd(Tensor q, Tensor k, Tensor v, bool causal, float scale) -> Tensor");
  m.def(
      "sdpa_fwd_partial(Tensor q, Tensor k, Tensor v, bool causal, float scale, int kv_begin, "
      "int kv_end, int n_split) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(tiledattention_b200, CUDA, m) {
  m.impl("sdpa_fwd", &sdpa_fwd_cuda);
  m.impl("sdpa_fwd_partial", &sdpa_fwd_partial_cuda);
}

TORCH_LIBRARY_IMPL(tiledattention_b200, Meta, m) {
  m.impl("sdpa_fwd", &sdpa_fwd_meta);
  m.impl("sdpa_fwd_partial", &sdpa_fwd_partial_meta);
}

PyMODINIT_FUNC PyInit__fast_launch() { return PyModule_Create(&kModule); }
