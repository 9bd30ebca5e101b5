// _torchcall: the decode call path of lowbit.ops (ops.gemv / ops.linear at versions 5 and 6) as one CPython call
// that takes torch tensors. It unpacks them in C++ (no per-attribute Python calls), checks what the C ABI cannot
// see -- dtype, device, shape, contiguity of x, out and bias, and that x's device is the current one -- allocates
// the output when none is given, and calls the C ABI of liblowbit_b200.so on torch's current stream. Anything
// unusual returns None, and the Python caller then takes its fully checked path (which raises the reference's
// errors); a refusal by the C ABI raises RuntimeError with lb_last_error().
//
//   gemv(x, w_ptr, s_ptr, device, n, k, group, version, out=None, bias=None) -> Tensor | None
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>

#include "../../include/lowbit_b200.h"

namespace {

bool half_cuda_on(const at::Tensor& t, int dev) {
  return t.scalar_type() == at::kHalf && t.is_cuda() && t.get_device() == dev && t.is_contiguous();
}

PyObject* tc_gemv(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs < 8 || nargs > 10) {
    PyErr_SetString(PyExc_TypeError, "gemv(x, w_ptr, s_ptr, device, n, k, group, version, out=None, bias=None)");
    return nullptr;
  }
  if (!THPVariable_Check(args[0])) Py_RETURN_NONE;
  long long v[7];
  for (int i = 0; i < 7; ++i) {
    v[i] = PyLong_AsLongLong(args[1 + i]);
    if (v[i] == -1 && PyErr_Occurred()) return nullptr;
  }
  const void* w = reinterpret_cast<const void*>(static_cast<uintptr_t>(v[0]));
  const void* s = reinterpret_cast<const void*>(static_cast<uintptr_t>(v[1]));
  const int dev = static_cast<int>(v[2]), version = static_cast<int>(v[6]);
  const int64_t n = v[3], k = v[4], group = v[5];
  PyObject* out_obj = nargs > 8 ? args[8] : Py_None;
  PyObject* bias_obj = nargs > 9 ? args[9] : Py_None;

  const at::Tensor& x = THPVariable_Unpack(args[0]);
  if (!half_cuda_on(x, dev) || x.dim() != 2 || x.size(1) != k || x.size(0) == 0 ||
      c10::cuda::current_device() != dev)
    Py_RETURN_NONE;
  const int64_t m = x.size(0);
  const void* bias = nullptr;
  if (bias_obj != Py_None) {
    if (!THPVariable_Check(bias_obj)) Py_RETURN_NONE;
    const at::Tensor& b = THPVariable_Unpack(bias_obj);
    if (!half_cuda_on(b, dev) || b.dim() != 1 || b.size(0) != n) Py_RETURN_NONE;
    bias = b.data_ptr();
  }
  at::Tensor y;
  if (out_obj == Py_None) {
    y = at::empty({m, n}, x.options());
  } else {
    if (!THPVariable_Check(out_obj)) Py_RETURN_NONE;
    const at::Tensor& o = THPVariable_Unpack(out_obj);
    if (!half_cuda_on(o, dev) || o.dim() != 2 || o.size(0) != m || o.size(1) != n) Py_RETURN_NONE;
    y = o;
  }
  const auto st = reinterpret_cast<lb_stream_t>(c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream());
  int rc;
  if (bias)
    rc = lb_w4_linear(x.data_ptr(), w, s, bias, y.data_ptr(), m, n, k, group, version, st);
  else if (version == 5)
    rc = lb_w4_gemm_tc(x.data_ptr(), w, s, y.data_ptr(), m, n, k, group, 0, st);
  else
    rc = lb_w4_gemv(x.data_ptr(), w, s, y.data_ptr(), m, n, k, group, version, 0, st);
  if (rc) {
    const char* msg = lb_last_error();
    PyErr_SetString(PyExc_RuntimeError, (msg && msg[0]) ? msg : lb_status_string(rc));
    return nullptr;
  }
  if (out_obj != Py_None) {
    Py_INCREF(out_obj);
    return out_obj;
  }
  return THPVariable_Wrap(std::move(y));
}

PyMethodDef methods[] = {
    {"gemv", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)(void)>(tc_gemv)), METH_FASTCALL,
     "gemv(x, w_ptr, s_ptr, device, n, k, group, version, out=None, bias=None) -> Tensor, or None for the checked "
     "path"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef module = {PyModuleDef_HEAD_INIT, "_torchcall", nullptr, -1, methods, nullptr, nullptr, nullptr, nullptr};

}  // namespace

PyMODINIT_FUNC PyInit__torchcall(void) { return PyModule_Create(&module); }
