/*
 * _fastcall: the decode call path of lowbit.ops without ctypes. A CPython extension whose functions take the
 * launch arguments as plain Python integers (pointers, sizes, the stream handle) through vectorcall and call the
 * C ABI of liblowbit_b200.so directly -- the same library and entry points ctypes binds, minus its per-argument
 * conversion (about 2 us of an 11-argument call). No torch headers: the caller passes data_ptr() values.
 *
 *   gemv(x, w, s, y, m, n, k, group, version, stream) -> status   lb_w4_gemv (version 1-4, 6) or lb_w4_gemm_tc (5)
 *   linear(x, w, s, bias, y, m, n, k, group, version, stream) -> status                           lb_w4_linear
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include "../../include/lowbit_b200.h"

static int as_args(PyObject* const* args, Py_ssize_t nargs, Py_ssize_t want, long long* out) {
  if (nargs != want) {
    PyErr_Format(PyExc_TypeError, "expected %zd integer arguments, got %zd", want, nargs);
    return -1;
  }
  for (Py_ssize_t i = 0; i < nargs; ++i) {
    if (args[i] == Py_None) {
      out[i] = 0;
      continue;
    }
    out[i] = PyLong_AsLongLong(args[i]);
    if (out[i] == -1 && PyErr_Occurred()) return -1;
  }
  return 0;
}

#define PTR(v) ((const void*)(uintptr_t)(v))

static PyObject* fc_gemv(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  long long a[10];
  (void)self;
  if (as_args(args, nargs, 10, a)) return NULL;
  int rc;
  if (a[8] == 5)
    rc = lb_w4_gemm_tc(PTR(a[0]), PTR(a[1]), PTR(a[2]), (void*)(uintptr_t)a[3], a[4], a[5], a[6], a[7], 0,
                       (lb_stream_t)(uintptr_t)a[9]);
  else
    rc = lb_w4_gemv(PTR(a[0]), PTR(a[1]), PTR(a[2]), (void*)(uintptr_t)a[3], a[4], a[5], a[6], a[7], (int)a[8], 0,
                    (lb_stream_t)(uintptr_t)a[9]);
  return PyLong_FromLong(rc);
}

static PyObject* fc_linear(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  long long a[11];
  (void)self;
  if (as_args(args, nargs, 11, a)) return NULL;
  int rc = lb_w4_linear(PTR(a[0]), PTR(a[1]), PTR(a[2]), PTR(a[3]), (void*)(uintptr_t)a[4], a[5], a[6], a[7], a[8],
                        (int)a[9], (lb_stream_t)(uintptr_t)a[10]);
  return PyLong_FromLong(rc);
}

static PyMethodDef methods[] = {
    {"gemv", (PyCFunction)(void (*)(void))fc_gemv, METH_FASTCALL,
     "gemv(x, w, s, y, m, n, k, group, version, stream) -> lb_status (lb_w4_gemv; version 5: lb_w4_gemm_tc)"},
    {"linear", (PyCFunction)(void (*)(void))fc_linear, METH_FASTCALL,
     "linear(x, w, s, bias, y, m, n, k, group, version, stream) -> lb_status (lb_w4_linear)"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_fastcall", NULL, -1, methods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__fastcall(void) { return PyModule_Create(&module); }
