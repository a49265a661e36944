// Python fast-call entry points for the hot C-ABI calls (module
// pico_kernels_b200._pkfast). The same functions are reachable through
// ctypes (_lib.py); on a slow host CPU, ctypes' per-argument conversion of a
// 17-argument call costs several microseconds, more than a decode GEMM's
// kernel. These wrappers take the arguments as a vector of Python ints and
// floats (pointers as ints, None as 0) and call into libpico_b200.so.
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <cstdint>

#include "pico_b200.h"

namespace {

// The arguments of one call: integers and pointers as 64-bit words, the one
// float apart. kinds[i]: 'p' pointer (or None), 'i' integer, 'f' float.
struct Args {
  uint64_t w[17];
  float f;
};

bool parse(PyObject* const* args, Py_ssize_t n, const char* kinds, Args* a, const char* name) {
  if (n != 17) {
    PyErr_Format(PyExc_TypeError, "%s takes 17 arguments (%zd given)", name, n);
    return false;
  }
  for (int i = 0; i < 17; ++i) {
    PyObject* o = args[i];
    if (kinds[i] == 'f') {
      const double d = PyFloat_AsDouble(o);
      if (d == -1.0 && PyErr_Occurred()) return false;
      a->f = static_cast<float>(d);
      a->w[i] = 0;
    } else if (kinds[i] == 'p') {
      if (o == Py_None) {
        a->w[i] = 0;
        continue;
      }
      const unsigned long long v = PyLong_AsUnsignedLongLong(o);
      if (v == static_cast<unsigned long long>(-1) && PyErr_Occurred()) return false;
      a->w[i] = v;
    } else {
      const long long v = PyLong_AsLongLong(o);
      if (v == -1 && PyErr_Occurred()) return false;
      a->w[i] = static_cast<uint64_t>(v);
    }
  }
  return true;
}

template <typename P>
P* ptr(uint64_t w) {
  return reinterpret_cast<P*>(static_cast<uintptr_t>(w));
}
int64_t i64(uint64_t w) { return static_cast<int64_t>(w); }

// w4a16_gemm(a, a_dtype, lda, wp, scales, scalar_scale, group_size, M, N, K,
//            out, out_dtype, ldo, split_k, workspace, workspace_bytes, stream)
PyObject* w4a16_gemm(PyObject*, PyObject* const* args, Py_ssize_t n) {
  Args a;
  if (!parse(args, n, "piippfiiiipiiipip", &a, "w4a16_gemm")) return nullptr;
  const uint64_t* w = a.w;
  const int st = pk_w4a16_gemm(ptr<const void>(w[0]), static_cast<int>(w[1]), i64(w[2]),
                               ptr<const uint8_t>(w[3]), ptr<const void>(w[4]), a.f,
                               static_cast<int>(w[6]), i64(w[7]), i64(w[8]), i64(w[9]),
                               ptr<void>(w[10]), static_cast<int>(w[11]), i64(w[12]),
                               static_cast<int>(w[13]), ptr<void>(w[14]),
                               static_cast<size_t>(w[15]), ptr<void>(w[16]));
  return PyLong_FromLong(st);
}

// w4a16_gemm_host(a_host, a_dtype, lda, wp, scales, scalar_scale, group_size,
//                 M, N, K, y_host, out_dtype, a_dev, y_dev, workspace,
//                 workspace_bytes, stream)
PyObject* w4a16_gemm_host(PyObject*, PyObject* const* args, Py_ssize_t n) {
  Args a;
  if (!parse(args, n, "piippfiiiipipppip", &a, "w4a16_gemm_host")) return nullptr;
  const uint64_t* w = a.w;
  const int st = pk_w4a16_gemm_host(ptr<const void>(w[0]), static_cast<int>(w[1]), i64(w[2]),
                                    ptr<const uint8_t>(w[3]), ptr<const void>(w[4]), a.f,
                                    static_cast<int>(w[6]), i64(w[7]), i64(w[8]), i64(w[9]),
                                    ptr<void>(w[10]), static_cast<int>(w[11]), ptr<void>(w[12]),
                                    ptr<void>(w[13]), ptr<void>(w[14]),
                                    static_cast<size_t>(w[15]), ptr<void>(w[16]));
  return PyLong_FromLong(st);
}

PyMethodDef kMethods[] = {
    {"w4a16_gemm", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(w4a16_gemm)),
     METH_FASTCALL, "pk_w4a16_gemm with the C ABI's 17 arguments; returns the status."},
    {"w4a16_gemm_host",
     reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(w4a16_gemm_host)), METH_FASTCALL,
     "pk_w4a16_gemm_host with the C ABI's 17 arguments; returns the status."},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_pkfast",
                       "Fast-call entry points of libpico_b200.so.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__pkfast() { return PyModule_Create(&kModule); }
