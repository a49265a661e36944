// Torch-aware fast-call entry points (module pico_kernels_b200._pktorch).
//
// gemm_int4.int4_gemm and int4_gemm_host check a dozen tensor attributes
// before their C-ABI call; on a slow host CPU each attribute read from Python
// costs 0.1-0.3 us, together more than the decode GEMM's kernel. These
// functions make the same checks on the tensors in C++ and call
// libpico_b200.so directly (linked by its soname, so the library instance is
// the one ctypes loaded). Each returns the output tensor, or the C ABI's
// status when the call failed, or -1 when the call is not one it serves
// (inputs that need a copy or a cast, a workspace not yet allocated, a host
// output not given, anything unexpected): the caller then takes the Python
// path, which raises the documented errors or allocates. Calls run with the
// GIL held (the shape cache below relies on it). The
// workspaces are the ones pico_kernels_b200._lib keeps (its dict is bound
// once with bind()), so reset_workspaces() covers both paths.
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/Dtype.h>
#include <torch/csrc/autograd/python_variable.h>

#include <cstdint>

#include "pico_b200.h"

namespace {

constexpr long kNotServed = -1;

PyObject* g_workspaces = nullptr;  // _lib._workspaces: {(device, stream, tag): uint8 tensor}
PyObject* g_tag_splitk = nullptr;
PyObject* g_tag_a = nullptr;
PyObject* g_tag_y = nullptr;

int code_of(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return PK_F16;
    case at::kBFloat16: return PK_BF16;
    case at::kFloat: return PK_F32;
    default: return -1;
  }
}

// Pointer of the cached workspace (device, stream, tag) when it holds at
// least `nbytes`; nullptr otherwise (the Python path allocates it).
void* workspace(int device, uint64_t stream, PyObject* tag, size_t nbytes) {
  if (g_workspaces == nullptr) return nullptr;
  PyObject* key = Py_BuildValue("(iKO)", device, static_cast<unsigned long long>(stream), tag);
  if (key == nullptr) {
    PyErr_Clear();
    return nullptr;
  }
  PyObject* buf = PyDict_GetItemWithError(g_workspaces, key);  // borrowed
  Py_DECREF(key);
  if (buf == nullptr) {
    PyErr_Clear();
    return nullptr;
  }
  if (!THPVariable_Check(buf)) return nullptr;
  const at::Tensor& t = THPVariable_Unpack(buf);
  if (static_cast<size_t>(t.numel()) < nbytes || t.scalar_type() != at::kByte) return nullptr;
  return t.data_ptr();
}

// pk_w4a16_workspace_size per (M, N, K, split_k): a pure function of the shape.
size_t workspace_bytes(int64_t M, int64_t N, int64_t K, int split_k) {
  struct Entry {
    int64_t M, N, K;
    int split;
    size_t bytes;
  };
  static Entry cache[16];
  static int used = 0, next = 0;
  for (int i = 0; i < used; ++i)
    if (cache[i].M == M && cache[i].N == N && cache[i].K == K && cache[i].split == split_k)
      return cache[i].bytes;
  const size_t b = pk_w4a16_workspace_size(M, N, K, split_k);
  cache[next] = Entry{M, N, K, split_k, b};
  next = (next + 1) % 16;
  if (used < 16) ++used;
  return b;
}

// The weights and scales of a W4A16 call: w_packed [K, N/2] uint8 on `device`
// (contiguous), scale a [G, N] tensor of a's dtype (contiguous, same device)
// or a Python number. False when the Python path must handle them.
struct Weights {
  const void* wp;
  const void* scales;
  float scalar;
  int group;
  int64_t N;
};
bool weights(PyObject* w_obj, PyObject* scale_obj, PyObject* group_obj, int64_t K,
             at::ScalarType a_type, int device, Weights* w) {
  if (!THPVariable_Check(w_obj)) return false;
  const at::Tensor& wp = THPVariable_Unpack(w_obj);
  if (!wp.is_cuda() || wp.get_device() != device || wp.scalar_type() != at::kByte ||
      wp.dim() != 2 || wp.size(0) != K || !wp.is_contiguous())
    return false;
  w->wp = wp.data_ptr();
  w->N = 2 * wp.size(1);
  if (THPVariable_Check(scale_obj)) {
    const at::Tensor& s = THPVariable_Unpack(scale_obj);
    if (s.numel() <= 1) return false;  // a one-element tensor: the Python path reads it
    if (!s.is_cuda() || s.get_device() != device || s.dim() != 2 || s.size(1) != w->N ||
        s.scalar_type() != a_type || !s.is_contiguous())
      return false;
    const int64_t G = s.size(0);
    int64_t group = 0;
    if (group_obj == Py_None) {  // prefer 128 when several sizes give G groups
      for (int64_t g : {static_cast<int64_t>(128), K / G})
        if (g > 0 && (K + g - 1) / g == G) {
          group = g;
          break;
        }
    } else {
      group = PyLong_AsLongLong(group_obj);
      if (group == -1 && PyErr_Occurred()) {
        PyErr_Clear();
        return false;
      }
    }
    if (group <= 0 || (K + group - 1) / group != G || group > (1ll << 30)) return false;
    w->scales = s.data_ptr();
    w->scalar = 1.0f;
    w->group = static_cast<int>(group);
    return true;
  }
  if (!PyFloat_Check(scale_obj) && !PyLong_Check(scale_obj)) return false;
  const double v = PyFloat_AsDouble(scale_obj);
  if (v == -1.0 && PyErr_Occurred()) {
    PyErr_Clear();
    return false;
  }
  w->scales = nullptr;
  w->scalar = static_cast<float>(v);
  w->group = 0;
  return true;
}

// out_dtype (a torch.dtype) and out: a contiguous [M, N] tensor of that
// dtype (fp32 or bf16), on CUDA `device` (device >= 0) or on the host (-1).
bool output(PyObject* out_obj, PyObject* dtype_obj, int64_t M, int64_t N, int device, void** ptr,
            int* code, int64_t* elt) {
  if (!THPVariable_Check(out_obj) || !THPDtype_Check(dtype_obj)) return false;
  const at::ScalarType want = reinterpret_cast<THPDtype*>(dtype_obj)->scalar_type;
  const at::Tensor& out = THPVariable_Unpack(out_obj);
  if (out.scalar_type() != want || (want != at::kFloat && want != at::kBFloat16)) return false;
  if (device >= 0 ? (!out.is_cuda() || out.get_device() != device) : out.is_cuda()) return false;
  if (out.dim() != 2 || out.size(0) != M || out.size(1) != N || !out.is_contiguous())
    return false;
  *ptr = out.data_ptr();
  *code = code_of(want);
  *elt = out.element_size();
  return true;
}

// int4_gemm(a, w_packed, scale, group_size, out, out_dtype, split_k)
//   -> out (allocated here when None), or the status, or -1
PyObject* int4_gemm(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 7) {
    PyErr_Format(PyExc_TypeError, "int4_gemm takes 7 arguments (%zd given)", n);
    return nullptr;
  }
  try {
    if (!THPVariable_Check(args[0])) return PyLong_FromLong(kNotServed);
    const at::Tensor& a = THPVariable_Unpack(args[0]);
    const int a_code = code_of(a.scalar_type());
    if (!a.is_cuda() || (a_code != PK_F16 && a_code != PK_BF16) || a.dim() != 2)
      return PyLong_FromLong(kNotServed);
    const int64_t M = a.size(0), K = a.size(1);
    if (a.stride(1) != 1 || a.stride(0) < K) return PyLong_FromLong(kNotServed);
    const int device = a.get_device();
    Weights w;
    if (!weights(args[1], args[2], args[3], K, a.scalar_type(), device, &w))
      return PyLong_FromLong(kNotServed);
    void* out = nullptr;
    int out_code = 0;
    int64_t elt = 0;
    const bool alloc = args[4] == Py_None;
    if (alloc) {
      if (!THPDtype_Check(args[5])) return PyLong_FromLong(kNotServed);
      const at::ScalarType want = reinterpret_cast<THPDtype*>(args[5])->scalar_type;
      if (want != at::kFloat && want != at::kBFloat16) return PyLong_FromLong(kNotServed);
      out_code = code_of(want);
    } else if (!output(args[4], args[5], M, w.N, device, &out, &out_code, &elt)) {
      return PyLong_FromLong(kNotServed);
    }
    const long split = PyLong_AsLong(args[6]);
    if (split == -1 && PyErr_Occurred()) {
      PyErr_Clear();
      return PyLong_FromLong(kNotServed);
    }
    const uint64_t stream =
        reinterpret_cast<uint64_t>(c10::cuda::getCurrentCUDAStream(device).stream());
    const size_t ws_bytes = workspace_bytes(M, w.N, K, static_cast<int>(split));
    void* ws = nullptr;
    if (ws_bytes > 0) {
      ws = workspace(device, stream, g_tag_splitk, ws_bytes);
      if (ws == nullptr) return PyLong_FromLong(kNotServed);
    }
    at::Tensor y;
    if (alloc) {
      y = at::empty({M, w.N}, at::TensorOptions()
                                  .dtype(out_code == PK_F32 ? at::kFloat : at::kBFloat16)
                                  .device(at::Device(at::kCUDA, static_cast<int8_t>(device))));
      out = y.data_ptr();
    }
    const int st = pk_w4a16_gemm(a.data_ptr(), a_code, a.stride(0),
                                 static_cast<const uint8_t*>(w.wp), w.scales, w.scalar, w.group,
                                 M, w.N, K, out, out_code, w.N, static_cast<int>(split), ws,
                                 ws_bytes, reinterpret_cast<void*>(stream));
    if (st != PK_OK) return PyLong_FromLong(st);
    if (alloc) return THPVariable_Wrap(std::move(y));
    Py_INCREF(args[4]);
    return args[4];
  } catch (...) {
    PyErr_Clear();
    return PyLong_FromLong(kNotServed);
  }
}

// int4_gemm_host(a, w_packed, scale, group_size, out, out_dtype) -> out, or the status, or -1
// (a and out: host tensors; the staging buffers "stage_a" / "stage_y" and the
// workspace are the cached ones of the weights' device and current stream)
PyObject* int4_gemm_host(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 6) {
    PyErr_Format(PyExc_TypeError, "int4_gemm_host takes 6 arguments (%zd given)", n);
    return nullptr;
  }
  try {
    if (!THPVariable_Check(args[0]) || !THPVariable_Check(args[1]))
      return PyLong_FromLong(kNotServed);
    const at::Tensor& a = THPVariable_Unpack(args[0]);
    const int a_code = code_of(a.scalar_type());
    if (a.is_cuda() || (a_code != PK_F16 && a_code != PK_BF16) || a.dim() != 2)
      return PyLong_FromLong(kNotServed);
    const int64_t M = a.size(0), K = a.size(1);
    if (a.stride(1) != 1 || a.stride(0) < K) return PyLong_FromLong(kNotServed);
    const at::Tensor& wp = THPVariable_Unpack(args[1]);
    if (!wp.is_cuda()) return PyLong_FromLong(kNotServed);
    const int device = wp.get_device();
    Weights w;
    if (!weights(args[1], args[2], args[3], K, a.scalar_type(), device, &w))
      return PyLong_FromLong(kNotServed);
    void* out;
    int out_code;
    int64_t elt;
    if (!output(args[4], args[5], M, w.N, -1, &out, &out_code, &elt))
      return PyLong_FromLong(kNotServed);
    const uint64_t stream =
        reinterpret_cast<uint64_t>(c10::cuda::getCurrentCUDAStream(device).stream());
    const size_t ws_bytes = workspace_bytes(M, w.N, K, 0);
    void* ws = nullptr;
    if (ws_bytes > 0) {
      ws = workspace(device, stream, g_tag_splitk, ws_bytes);
      if (ws == nullptr) return PyLong_FromLong(kNotServed);
    }
    void* a_dev = workspace(device, stream, g_tag_a, static_cast<size_t>(M * K * 2));
    void* y_dev = workspace(device, stream, g_tag_y, static_cast<size_t>(M * w.N * elt));
    if (a_dev == nullptr || y_dev == nullptr) return PyLong_FromLong(kNotServed);
    const int st = pk_w4a16_gemm_host(a.data_ptr(), a_code, a.stride(0),
                                      static_cast<const uint8_t*>(w.wp), w.scales, w.scalar,
                                      w.group, M, w.N, K, out, out_code, a_dev, y_dev, ws,
                                      ws_bytes, reinterpret_cast<void*>(stream));
    if (st != PK_OK) return PyLong_FromLong(st);
    Py_INCREF(args[4]);
    return args[4];
  } catch (...) {
    PyErr_Clear();
    return PyLong_FromLong(kNotServed);
  }
}

// bind(workspaces): the dict of cached workspaces the Python path fills.
PyObject* bind(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (n != 1 || !PyDict_Check(args[0])) {
    PyErr_SetString(PyExc_TypeError, "bind takes the workspace dict");
    return nullptr;
  }
  Py_INCREF(args[0]);
  Py_XDECREF(g_workspaces);
  g_workspaces = args[0];
  Py_RETURN_NONE;
}

PyMethodDef kMethods[] = {
    {"int4_gemm", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(int4_gemm)),
     METH_FASTCALL,
     "int4_gemm(a, w_packed, scale, group_size, out, out_dtype, split_k): the output tensor, "
     "the C ABI's status on failure, or -1 when the Python path must take the call."},
    {"int4_gemm_host",
     reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(int4_gemm_host)), METH_FASTCALL,
     "int4_gemm_host(a, w_packed, scale, group_size, out, out_dtype): out, the C ABI's status "
     "on failure, or -1 when the Python path must take the call."},
    {"bind", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(bind)), METH_FASTCALL,
     "bind(workspaces): the workspace dict of pico_kernels_b200._lib."},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_pktorch",
                       "Torch-aware fast-call entry points of libpico_b200.so.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__pktorch() {
  g_tag_splitk = PyUnicode_InternFromString("splitk");
  g_tag_a = PyUnicode_InternFromString("stage_a");
  g_tag_y = PyUnicode_InternFromString("stage_y");
  if (!g_tag_splitk || !g_tag_a || !g_tag_y) return nullptr;
  return PyModule_Create(&kModule);
}
