// _srs_host: host-side helper of the fused optimizer steps (a CPython module).
//
// signature(params, state, names) -> bytes describes every tensor a step of a
// parameter group touches: for each parameter, the parameter, its gradient,
// its state dict and the named state tensors, each as object identity plus
// (for tensors) data address, element count, dtype, contiguity, device and
// shape.  Two equal signatures mean the same objects with the same storage
// and layout, so the row tables and checks of the earlier step still hold.
// It replaces a per-tensor Python loop (~1 us per parameter) with one call.
//
// A tensor without strided storage (sparse, meta) makes the signature None:
// the caller then takes the full preparation, which raises the proper error.
#include <Python.h>

#include <cstdint>
#include <unordered_map>
#include <vector>

#include <torch/csrc/autograd/python_variable.h>

namespace {

// false: not describable (the signature is then None).
bool describe(PyObject* obj, std::vector<int64_t>& out) {
  out.push_back(static_cast<int64_t>(reinterpret_cast<intptr_t>(obj)));
  if (obj == nullptr || obj == Py_None || !THPVariable_Check(obj)) return true;
  const at::Tensor& t = THPVariable_Unpack(obj);
  if (!t.defined() || t.layout() != c10::kStrided || !t.has_storage()) return false;
  out.push_back(static_cast<int64_t>(reinterpret_cast<intptr_t>(t.data_ptr())));
  out.push_back(t.numel());
  out.push_back(static_cast<int64_t>(t.scalar_type()));
  out.push_back(t.is_contiguous() ? 1 : 0);
  out.push_back(static_cast<int64_t>(t.device().type()) * 1024 + t.device().index());
  out.push_back(t.dim());
  for (const int64_t s : t.sizes()) out.push_back(s);
  return true;
}

PyObject* signature(PyObject*, PyObject* args) {
  PyObject *params, *state, *names;
  if (!PyArg_ParseTuple(args, "OO!O!", &params, &PyDict_Type, &state, &PyTuple_Type, &names))
    return nullptr;
  PyObject* seq = PySequence_Fast(params, "params must be a sequence");
  if (seq == nullptr) return nullptr;
  static PyObject* grad_name = PyUnicode_InternFromString("grad");
  // The state dict by key identity, read once: tensors hash by id, so this is
  // the dict's own lookup without calling the tensors' Python __hash__.
  std::unordered_map<PyObject*, PyObject*> states;
  states.reserve(static_cast<size_t>(PyDict_GET_SIZE(state)) * 2);
  {
    Py_ssize_t pos = 0;
    PyObject *key, *value;
    while (PyDict_Next(state, &pos, &key, &value)) states.emplace(key, value);
  }
  std::vector<int64_t> out;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  out.reserve(static_cast<size_t>(n) * 24 + 1);
  out.push_back(n);
  bool ok = true;
  try {
    for (Py_ssize_t i = 0; ok && i < n; ++i) {
      PyObject* p = PySequence_Fast_GET_ITEM(seq, i);
      ok = describe(p, out);
      PyObject* g = PyObject_GetAttr(p, grad_name);
      if (g == nullptr) {
        Py_DECREF(seq);
        return nullptr;
      }
      ok = ok && describe(g, out);
      Py_DECREF(g);
      const auto found = states.find(p);  // no default insertion
      PyObject* st = found == states.end() ? nullptr : found->second;
      out.push_back(static_cast<int64_t>(reinterpret_cast<intptr_t>(st)));
      if (st == nullptr || !PyDict_Check(st)) continue;
      for (Py_ssize_t k = 0; ok && k < PyTuple_GET_SIZE(names); ++k) {
        PyObject* s = PyDict_GetItemWithError(st, PyTuple_GET_ITEM(names, k));
        if (s == nullptr && PyErr_Occurred()) {
          Py_DECREF(seq);
          return nullptr;
        }
        ok = describe(s, out);
      }
    }
  } catch (const std::exception&) {
    ok = false;
  }
  Py_DECREF(seq);
  if (!ok) Py_RETURN_NONE;
  return PyBytes_FromStringAndSize(reinterpret_cast<const char*>(out.data()),
                                   static_cast<Py_ssize_t>(out.size() * sizeof(int64_t)));
}

PyMethodDef kMethods[] = {
    {"signature", signature, METH_VARARGS,
     "signature(params, state, names) -> bytes or None: identity, storage and layout of "
     "every parameter, gradient, state dict and named state tensor of a group."},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_srs_host",
                       "Host-side helpers of the sm_100a optimizer steps.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__srs_host(void) { return PyModule_Create(&kModule); }
