// libkorith_b200.so: the C ABI of korith.h over the framework's Python runtime.
//
// Every entry point takes the library mutex and the Python GIL, then calls the
// matching method of axropus_deploy_b200.capi (one CSession: model, paged KV cache,
// kernels). Loaded into a Python process (ctypes, cffi) the library uses that process's
// interpreter; loaded by a plain C/C++ program it initialises one on the first call and
// puts the framework and its site-packages (recorded at build time) on sys.path.
// Errors are returned as false / -1 with the message in korith_last_error().
#include "korith.h"

#include <Python.h>
#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

#ifndef AXR_SITE_PACKAGES
#define AXR_SITE_PACKAGES ""
#endif

namespace {

std::mutex g_mu;
std::string g_err;
PyObject* g_mod = nullptr;  // axropus_deploy_b200.capi (owned)

struct Gil {
  PyGILState_STATE s;
  Gil() : s(PyGILState_Ensure()) {}
  ~Gil() { PyGILState_Release(s); }
};

std::string repo_root() {
  Dl_info info{};
  if (dladdr(reinterpret_cast<void*>(&repo_root), &info) == 0 || info.dli_fname == nullptr) return "";
  std::string p(info.dli_fname);  // <root>/axropus_deploy_b200/libkorith_b200.so
  for (int i = 0; i < 2; ++i) {
    const auto k = p.find_last_of('/');
    if (k == std::string::npos) return ".";
    p = p.substr(0, k);
  }
  return p;
}

void take_python_error(const char* where) {
  PyObject *type = nullptr, *value = nullptr, *tb = nullptr;
  PyErr_Fetch(&type, &value, &tb);
  std::string msg = where;
  if (value != nullptr) {
    PyObject* s = PyObject_Str(value);
    if (s != nullptr) {
      const char* c = PyUnicode_AsUTF8(s);
      if (c != nullptr) msg += std::string(": ") + c;
      Py_DECREF(s);
    }
  }
  Py_XDECREF(type);
  Py_XDECREF(value);
  Py_XDECREF(tb);
  PyErr_Clear();
  g_err = msg;
}

// Caller holds g_mu. Leaves the GIL released.
bool ensure_runtime() {
  if (!Py_IsInitialized()) {
    Py_InitializeEx(0);
    PyEval_SaveThread();  // every call below takes the GIL through PyGILState_Ensure
  }
  if (g_mod != nullptr) return true;
  Gil gil;
  PyObject* path = PySys_GetObject("path");  // borrowed
  if (path != nullptr) {
    const std::string root = repo_root();
    for (const std::string& d : {std::string(AXR_SITE_PACKAGES), root}) {
      if (d.empty()) continue;
      PyObject* s = PyUnicode_FromString(d.c_str());
      if (PySequence_Contains(path, s) == 0) PyList_Insert(path, 0, s);
      Py_DECREF(s);
    }
  }
  g_mod = PyImport_ImportModule("axropus_deploy_b200.capi");
  if (g_mod == nullptr) {
    take_python_error("import axropus_deploy_b200.capi");
    return false;
  }
  return true;
}

// New reference to capi.<fn>(*args) (args stolen), nullptr on error. Caller holds the GIL.
PyObject* call_module(const char* fn, PyObject* args) {
  PyObject* f = PyObject_GetAttrString(g_mod, fn);
  if (f == nullptr) {
    Py_XDECREF(args);
    take_python_error(fn);
    return nullptr;
  }
  PyObject* r = PyObject_CallObject(f, args);
  Py_DECREF(f);
  Py_XDECREF(args);
  if (r == nullptr) take_python_error(fn);
  return r;
}

// New reference to capi.session().<meth>(*args) (args stolen). Caller holds the GIL.
PyObject* call_session(const char* meth, PyObject* args) {
  PyObject* s = call_module("session", nullptr);
  if (s == nullptr) {
    Py_XDECREF(args);
    return nullptr;
  }
  PyObject* m = PyObject_GetAttrString(s, meth);
  Py_DECREF(s);
  if (m == nullptr) {
    Py_XDECREF(args);
    take_python_error(meth);
    return nullptr;
  }
  PyObject* r = PyObject_CallObject(m, args);
  Py_DECREF(m);
  Py_XDECREF(args);
  if (r == nullptr) take_python_error(meth);
  return r;
}

PyObject* int_list(const int32_t* v, int32_t n) {
  PyObject* l = PyList_New(n);
  for (int32_t i = 0; i < n; ++i) PyList_SET_ITEM(l, i, PyLong_FromLong(v[i]));
  return l;
}

bool truthy(PyObject* r) {
  if (r == nullptr) return false;
  const bool ok = PyObject_IsTrue(r) == 1;
  Py_DECREF(r);
  return ok;
}

long as_long(PyObject* r, long fallback) {
  if (r == nullptr) return fallback;
  const long v = PyLong_AsLong(r);
  Py_DECREF(r);
  if (PyErr_Occurred()) {
    take_python_error("result");
    return fallback;
  }
  return v;
}

bool init_common(const char* model_path, int n_ctx) {
  if (model_path == nullptr || model_path[0] == '\0' || n_ctx <= 0) {
    g_err = "model_path and a positive n_ctx are required";
    return false;
  }
  if (!ensure_runtime()) return false;
  Gil gil;
  return truthy(call_module("init", Py_BuildValue("(si)", model_path, n_ctx)));
}

}  // namespace

extern "C" {

const char* korith_last_error(void) { return g_err.c_str(); }

// ------------------------------------------------------------------ korith_*
bool korith_init(const char* model_path, int n_ctx) {
  std::lock_guard<std::mutex> lk(g_mu);
  return init_common(model_path, n_ctx);
}

int korith_tokenize(const char* prompt) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (prompt == nullptr || !ensure_runtime()) return -1;
  Gil gil;
  return static_cast<int>(as_long(call_session("tokenize", Py_BuildValue("(s)", prompt)), -1));
}

int korith_step(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!ensure_runtime()) return -1;
  Gil gil;
  return static_cast<int>(as_long(call_session("step", nullptr), -1));
}

void korith_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_mod == nullptr) return;
  Gil gil;
  PyObject* r = call_module("shutdown", nullptr);
  Py_XDECREF(r);
}

// ------------------------------------------------------------------ korith_engine_*
bool korith_engine_init_model(const struct korith_engine_params* params) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (params == nullptr) return false;
  return init_common(params->model_path, params->n_ctx);
}

bool korith_engine_prefill(const int32_t* tokens, int32_t n_tokens) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (tokens == nullptr || n_tokens <= 0 || !ensure_runtime()) return false;
  Gil gil;
  return truthy(call_session("prefill", Py_BuildValue("(N)", int_list(tokens, n_tokens))));
}

bool korith_engine_decode_step(int32_t* token_out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (token_out == nullptr || !ensure_runtime()) return false;
  Gil gil;
  const long t = as_long(call_session("step", nullptr), -1);
  if (t < 0) return false;
  *token_out = static_cast<int32_t>(t);
  return true;
}

bool korith_engine_get_logits(float* out_logits, int32_t n_vocab) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (out_logits == nullptr || n_vocab <= 0 || !ensure_runtime()) return false;
  Gil gil;
  PyObject* a = call_session("get_logits", nullptr);
  if (a == nullptr) return false;
  bool ok = false;
  if (a != Py_None) {
    Py_buffer view;
    if (PyObject_GetBuffer(a, &view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) == 0) {
      const Py_ssize_t n = view.len / static_cast<Py_ssize_t>(sizeof(float));
      if (view.itemsize == sizeof(float) && n_vocab <= n) {
        std::memcpy(out_logits, view.buf, static_cast<size_t>(n_vocab) * sizeof(float));
        ok = true;
      } else {
        g_err = "get_logits: n_vocab larger than the model's vocabulary";
      }
      PyBuffer_Release(&view);
    } else {
      take_python_error("get_logits buffer");
    }
  } else {
    g_err = "get_logits: no logits yet (prefill first)";
  }
  Py_DECREF(a);
  return ok;
}

bool korith_engine_apply_kv_replay(const uint8_t* blob, size_t n_bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (blob == nullptr || n_bytes == 0 || !ensure_runtime()) return false;
  Gil gil;
  PyObject* b = PyBytes_FromStringAndSize(reinterpret_cast<const char*>(blob), static_cast<Py_ssize_t>(n_bytes));
  return truthy(call_session("apply_kv_replay", Py_BuildValue("(N)", b)));
}

bool korith_engine_export_snapshot(const char* path) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (path == nullptr || path[0] == '\0' || !ensure_runtime()) return false;
  Gil gil;
  return truthy(call_session("export_snapshot", Py_BuildValue("(s)", path)));
}

bool korith_engine_import_snapshot(const char* path) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (path == nullptr || path[0] == '\0' || !ensure_runtime()) return false;
  Gil gil;
  return truthy(call_session("import_snapshot", Py_BuildValue("(s)", path)));
}

bool korith_engine_verify_tokens(const int32_t* proposed_tokens, int32_t n_tokens, int32_t* accepted_prefix) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (proposed_tokens == nullptr || accepted_prefix == nullptr || n_tokens < 0 || !ensure_runtime()) return false;
  if (n_tokens == 0) {
    *accepted_prefix = 0;
    return true;
  }
  Gil gil;
  const long a = as_long(call_session("verify", Py_BuildValue("(N)", int_list(proposed_tokens, n_tokens))), -1);
  if (a < 0) return false;
  *accepted_prefix = static_cast<int32_t>(a);
  return true;
}

void korith_engine_get_metrics(struct korith_engine_metrics* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (out == nullptr) return;
  std::memset(out, 0, sizeof(*out));
  if (g_mod == nullptr) return;
  Gil gil;
  PyObject* d = call_session("metrics", nullptr);
  if (d == nullptr) return;
  auto f = [&](const char* k) {
    PyObject* v = PyDict_GetItemString(d, k);  // borrowed
    return v ? PyFloat_AsDouble(v) : 0.0;
  };
  out->prefill_ms = f("prefill_ms");
  out->decode_ms = f("decode_ms");
  out->total_ms = f("total_ms");
  out->restore_ms = f("restore_ms");
  out->verify_ms = f("verify_ms");
  out->draft_ms = f("draft_ms");
  out->tokens_out = static_cast<int32_t>(f("tokens_out"));
  out->accepted_tokens = static_cast<int32_t>(f("accepted_tokens"));
  out->rejected_tokens = static_cast<int32_t>(f("rejected_tokens"));
  Py_DECREF(d);
  PyErr_Clear();
}

void korith_engine_shutdown(void) { korith_shutdown(); }

bool korith_engine_cuda_probe(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!ensure_runtime()) return false;
  Gil gil;
  return truthy(call_module("cuda_probe", nullptr));
}

}  // extern "C"
