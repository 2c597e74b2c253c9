/* CPython binding of one C-ABI entry, avo_b200_attn_fwd_ws, for the per-call path of
 * attention().  Small problems are bound by host time per call (the B1 H4 S512 case of the
 * scorer runs ~15 us of GPU work per launch); a ctypes call with fifteen arguments costs
 * ~2 us of argument conversion, a METH_FASTCALL function a fraction of that.  The function
 * address comes from the library ctypes already loaded (bind), so this module links to
 * nothing but Python and calls exactly the same native entry.
 *
 * fwd_ws(q, k, v, o, lse_or_None, batch, heads, seq, head_dim, causal, scale,
 *        workspace, workspace_bytes, status, stream) -> int status code
 * Pointer arguments are integers (tensor.data_ptr()), lse may be None; the return value is
 * the entry's own status code. */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stddef.h>

typedef int (*fwd_ws_fn)(const void*, const void*, const void*, void*, float*, int, int, int, int, int, float,
                         void*, size_t, int*, void*);

static fwd_ws_fn g_fwd_ws = NULL;

static PyObject* bind(PyObject* self, PyObject* addr) {
  (void)self;
  void* fn = PyLong_AsVoidPtr(addr);
  if (fn == NULL) {
    if (!PyErr_Occurred()) PyErr_SetString(PyExc_ValueError, "null function address");
    return NULL;
  }
  g_fwd_ws = (fwd_ws_fn)fn;
  Py_RETURN_NONE;
}

static int as_ptr(PyObject* obj, void** out) {
  if (obj == Py_None) {
    *out = NULL;
    return 0;
  }
  *out = PyLong_AsVoidPtr(obj);
  return (*out == NULL && PyErr_Occurred()) ? -1 : 0;
}

static int as_int(PyObject* obj, int* out) {
  long v = PyLong_AsLong(obj);
  if (v == -1 && PyErr_Occurred()) return -1;
  if (v < -2147483647L - 1L || v > 2147483647L) {
    PyErr_SetString(PyExc_OverflowError, "argument out of int range");
    return -1;
  }
  *out = (int)v;
  return 0;
}

static PyObject* fwd_ws(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 15) {
    PyErr_SetString(PyExc_TypeError, "fwd_ws takes 15 arguments");
    return NULL;
  }
  if (g_fwd_ws == NULL) {
    PyErr_SetString(PyExc_RuntimeError, "fwd_ws is not bound to the library yet");
    return NULL;
  }
  void *q, *k, *v, *o, *lse, *ws, *status, *stream;
  int batch, heads, seq, head_dim, causal;
  if (as_ptr(args[0], &q) || as_ptr(args[1], &k) || as_ptr(args[2], &v) || as_ptr(args[3], &o) ||
      as_ptr(args[4], &lse) || as_int(args[5], &batch) || as_int(args[6], &heads) || as_int(args[7], &seq) ||
      as_int(args[8], &head_dim) || as_int(args[9], &causal))
    return NULL;
  const double scale = PyFloat_AsDouble(args[10]);
  if (scale == -1.0 && PyErr_Occurred()) return NULL;
  if (as_ptr(args[11], &ws)) return NULL;
  const size_t ws_bytes = PyLong_AsSize_t(args[12]);
  if (ws_bytes == (size_t)-1 && PyErr_Occurred()) return NULL;
  if (as_ptr(args[13], &status) || as_ptr(args[14], &stream)) return NULL;
  const int rc = g_fwd_ws(q, k, v, o, (float*)lse, batch, heads, seq, head_dim, causal, (float)scale, ws, ws_bytes,
                          (int*)status, stream);
  return PyLong_FromLong(rc);
}

static PyMethodDef methods[] = {
    {"bind", (PyCFunction)bind, METH_O, "bind(address of avo_b200_attn_fwd_ws)"},
    {"fwd_ws", (PyCFunction)(void (*)(void))fwd_ws, METH_FASTCALL, "avo_b200_attn_fwd_ws through the bound address"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_avo_b200_fast", NULL, -1, methods,
                                    NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__avo_b200_fast(void) { return PyModule_Create(&module); }
