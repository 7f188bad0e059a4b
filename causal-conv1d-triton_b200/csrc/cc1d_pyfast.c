/*
 * CPython binding of the hot launch entry points of libcausal_conv1d_b200.so (cc1d_fwd,
 * cc1d_bwd_workspace_bytes, cc1d_bwd, cc1d_update), for the package's Python layer.
 *
 * Each function takes the C entry point's arguments positionally, in the order of
 * include/causal_conv1d_b200.h: pointers as Python ints (None for NULL), sizes and codes as
 * ints, and returns the entry point's int result. It parses them with METH_FASTCALL, about
 * 0.3 us per call, where ctypes' per-argument conversion costs 3-5 us: at small shapes those
 * microseconds are a large share of a step. The other entry points are called through ctypes
 * (causal_conv1d_b200/_native.py). Both routes reach the same loaded library.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "causal_conv1d_b200.h"

static int arg_ptr(PyObject* o, void** out) {
  if (o == Py_None) {
    *out = NULL;
    return 0;
  }
  *out = PyLong_AsVoidPtr(o);
  return (*out == NULL && PyErr_Occurred()) ? -1 : 0;
}

static int arg_i64(PyObject* o, int64_t* out) {
  const long long v = PyLong_AsLongLong(o);
  if (v == -1 && PyErr_Occurred()) return -1;
  *out = (int64_t)v;
  return 0;
}

static int arg_int(PyObject* o, int* out) {
  const long v = PyLong_AsLong(o);
  if (v == -1 && PyErr_Occurred()) return -1;
  if (v < INT32_MIN || v > INT32_MAX) {
    PyErr_SetString(PyExc_OverflowError, "int argument out of range");
    return -1;
  }
  *out = (int)v;
  return 0;
}

/* Parses args[0..n) by the format string: 'p' pointer, 'l' int64, 'i' int. */
static int parse(PyObject* const* args, Py_ssize_t n, const char* fmt, void** p, int64_t* l, int* i,
                 const char* name) {
  Py_ssize_t want = 0;
  for (const char* c = fmt; *c; ++c) ++want;
  if (n != want) {
    PyErr_Format(PyExc_TypeError, "%s takes %zd arguments (%zd given)", name, want, n);
    return -1;
  }
  int np = 0, nl = 0, ni = 0;
  for (Py_ssize_t k = 0; k < n; ++k) {
    int rc = 0;
    switch (fmt[k]) {
      case 'p': rc = arg_ptr(args[k], &p[np++]); break;
      case 'l': rc = arg_i64(args[k], &l[nl++]); break;
      default: rc = arg_int(args[k], &i[ni++]); break;
    }
    if (rc != 0) return -1;
  }
  return 0;
}

static PyObject* py_fwd(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  (void)self;
  void* p[8];
  int64_t l[6];
  int i[5];
  /* x sxb sxt weight bias init seq out final B T D W x_dt w_dt b_dt i_dt silu stream */
  if (parse(args, n, "pllpppppplllliiiiip", p, l, i, "cc1d_fwd") != 0) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = cc1d_fwd(p[0], l[0], l[1], p[1], p[2], p[3], (const int32_t*)p[4], p[5], p[6], l[2], l[3], l[4], l[5],
                i[0], i[1], i[2], i[3], i[4], p[7]);
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject* py_bwd_workspace_bytes(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  (void)self;
  void* p[2];
  int64_t l[8];
  int i[1];
  /* x sxb sxt dout syb syt B T D W x_dt */
  if (parse(args, n, "pllplllllli", p, l, i, "cc1d_bwd_workspace_bytes") != 0) return NULL;
  const int64_t r = cc1d_bwd_workspace_bytes(p[0], l[0], l[1], p[1], l[2], l[3], l[4], l[5], l[6], l[7], i[0]);
  return PyLong_FromLongLong((long long)r);
}

static PyObject* py_bwd(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  (void)self;
  void* p[14];
  int64_t l[9];
  int i[5];
  /* x sxb sxt weight bias init seq dout syb syt dfinal dx dweight dbias dinit grad_f32 workspace
     ws_bytes B T D W x_dt w_dt b_dt i_dt silu stream */
  if (parse(args, n, "pllpppppllpppppppllllliiiiip", p, l, i, "cc1d_bwd") != 0) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = cc1d_bwd(p[0], l[0], l[1], p[1], p[2], p[3], (const int32_t*)p[4], p[5], l[2], l[3], p[6], p[7], p[8], p[9],
                p[10], (float*)p[11], p[12], l[4], l[5], l[6], l[7], l[8], i[0], i[1], i[2], i[3], i[4], p[13]);
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject* py_update(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  (void)self;
  void* p[7];
  int64_t l[6];
  int i[5];
  /* x sxb sxt conv_state indices weight bias out B L D W x_dt s_dt w_dt b_dt silu stream */
  if (parse(args, n, "pllppppplllliiiiip", p, l, i, "cc1d_update") != 0) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = cc1d_update(p[0], l[0], l[1], p[1], (const int32_t*)p[2], p[3], p[4], p[5], l[2], l[3], l[4], l[5], i[0],
                   i[1], i[2], i[3], i[4], p[6]);
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyMethodDef methods[] = {
    {"fwd", (PyCFunction)(void (*)(void))py_fwd, METH_FASTCALL, "cc1d_fwd(...) -> int"},
    {"bwd_workspace_bytes", (PyCFunction)(void (*)(void))py_bwd_workspace_bytes, METH_FASTCALL,
     "cc1d_bwd_workspace_bytes(...) -> int"},
    {"bwd", (PyCFunction)(void (*)(void))py_bwd, METH_FASTCALL, "cc1d_bwd(...) -> int"},
    {"update", (PyCFunction)(void (*)(void))py_update, METH_FASTCALL, "cc1d_update(...) -> int"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_cc1d_fast", NULL, -1, methods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__cc1d_fast(void) { return PyModule_Create(&module); }
