/*
 * _titan_pybind: vectorcall (METH_FASTCALL) bindings of the hot launchers of
 * libtitan_b200.so for the Python modules.
 *
 * ctypes converts each argument through its argtypes machinery (~0.15 us per
 * argument, ~3.7 us for the 21-argument MLA launcher), which made an eager
 * decode call host-bound.  These wrappers parse Python ints / floats straight
 * into the C types of include/titan_b200.h and call the library.  They do not
 * link the library: `bind` receives the addresses of the entry points of the
 * copy ctypes loaded (titan_native.load()), so both paths call the same code.
 *
 * Argument kinds: 'p' pointer (Python int or None), 'i' int64, 'f' float.
 * Every argument is converted before the call; a conversion error raises
 * without launching anything.  The launcher runs with the GIL released (as
 * under ctypes), so threads driving different streams or GPUs overlap; each
 * wrapper returns the launcher's status.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>
#include <string.h>

#include "../../include/titan_b200.h"

static __typeof__(&titan_mla_sparse_attention) p_mla;
static __typeof__(&titan_mla_sparse_attention_sem) p_mla_sem;
static __typeof__(&titan_mla_sparse_attention_paged) p_mla_paged;
static __typeof__(&titan_copy_ex) p_copy;
static __typeof__(&titan_store_int8) p_store_int8;
static __typeof__(&titan_moe_align_small) p_moe_align;
static __typeof__(&titan_convert_req_index_to_global) p_convert;
static __typeof__(&titan_device_pointer) p_device_pointer;

#define MAX_ARGS 32

/* Converts a[0..n) by `kinds` into iv (ints, pointers) and fv (floats).
 * Returns 0, or -1 with a Python exception set. */
static int parse(const char *name, PyObject *const *a, Py_ssize_t n, const char *kinds, int64_t *iv, double *fv) {
  Py_ssize_t want = (Py_ssize_t)strlen(kinds);
  if (n != want) {
    PyErr_Format(PyExc_TypeError, "%s: expected %zd arguments, got %zd", name, want, n);
    return -1;
  }
  for (Py_ssize_t k = 0; k < n; ++k) {
    PyObject *o = a[k];
    switch (kinds[k]) {
      case 'p':
        iv[k] = o == Py_None ? 0 : (int64_t)(uintptr_t)PyLong_AsVoidPtr(o);
        break;
      case 'i':
        iv[k] = PyLong_AsLongLong(o);
        break;
      case 'f':
        fv[k] = PyFloat_AsDouble(o);
        break;
      default:
        PyErr_SetString(PyExc_SystemError, "bad argument kind");
        return -1;
    }
    if (PyErr_Occurred()) {
      PyErr_Format(PyExc_TypeError, "%s: argument %zd has the wrong type", name, k);
      return -1;
    }
  }
  return 0;
}

#define P(k) ((void *)(uintptr_t)iv[k])
#define I(k) (iv[k])
#define F(k) ((float)fv[k])
#define UNBOUND(fn)                                                        \
  if (fn == NULL) {                                                        \
    PyErr_SetString(PyExc_RuntimeError, "_titan_pybind: bind() not called"); \
    return NULL;                                                           \
  }

static PyObject *py_mla(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_mla);
  if (parse("mla", a, n, "piipiipiipiiiifipip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_mla(P(0), I(1), I(2), P(3), I(4), I(5), (const int32_t *)P(6), I(7), I(8), P(9), I(10), I(11), I(12),
                   I(13), F(14), I(15), P(16), I(17), (titan_stream_t)P(18));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_mla_sem(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_mla_sem);
  if (parse("mla_sem", a, n, "piipiipiipiiiifipipip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_mla_sem(P(0), I(1), I(2), P(3), I(4), I(5), (const int32_t *)P(6), I(7), I(8), P(9), I(10), I(11),
                       I(12), I(13), F(14), I(15), P(16), I(17), (int32_t *)P(18), I(19), (titan_stream_t)P(20));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_mla_paged(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_mla_paged);
  if (parse("mla_paged", a, n, "piipiipiipipiiiiipiiiifipipip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_mla_paged(P(0), I(1), I(2), P(3), I(4), I(5), (const int32_t *)P(6), I(7), I(8), (const int32_t *)P(9),
                         I(10), (const int32_t *)P(11), I(12), I(13), I(14), I(15), I(16), P(17), I(18), I(19), I(20),
                         I(21), F(22), I(23), P(24), I(25), (int32_t *)P(26), I(27), (titan_stream_t)P(28));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_copy(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_copy);
  if (parse("copy", a, n, "ppiip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_copy(P(0), P(1), I(2), (int)I(3), (titan_stream_t)P(4));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_store_int8(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_store_int8);
  if (parse("store_int8", a, n, "pipiiiipiip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_store_int8(P(0), I(1), P(2), I(3), I(4), I(5), I(6), P(7), (int)I(8), I(9), (titan_stream_t)P(10));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_moe_align(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_moe_align);
  if (parse("moe_align", a, n, "piipppip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_moe_align(P(0), (int)I(1), I(2), (int32_t *)P(3), (int32_t *)P(4), (int32_t *)P(5),
                                       (int)I(6), (titan_stream_t)P(7));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject *py_convert(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_convert);
  if (parse("convert", a, n, "pipiiipiipiiiip", iv, fv)) return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_convert((const int32_t *)P(0), I(1), (const int32_t *)P(2), I(3), I(4), I(5),
                                     (const int32_t *)P(6), I(7), I(8), (int32_t *)P(9), I(10), I(11), I(12), I(13),
                                     (titan_stream_t)P(14));
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

/* device_pointer(ptr) -> (status, device address): titan_device_pointer. */
static PyObject *py_device_pointer(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  UNBOUND(p_device_pointer);
  if (parse("device_pointer", a, n, "p", iv, fv)) return NULL;
  void *dev = NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
    rc = p_device_pointer(P(0), &dev);
  Py_END_ALLOW_THREADS
  return Py_BuildValue("(iK)", rc, (unsigned long long)(uintptr_t)dev);
}

/* bind(mla, mla_sem, mla_paged, copy, store_int8, moe_align, convert,
 * device_pointer): entry point addresses (Python ints) of the loaded library. */
static PyObject *py_bind(PyObject *self, PyObject *const *a, Py_ssize_t n) {
  int64_t iv[MAX_ARGS];
  double fv[MAX_ARGS];
  if (parse("bind", a, n, "pppppppp", iv, fv)) return NULL;
  for (int k = 0; k < 8; ++k)
    if (iv[k] == 0) {
      PyErr_SetString(PyExc_ValueError, "bind: null entry point");
      return NULL;
    }
  p_mla = (__typeof__(p_mla))P(0);
  p_mla_sem = (__typeof__(p_mla_sem))P(1);
  p_mla_paged = (__typeof__(p_mla_paged))P(2);
  p_copy = (__typeof__(p_copy))P(3);
  p_store_int8 = (__typeof__(p_store_int8))P(4);
  p_moe_align = (__typeof__(p_moe_align))P(5);
  p_convert = (__typeof__(p_convert))P(6);
  p_device_pointer = (__typeof__(p_device_pointer))P(7);
  Py_RETURN_NONE;
}

static PyMethodDef methods[] = {
    {"bind", (PyCFunction)(void (*)(void))py_bind, METH_FASTCALL, "bind(entry point addresses)"},
    {"mla", (PyCFunction)(void (*)(void))py_mla, METH_FASTCALL, "titan_mla_sparse_attention"},
    {"mla_sem", (PyCFunction)(void (*)(void))py_mla_sem, METH_FASTCALL, "titan_mla_sparse_attention_sem"},
    {"mla_paged", (PyCFunction)(void (*)(void))py_mla_paged, METH_FASTCALL, "titan_mla_sparse_attention_paged"},
    {"copy", (PyCFunction)(void (*)(void))py_copy, METH_FASTCALL, "titan_copy_ex"},
    {"store_int8", (PyCFunction)(void (*)(void))py_store_int8, METH_FASTCALL, "titan_store_int8"},
    {"moe_align", (PyCFunction)(void (*)(void))py_moe_align, METH_FASTCALL, "titan_moe_align_small"},
    {"convert", (PyCFunction)(void (*)(void))py_convert, METH_FASTCALL, "titan_convert_req_index_to_global"},
    {"device_pointer", (PyCFunction)(void (*)(void))py_device_pointer, METH_FASTCALL, "titan_device_pointer"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_titan_pybind",
                                    "Fast-call bindings of libtitan_b200.so", -1, methods};

PyMODINIT_FUNC PyInit__titan_pybind(void) { return PyModule_Create(&module); }
