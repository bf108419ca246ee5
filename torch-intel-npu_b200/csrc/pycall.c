/* _lowbit_call: a CPython fast path for the per-call C-ABI entry point lb_linear_path.
 *
 * ctypes converts each of lb_linear_path's 17 arguments through its argtypes on every call
 * (~3 us on a host core), which at decode sizes costs as much as the GPU work.  This module
 * takes the same plain integers (pointers as Python ints, None for a null pointer) and calls
 * the entry point directly.  It does not link against liblowbit: lowbit_runtime hands it the
 * address of lb_linear_path from the library it loaded (bind()), so both paths always call
 * the same library.  No torch types cross this boundary.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stddef.h>
#include <stdint.h>

typedef int (*linear_path_fn)(int, int, int, int, int, int, const void *, const void *, const void *, const void *,
                              const void *, int, const void *, void *, void *, size_t, void *);

static linear_path_fn g_linear_path = NULL;

static PyObject *bind(PyObject *self, PyObject *arg) {
  (void)self;
  const unsigned long long a = PyLong_AsUnsignedLongLong(arg);
  if (PyErr_Occurred()) return NULL;
  g_linear_path = (linear_path_fn)(uintptr_t)a;
  Py_RETURN_NONE;
}

static int as_int(PyObject *o, int *out) {
  const long v = PyLong_AsLong(o);
  if (v == -1 && PyErr_Occurred()) return 0;
  if (v < INT32_MIN || v > INT32_MAX) {
    PyErr_SetString(PyExc_OverflowError, "argument does not fit a C int");
    return 0;
  }
  *out = (int)v;
  return 1;
}

static int as_ptr(PyObject *o, void **out) {
  if (o == Py_None) {
    *out = NULL;
    return 1;
  }
  const unsigned long long v = PyLong_AsUnsignedLongLong(o);
  if (v == (unsigned long long)-1 && PyErr_Occurred()) return 0;
  *out = (void *)(uintptr_t)v;
  return 1;
}

/* linear_path(path, fmt, group, m, n, k, x, codes, scales, down, up, rank, bias, y, ws, ws_bytes, stream)
 * -> lb_status, the same arguments in the same order as lb_linear_path in include/lowbit.h. */
static PyObject *linear_path(PyObject *self, PyObject *const *args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 17) {
    PyErr_SetString(PyExc_TypeError, "linear_path takes 17 arguments");
    return NULL;
  }
  if (!g_linear_path) {
    PyErr_SetString(PyExc_RuntimeError, "linear_path called before bind()");
    return NULL;
  }
  int iv[7];
  void *pv[10];
  static const int int_slots[7] = {0, 1, 2, 3, 4, 5, 11};
  static const int ptr_slots[10] = {6, 7, 8, 9, 10, 12, 13, 14, 15, 16};
  for (int i = 0; i < 7; ++i)
    if (!as_int(args[int_slots[i]], &iv[i])) return NULL;
  for (int i = 0; i < 10; ++i)
    if (!as_ptr(args[ptr_slots[i]], &pv[i])) return NULL;
  const int status = g_linear_path(iv[0], iv[1], iv[2], iv[3], iv[4], iv[5], pv[0], pv[1], pv[2], pv[3], pv[4], iv[6],
                                   pv[5], pv[6], pv[7], (size_t)(uintptr_t)pv[8], pv[9]);
  return PyLong_FromLong(status);
}

static PyMethodDef methods[] = {
    {"bind", (PyCFunction)bind, METH_O, "bind(address of lb_linear_path)"},
    {"linear_path", (PyCFunction)(void (*)(void))linear_path, METH_FASTCALL, "lb_linear_path with plain integers"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_lowbit_call", NULL, -1, methods};

PyMODINIT_FUNC PyInit__lowbit_call(void) { return PyModule_Create(&module); }
