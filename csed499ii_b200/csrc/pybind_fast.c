/*
 * CPython binding of the GEMM entry points for the Python operator
 * (csed499ii_b200.mul_2_4 and friends): the same C ABI as the ctypes table
 * in _ext.py, called with plain integers.  The reference reaches its kernel
 * through a compiled pybind11 extension (marlin_cuda.mul_2_4,
 * kernel_experiments/sparse_marlin/src/marlin/marlin_cuda.cpp:66-99); with
 * ctypes the argument conversion alone cost ~2.5 us per call, as much as a
 * quarter of a decode GEMM, which made an eager decode step host-bound.
 *
 * mul(A, B, meta, C, s, prob_m, prob_n, prob_k, workspace, groupsize, dev,
 *     stream, thread_k, thread_m, sms, max_par, meta_bits, bias, activation)
 * -> int status.  Pointers and the stream are integers (0 = none).
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/sm100_marlin.h"

static PyObject* fast_mul(PyObject* self, PyObject* args) {
  unsigned long long a, b, meta, c, s, ws, stream, bias;
  int prob_m, prob_n, prob_k, groupsize, dev, thread_k, thread_m, sms, max_par, meta_bits, act;
  (void)self;
  if (!PyArg_ParseTuple(args, "KKKKKiiiKiiKiiiiiKi", &a, &b, &meta, &c, &s, &prob_m, &prob_n,
                        &prob_k, &ws, &groupsize, &dev, &stream, &thread_k, &thread_m, &sms,
                        &max_par, &meta_bits, &bias, &act))
    return NULL;
  int rc;
  Py_BEGIN_ALLOW_THREADS
  if (bias == 0 && act == 0) {
    if (meta_bits == 4)
      rc = sm100_marlin_mul_2_4((const void*)a, (const void*)b, (const void*)meta, (void*)c,
                                (const void*)s, prob_m, prob_n, prob_k, (void*)ws, groupsize, dev,
                                (void*)stream, thread_k, thread_m, sms, max_par);
    else
      rc = sm100_marlin_mul_2_4_meta3((const void*)a, (const void*)b, (const void*)meta, (void*)c,
                                      (const void*)s, prob_m, prob_n, prob_k, (void*)ws, groupsize,
                                      dev, (void*)stream, thread_k, thread_m, sms, max_par);
  } else {
    rc = sm100_marlin_mul_2_4_epilogue((const void*)a, (const void*)b, (const void*)meta, (void*)c,
                                       (const void*)s, prob_m, prob_n, prob_k, (void*)ws, groupsize,
                                       dev, (void*)stream, thread_k, thread_m, sms, max_par,
                                       meta_bits, (const void*)bias, act);
  }
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyMethodDef kMethods[] = {
    {"mul", fast_mul, METH_VARARGS, "2:4 W4A16 GEMM through the C ABI (status code)."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_fastcall", NULL, -1, kMethods,
                                     NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__fastcall(void) { return PyModule_Create(&kModule); }
