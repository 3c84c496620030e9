/* Host-side step packing for ModelRunner: needle's per-sequence block tables
 * (Python lists of ints, needle/backend/scheduler.py:127-130 hands a fresh
 * list per sequence every step) written straight into the padded int32
 * [rows, width] block table at a raw address -- the pinned staging buffer
 * that is copied to the device in one transfer.  One pass in C over the
 * list items replaces a Python-level conversion of every block id. */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

static PyObject* fill_block_table(PyObject* self, PyObject* args) {
  PyObject* rows;
  unsigned long long addr;
  Py_ssize_t cap;
  int width, pad;
  (void)self;
  if (!PyArg_ParseTuple(args, "OKnii", &rows, &addr, &cap, &width, &pad)) return NULL;
  PyObject* seq = PySequence_Fast(rows, "rows must be a sequence of sequences");
  if (!seq) return NULL;
  const Py_ssize_t n_rows = PySequence_Fast_GET_SIZE(seq);
  if (width <= 0 || addr == 0 || cap < 0 ||
      (unsigned long long)n_rows * (unsigned long long)width * 4ull > (unsigned long long)cap) {
    Py_DECREF(seq);
    PyErr_SetString(PyExc_ValueError, "block table does not fit the destination buffer");
    return NULL;
  }
  int32_t* out = (int32_t*)(uintptr_t)addr;
  for (Py_ssize_t i = 0; i < n_rows; ++i) {
    PyObject* row = PySequence_Fast(PySequence_Fast_GET_ITEM(seq, i), "each row must be a sequence");
    if (!row) {
      Py_DECREF(seq);
      return NULL;
    }
    const Py_ssize_t n = PySequence_Fast_GET_SIZE(row);
    if (n > width) {
      Py_DECREF(row);
      Py_DECREF(seq);
      PyErr_Format(PyExc_ValueError, "row %zd has %zd blocks, more than the width %d", i, n, width);
      return NULL;
    }
    PyObject** items = PySequence_Fast_ITEMS(row);
    int32_t* o = out + (size_t)i * (size_t)width;
    for (Py_ssize_t j = 0; j < n; ++j) {
      const long v = PyLong_AsLong(items[j]);
      if ((v == -1 && PyErr_Occurred()) || v < INT32_MIN || v > INT32_MAX) {
        Py_DECREF(row);
        Py_DECREF(seq);
        if (!PyErr_Occurred()) PyErr_SetString(PyExc_OverflowError, "block id out of int32 range");
        return NULL;
      }
      o[j] = (int32_t)v;
    }
    for (Py_ssize_t j = n; j < width; ++j) o[j] = pad;
    Py_DECREF(row);
  }
  Py_DECREF(seq);
  Py_RETURN_NONE;
}

static PyMethodDef methods[] = {
    {"fill_block_table", fill_block_table, METH_VARARGS,
     "fill_block_table(rows, address, capacity_bytes, width, pad): write rows (sequences of "
     "ints) as a padded int32 [len(rows), width] table at address."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_steppack",
                                    "Host-side step packing for ModelRunner.", -1, methods};

PyMODINIT_FUNC PyInit__steppack(void) { return PyModule_Create(&module); }
