// Host side of ActorInferenceServer.service() for wave requests, in C++
// (CPython API): packs the wire objects of one service() call into the flat
// arrays a step is planned from, and builds the per-request response rows
// from the step's results.  The Python-level loops these replace cost
// ~2-3 us per row (src/imba_chess/eval/actor_server.py:806-925 does the same
// work with per-row tensor builds).
//
// pack_wave_rows(requests, out_piece, out_side) ->
//     (rows, legal_off bytes, legal_ids bytes, node_ids bytes, parent_ids bytes)
//   requests: sequence of objects with .rows, each row with .node_id,
//   .parent_id (int or None), .prev_move_vocab_id, .board_state (a mapping
//   with "piece_ids" (64 ints in 0..12) and the five side fields) and
//   .legal_vocab_ids (a sequence of ints).  out_piece: writable buffer of
//   R*64 bytes, out_side: writable int32 buffer [R, 7] (column 0 is left to
//   the caller).  legal_off is int32 [R+1], legal_ids int32, node / parent
//   ids int64 (parent INT64_MIN for None).  Raises ValueError for piece ids outside
//   0..12 or boards without 64 squares, TypeError for non-integers.
//
// wave_responses(counts, values, legal, offsets) -> list of row lists
//   counts: rows per request; values: float32 [R]; legal: float32 [NL];
//   offsets: int32 [R+1].  Returns, per request, [(value, [legal...]), ...].
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <cstdint>
#include <cstring>
#include <vector>

namespace {

PyObject* s_rows;
PyObject* s_node_id;
PyObject* s_parent_id;
PyObject* s_prev_move;
PyObject* s_board_state;
PyObject* s_legal;
PyObject* s_piece_ids;
PyObject* s_fields[5];

bool intern_all() {
  s_rows = PyUnicode_InternFromString("rows");
  s_node_id = PyUnicode_InternFromString("node_id");
  s_parent_id = PyUnicode_InternFromString("parent_id");
  s_prev_move = PyUnicode_InternFromString("prev_move_vocab_id");
  s_board_state = PyUnicode_InternFromString("board_state");
  s_legal = PyUnicode_InternFromString("legal_vocab_ids");
  s_piece_ids = PyUnicode_InternFromString("piece_ids");
  const char* f[5] = {"turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id"};
  for (int i = 0; i < 5; ++i) s_fields[i] = PyUnicode_InternFromString(f[i]);
  return s_rows && s_node_id && s_parent_id && s_prev_move && s_board_state && s_legal && s_piece_ids &&
         s_fields[0] && s_fields[1] && s_fields[2] && s_fields[3] && s_fields[4];
}

// Owned reference holder.
struct Ref {
  PyObject* p = nullptr;
  Ref() = default;
  explicit Ref(PyObject* o) : p(o) {}
  Ref(const Ref&) = delete;
  Ref& operator=(const Ref&) = delete;
  ~Ref() { Py_XDECREF(p); }
  PyObject* get() const { return p; }
  explicit operator bool() const { return p != nullptr; }
};

bool as_long(PyObject* o, long long* out) {
#if PY_VERSION_HEX >= 0x030C0000
  // Exact ints that fit one digit (every id and piece code on the wire) are
  // read inline, without the general conversion.
  if (PyLong_CheckExact(o) && PyUnstable_Long_IsCompact(reinterpret_cast<PyLongObject*>(o))) {
    *out = (long long)PyUnstable_Long_CompactValue(reinterpret_cast<PyLongObject*>(o));
    return true;
  }
#endif
  if (!PyLong_Check(o)) {
    // numpy integers and other __index__ types
    Ref i(PyNumber_Index(o));
    if (!i) return false;
    *out = PyLong_AsLongLong(i.get());
  } else {
    *out = PyLong_AsLongLong(o);
  }
  return !(*out == -1 && PyErr_Occurred());
}

// Mapping item or attribute (board_state may be a dict or an object).
PyObject* get_item(PyObject* m, PyObject* key) {
  if (PyDict_Check(m)) {
    PyObject* v = PyDict_GetItemWithError(m, key);
    if (!v) {
      if (!PyErr_Occurred()) PyErr_SetObject(PyExc_KeyError, key);
      return nullptr;
    }
    Py_INCREF(v);
    return v;
  }
  return PyObject_GetItem(m, key);
}

struct Buf {
  Py_buffer view{};
  bool ok = false;
  ~Buf() {
    if (ok) PyBuffer_Release(&view);
  }
};

PyObject* pack_wave_rows(PyObject*, PyObject* args) {
  PyObject *requests, *out_piece, *out_side;
  if (!PyArg_ParseTuple(args, "OOO", &requests, &out_piece, &out_side)) return nullptr;
  Ref reqs(PySequence_Fast(requests, "requests must be a sequence"));
  if (!reqs) return nullptr;
  const Py_ssize_t G = PySequence_Fast_GET_SIZE(reqs.get());
  // Rows of every request (kept alive while packing).
  std::vector<PyObject*> row_lists;
  row_lists.reserve(G);
  struct Cleanup {
    std::vector<PyObject*>& v;
    ~Cleanup() {
      for (PyObject* o : v) Py_XDECREF(o);
    }
  } cleanup{row_lists};
  Py_ssize_t R = 0;
  for (Py_ssize_t g = 0; g < G; ++g) {
    Ref rows(PyObject_GetAttr(PySequence_Fast_GET_ITEM(reqs.get(), g), s_rows));
    if (!rows) return nullptr;
    PyObject* fast = PySequence_Fast(rows.get(), "rows must be a sequence");
    if (!fast) return nullptr;
    row_lists.push_back(fast);
    R += PySequence_Fast_GET_SIZE(fast);
  }
  Buf piece, side;
  if (PyObject_GetBuffer(out_piece, &piece.view, PyBUF_WRITABLE | PyBUF_C_CONTIGUOUS) != 0) return nullptr;
  piece.ok = true;
  if (PyObject_GetBuffer(out_side, &side.view, PyBUF_WRITABLE | PyBUF_C_CONTIGUOUS) != 0) return nullptr;
  side.ok = true;
  if (piece.view.len < (Py_ssize_t)R * 64 || side.view.len < (Py_ssize_t)R * 7 * 4) {
    PyErr_SetString(PyExc_ValueError, "output buffers too small for the wave's rows");
    return nullptr;
  }
  uint8_t* pc = static_cast<uint8_t*>(piece.view.buf);
  int32_t* sd = static_cast<int32_t*>(side.view.buf);
  std::vector<int32_t> loff((size_t)R + 1, 0);
  std::vector<int32_t> lids;
  std::vector<int64_t> node((size_t)R), parent((size_t)R);
  lids.reserve((size_t)R * 40);
  Py_ssize_t r = 0;
  for (PyObject* rows : row_lists) {
    const Py_ssize_t n = PySequence_Fast_GET_SIZE(rows);
    for (Py_ssize_t i = 0; i < n; ++i, ++r) {
      PyObject* row = PySequence_Fast_GET_ITEM(rows, i);
      long long v;
      {
        Ref o(PyObject_GetAttr(row, s_node_id));
        if (!o || !as_long(o.get(), &v)) return nullptr;
        node[r] = v;
      }
      {
        Ref o(PyObject_GetAttr(row, s_parent_id));
        if (!o) return nullptr;
        if (o.get() == Py_None) {
          parent[r] = INT64_MIN;
        } else {
          if (!as_long(o.get(), &v)) return nullptr;
          parent[r] = v;
        }
      }
      int32_t* srow = sd + (size_t)r * 7;
      {
        Ref o(PyObject_GetAttr(row, s_prev_move));
        if (!o || !as_long(o.get(), &v)) return nullptr;
        srow[6] = v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
      }
      Ref bs(PyObject_GetAttr(row, s_board_state));
      if (!bs) return nullptr;
      for (int f = 0; f < 5; ++f) {
        Ref o(get_item(bs.get(), s_fields[f]));
        if (!o || !as_long(o.get(), &v)) return nullptr;
        srow[1 + f] = v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
      }
      {
        Ref pl(get_item(bs.get(), s_piece_ids));
        if (!pl) return nullptr;
        Ref fast(PySequence_Fast(pl.get(), "piece_ids must be a sequence"));
        if (!fast) return nullptr;
        if (PySequence_Fast_GET_SIZE(fast.get()) != 64) {
          PyErr_SetString(PyExc_ValueError, "every board_state must carry 64 piece_ids");
          return nullptr;
        }
        uint8_t* prow = pc + (size_t)r * 64;
        for (int k = 0; k < 64; ++k) {
          if (!as_long(PySequence_Fast_GET_ITEM(fast.get(), k), &v)) return nullptr;
          if (v < 0 || v > 12) {
            PyErr_SetString(PyExc_ValueError, "piece_ids values must be in [0, 12]");
            return nullptr;
          }
          prow[k] = (uint8_t)v;
        }
      }
      {
        Ref ll(PyObject_GetAttr(row, s_legal));
        if (!ll) return nullptr;
        Ref fast(PySequence_Fast(ll.get(), "legal_vocab_ids must be a sequence"));
        if (!fast) return nullptr;
        const Py_ssize_t m = PySequence_Fast_GET_SIZE(fast.get());
        for (Py_ssize_t k = 0; k < m; ++k) {
          if (!as_long(PySequence_Fast_GET_ITEM(fast.get(), k), &v)) return nullptr;
          lids.push_back(v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v));
        }
        if ((long long)lids.size() > INT32_MAX) {
          PyErr_SetString(PyExc_ValueError, "too many legal ids in one wave");
          return nullptr;
        }
        loff[r + 1] = (int32_t)lids.size();
      }
    }
  }
  return Py_BuildValue("(ny#y#y#y#)", R, reinterpret_cast<const char*>(loff.data()),
                       (Py_ssize_t)(loff.size() * 4), reinterpret_cast<const char*>(lids.data()),
                       (Py_ssize_t)(lids.size() * 4), reinterpret_cast<const char*>(node.data()),
                       (Py_ssize_t)(node.size() * 8), reinterpret_cast<const char*>(parent.data()),
                       (Py_ssize_t)(parent.size() * 8));
}

PyObject* wave_responses(PyObject*, PyObject* args) {
  PyObject *counts, *values, *legal, *offsets;
  if (!PyArg_ParseTuple(args, "OOOO", &counts, &values, &legal, &offsets)) return nullptr;
  Ref cf(PySequence_Fast(counts, "counts must be a sequence"));
  if (!cf) return nullptr;
  Buf vb, lb, ob;
  if (PyObject_GetBuffer(values, &vb.view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) != 0) return nullptr;
  vb.ok = true;
  if (PyObject_GetBuffer(legal, &lb.view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) != 0) return nullptr;
  lb.ok = true;
  if (PyObject_GetBuffer(offsets, &ob.view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) != 0) return nullptr;
  ob.ok = true;
  if (vb.view.itemsize != 4 || lb.view.itemsize != 4 || ob.view.itemsize != 4 ||
      (vb.view.format && strcmp(vb.view.format, "f") != 0) || (lb.view.format && strcmp(lb.view.format, "f") != 0) ||
      (ob.view.format && strcmp(ob.view.format, "i") != 0)) {
    PyErr_SetString(PyExc_TypeError, "values / legal must be float32 and offsets int32");
    return nullptr;
  }
  const float* val = static_cast<const float*>(vb.view.buf);
  const float* leg = static_cast<const float*>(lb.view.buf);
  const int32_t* off = static_cast<const int32_t*>(ob.view.buf);
  const Py_ssize_t R = vb.view.len / 4, NL = lb.view.len / 4;
  if (ob.view.len / 4 != R + 1) {
    PyErr_SetString(PyExc_ValueError, "offsets must have one entry more than values");
    return nullptr;
  }
  const Py_ssize_t G = PySequence_Fast_GET_SIZE(cf.get());
  Ref out(PyList_New(G));
  if (!out) return nullptr;
  Py_ssize_t r = 0;
  for (Py_ssize_t g = 0; g < G; ++g) {
    long long n;
    if (!as_long(PySequence_Fast_GET_ITEM(cf.get(), g), &n)) return nullptr;
    if (n < 0 || r + n > R) {
      PyErr_SetString(PyExc_ValueError, "counts do not match the rows");
      return nullptr;
    }
    PyObject* lst = PyList_New((Py_ssize_t)n);
    if (!lst) return nullptr;
    PyList_SET_ITEM(out.get(), g, lst);  // steals
    for (Py_ssize_t i = 0; i < n; ++i, ++r) {
      const int32_t a = off[r], b = off[r + 1];
      if (a < 0 || b < a || b > NL) {
        PyErr_SetString(PyExc_ValueError, "legal offsets out of range");
        return nullptr;
      }
      PyObject* ll = PyList_New(b - a);
      if (!ll) return nullptr;
      for (int32_t k = a; k < b; ++k) {
        PyObject* f = PyFloat_FromDouble((double)leg[k]);
        if (!f) {
          Py_DECREF(ll);
          return nullptr;
        }
        PyList_SET_ITEM(ll, k - a, f);
      }
      PyObject* v = PyFloat_FromDouble((double)val[r]);
      if (!v) {
        Py_DECREF(ll);
        return nullptr;
      }
      PyObject* tup = PyTuple_Pack(2, v, ll);
      Py_DECREF(v);
      Py_DECREF(ll);
      if (!tup) return nullptr;
      PyList_SET_ITEM(lst, i, tup);
    }
  }
  return Py_NewRef(out.get());
}

PyMethodDef kMethods[] = {
    {"pack_wave_rows", pack_wave_rows, METH_VARARGS, "Pack the rows of wave requests into flat arrays."},
    {"wave_responses", wave_responses, METH_VARARGS, "Per-request response rows from a step's results."},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_hostpath", "C++ host path of the wave service.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__hostpath(void) {
  if (!intern_all()) return nullptr;
  return PyModule_Create(&kModule);
}
