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
//   0..12 or boards without 64 squares, TypeError for non-integers.  The
//   attributes are read on the calling thread; the elements of the integer
//   lists (64 piece ids and the legal ids of every row) are converted by a
//   few worker threads that only read the int objects' memory, while the
//   calling thread holds the GIL and waits for them.
//
// wave_chains(dicts, counts, parent_ids) -> (depths, chain rows) and
// record_chains(dicts, counts, node_ids, parent_ids, own_start): the turn
// node-chain bookkeeping of a wave (see the functions below).
//
// wave_responses(counts, values, legal, offsets) -> list of row lists
//   counts: rows per request; values: float32 [R]; legal: float32 [NL];
//   offsets: int32 [R+1].  Returns, per request, [(value, [legal...]), ...];
//   the rows are not tracked by the cyclic garbage collector (they hold
//   only floats).
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
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

// An exact int that fits one digit, read without any API call (safe from
// worker threads while the calling thread holds the GIL and waits).
inline bool compact_int(PyObject* o, long long* out) {
#if PY_VERSION_HEX >= 0x030C0000
  if (PyLong_CheckExact(o) && PyUnstable_Long_IsCompact(reinterpret_cast<PyLongObject*>(o))) {
    *out = (long long)PyUnstable_Long_CompactValue(reinterpret_cast<PyLongObject*>(o));
    return true;
  }
#endif
  (void)o;
  (void)out;
  return false;
}

inline int32_t clamp32(long long v) {
  return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}

// Piece ids and legal ids of one row, from the borrowed item arrays of its
// lists; false when an element needs the general conversion (or is out of
// range), which the calling thread then redoes with the Python API.
bool convert_row_fast(PyObject* const* pieces, PyObject* const* legal, Py_ssize_t nlegal, uint8_t* prow,
                      int32_t* lrow) {
  for (int k = 0; k < 64; ++k) {
    long long v;
    if (!compact_int(pieces[k], &v) || v < 0 || v > 12) return false;
    prow[k] = (uint8_t)v;
  }
  for (Py_ssize_t k = 0; k < nlegal; ++k) {
    long long v;
    if (!compact_int(legal[k], &v)) return false;
    lrow[k] = clamp32(v);
  }
  return true;
}

// The same with the general conversions and the error messages.
bool convert_row_slow(PyObject* const* pieces, PyObject* const* legal, Py_ssize_t nlegal, uint8_t* prow,
                      int32_t* lrow) {
  for (int k = 0; k < 64; ++k) {
    long long v;
    if (!as_long(pieces[k], &v)) return false;
    if (v < 0 || v > 12) {
      PyErr_SetString(PyExc_ValueError, "piece_ids values must be in [0, 12]");
      return false;
    }
    prow[k] = (uint8_t)v;
  }
  for (Py_ssize_t k = 0; k < nlegal; ++k) {
    long long v;
    if (!as_long(legal[k], &v)) return false;
    lrow[k] = clamp32(v);
  }
  return true;
}

PyObject* pack_wave_rows(PyObject*, PyObject* args) {
  PyObject *requests, *out_piece, *out_side;
  if (!PyArg_ParseTuple(args, "OOO", &requests, &out_piece, &out_side)) return nullptr;
  Ref reqs(PySequence_Fast(requests, "requests must be a sequence"));
  if (!reqs) return nullptr;
  const Py_ssize_t G = PySequence_Fast_GET_SIZE(reqs.get());
  // Every sequence object read below is kept alive until the end.
  std::vector<PyObject*> keep;
  struct Cleanup {
    std::vector<PyObject*>& v;
    ~Cleanup() {
      for (PyObject* o : v) Py_XDECREF(o);
    }
  } cleanup{keep};
  std::vector<PyObject*> row_lists;
  row_lists.reserve(G);
  Py_ssize_t R = 0;
  for (Py_ssize_t g = 0; g < G; ++g) {
    Ref rows(PyObject_GetAttr(PySequence_Fast_GET_ITEM(reqs.get(), g), s_rows));
    if (!rows) return nullptr;
    PyObject* fast = PySequence_Fast(rows.get(), "rows must be a sequence");
    if (!fast) return nullptr;
    keep.push_back(fast);
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
  std::vector<int64_t> node((size_t)R), parent((size_t)R);
  std::vector<PyObject* const*> pitems((size_t)R), litems((size_t)R);
  keep.reserve(keep.size() + 2 * (size_t)R);
  // Pass 1 (this thread): attributes, side fields, ids and the item arrays
  // of every row's two integer lists.
  Py_ssize_t r = 0;
  long long total_legal = 0;
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
        srow[6] = clamp32(v);
      }
      Ref bs(PyObject_GetAttr(row, s_board_state));
      if (!bs) return nullptr;
      for (int f = 0; f < 5; ++f) {
        Ref o(get_item(bs.get(), s_fields[f]));
        if (!o || !as_long(o.get(), &v)) return nullptr;
        srow[1 + f] = clamp32(v);
      }
      {
        Ref pl(get_item(bs.get(), s_piece_ids));
        if (!pl) return nullptr;
        PyObject* fast = PySequence_Fast(pl.get(), "piece_ids must be a sequence");
        if (!fast) return nullptr;
        keep.push_back(fast);
        if (PySequence_Fast_GET_SIZE(fast) != 64) {
          PyErr_SetString(PyExc_ValueError, "every board_state must carry 64 piece_ids");
          return nullptr;
        }
        pitems[r] = PySequence_Fast_ITEMS(fast);
      }
      {
        Ref ll(PyObject_GetAttr(row, s_legal));
        if (!ll) return nullptr;
        PyObject* fast = PySequence_Fast(ll.get(), "legal_vocab_ids must be a sequence");
        if (!fast) return nullptr;
        keep.push_back(fast);
        total_legal += PySequence_Fast_GET_SIZE(fast);
        if (total_legal > INT32_MAX) {
          PyErr_SetString(PyExc_ValueError, "too many legal ids in one wave");
          return nullptr;
        }
        litems[r] = PySequence_Fast_ITEMS(fast);
        loff[r + 1] = (int32_t)total_legal;
      }
    }
  }
  // Pass 2 (worker threads, no Python API): the integer lists' elements.
  std::vector<int32_t> lids((size_t)total_legal);
  std::vector<uint8_t> slow((size_t)R, 0);
  auto work = [&](Py_ssize_t lo, Py_ssize_t hi) {
    for (Py_ssize_t q = lo; q < hi; ++q)
      if (!convert_row_fast(pitems[q], litems[q], loff[q + 1] - loff[q], pc + (size_t)q * 64, lids.data() + loff[q]))
        slow[q] = 1;
  };
  const unsigned hw = std::thread::hardware_concurrency();
  const Py_ssize_t nthreads = std::min<Py_ssize_t>(std::max<Py_ssize_t>(1, R / 512), hw > 1 ? (Py_ssize_t)hw : 1);
  const Py_ssize_t T = std::min<Py_ssize_t>(nthreads, 8);
  if (T <= 1) {
    work(0, R);
  } else {
    std::vector<std::thread> pool;
    pool.reserve((size_t)T - 1);
    const Py_ssize_t per = (R + T - 1) / T;
    for (Py_ssize_t t = 1; t < T; ++t) pool.emplace_back(work, t * per, std::min(R, (t + 1) * per));
    work(0, std::min(R, per));
    for (auto& th : pool) th.join();
  }
  // Pass 3 (this thread): rows with other integer types, or errors.
  for (Py_ssize_t q = 0; q < R; ++q)
    if (slow[q] &&
        !convert_row_slow(pitems[q], litems[q], loff[q + 1] - loff[q], pc + (size_t)q * 64, lids.data() + loff[q]))
      return nullptr;
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
      // A row is a float and a list of floats: it can never be part of a
      // reference cycle, so it stays out of the cyclic collector's lists
      // (whose next pass would otherwise scan every row of the wave).
      PyObject_GC_UnTrack(ll);
      PyObject_GC_UnTrack(tup);
      PyList_SET_ITEM(lst, i, tup);
    }
  }
  return Py_NewRef(out.get());
}

// Reads an int64 buffer argument.
bool int64_view(PyObject* o, Buf* b, const int64_t** data, Py_ssize_t* n) {
  if (PyObject_GetBuffer(o, &b->view, PyBUF_C_CONTIGUOUS) != 0) return false;
  b->ok = true;
  if (b->view.len % 8) {
    PyErr_SetString(PyExc_ValueError, "expected an int64 buffer");
    return false;
  }
  *data = static_cast<const int64_t*>(b->view.buf);
  *n = b->view.len / 8;
  return true;
}

// Per-request row counts as a vector (and their sum).
bool read_counts(PyObject* counts, std::vector<Py_ssize_t>* out, Py_ssize_t* total) {
  Ref cf(PySequence_Fast(counts, "counts must be a sequence"));
  if (!cf) return false;
  const Py_ssize_t G = PySequence_Fast_GET_SIZE(cf.get());
  out->resize(G);
  *total = 0;
  for (Py_ssize_t g = 0; g < G; ++g) {
    long long n;
    if (!as_long(PySequence_Fast_GET_ITEM(cf.get(), g), &n)) return false;
    if (n < 0) {
      PyErr_SetString(PyExc_ValueError, "negative row count");
      return false;
    }
    (*out)[g] = (Py_ssize_t)n;
    *total += (Py_ssize_t)n;
  }
  return true;
}

// The parent chain (arena rows, root -> parent) of one row: a borrowed list
// from the turn's node_chains, or nullptr for a child of the root.  KeyError
// for a parent the turn does not know (actor_server.py:839-850 indexes
// node_chains[parent_id] the same way).
bool parent_chain(PyObject* dict, int64_t parent, PyObject** chain) {
  *chain = nullptr;
  if (parent == INT64_MIN) return true;
  Ref key(PyLong_FromLongLong(parent));
  if (!key) return false;
  PyObject* c = PyDict_GetItemWithError(dict, key.get());
  if (!c) {
    if (!PyErr_Occurred()) PyErr_SetObject(PyExc_KeyError, key.get());
    return false;
  }
  if (!PyList_Check(c)) {
    PyErr_SetString(PyExc_TypeError, "node chains must be lists of arena rows");
    return false;
  }
  *chain = c;
  return true;
}

// wave_chains(dicts, counts, parent_ids) -> (depths bytes, chain rows bytes)
//   dicts: per request, its turn's node_chains (node id -> list of arena
//   rows); counts: rows per request; parent_ids: int64 per row (INT64_MIN:
//   a child of the root).  depths: int64 per row (the parent chain's
//   length); chain rows: int64, every row's parent chain, concatenated.
PyObject* wave_chains(PyObject*, PyObject* args) {
  PyObject *dicts, *counts, *parents;
  if (!PyArg_ParseTuple(args, "OOO", &dicts, &counts, &parents)) return nullptr;
  Ref df(PySequence_Fast(dicts, "dicts must be a sequence"));
  if (!df) return nullptr;
  std::vector<Py_ssize_t> cnt;
  Py_ssize_t R = 0;
  if (!read_counts(counts, &cnt, &R)) return nullptr;
  Buf pb;
  const int64_t* par;
  Py_ssize_t np_;
  if (!int64_view(parents, &pb, &par, &np_)) return nullptr;
  if (np_ != R || PySequence_Fast_GET_SIZE(df.get()) != (Py_ssize_t)cnt.size()) {
    PyErr_SetString(PyExc_ValueError, "counts, dicts and parent ids disagree");
    return nullptr;
  }
  std::vector<int64_t> depth((size_t)R), flat;
  flat.reserve((size_t)R * 2);
  Py_ssize_t r = 0;
  for (size_t g = 0; g < cnt.size(); ++g) {
    PyObject* d = PySequence_Fast_GET_ITEM(df.get(), (Py_ssize_t)g);
    if (!PyDict_Check(d)) {
      PyErr_SetString(PyExc_TypeError, "node chains must be dicts");
      return nullptr;
    }
    for (Py_ssize_t i = 0; i < cnt[g]; ++i, ++r) {
      PyObject* c;
      if (!parent_chain(d, par[r], &c)) return nullptr;
      const Py_ssize_t n = c ? PyList_GET_SIZE(c) : 0;
      depth[r] = n;
      for (Py_ssize_t k = 0; k < n; ++k) {
        long long v;
        if (!as_long(PyList_GET_ITEM(c, k), &v)) return nullptr;
        flat.push_back(v);
      }
    }
  }
  return Py_BuildValue("(y#y#)", reinterpret_cast<const char*>(depth.data()), (Py_ssize_t)(depth.size() * 8),
                       reinterpret_cast<const char*>(flat.data()), (Py_ssize_t)(flat.size() * 8));
}

// record_chains(dicts, counts, node_ids, parent_ids, own_start)
//   After a wave: node_chains[node] = node_chains[parent] + [own row] for
//   every row, own row = own_start[request] + its index within the request
//   (actor_server.py:904-914; the rows the wave minted, in wave order).
PyObject* record_chains(PyObject*, PyObject* args) {
  PyObject *dicts, *counts, *nodes, *parents, *starts;
  if (!PyArg_ParseTuple(args, "OOOOO", &dicts, &counts, &nodes, &parents, &starts)) return nullptr;
  Ref df(PySequence_Fast(dicts, "dicts must be a sequence"));
  if (!df) return nullptr;
  std::vector<Py_ssize_t> cnt;
  Py_ssize_t R = 0;
  if (!read_counts(counts, &cnt, &R)) return nullptr;
  Buf nb, pb, sb;
  const int64_t *nod, *par, *st;
  Py_ssize_t nn, np_, ns;
  if (!int64_view(nodes, &nb, &nod, &nn) || !int64_view(parents, &pb, &par, &np_) ||
      !int64_view(starts, &sb, &st, &ns))
    return nullptr;
  if (nn != R || np_ != R || ns != (Py_ssize_t)cnt.size() ||
      PySequence_Fast_GET_SIZE(df.get()) != (Py_ssize_t)cnt.size()) {
    PyErr_SetString(PyExc_ValueError, "counts, dicts, node / parent ids and starts disagree");
    return nullptr;
  }
  Py_ssize_t r = 0;
  for (size_t g = 0; g < cnt.size(); ++g) {
    PyObject* d = PySequence_Fast_GET_ITEM(df.get(), (Py_ssize_t)g);
    if (!PyDict_Check(d)) {
      PyErr_SetString(PyExc_TypeError, "node chains must be dicts");
      return nullptr;
    }
    // Parents first: a row whose parent is recorded by this same wave sees
    // the chain the parent had before the wave, as the reference does.
    std::vector<PyObject*> chains((size_t)cnt[g]);
    for (Py_ssize_t i = 0; i < cnt[g]; ++i) {
      if (!parent_chain(d, par[r + i], &chains[(size_t)i])) return nullptr;
    }
    std::vector<Ref> fresh((size_t)cnt[g]);
    for (Py_ssize_t i = 0; i < cnt[g]; ++i) {
      PyObject* c = chains[(size_t)i];
      const Py_ssize_t n = c ? PyList_GET_SIZE(c) : 0;
      PyObject* lst = PyList_New(n + 1);
      if (!lst) return nullptr;
      fresh[(size_t)i].p = lst;
      for (Py_ssize_t k = 0; k < n; ++k) {
        PyObject* v = PyList_GET_ITEM(c, k);
        Py_INCREF(v);
        PyList_SET_ITEM(lst, k, v);
      }
      PyObject* own = PyLong_FromLongLong(st[g] + i);
      if (!own) return nullptr;
      PyList_SET_ITEM(lst, n, own);
      PyObject_GC_UnTrack(lst);  // a list of ints: no cycles, nothing for the collector to scan
    }
    for (Py_ssize_t i = 0; i < cnt[g]; ++i, ++r) {
      Ref key(PyLong_FromLongLong(nod[r]));
      if (!key || PyDict_SetItem(d, key.get(), fresh[(size_t)i].get()) != 0) return nullptr;
    }
  }
  Py_RETURN_NONE;
}

// ids_csr(rows) -> (offsets bytes, ids bytes): the CSR of per-row integer
// sequences (int32 offsets [R+1], int32 ids), e.g. every row's legal move
// ids.  Lists and tuples of exact one-digit ints are read inline; other
// sequences and integer types take the general conversion (TypeError for
// non-integers).
PyObject* ids_csr(PyObject*, PyObject* args) {
  PyObject* rows;
  if (!PyArg_ParseTuple(args, "O", &rows)) return nullptr;
  Ref seq(PySequence_Fast(rows, "ids_csr expects a sequence of id sequences"));
  if (!seq) return nullptr;
  const Py_ssize_t R = PySequence_Fast_GET_SIZE(seq.get());
  PyObject** items = PySequence_Fast_ITEMS(seq.get());
  std::vector<int32_t> off((size_t)R + 1, 0);
  std::vector<int32_t> ids;
  ids.reserve((size_t)R * 32);
  for (Py_ssize_t r = 0; r < R; ++r) {
    Ref row(PySequence_Fast(items[r], "ids_csr: each row must be a sequence of ints"));
    if (!row) return nullptr;
    const Py_ssize_t n = PySequence_Fast_GET_SIZE(row.get());
    PyObject** e = PySequence_Fast_ITEMS(row.get());
    for (Py_ssize_t k = 0; k < n; ++k) {
      long long v;
      if (!as_long(e[k], &v)) return nullptr;
      ids.push_back(clamp32(v));
    }
    if (ids.size() > (size_t)INT32_MAX) {
      PyErr_SetString(PyExc_OverflowError, "ids_csr: more than 2^31 ids");
      return nullptr;
    }
    off[(size_t)r + 1] = (int32_t)ids.size();
  }
  static const char kEmpty[1] = {0};
  const char* idp = ids.empty() ? kEmpty : reinterpret_cast<const char*>(ids.data());
  return Py_BuildValue("(y#y#)", reinterpret_cast<const char*>(off.data()), (Py_ssize_t)(off.size() * 4), idp,
                       (Py_ssize_t)(ids.size() * 4));
}

PyMethodDef kMethods[] = {
    {"ids_csr", ids_csr, METH_VARARGS, "CSR (int32 offsets, int32 ids) of per-row integer sequences."},
    {"pack_wave_rows", pack_wave_rows, METH_VARARGS, "Pack the rows of wave requests into flat arrays."},
    {"wave_responses", wave_responses, METH_VARARGS, "Per-request response rows from a step's results."},
    {"wave_chains", wave_chains, METH_VARARGS, "Depths and parent-chain arena rows of a wave's rows."},
    {"record_chains", record_chains, METH_VARARGS, "Record the node chains of a wave's rows."},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_hostpath", "C++ host path of the wave service.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__hostpath(void) {
  if (!intern_all()) return nullptr;
  return PyModule_Create(&kModule);
}
