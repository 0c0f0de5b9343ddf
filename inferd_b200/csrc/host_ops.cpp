// host_ops.cpp -- the per-sequence loops of PagedKVCache's decode path, in C.
//
// The page tables stay Python objects (SequencePageTable: .length, .blocks, .dirty_from),
// and the allocator its LIFO free list and allocated set, exactly as the reference keeps
// them (core/paged_cache.py:27-92); these functions only walk them without the
// interpreter's per-bytecode cost.  Each has a pure-Python twin in paged_cache.py with the
// same results, which the tests compare against.
//
//   plan_slots(tables, per, block_size, free_list, allocated, slots_out)
//       -> (reserved, failed_index)
//     Reserves the pages `per` more tokens need (a table's new blocks are popped from the
//     end of free_list, as BlockAllocator.allocate does), marks each table's lowest changed
//     page, and writes the int64 slots (block * block_size + offset) of positions
//     length .. length + per - 1 of every table, in table order, to slots_out.  reserved
//     lists (table, new_blocks) per table that grew.  When the free list runs short at
//     table i, nothing more is taken and failed_index = i (the caller rolls back and raises
//     MemoryError); else -1.
//   advance(tables, per)            every table's length += per
//   truncate(tables, lengths, block_size, free_list, allocated) -> freed blocks
//     All lengths are checked first (ValueError); then each table keeps
//     ceil(length / block_size) blocks and its tail goes back to free_list in table order.
//   scan(tables, extra, lens_out) -> (nblk, width, max_len)
//     lens_out[i] = length + extra (int32), the page counts and the widest table.
//   pack_changes(tables, prev_ids, prev_nblk, clean, out) -> (pairs, ids, nblk)
//     For each table whose page list changed since the last call (dirty_from != clean, or
//     its list object replaced), the (column, block) pairs of pages dirty_from .. len - 1
//     and (column, 0) for pages it lost; row i's count goes to out[i] (int32).  Resets
//     dirty_from.  Returns the flat pair list (int32 buffer bytes) and the current list ids
//     and lengths.
//   pack_staged(tables, prev_ids, prev_nblk, clean, row_ptr, pairs_out) -> (total, ids, nblk)
//     pack_changes written straight into staging: row_ptr[0 .. n] (int32) the exclusive
//     prefix of the per-row pair counts, pairs_out (int32) the flat (column, block) pairs
//     while they fit.  total is the number of pairs; above pairs_out's capacity the caller
//     sends whole tables instead (the pairs past the capacity are counted, not written).
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <cstdint>
#include <cstring>
#include <vector>

namespace {

PyObject* s_length = nullptr;
PyObject* s_blocks = nullptr;
PyObject* s_dirty = nullptr;

bool get_long(PyObject* obj, PyObject* name, long long* out) {
  PyObject* v = PyObject_GetAttr(obj, name);
  if (!v) return false;
  *out = PyLong_AsLongLong(v);
  Py_DECREF(v);
  return !(*out == -1 && PyErr_Occurred());
}

bool set_long(PyObject* obj, PyObject* name, long long value) {
  PyObject* v = PyLong_FromLongLong(value);
  if (!v) return false;
  const int r = PyObject_SetAttr(obj, name, v);
  Py_DECREF(v);
  return r == 0;
}

// True for a struct-module format naming a signed integer of `itemsize` bytes in native
// byte order ("i", "l", "q", optionally prefixed with "@" or "=").
bool signed_int_format(const char* fmt, Py_ssize_t itemsize) {
  if (fmt == nullptr) return false;
  if (*fmt == '@' || *fmt == '=') ++fmt;
  if (fmt[0] == '\0' || fmt[1] != '\0') return false;
  switch (fmt[0]) {
    case 'i': return itemsize == static_cast<Py_ssize_t>(sizeof(int));
    case 'l': return itemsize == static_cast<Py_ssize_t>(sizeof(long));
    case 'q': return itemsize == static_cast<Py_ssize_t>(sizeof(long long));
    default: return false;
  }
}

// writable C-contiguous buffer of signed integers of `itemsize` bytes (int32 or int64),
// at least `bytes` bytes long; anything else (another item size, floats, unsigned) is a
// TypeError, so a mistyped view can never be read or written as the wrong integer width
bool get_buffer(PyObject* obj, Py_buffer* view, Py_ssize_t bytes, Py_ssize_t itemsize) {
  if (PyObject_GetBuffer(obj, view, PyBUF_WRITABLE | PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) != 0)
    return false;
  if (view->itemsize != itemsize || !signed_int_format(view->format, view->itemsize)) {
    PyErr_Format(PyExc_TypeError, "expected a buffer of int%d, got format '%s' with %zd-byte items",
                 static_cast<int>(itemsize * 8), view->format ? view->format : "B", view->itemsize);
    PyBuffer_Release(view);
    return false;
  }
  if (view->len < bytes) {
    PyBuffer_Release(view);
    PyErr_SetString(PyExc_ValueError, "output buffer too small");
    return false;
  }
  return true;
}

PyObject* plan_slots(PyObject*, PyObject* args) {
  PyObject *tables, *free_list, *allocated, *slots_obj;
  long long per, bs;
  if (!PyArg_ParseTuple(args, "O!LLO!O!O", &PyList_Type, &tables, &per, &bs, &PyList_Type, &free_list,
                        &PySet_Type, &allocated, &slots_obj))
    return nullptr;
  if (per <= 0 || bs <= 0) {
    PyErr_SetString(PyExc_ValueError, "per and block_size must be positive");
    return nullptr;
  }
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  Py_buffer view;
  if (!get_buffer(slots_obj, &view, static_cast<Py_ssize_t>(n * per * 8), 8)) return nullptr;
  int64_t* slots = static_cast<int64_t*>(view.buf);
  PyObject* reserved = PyList_New(0);
  Py_ssize_t failed = -1;
  if (!reserved) goto error;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* t = PyList_GET_ITEM(tables, i);
    long long pos, dirty;
    if (!get_long(t, s_length, &pos)) goto error;
    PyObject* blocks = PyObject_GetAttr(t, s_blocks);
    if (!blocks) goto error;
    if (!PyList_Check(blocks)) {
      Py_DECREF(blocks);
      PyErr_SetString(PyExc_TypeError, "page table blocks must be a list");
      goto error;
    }
    const Py_ssize_t nb = PyList_GET_SIZE(blocks);
    const long long need = (pos + per + bs - 1) / bs - nb;
    if (need > 0) {
      const Py_ssize_t nfree = PyList_GET_SIZE(free_list);
      if (need > nfree) {
        Py_DECREF(blocks);
        failed = i;
        break;
      }
      PyObject* fresh = PyList_New(static_cast<Py_ssize_t>(need));
      if (!fresh) {
        Py_DECREF(blocks);
        goto error;
      }
      for (long long j = 0; j < need; ++j) {  // pop() order: last free block first
        PyObject* b = PyList_GET_ITEM(free_list, nfree - 1 - j);
        Py_INCREF(b);
        PyList_SET_ITEM(fresh, static_cast<Py_ssize_t>(j), b);
        if (PySet_Add(allocated, b) != 0 || PyList_Append(blocks, b) != 0) {
          Py_DECREF(fresh);
          Py_DECREF(blocks);
          goto error;
        }
      }
      if (PyList_SetSlice(free_list, nfree - static_cast<Py_ssize_t>(need), nfree, nullptr) != 0) {
        Py_DECREF(fresh);
        Py_DECREF(blocks);
        goto error;
      }
      if (!get_long(t, s_dirty, &dirty) || (nb < dirty && !set_long(t, s_dirty, nb))) {
        Py_DECREF(fresh);
        Py_DECREF(blocks);
        goto error;
      }
      PyObject* pair = PyTuple_Pack(2, t, fresh);
      Py_DECREF(fresh);
      if (!pair || PyList_Append(reserved, pair) != 0) {
        Py_XDECREF(pair);
        Py_DECREF(blocks);
        goto error;
      }
      Py_DECREF(pair);
    }
    for (long long q = pos; q < pos + per; ++q) {
      const long long page = q / bs;
      const long long blk = PyLong_AsLongLong(PyList_GET_ITEM(blocks, static_cast<Py_ssize_t>(page)));
      if (blk == -1 && PyErr_Occurred()) {
        Py_DECREF(blocks);
        goto error;
      }
      *slots++ = blk * bs + (q - page * bs);
    }
    Py_DECREF(blocks);
  }
  PyBuffer_Release(&view);
  {
    PyObject* res = Py_BuildValue("(Nn)", reserved, failed);
    return res;
  }
error:
  PyBuffer_Release(&view);
  Py_XDECREF(reserved);
  return nullptr;
}

PyObject* advance(PyObject*, PyObject* args) {
  PyObject* tables;
  long long per;
  if (!PyArg_ParseTuple(args, "O!L", &PyList_Type, &tables, &per)) return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* t = PyList_GET_ITEM(tables, i);
    long long len;
    if (!get_long(t, s_length, &len) || !set_long(t, s_length, len + per)) return nullptr;
  }
  Py_RETURN_NONE;
}

PyObject* truncate(PyObject*, PyObject* args) {
  PyObject *tables, *lengths, *free_list, *allocated;
  long long bs;
  if (!PyArg_ParseTuple(args, "O!O!LO!O!", &PyList_Type, &tables, &PyList_Type, &lengths, &bs, &PyList_Type,
                        &free_list, &PySet_Type, &allocated))
    return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  if (PyList_GET_SIZE(lengths) != n) {
    PyErr_SetString(PyExc_ValueError, "one length per sequence");
    return nullptr;
  }
  std::vector<long long> want(static_cast<size_t>(n));
  for (Py_ssize_t i = 0; i < n; ++i) {
    long long cur;
    const long long w = PyLong_AsLongLong(PyList_GET_ITEM(lengths, i));
    if (w == -1 && PyErr_Occurred()) return nullptr;
    if (!get_long(PyList_GET_ITEM(tables, i), s_length, &cur)) return nullptr;
    if (w < 0 || w > cur) {
      PyErr_Format(PyExc_ValueError, "cannot truncate a sequence of length %lld to %lld", cur, w);
      return nullptr;
    }
    want[static_cast<size_t>(i)] = w;
  }
  PyObject* freed_all = PyList_New(0);
  if (!freed_all) return nullptr;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* t = PyList_GET_ITEM(tables, i);
    const long long w = want[static_cast<size_t>(i)];
    const long long keep = (w + bs - 1) / bs;
    PyObject* blocks = PyObject_GetAttr(t, s_blocks);
    if (!blocks) goto error;
    if (!PyList_Check(blocks)) {
      Py_DECREF(blocks);
      PyErr_SetString(PyExc_TypeError, "page table blocks must be a list");
      goto error;
    }
    const Py_ssize_t nb = PyList_GET_SIZE(blocks);
    if (keep < nb) {
      for (Py_ssize_t j = static_cast<Py_ssize_t>(keep); j < nb; ++j) {  // freed in table order
        PyObject* b = PyList_GET_ITEM(blocks, j);
        const int present = PySet_Contains(allocated, b);
        if (present != 1) {
          if (present == 0) PyErr_SetString(PyExc_ValueError, "block is not allocated");
          Py_DECREF(blocks);
          goto error;
        }
        if (PySet_Discard(allocated, b) < 0 || PyList_Append(free_list, b) != 0 || PyList_Append(freed_all, b) != 0) {
          Py_DECREF(blocks);
          goto error;
        }
      }
      if (PyList_SetSlice(blocks, static_cast<Py_ssize_t>(keep), nb, nullptr) != 0) {
        Py_DECREF(blocks);
        goto error;
      }
      long long dirty;
      if (!get_long(t, s_dirty, &dirty) || (keep < dirty && !set_long(t, s_dirty, keep))) {
        Py_DECREF(blocks);
        goto error;
      }
    }
    Py_DECREF(blocks);
    if (!set_long(t, s_length, w)) goto error;
  }
  return freed_all;
error:
  Py_DECREF(freed_all);
  return nullptr;
}

// Walk the tables for pack_changes / pack_staged: emit(row, column, block) for every changed
// entry, counts[row] = the row's pair count; resets dirty_from.  Fills ids / nblk (new
// references) with the current list ids and lengths.
template <typename Emit>
bool walk_changes(PyObject* tables, PyObject* prev_ids, PyObject* prev_nblk, long long clean,
                  int32_t* counts, PyObject* ids, PyObject* nblk, Emit emit) {
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* t = PyList_GET_ITEM(tables, i);
    PyObject* blocks = PyObject_GetAttr(t, s_blocks);
    if (!blocks) return false;
    if (!PyList_Check(blocks)) {
      Py_DECREF(blocks);
      PyErr_SetString(PyExc_TypeError, "page table blocks must be a list");
      return false;
    }
    const Py_ssize_t nb = PyList_GET_SIZE(blocks);
    PyObject* id = PyLong_FromVoidPtr(blocks);
    PyObject* nbo = PyLong_FromSsize_t(nb);
    if (!id || !nbo) {
      Py_XDECREF(id);
      Py_XDECREF(nbo);
      Py_DECREF(blocks);
      return false;
    }
    PyList_SET_ITEM(ids, i, id);
    PyList_SET_ITEM(nblk, i, nbo);
    long long dirty;
    if (!get_long(t, s_dirty, &dirty)) {
      Py_DECREF(blocks);
      return false;
    }
    const int same = PyObject_RichCompareBool(id, PyList_GET_ITEM(prev_ids, i), Py_EQ);
    if (same < 0) {
      Py_DECREF(blocks);
      return false;
    }
    const long long start = same ? dirty : 0;
    int32_t count = 0;
    if (start != clean) {
      const long long old = PyLong_AsLongLong(PyList_GET_ITEM(prev_nblk, i));
      if (old == -1 && PyErr_Occurred()) {
        Py_DECREF(blocks);
        return false;
      }
      for (long long c = start; c < nb; ++c) {
        const long long b = PyLong_AsLongLong(PyList_GET_ITEM(blocks, static_cast<Py_ssize_t>(c)));
        if (b == -1 && PyErr_Occurred()) {
          Py_DECREF(blocks);
          return false;
        }
        emit(static_cast<int32_t>(c), static_cast<int32_t>(b));
        ++count;
      }
      for (long long c = (nb > start ? nb : start); c < old; ++c) {
        emit(static_cast<int32_t>(c), 0);
        ++count;
      }
      if (!set_long(t, s_dirty, clean)) {
        Py_DECREF(blocks);
        return false;
      }
    }
    counts[i] = count;
    Py_DECREF(blocks);
  }
  return true;
}

PyObject* pack_changes(PyObject*, PyObject* args) {
  PyObject *tables, *prev_ids, *prev_nblk, *out_obj;
  long long clean;
  if (!PyArg_ParseTuple(args, "O!O!O!LO", &PyList_Type, &tables, &PyList_Type, &prev_ids, &PyList_Type, &prev_nblk,
                        &clean, &out_obj))
    return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  if (PyList_GET_SIZE(prev_ids) != n || PyList_GET_SIZE(prev_nblk) != n) {
    PyErr_SetString(PyExc_ValueError, "previous batch state does not match the tables");
    return nullptr;
  }
  Py_buffer view;
  if (!get_buffer(out_obj, &view, static_cast<Py_ssize_t>(n * 4), 4)) return nullptr;
  std::vector<int32_t> pairs;
  PyObject* ids = PyList_New(n);
  PyObject* nblk = PyList_New(n);
  if (!ids || !nblk ||
      !walk_changes(tables, prev_ids, prev_nblk, clean, static_cast<int32_t*>(view.buf), ids, nblk,
                    [&](int32_t c, int32_t b) {
                      pairs.push_back(c);
                      pairs.push_back(b);
                    })) {
    PyBuffer_Release(&view);
    Py_XDECREF(ids);
    Py_XDECREF(nblk);
    return nullptr;
  }
  PyBuffer_Release(&view);
  PyObject* pb = PyBytes_FromStringAndSize(reinterpret_cast<const char*>(pairs.data()),
                                           static_cast<Py_ssize_t>(pairs.size() * sizeof(int32_t)));
  if (!pb) {
    Py_DECREF(ids);
    Py_DECREF(nblk);
    return nullptr;
  }
  return Py_BuildValue("(NNN)", pb, ids, nblk);
}

PyObject* pack_staged(PyObject*, PyObject* args) {
  PyObject *tables, *prev_ids, *prev_nblk, *rp_obj, *pairs_obj;
  long long clean;
  if (!PyArg_ParseTuple(args, "O!O!O!LOO", &PyList_Type, &tables, &PyList_Type, &prev_ids, &PyList_Type,
                        &prev_nblk, &clean, &rp_obj, &pairs_obj))
    return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  if (PyList_GET_SIZE(prev_ids) != n || PyList_GET_SIZE(prev_nblk) != n) {
    PyErr_SetString(PyExc_ValueError, "previous batch state does not match the tables");
    return nullptr;
  }
  Py_buffer rp_view, pv;
  if (!get_buffer(rp_obj, &rp_view, static_cast<Py_ssize_t>((n + 1) * 4), 4)) return nullptr;
  if (!get_buffer(pairs_obj, &pv, 0, 4)) {
    PyBuffer_Release(&rp_view);
    return nullptr;
  }
  int32_t* row_ptr = static_cast<int32_t*>(rp_view.buf);
  int32_t* out = static_cast<int32_t*>(pv.buf);
  const long long cap = static_cast<long long>(pv.len / 8);  // pairs that fit
  long long total = 0;
  PyObject* ids = PyList_New(n);
  PyObject* nblk = PyList_New(n);
  const bool ok = ids && nblk &&
                  walk_changes(tables, prev_ids, prev_nblk, clean, row_ptr + 1, ids, nblk,
                               [&](int32_t c, int32_t b) {
                                 if (total < cap) {
                                   out[2 * total] = c;
                                   out[2 * total + 1] = b;
                                 }
                                 ++total;
                               });
  if (ok) {  // counts -> exclusive prefix
    row_ptr[0] = 0;
    for (Py_ssize_t i = 0; i < n; ++i) row_ptr[i + 1] += row_ptr[i];
  }
  PyBuffer_Release(&rp_view);
  PyBuffer_Release(&pv);
  if (!ok) {
    Py_XDECREF(ids);
    Py_XDECREF(nblk);
    return nullptr;
  }
  return Py_BuildValue("(LNN)", total, ids, nblk);
}

// scan(tables, extra, lens_out) -> (nblk, width, max_len): lens_out[i] = length + extra
// (int32), nblk the list of page counts, width the largest (at least 1)
PyObject* scan(PyObject*, PyObject* args) {
  PyObject *tables, *out_obj;
  long long extra;
  if (!PyArg_ParseTuple(args, "O!LO", &PyList_Type, &tables, &extra, &out_obj)) return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(tables);
  Py_buffer view;
  if (!get_buffer(out_obj, &view, static_cast<Py_ssize_t>(n * 4), 4)) return nullptr;
  int32_t* lens = static_cast<int32_t*>(view.buf);
  PyObject* nblk = PyList_New(n);
  if (!nblk) {
    PyBuffer_Release(&view);
    return nullptr;
  }
  Py_ssize_t width = 1;
  long long max_len = 0;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* t = PyList_GET_ITEM(tables, i);
    long long len;
    PyObject* blocks = nullptr;
    if (!get_long(t, s_length, &len) || !(blocks = PyObject_GetAttr(t, s_blocks))) {
      PyBuffer_Release(&view);
      Py_DECREF(nblk);
      return nullptr;
    }
    const Py_ssize_t nb = PyObject_Length(blocks);
    Py_DECREF(blocks);
    PyObject* nbo = nb < 0 ? nullptr : PyLong_FromSsize_t(nb);
    if (!nbo) {
      PyBuffer_Release(&view);
      Py_DECREF(nblk);
      return nullptr;
    }
    PyList_SET_ITEM(nblk, i, nbo);
    if (nb > width) width = nb;
    lens[i] = static_cast<int32_t>(len + extra);
    if (len + extra > max_len) max_len = len + extra;
  }
  PyBuffer_Release(&view);
  return Py_BuildValue("(NnL)", nblk, width, max_len);
}

PyMethodDef kMethods[] = {
    {"scan", scan, METH_VARARGS, "lengths, page counts and the widest table of a batch"},
    {"plan_slots", plan_slots, METH_VARARGS, "reserve pages and write the slots of an append"},
    {"advance", advance, METH_VARARGS, "advance every table's length"},
    {"truncate", truncate, METH_VARARGS, "batched truncation returning the freed blocks"},
    {"pack_changes", pack_changes, METH_VARARGS, "sparse page-table changes since the last call"},
    {"pack_staged", pack_staged, METH_VARARGS, "pack_changes written straight into staging buffers"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_hostops", "Page-table loops of the decode path.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__hostops(void) {
  s_length = PyUnicode_InternFromString("length");
  s_blocks = PyUnicode_InternFromString("blocks");
  s_dirty = PyUnicode_InternFromString("dirty_from");
  if (!s_length || !s_blocks || !s_dirty) return nullptr;
  return PyModule_Create(&kModule);
}
