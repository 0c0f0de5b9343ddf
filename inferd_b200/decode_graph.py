"""One decode (or speculative-verify) step of a fixed batch, replayed as a CUDA graph.

The reference's decode loop issues, per step and per sequence, Python-level cache updates
and attention calls (core/scheduler.py:142-159, core/paged_attn_interface.py:25-62).  Here a
step of a whole batch is one graph replay:

    one host->device copy of the step's inputs (queries, new K and V, slots, lengths and
    page-table changes) from pinned memory
    -> sparse page-table update of a device-resident [B, capacity] table
    -> KV append (reshape_and_cache) -> paged attention over the table, whose epilogue
       copies each finished block of output rows to pinned host memory as the grid runs
       (a device->host copy after the grid where the kernel's tensor-core path does not
       apply)

The host side of a step -- reserving pages, computing slots, lengths and the table changes --
runs in C (csrc/host_ops.cpp) on the PagedKVCache's own page tables and lands in pinned
staging buffers that the graph reads.  Two staging sets (and two graphs) alternate, so the
next step can be prepared while the current one runs.

    g = DecodeGraph(cache, seq_ids, num_q_heads=32)       # q_len=1 decode (or q_len=k+1)
    g.prepare()                                          # step 0's pages and slots
    q, k, v = g.inputs()                                 # pinned views: fill them
    g.launch()                                           # one replay; lengths advance
    g.prepare()                                          # next step, while this one runs
    torch.cuda.current_stream().synchronize()
    out = g.result()                                     # pinned [B, q_len, Hq, D]

While a DecodeGraph drives a batch, its sequences change only through prepare/launch and
DecodeGraph.rollback or PagedKVCache.truncate_batched / truncate_sequence (the rollback of a
verify window); other
page-table consumers (decode_metadata, plan_append) must not run on the same sequences.
A table that outgrows the captured capacity, or a step with more table changes than the
staging holds, is handled by re-uploading the table (and re-capturing when the capacity
grows) before the replay.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from .paged_attn import paged_attention_batched
from .paged_cache import _CLEAN, PagedKVCache, _hostops


class _HostRows:
    """A step's pinned host output as the one destination of the attention's epilogue copy
    (paged_attention_batched's `gather` protocol: device, rows, tail, dtype, begin,
    publish).  The kernel stores every finished block of rows to the host as 16-byte
    vectors while the rest of the grid runs, so no device-to-host copy follows the grid."""

    def __init__(self, host: torch.Tensor, device: torch.device) -> None:
        lib = _lib.load()
        dptr = ctypes.c_void_p()
        _lib.check(lib.inferd_host_device_pointer(host.data_ptr(), ctypes.byref(dptr)),
                   "host_device_pointer")
        self.device = device
        self.rows = host.shape[0]
        self.tail = tuple(host.shape[1:])
        self.dtype = host.dtype
        self._dst = torch.tensor([dptr.value], dtype=torch.int64, device=device)

    def begin(self) -> tuple[int, int, int]:
        return self._dst.data_ptr(), 1, 0

    def publish(self) -> None:
        pass


class DecodeGraph:
    """A step of a fixed batch of sequences of one PagedKVCache layer as a CUDA graph."""

    def __init__(self, cache: PagedKVCache, seq_ids: list[int], *, num_q_heads: int, q_len: int = 1,
                 layer: int = 0, scale: float | None = None, headroom_pages: int = 64,
                 copy_out: bool = True) -> None:
        if _hostops is None:
            raise RuntimeError("DecodeGraph needs the _hostops module (python -m inferd_b200.build)")
        if cache.device.type != "cuda":
            raise RuntimeError("DecodeGraph runs on CUDA pools only")
        if len(set(seq_ids)) != len(seq_ids) or not seq_ids:
            raise ValueError("seq_ids must be a non-empty list of distinct sequences")
        if num_q_heads % cache.num_kv_heads != 0:
            raise ValueError("num_q_heads must be a multiple of the cache's kv heads")
        cache._check_layer(layer)
        self.cache, self.ids, self.layer, self.q_len = cache, list(seq_ids), layer, int(q_len)
        self.tables = [cache._table(s) for s in self.ids]
        self.num_q_heads = num_q_heads
        self.scale = 1.0 / math.sqrt(cache.head_dim) if scale is None else float(scale)
        self.headroom = int(headroom_pages)
        self.copy_out = copy_out
        dev, dt = cache.device, cache.dtype
        b, ql, hkv, d = len(self.ids), self.q_len, cache.num_kv_heads, cache.head_dim
        self._b = b
        self._nq = b * ql * num_q_heads * d
        self._nk = b * ql * hkv * d
        n_in = self._nq + 2 * self._nk
        # per step each row gains at most ceil(q_len / block) + 1 pages and may lose as many
        self._max_pairs = b * (2 * (ql // cache.block_size + 2)) + 64
        n_meta = 2 * b + 1 + 2 * self._max_pairs
        # One staging area per set, [inputs | slots (int64) | lengths, row offsets, changes
        # (int32)], so a step's inputs cross the host link as ONE copy: each copy costs a
        # few microseconds of its own, which three small copies paid three times.
        es = torch.empty(0, dtype=dt).element_size()
        self._off_slots = _align(n_in * es)
        self._off_meta = _align(self._off_slots + b * ql * 8)
        self._nbytes = self._off_meta + n_meta * 4
        self._stage_h = [torch.empty(self._nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self._stage_d = torch.zeros(self._nbytes, dtype=torch.uint8, device=dev)
        self._inp_h, self._slots_h, self._meta_h = zip(*(self._views(h, n_in, n_meta) for h in self._stage_h))
        self._inp_d, self._slots_d, self._meta_d = self._views(self._stage_d, n_in, n_meta)
        for i in range(2):
            self._slots_h[i].fill_(-1)
            self._meta_h[i].zero_()
        self._out_h = [torch.empty((b, ql, num_q_heads, d), dtype=dt, pin_memory=True) for _ in range(2)]
        self._out_d = torch.empty((b, ql, num_q_heads, d), dtype=dt, device=dev)
        # the attention writes the pinned outputs itself when its tensor-core path applies
        # (decided by the first warm-up step); otherwise one copy follows it in the graph
        self._host_rows = None
        if copy_out:
            try:
                self._host_rows = [_HostRows(h, self._out_d.device) for h in self._out_h]
            except (ValueError, RuntimeError):
                self._host_rows = None
        self._events = [torch.cuda.Event(), torch.cuda.Event()]
        self._recorded = [False, False]
        self._set = 0            # staging set the next prepare/launch uses
        self._last = None        # set of the last launch
        self._prepared = None    # (set, reserved) between prepare and launch
        self._graphs: list[torch.cuda.CUDAGraph] = []
        self._master = None
        self._cap = 0
        self._build(max(len(t.blocks) for t in self.tables))

    # ------------------------------------------------------------ set-up
    def _views(self, buf: torch.Tensor, n_in: int, n_meta: int):
        """(inputs, slots, metadata) views of one staging byte buffer."""
        b, ql, dt = self._b, self.q_len, self.cache.dtype
        es = torch.empty(0, dtype=dt).element_size()
        return (buf[:n_in * es].view(dt),
                buf[self._off_slots:self._off_slots + b * ql * 8].view(torch.int64),
                buf[self._off_meta:self._off_meta + n_meta * 4].view(torch.int32))

    def _upload_dense(self) -> None:
        """Copy every table to the device master (stream-ordered after earlier replays)."""
        host = np.zeros((self._b, self._cap), dtype=np.int32)
        for i, t in enumerate(self.tables):
            host[i, :len(t.blocks)] = t.blocks
            t.dirty_from = _CLEAN
        self._master.copy_(torch.from_numpy(host).pin_memory(), non_blocking=True)
        self._prev_ids = [id(t.blocks) for t in self.tables]
        self._prev_nblk = [len(t.blocks) for t in self.tables]

    def _build(self, width: int) -> None:
        dev = self.cache.device
        self._cap = (width + self.headroom + 63) // 64 * 64
        self._master = torch.zeros((self._b, self._cap), dtype=torch.int32, device=dev)
        self._upload_dense()
        # staging that writes nothing: every slot -1 (skipped by the append), no table changes
        for i in range(2):
            self._slots_h[i].fill_(-1)
            self._meta_h[i].zero_()
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            for i in range(2):  # warm-up: kernel attributes and the attention workspace
                self._body(i)
        torch.cuda.current_stream(dev).wait_stream(stream)
        torch.cuda.synchronize(dev)
        self._graphs = []
        for i in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._body(i)
            self._graphs.append(g)
        torch.cuda.synchronize(dev)

    def _body(self, i: int) -> None:
        cache, b, ql, hq, d = self.cache, self._b, self.q_len, self.num_q_heads, self.cache.head_dim
        dev = cache.device
        self._stage_d.copy_(self._stage_h[i], non_blocking=True)
        lib = _lib.load()
        rp = self._meta_d[b:2 * b + 1]
        upd = self._meta_d[2 * b + 1:]
        _lib.check(lib.inferd_block_tables_refresh(self._master.data_ptr(), self._cap, rp.data_ptr(),
                                                   upd.data_ptr(), 0, b, 0, self._master.data_ptr(),
                                                   _lib.stream_of(dev)), "block_tables_refresh")
        q = self._inp_d[:self._nq].view(b, ql, hq, d)
        k = self._inp_d[self._nq:self._nq + self._nk].view(b * ql, cache.num_kv_heads, d)
        v = self._inp_d[self._nq + self._nk:].view(b * ql, cache.num_kv_heads, d)
        cache._write(self.layer, k, v, self._slots_d)
        args = (q, cache.key_cache[self.layer], cache.value_cache[self.layer], self._master,
                self._meta_d[:b])
        kw = dict(scale=self.scale, max_context_len=self._cap * cache.block_size, out=self._out_d)
        if self._host_rows is not None:
            try:
                paged_attention_batched(*args, gather=self._host_rows[i], **kw)
                return
            except ValueError:  # shapes outside the tensor-core path: copy after the grid
                self._host_rows = None
        paged_attention_batched(*args, **kw)
        if self.copy_out:
            self._out_h[i].copy_(self._out_d, non_blocking=True)

    # ------------------------------------------------------------ steps
    def inputs(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Pinned views (q [B, q_len, Hq, D], k and v [B * q_len, Hkv, D]) of the staging set
        the next launch reads; fill them between prepare and launch."""
        h = self._inp_h[self._set]
        b, ql, d = self._b, self.q_len, self.cache.head_dim
        return (h[:self._nq].view(b, ql, self.num_q_heads, d),
                h[self._nq:self._nq + self._nk].view(b * ql, self.cache.num_kv_heads, d),
                h[self._nq + self._nk:].view(b * ql, self.cache.num_kv_heads, d))

    def input_buffers(self) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """The pinned (q, k, v) views of both staging sets, for callers that stage inputs
        ahead; launch i reads set i % 2."""
        out = []
        for i in range(2):
            self._set, cur = i, self._set
            out.append(self.inputs())
            self._set = cur
        return out

    def prepare(self) -> None:
        """Reserve the next step's pages and stage its slots, lengths and table changes (host
        work only; MemoryError leaves the cache unchanged)."""
        if self._prepared is not None:
            raise RuntimeError("a step is already prepared")
        i = self._set
        if self._recorded[i]:
            self._events[i].synchronize()  # the replay that last read this set is done
        cache, b, ql, bs = self.cache, self._b, self.q_len, self.cache.block_size
        slots = self._slots_h[i].numpy()
        reserved, failed = _hostops.plan_slots(self.tables, ql, bs, cache.allocator._free,
                                               cache.allocator._allocated, slots)
        if failed >= 0:
            t = self.tables[failed]
            need = (t.length + ql + bs - 1) // bs - len(t.blocks)
            msg = f"requested {need} blocks, only {cache.allocator.free_count} free"
            for tt, nb in reversed(reserved):
                cache._rollback(tt, nb)
            raise MemoryError(msg)
        meta = self._meta_h[i].numpy()
        nblk, width, _ = _hostops.scan(self.tables, ql, meta[:b])
        if width > self._cap:
            # a table outgrew the captured capacity: new master and graphs (the rebuild
            # sends every table whole and resets the staging, so keep this step's slots)
            saved_slots, saved_lens = slots.copy(), meta[:b].copy()
            self._rebuild_for(width, i)
            slots[:] = saved_slots
            meta[:b] = saved_lens
        # row offsets and (column, block) pairs of the table changes, written in place
        total, ids, _ = _hostops.pack_staged(self.tables, self._prev_ids, self._prev_nblk, _CLEAN,
                                             meta[b:2 * b + 1], meta[2 * b + 1:])
        if total > self._max_pairs:
            # more changes than the staging holds: send the whole table before the replay
            meta[b:2 * b + 1] = 0
            self._upload_dense()
        else:
            self._prev_ids, self._prev_nblk = ids, nblk
        self._prepared = (i, reserved)

    def _rebuild_for(self, width: int, i: int) -> None:
        torch.cuda.synchronize(self.cache.device)
        self._build(width)
        self._recorded = [False, False]

    def launch(self) -> None:
        """Replay the prepared step on the current stream; the lengths advance (the K/V of
        these tokens are written in stream order)."""
        if self._prepared is None:
            raise RuntimeError("prepare() the step first")
        i, _ = self._prepared
        self._graphs[i].replay()
        self._events[i].record(torch.cuda.current_stream(self.cache.device))
        self._recorded[i] = True
        _hostops.advance(self.tables, self.q_len)
        self._prepared = None
        self._last = i
        self._set = i ^ 1

    def rollback(self, keep) -> list[int]:
        """Roll back the verify window of the last launched step: sequence i keeps the first
        keep[i] (0 .. q_len) tokens of the window and releases the rest, with any pages only
        they used (PagedKVCache.truncate_batched on this graph's sequences, without the
        per-sequence lookups).  Call it between launch() and the next prepare(); the pages
        it frees are reused only by later steps, which the stream orders after this one.
        Returns the freed blocks."""
        if self._prepared is not None:
            raise RuntimeError("rollback() comes before prepare()")
        if self._last is None:
            raise RuntimeError("no step has been launched")
        if len(keep) != len(self.tables):
            raise ValueError("one keep count per sequence")
        ql = self.q_len
        lengths = []
        for t, k in zip(self.tables, keep):
            k = int(k)
            if k < 0 or k > ql:
                raise ValueError(f"keep counts lie in 0 .. {ql}")
            lengths.append(t.length - ql + k)
        cache = self.cache
        return _hostops.truncate(self.tables, lengths, cache.block_size, cache.allocator._free,
                                 cache.allocator._allocated)

    def abort(self) -> None:
        """Release the pages of a prepared step that will not be launched."""
        if self._prepared is None:
            return
        _, reserved = self._prepared
        for t, nb in reversed(reserved):
            self.cache._rollback(t, nb)
        self._prepared = None

    def result(self) -> torch.Tensor:
        """The last launch's output in pinned host memory ([B, q_len, Hq, D]); read it after
        the stream has synchronised."""
        if self._last is None:
            raise RuntimeError("no step has been launched")
        return self._out_h[self._last]

    @property
    def output(self) -> torch.Tensor:
        """The last launch's output on the device."""
        return self._out_d

    def staged_bytes(self) -> int:
        """Host-to-device bytes one replay copies (inputs, slots, lengths and changes, with
        the alignment gaps between them)."""
        return self._nbytes


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a
