"""Host-side logic of inferd_b200 on CPU: allocator, page tables, validation, rollback.

The allocator and page-table semantics are pinned to a trace recorded from the
reference's PagedKVCache (tests/golden/cache_trace.json, made by
tests/golden/make_golden.py).  K/V writes are replaced by a recording stub here; the
kernels themselves are covered by the gpu-marked tests.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from inferd_b200.paged_cache import BlockAllocator, PagedKVCache, SequencePageTable


class RecordingCache(PagedKVCache):
    """PagedKVCache whose K/V writes are recorded instead of launched."""

    def __init__(self, *a, fail_write=False, **k):
        super().__init__(*a, **k)
        self.writes = []
        self.fail_write = fail_write

    def _write(self, layer, keys, values, slots):
        if self.fail_write:
            raise RuntimeError("injected write failure")
        self.writes.append((layer, slots.tolist()))


def test_allocator_lifo_and_errors():
    a = BlockAllocator(4)
    assert a.allocate(2) == [0, 1]
    a.free([1, 0])
    assert a.allocate(2) == [0, 1]
    with pytest.raises(MemoryError):
        a.allocate(3)
    with pytest.raises(ValueError):
        a.allocate(-1)
    with pytest.raises(ValueError):
        a.free([0, 0])
    with pytest.raises(ValueError):
        a.free([3])
    with pytest.raises(ValueError):
        BlockAllocator(0)


def test_reuse_order_matches_reference(cache_trace):
    cache = RecordingCache(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    cache.create_sequence(1)
    cache.create_sequence(2)
    one = [torch.ones(3, 1, 1)]
    cache.append_tokens(1, one, one)
    first = list(cache.sequences[1].blocks)
    cache.free_sequence(1)
    cache.append_tokens(2, one, one)
    assert first == cache_trace["reuse"]["first"]
    assert cache.sequences[2].blocks == cache_trace["reuse"]["second"] == first[::-1]


def test_random_trace_matches_reference(cache_trace):
    cache = RecordingCache(num_layers=2, num_blocks=cache_trace["num_blocks"],
                           block_size=cache_trace["block_size"], num_kv_heads=1, head_dim=2,
                           dtype=torch.float32)
    for op in cache_trace["ops"]:
        if op["op"] == "create":
            cache.create_sequence(op["seq"])
        elif op["op"] == "append":
            kv = [torch.zeros(op["n"], 1, 2) for _ in range(2)]
            try:
                cache.append_tokens(op["seq"], kv, kv)
                res = "ok"
            except MemoryError:
                res = "MemoryError"
            assert res == op["result"]
            t = cache.sequences[op["seq"]]
            assert t.blocks == op["blocks"]
            assert t.length == op["length"]
            assert cache.allocator.free_count == op["free"]
        else:
            cache.free_sequence(op["seq"])
            assert cache.allocator.free_count == op["free"]
        cache.assert_consistent()


def test_slots_follow_page_table():
    cache = RecordingCache(num_layers=2, num_blocks=8, block_size=4, num_kv_heads=1, head_dim=2,
                           dtype=torch.float32)
    cache.create_sequence(0)
    cache.create_sequence(1)
    cache.append_tokens(1, [torch.zeros(2, 1, 2)] * 2, [torch.zeros(2, 1, 2)] * 2)
    cache.append_tokens(0, [torch.zeros(6, 1, 2)] * 2, [torch.zeros(6, 1, 2)] * 2)
    # seq 1 owns block 0, seq 0 owns blocks 1, 2: slot = block * 4 + offset
    assert cache.writes[-1] == (1, [4, 5, 6, 7, 8, 9])
    assert cache.sequences[0].slots(4, 2) == [8, 9]
    assert cache.sequences[0].block_for_pos(5) == (2, 1)
    with pytest.raises(IndexError):
        cache.sequences[0].block_for_pos(6)


def test_batched_append_is_all_or_nothing():
    cache = RecordingCache(num_layers=1, num_blocks=3, block_size=2, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    for s in range(3):
        cache.create_sequence(s)
    kv = [torch.zeros(6, 1, 1)]   # 2 tokens each -> one block each
    cache.append_tokens_batched([0, 1, 2], kv, kv)
    assert [cache.sequence_length(s) for s in range(3)] == [2, 2, 2]
    assert cache.writes[-1][1] == [0, 1, 2, 3, 4, 5]
    with pytest.raises(MemoryError):   # needs 3 more blocks, none free
        cache.append_tokens_batched([0, 1, 2], kv, kv)
    assert [len(cache.sequences[s].blocks) for s in range(3)] == [1, 1, 1]
    assert cache.allocator.free_count == 0
    cache.assert_consistent()


def test_write_failure_rolls_back_new_blocks():
    cache = RecordingCache(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32, fail_write=True)
    cache.create_sequence(0)
    with pytest.raises(RuntimeError):
        cache.append_tokens(0, [torch.zeros(3, 1, 1)], [torch.zeros(3, 1, 1)])
    assert cache.sequences[0].blocks == [] and cache.sequence_length(0) == 0
    assert cache.allocator.free_count == 4


def test_cpu_cache_has_no_cpu_fallback():
    cache = PagedKVCache(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1, head_dim=1,
                         dtype=torch.float32)
    cache.create_sequence(0)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cache.append_tokens(0, [torch.zeros(3, 1, 1)], [torch.zeros(3, 1, 1)])
    assert cache.sequences[0].blocks == [] and cache.allocator.free_count == 4


def test_validation_errors_match_reference():
    cache = RecordingCache(num_layers=2, num_blocks=4, block_size=2, num_kv_heads=2, head_dim=3,
                           dtype=torch.float32)
    cache.create_sequence(0)
    with pytest.raises(ValueError):
        cache.create_sequence(0)
    with pytest.raises(KeyError):
        cache.append_tokens(9, [], [])
    with pytest.raises(ValueError):
        cache.append_tokens(0, [torch.zeros(1, 2, 3)], [torch.zeros(1, 2, 3)])
    with pytest.raises(ValueError):
        cache.append_tokens(0, [torch.zeros(1, 2, 4)] * 2, [torch.zeros(1, 2, 4)] * 2)
    with pytest.raises(ValueError):
        cache.append_tokens(0, [torch.zeros(1, 2, 3), torch.zeros(2, 2, 3)],
                            [torch.zeros(1, 2, 3)] * 2)
    with pytest.raises(IndexError):
        cache.gather_layer(0, 2)
    for bad in (dict(num_layers=0), dict(block_size=0), dict(num_kv_heads=0)):
        kw = dict(num_layers=1, num_blocks=4, block_size=2, num_kv_heads=1, head_dim=1)
        kw.update(bad)
        with pytest.raises(ValueError):
            PagedKVCache(**kw)
    cache.append_tokens(0, [torch.zeros(0, 2, 3)] * 2, [torch.zeros(0, 2, 3)] * 2)
    assert cache.writes == []


def test_decode_metadata_packing():
    cache = RecordingCache(num_layers=1, num_blocks=16, block_size=4, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    for s, n in [(0, 5), (1, 1), (2, 12)]:
        cache.create_sequence(s)
        cache.append_tokens(s, [torch.zeros(n, 1, 1)], [torch.zeros(n, 1, 1)])
    bt, cl, mx = cache.decode_metadata([2, 0, 1])
    assert bt.dtype == torch.int32 and cl.dtype == torch.int32
    assert bt.tolist() == [[3, 4, 5], [0, 1, 0], [2, 0, 0]]
    assert cl.tolist() == [12, 5, 1] and mx == 12
    bt, cl, mx = cache.decode_metadata([1], extra_tokens=3, pad_pages=4)
    assert bt.shape == (1, 4) and cl.tolist() == [4] and mx == 4


def test_sequence_page_table_properties():
    t = SequencePageTable(seq_id=0, block_size=4, blocks=[3, 1], length=5)
    assert t.block_count == 2 and t.capacity_tokens == 8 and t.free_slots == 3


def test_truncate_sequence_rolls_back_without_copies():
    cache = RecordingCache(num_layers=1, num_blocks=8, block_size=4, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    cache.create_sequence(0)
    cache.append_tokens(0, [torch.zeros(10, 1, 1)], [torch.zeros(10, 1, 1)])
    assert cache.sequences[0].blocks == [0, 1, 2]
    n_writes = len(cache.writes)
    assert cache.truncate_sequence(0, 5) == [2]
    assert cache.sequence_length(0) == 5 and cache.sequences[0].blocks == [0, 1]
    assert len(cache.writes) == n_writes          # no K/V movement
    assert cache.truncate_sequence(0, 5) == []
    with pytest.raises(ValueError):
        cache.truncate_sequence(0, 6)
    cache.append_tokens(0, [torch.zeros(4, 1, 1)], [torch.zeros(4, 1, 1)])
    assert cache.sequences[0].blocks == [0, 1, 2]  # the freed block is reused first
    assert cache.writes[-1][1] == [5, 6, 7, 8]
    cache.assert_consistent()


def test_decode_metadata_incremental_rows_match_rebuild():
    # the host table is updated row by row between calls; it must always equal a table
    # rebuilt from the page tables (appends, block-crossing growth, truncation, reordering)
    cache = RecordingCache(num_layers=1, num_blocks=400, block_size=4, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    rng = np.random.default_rng(3)
    ids = list(range(6))
    for s in ids:
        cache.create_sequence(s)
        n = int(rng.integers(1, 30))
        cache.append_tokens(s, [torch.zeros(n, 1, 1)], [torch.zeros(n, 1, 1)])

    def rebuilt(order, extra=0):
        width = max(len(cache.sequences[s].blocks) for s in order)
        rows = [cache.sequences[s].blocks + [0] * (width - len(cache.sequences[s].blocks)) for s in order]
        return rows, [cache.sequences[s].length + extra for s in order]

    for step in range(120):
        cache.append_tokens_batched(ids, [torch.zeros(len(ids), 1, 1)], [torch.zeros(len(ids), 1, 1)])
        if step % 9 == 4:
            s = int(rng.integers(0, len(ids)))
            cache.truncate_sequence(s, max(0, cache.sequence_length(s) - int(rng.integers(1, 9))))
        order = ids if step % 17 else ids[::-1]
        bt, cl, mx = cache.decode_metadata(order)
        rows, lens = rebuilt(order)
        assert bt.tolist() == rows and cl.tolist() == lens and mx == max(lens)


def test_decode_metadata_sparse_updates_after_rollbacks_across_sequences():
    # rollbacks of several sequences, then re-growth, hand freed blocks between sequences
    # (LIFO): rows whose last block is unchanged but whose middle moved must still be right
    cache = RecordingCache(num_layers=1, num_blocks=64, block_size=2, num_kv_heads=1, head_dim=1,
                           dtype=torch.float32)
    ids = [0, 1, 2]
    for s, n in zip(ids, (7, 5, 9)):
        cache.create_sequence(s)
        cache.append_tokens(s, [torch.zeros(n, 1, 1)], [torch.zeros(n, 1, 1)])
    rng = np.random.default_rng(11)
    for step in range(200):
        for s in ids:
            if rng.random() < 0.4:
                cache.truncate_sequence(s, int(rng.integers(0, cache.sequence_length(s) + 1)))
        per = int(rng.integers(1, 4))
        cache.append_tokens_batched(ids, [torch.zeros(3 * per, 1, 1)], [torch.zeros(3 * per, 1, 1)])
        if step % 23 == 7:  # a table replaced from outside the class
            t = cache.sequences[1]
            t.blocks = list(t.blocks)
        bt, cl, mx = cache.decode_metadata(ids, extra_tokens=step % 2)
        width = max(len(cache.sequences[s].blocks) for s in ids)
        rows = [cache.sequences[s].blocks + [0] * (width - len(cache.sequences[s].blocks)) for s in ids]
        assert bt.tolist() == rows
        assert cl.tolist() == [cache.sequence_length(s) + step % 2 for s in ids]
    cache.assert_consistent()


def test_truncate_batched_matches_per_sequence_truncation():
    rng = np.random.default_rng(2)
    a = RecordingCache(num_layers=1, num_blocks=300, block_size=4, num_kv_heads=1, head_dim=1,
                       dtype=torch.float32)
    b = RecordingCache(num_layers=1, num_blocks=300, block_size=4, num_kv_heads=1, head_dim=1,
                       dtype=torch.float32)
    ids = [3, 1, 4, 0]
    for cache in (a, b):
        for s in ids:
            cache.create_sequence(s)
    for step in range(60):
        per = int(rng.integers(1, 7))
        for cache in (a, b):
            cache.append_tokens_batched(ids, [torch.zeros(4 * per, 1, 1)], [torch.zeros(4 * per, 1, 1)])
        lens = [int(rng.integers(0, a.sequence_length(s) + 1)) for s in ids]
        freed = a.truncate_batched(ids, lens)
        freed_ref = []
        for s, n in zip(ids, lens):
            freed_ref += b.truncate_sequence(s, n)
        assert freed == freed_ref
        assert [a.sequences[s].blocks for s in ids] == [b.sequences[s].blocks for s in ids]
        assert a.allocator._free == b.allocator._free
    with pytest.raises(ValueError):  # checked before any table changes
        a.truncate_batched(ids, [0, 0, 0, a.sequence_length(0) + 1])
    assert [a.sequence_length(s) for s in ids] == [b.sequence_length(s) for s in ids]
    with pytest.raises(ValueError):
        a.truncate_batched(ids, [0])
    a.assert_consistent()


def test_plan_and_commit_equal_append_then_metadata():
    from inferd_b200.paged_cache import AppendPlan  # noqa: F401
    rng = np.random.default_rng(4)
    a = RecordingCache(num_layers=2, num_blocks=200, block_size=4, num_kv_heads=1, head_dim=1,
                       dtype=torch.float32)
    b = RecordingCache(num_layers=2, num_blocks=200, block_size=4, num_kv_heads=1, head_dim=1,
                       dtype=torch.float32)
    ids = [5, 2, 9]
    for cache in (a, b):
        for s in ids:
            cache.create_sequence(s)
    for step in range(40):
        per = int(rng.integers(1, 6))
        kv = [torch.zeros(3 * per, 1, 1)] * 2
        plan = a.plan_append(ids, per)
        a.commit_append(plan, kv, kv)
        b.append_tokens_batched(ids, kv, kv)
        bt, cl, mx = b.decode_metadata(ids)
        assert plan.block_tables.tolist() == bt.tolist() and plan.context_lens.tolist() == cl.tolist()
        assert plan.max_context_len == mx and a.writes[-1] == b.writes[-1]
        assert [a.sequences[s].blocks for s in ids] == [b.sequences[s].blocks for s in ids]
        with pytest.raises(ValueError):
            a.commit_append(plan, kv, kv)
    # abort releases the reservation; a failed commit aborts
    free = a.allocator.free_count
    plan = a.plan_append(ids, 9)
    assert a.allocator.free_count < free
    a.abort_append(plan)
    assert a.allocator.free_count == free and [a.sequence_length(s) for s in ids] == [b.sequence_length(s) for s in ids]
    plan = a.plan_append(ids, 2)
    with pytest.raises(ValueError):
        a.commit_append(plan, [torch.zeros(5, 1, 1)] * 2, [torch.zeros(5, 1, 1)] * 2)
    assert a.allocator.free_count == free
    with pytest.raises(MemoryError):
        a.plan_append(ids, 10_000)
    assert a.allocator.free_count == free
    a.assert_consistent()


def test_native_page_table_loops_match_python():
    # csrc/host_ops.cpp walks the same Python page tables and allocator as the pure-Python
    # loops: identical tables, free lists, slots and metadata on a random decode / verify /
    # rollback sequence, including an exhausted pool (MemoryError with nothing taken)
    from inferd_b200 import paged_cache
    if paged_cache._hostops is None:
        pytest.skip("_hostops not built")
    caches = {}
    for native in (True, False):
        caches[native] = RecordingCache(num_layers=1, num_blocks=120, block_size=4, num_kv_heads=1,
                                        head_dim=1, dtype=torch.float32)
    ids = [7, 3, 11, 5]

    def run(native, fn):
        old = paged_cache._NATIVE
        paged_cache._NATIVE = native
        try:
            return fn(caches[native])
        except MemoryError as e:
            return ("MemoryError", str(e))
        finally:
            paged_cache._NATIVE = old

    for native in (True, False):
        for s in ids:
            caches[native].create_sequence(s)
    rng = np.random.default_rng(17)
    for step in range(300):
        per = int(rng.choice([1, 1, 2, 5, 9]))
        def plan_commit(c, per=per):
            plan = c.plan_append(ids, per)
            c.commit_append(plan, [torch.zeros(4 * per, 1, 1)], [torch.zeros(4 * per, 1, 1)])
            return (plan.slots.tolist(), plan.block_tables.tolist(), plan.context_lens.tolist(),
                    plan.max_context_len)
        a, b = run(True, plan_commit), run(False, plan_commit)
        assert a == b, f"step {step}"
        if rng.random() < 0.5:
            lens = [int(rng.integers(0, caches[True].sequence_length(s) + 1)) for s in ids]
            fa = run(True, lambda c: c.truncate_batched(ids, lens))
            fb = run(False, lambda c: c.truncate_batched(ids, lens))
            assert fa == fb
        if step % 50 == 25:  # the pool runs out part-way: earlier tables' pages roll back
            free = caches[True].allocator.free_count
            big = 4 * (free // 3 + 1)
            def plan_big(c, big=big):
                c.plan_append(ids, big)
            ea, eb = run(True, plan_big), run(False, plan_big)
            assert ea == eb and ea is not None and ea[0] == "MemoryError"
            assert caches[True].allocator.free_count == free
        if step % 37 == 5:  # a list replaced from outside the class
            for native in (True, False):
                t = caches[native].sequences[3]
                t.blocks = list(t.blocks)
        ma = run(True, lambda c: [x.tolist() if hasattr(x, "tolist") else x for x in c.decode_metadata(ids)])
        mb = run(False, lambda c: [x.tolist() if hasattr(x, "tolist") else x for x in c.decode_metadata(ids)])
        assert ma == mb
        assert [caches[True].sequences[s].blocks for s in ids] == [caches[False].sequences[s].blocks for s in ids]
        assert caches[True].allocator._free == caches[False].allocator._free
        assert caches[True].allocator._allocated == caches[False].allocator._allocated
    for native in (True, False):
        caches[native].assert_consistent()
    with pytest.raises(ValueError):
        run(True, lambda c: c.truncate_batched(ids, [10 ** 6] * 4))


def test_pack_staged_matches_pack_changes():
    # DecodeGraph's staging path: pack_staged writes the exclusive row offsets and the
    # (column, block) pairs in place; it must equal pack_changes + a prefix sum, and past
    # the pairs buffer's capacity it counts without writing
    from inferd_b200.paged_cache import _CLEAN, _hostops
    if _hostops is None:
        pytest.skip("_hostops not built")
    rng = np.random.default_rng(23)

    def make():
        tabs = []
        for s in range(6):
            t = SequencePageTable(seq_id=s, block_size=4)
            t.blocks = [int(x) for x in rng.integers(0, 1000, int(rng.integers(0, 9)))]
            t.length = 4 * len(t.blocks)
            t.dirty_from = _CLEAN
            tabs.append(t)
        return tabs

    a = make()
    b = [SequencePageTable(seq_id=t.seq_id, block_size=4, blocks=list(t.blocks), length=t.length) for t in a]
    for t in b:
        t.dirty_from = _CLEAN
    prev_a = ([id(t.blocks) for t in a], [len(t.blocks) for t in a])
    prev_b = ([id(t.blocks) for t in b], [len(t.blocks) for t in b])
    for step in range(200):
        for ta, tb in zip(a, b):  # the same random tail edits on both sets
            r = rng.random()
            if r < 0.3:
                new = [int(x) for x in rng.integers(0, 1000, int(rng.integers(1, 4)))]
                for t in (ta, tb):
                    t.dirty_from = min(t.dirty_from, len(t.blocks))
                    t.blocks.extend(new)
            elif r < 0.5 and ta.blocks:
                keep = int(rng.integers(0, len(ta.blocks)))
                for t in (ta, tb):
                    del t.blocks[keep:]
                    t.dirty_from = min(t.dirty_from, keep)
            elif r < 0.55:
                ta.blocks = list(ta.blocks)  # a list replaced from outside
                tb.blocks = list(tb.blocks)
        counts = np.zeros(len(a), dtype=np.int32)
        pairs, ids_a, nb_a = _hostops.pack_changes(a, prev_a[0], prev_a[1], _CLEAN, counts)
        want_pairs = np.frombuffer(pairs, dtype=np.int32)
        want_rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        cap = int(rng.choice([0, 3, 1000]))
        rp = np.full(len(b) + 1, -7, dtype=np.int32)
        buf = np.full(2 * cap, -7, dtype=np.int32)
        total, ids_b, nb_b = _hostops.pack_staged(b, prev_b[0], prev_b[1], _CLEAN, rp, buf)
        assert total == want_pairs.size // 2
        assert np.array_equal(rp, want_rp)
        n_written = min(total, cap)
        assert np.array_equal(buf[:2 * n_written], want_pairs[:2 * n_written])
        assert np.all(buf[2 * n_written:] == -7)
        assert nb_a == nb_b and [t.dirty_from for t in a] == [t.dirty_from for t in b] == [_CLEAN] * len(a)
        prev_a, prev_b = (ids_a, nb_a), (ids_b, nb_b)


def test_native_loops_reject_mistyped_buffers():
    # the native loops read and write their buffers as int32 / int64: a view of another
    # item size or kind is refused before anything is read or written
    from inferd_b200.paged_cache import _CLEAN, _hostops
    if _hostops is None:
        pytest.skip("_hostops not built")
    tabs = []
    for s in range(3):
        t = SequencePageTable(seq_id=s, block_size=4, blocks=[s, s + 3], length=7)
        t.dirty_from = 0
        tabs.append(t)
    for bad in (np.zeros(3, np.int64), np.zeros(3, np.float32), np.zeros(3, np.uint32),
                np.zeros(12, np.uint8)):
        with pytest.raises(TypeError):
            _hostops.scan(tabs, 0, bad)
    ids, nblk = [0] * 3, [0] * 3
    with pytest.raises(TypeError):
        _hostops.pack_staged(tabs, ids, nblk, _CLEAN, np.zeros(4, np.int32), np.zeros(8, np.float32))
    with pytest.raises(TypeError):
        _hostops.pack_staged(tabs, ids, nblk, _CLEAN, np.zeros(4, np.int64), np.zeros(8, np.int32))
    with pytest.raises(TypeError):
        _hostops.plan_slots(tabs, 1, 4, [9, 10], set(range(9)), np.zeros(3, np.int32))
    # the right types still work, and nothing above changed the tables
    lens = np.zeros(3, np.int32)
    nb, width, mx = _hostops.scan(tabs, 1, lens)
    assert lens.tolist() == [8, 8, 8] and nb == [2, 2, 2] and width == 2 and mx == 8
    assert [t.dirty_from for t in tabs] == [0, 0, 0]
