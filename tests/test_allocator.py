"""The native page allocator (tkv_allocator_*, host only) against the
reference CudaAllocator's bookkeeping rules (cuda_allocator.cpp): lowest page
id first and LIFO reuse (:97-99,120-127), all-or-nothing allocation
(:129-158), reference-counted sharing (:187-203), -1 padded tables (:231-253),
eviction that releases pages and keeps their count (:318-378).  KIVI
specifics: n_q(L)/16 pages per sequence, one ring row per live sequence.
Also a seeded random operation sequence checked step by step against a
Python model, and concurrent use from threads.
"""
import importlib
import threading

import numpy as np
import pytest

L = importlib.import_module("truellm-engine_b200._lib")
A = importlib.import_module("truellm-engine_b200.allocator")
ops = importlib.import_module("truellm-engine_b200.ops")

FMT = ops.KiviFormat(128, 128, 128, 4, 8)     # G = R = 128: 8 pages per key group


def make(num_pages=64, max_seqs=4, width=32):
    return A.PageAllocator(FMT, num_pages, max_seqs, width)


def test_create_rejects_bad_arguments():
    with pytest.raises(L.TkvError):
        A.PageAllocator(FMT, 0, 4, 8)
    with pytest.raises(L.TkvError):
        A.PageAllocator(FMT, 8, 0, 8)
    a = make()
    assert a.stats()["blocks_free"] == 64 and a.stats()["rows_free"] == 4


@pytest.mark.parametrize("length,pages", [(0, 0), (100, 0), (255, 0), (256, 8), (383, 8),
                                          (384, 16), (1000, 48)])
def test_pages_cover_whole_key_groups_only(length, pages):
    a = make()
    assert a.pages_for(length) == pages == FMT.quantized_len(length) // 16


def test_lowest_ids_first_and_lifo_reuse():
    a = make()
    assert a.allocate_sequence(1, 256) and a.allocate_sequence(2, 256)
    bt, lens, rows = a.block_tables([1, 2])
    assert list(bt[0, :8]) == list(range(8)) and list(bt[1, :8]) == list(range(8, 16))
    assert (bt[:, 8:] == -1).all() and list(lens) == [256, 256] and list(rows) == [0, 1]
    a.free_sequence(1)
    assert a.allocate_sequence(3, 256)
    bt, _, rows = a.block_tables([3])
    assert sorted(bt[0, :8]) == list(range(8)) and rows[0] == 0   # freed pages and row reused


def test_all_or_nothing():
    a = make(num_pages=20, max_seqs=2)
    assert a.allocate_sequence(1, 256)                  # 8 pages
    before = a.stats()
    assert not a.allocate_sequence(2, 384)              # 16 > 12 free
    assert not a.allocate_sequence(1, 0)                # duplicate id
    assert not a.allocate_sequence(3, 16 * 33 + 128)    # beyond the table width
    assert a.stats() == before
    assert a.allocate_sequence(2, 200)                  # 0 pages, a ring row
    assert not a.allocate_sequence(3, 0)                # out of ring rows
    assert a.extend_sequence(2, 384) == -1              # 16 pages > 12 free: unchanged
    assert a.sequence(2) == {"len": 200, "n_pages": 0, "ring_row": 1, "evicted": False}
    assert a.extend_sequence(2, 256) == 8 and a.extend_sequence(2, 300) == 0
    assert a.extend_sequence(2, 299) == -1              # shorter
    assert a.extend_sequence(9, 300) == -1              # unknown
    assert a.stats()["blocks_free"] == 4


def test_fork_shares_pages_by_count():
    a = make()
    assert a.allocate_sequence(1, 384)
    src_row, dst_row = a.fork(1, 2)
    assert (src_row, dst_row) == (0, 1)
    s = a.stats()
    assert (s["blocks_used"], s["blocks_shared"], s["sequences"]) == (16, 16, 2)
    bt, lens, rows = a.block_tables([1, 2])
    assert (bt[0] == bt[1]).all() and list(lens) == [384, 384] and list(rows) == [0, 1]
    assert a.extend_sequence(2, 512) == 8               # dst grows on pages of its own
    bt, _, _ = a.block_tables([1, 2])
    assert set(bt[1, 16:24]).isdisjoint(bt[0, :16])
    a.free_sequence(1)
    assert a.stats()["blocks_used"] == 24 and a.stats()["blocks_shared"] == 0
    a.free_sequence(2)
    assert a.stats()["blocks_used"] == 0 and a.stats()["rows_free"] == 4
    with pytest.raises(L.TkvError):
        a.fork(7, 8)                                    # unknown source
    assert not a.copy_sequence(7, 8)
    a.free_sequence(7)                                  # unknown: no-op


def test_tables_reject_unknown_and_evicted():
    a = make()
    assert a.allocate_sequence(1, 256)
    with pytest.raises(L.TkvError):
        a.block_tables([1, 5])
    a.evict(1)
    with pytest.raises(L.TkvError):
        a.block_tables([1])


def test_evict_and_reload():
    a = make(num_pages=24, max_seqs=2)
    assert a.allocate_sequence(1, 384) and a.allocate_sequence(2, 256)
    pages, row = a.evict(1)
    assert list(pages) == list(range(16)) and row == 0
    info = a.sequence(1)
    assert info["evicted"] and info["n_pages"] == 16 and info["ring_row"] == -1
    assert a.stats()["blocks_free"] == 16 and a.stats()["evicted"] == 1
    with pytest.raises(L.TkvError):
        a.evict(1)
    assert a.extend_sequence(1, 512) == -1              # evicted: no growth
    assert a.allocate_sequence(3, 256)                  # takes 8 of the released pages
    with pytest.raises(L.TkvError) as e:                # 8 free < 16 and no ring row
        a.reload(1)
    assert e.value.status == L.TKV_OUT_OF_MEMORY and a.sequence(1)["evicted"]
    a.free_sequence(3)
    pages2, row2 = a.reload(1)
    assert len(pages2) == 16 and row2 >= 0 and not a.sequence(1)["evicted"]
    bt, lens, _ = a.block_tables([1])
    assert list(bt[0, :16]) == list(pages2) and lens[0] == 384


def test_fork_then_evict_keeps_the_sharer():
    a = make()
    assert a.allocate_sequence(1, 256)
    a.fork(1, 2)
    pages, _ = a.evict(1)
    assert a.stats()["blocks_used"] == 8               # still held by 2
    bt, _, _ = a.block_tables([2])
    assert list(bt[0, :8]) == list(pages)


class Model:
    """Python restatement of the allocator's rules, for the random walk."""

    def __init__(self, num_pages, max_seqs, width):
        self.free = list(range(num_pages))[::-1]
        self.rows = list(range(max_seqs))[::-1]
        self.refs = [0] * num_pages
        self.seqs = {}
        self.width = width

    def pages_for(self, n):
        return FMT.quantized_len(n) // 16

    def take(self):
        p = self.free.pop()
        self.refs[p] = 1
        return p

    def release(self, p):
        self.refs[p] -= 1
        if self.refs[p] == 0:
            self.free.append(p)

    def add(self, i, n):
        k = self.pages_for(n)
        if i in self.seqs or k > self.width or k > len(self.free) or not self.rows:
            return False
        self.seqs[i] = {"pages": [self.take() for _ in range(k)], "len": n,
                        "row": self.rows.pop(), "ev": 0}
        return True

    def extend(self, i, n):
        s = self.seqs.get(i)
        k = self.pages_for(n)
        if s is None or s["ev"] or n < s["len"] or k > self.width:
            return -1
        need = k - len(s["pages"])
        if need > len(self.free):
            return -1
        s["pages"] += [self.take() for _ in range(need)]
        s["len"] = n
        return max(need, 0)

    def free_seq(self, i):
        s = self.seqs.pop(i, None)
        if s is None:
            return
        for p in s["pages"]:
            self.release(p)
        if s["row"] >= 0:
            self.rows.append(s["row"])

    def fork(self, i, j):
        s = self.seqs.get(i)
        if s is None or s["ev"] or j in self.seqs or i == j or not self.rows:
            return False
        for p in s["pages"]:
            self.refs[p] += 1
        self.seqs[j] = {"pages": list(s["pages"]), "len": s["len"], "row": self.rows.pop(),
                        "ev": 0}
        return True

    def evict(self, i):
        s = self.seqs.get(i)
        if s is None or s["ev"]:
            return False
        for p in s["pages"]:
            self.release(p)
        self.rows.append(s["row"])
        s["ev"], s["pages"], s["row"] = len(s["pages"]) or -1, [], -1
        return True

    def reload(self, i):
        s = self.seqs.get(i)
        if s is None or not s["ev"]:
            return False
        need = max(s["ev"], 0)
        if need > len(self.free) or not self.rows:
            return False
        s["pages"] = [self.take() for _ in range(need)]
        s["row"], s["ev"] = self.rows.pop(), 0
        return True


def test_random_walk_matches_the_model():
    rng = np.random.default_rng(7)
    a, m = make(num_pages=96, max_seqs=8, width=24), Model(96, 8, 24)
    for step in range(3000):
        op = rng.integers(6)
        i = int(rng.integers(12))
        if op == 0:
            n = int(rng.integers(0, 520))
            assert a.allocate_sequence(i, n) == m.add(i, n), step
        elif op == 1:
            n = int(rng.integers(0, 520))
            assert a.extend_sequence(i, n) == m.extend(i, n), step
        elif op == 2:
            a.free_sequence(i)
            m.free_seq(i)
        elif op == 3:
            j = int(rng.integers(12))
            assert a.copy_sequence(i, j) == m.fork(i, j), step
        elif op == 4:
            try:
                a.evict(i)
                ok = True
            except L.TkvError:
                ok = False
            assert ok == m.evict(i), step
        else:
            try:
                a.reload(i)
                ok = True
            except L.TkvError:
                ok = False
            assert ok == m.reload(i), step
        live = sorted(k for k, s in m.seqs.items() if not s["ev"])
        if live:
            bt, lens, rows = a.block_tables(live)
            for r, k in enumerate(live):
                s = m.seqs[k]
                assert list(bt[r, :len(s["pages"])]) == s["pages"], step
                assert (bt[r, len(s["pages"]):] == -1).all()
                assert lens[r] == s["len"] and rows[r] == s["row"]
        st = a.stats()
        assert st["blocks_free"] == len(m.free) and st["rows_free"] == len(m.rows)
        assert st["blocks_shared"] == sum(1 for c in m.refs if c > 1)
        assert st["sequences"] == len(m.seqs)


def test_concurrent_threads():
    a = make(num_pages=4096, max_seqs=64, width=64)
    errors = []

    def worker(t):
        try:
            for k in range(300):
                i = t * 1000 + k
                if a.allocate_sequence(i, 256 + 16 * (k % 40)):
                    a.extend_sequence(i, 800)
                    if k % 3 == 0:
                        a.copy_sequence(i, i + 500)
                        a.free_sequence(i + 500)
                    a.free_sequence(i)
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(t,)) for t in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors
    s = a.stats()
    assert s["blocks_free"] == 4096 and s["rows_free"] == 64 and s["sequences"] == 0
