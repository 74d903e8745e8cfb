"""Page and ring-row moves and the allocator driving a serving loop, on the GPU.

* tkv_copy_pages / tkv_swap_pages / tkv_copy_ring_rows / tkv_swap_ring_rows
  move exactly the mapped bytes (pool <-> pool, pool <-> pinned host), flag
  out-of-range pairs without touching anything else, and reject pageable
  host memory before launching.
* A serving loop on KiviCacheAllocator (2 layers): prefill, one-token decode
  steps, a fork (copy_sequence) whose two sequences then diverge, an
  eviction to pinned host and a reload onto other pages, a free whose pages
  are reused by a new sequence; each new sequence's prefill attention is
  checked against the oracle.  At checkpoints every live sequence's pages
  equal, byte for byte, the oracle's pages for the same token history
  appended in one call, and decode attention through the allocator's tables
  and ring rows matches the oracle within 2e-3.
"""
import ctypes as C
import importlib
import math

import numpy as np
import pytest
import torch

from kivi_helpers import check_close, live_ring_values

pytestmark = pytest.mark.gpu

L = importlib.import_module("truellm-engine_b200._lib")
A = importlib.import_module("truellm-engine_b200.allocator")


def _random_cache(ops, cuda, fmt, num_pages, max_seqs, seed):
    c = ops.KiviPagedCache(fmt, num_pages, max_seqs, cuda)
    g = torch.Generator(device=cuda).manual_seed(seed)
    c.pool.copy_(torch.randint(0, 256, c.pool.shape, dtype=torch.uint8, device=cuda, generator=g))
    c.ring.view(torch.int16).copy_(torch.randint(-30000, 30000, c.ring.shape, dtype=torch.int16,
                                                 device=cuda, generator=g))
    return c


def _bits(t):
    """fp16 tensors compared by their bits (random ring bits include NaNs)."""
    return t.view(torch.int16)


def _map(pairs, cuda):
    return torch.tensor(pairs, dtype=torch.int32, device=cuda).reshape(-1, 2)


def test_copy_pages_and_rows(ops, cuda):
    fmt = ops.KiviFormat(128, 32, 32, 4, 4)
    c = _random_cache(ops, cuda, fmt, 40, 6, 1)
    pool0, ring0 = c.pool.clone(), c.ring.clone()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    pairs = [(3, 30), (0, 31), (17, 5), (39, 6)]
    ops.copy_pages(c, _map(pairs, cuda), err=err)
    ops.copy_ring_rows(c, _map([(1, 4), (5, 0)], cuda), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    exp = pool0.clone()
    for s, d in pairs:
        exp[d] = pool0[s]
    assert torch.equal(c.pool, exp)
    er = ring0.clone()
    er[4], er[0] = ring0[1], ring0[5]
    assert torch.equal(_bits(c.ring), _bits(er))
    # out-of-range pairs are flagged and skipped; the others still move
    ops.copy_pages(c, _map([(2, 40), (-1, 3), (8, 9)], cuda), err=err)
    ops.copy_ring_rows(c, _map([(0, 6)], cuda), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == L.TKV_ERR_BAD_PAGE | L.TKV_ERR_BAD_SLOT
    exp[9] = exp[8]
    assert torch.equal(c.pool, exp) and torch.equal(_bits(c.ring), _bits(er))


def test_swap_round_trip_through_pinned_host(ops, cuda):
    fmt = ops.KiviFormat(64, 16, 16, 2, 3)
    c = _random_cache(ops, cuda, fmt, 64, 4, 2)
    pool0, ring0 = c.pool.clone(), c.ring.clone()
    pages = [5, 60, 7, 33, 12]
    imgs = torch.empty((len(pages),) + tuple(c.pool.shape[1:]), dtype=torch.uint8,
                       pin_memory=True)
    rimg = torch.empty((2,) + tuple(c.ring.shape[1:]), dtype=torch.float16, pin_memory=True)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.swap_pages(c, imgs, _map([(p, i) for i, p in enumerate(pages)], cuda), 0, err=err)
    ops.swap_ring_rows(c, rimg, _map([(3, 0), (1, 1)], cuda), 0, err=err)
    torch.cuda.synchronize()
    assert torch.equal(imgs, pool0[pages].cpu())
    assert torch.equal(_bits(rimg), _bits(ring0[[3, 1]].cpu()))
    c.pool.zero_()
    c.ring.zero_()
    dst = [40, 41, 0, 1, 63]
    ops.swap_pages(c, imgs, _map([(i, d) for i, d in enumerate(dst)], cuda), 1, err=err)
    ops.swap_ring_rows(c, rimg, _map([(0, 2), (1, 0)], cuda), 1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(c.pool[dst], pool0[pages])
    assert torch.equal(_bits(c.ring[[2, 0]]), _bits(ring0[[3, 1]]))
    others = [p for p in range(64) if p not in dst]
    assert int(c.pool[others].count_nonzero()) == 0
    # image index beyond the capacity: flagged, nothing written
    ops.swap_pages(c, imgs, _map([(0, 5)], cuda), 0, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == L.TKV_ERR_BAD_PAGE


def test_pageable_host_memory_is_rejected_before_launch(ops, cuda):
    fmt = ops.KiviFormat(64, 16, 16, 4, 1)
    c = ops.KiviPagedCache(fmt, 4, 2, cuda)
    buf = np.zeros((4, 1, fmt.page_bytes), np.uint8)        # pageable numpy memory
    m = _map([(0, 0)], cuda)
    cs = c.c_struct()
    st = L.lib().tkv_swap_pages(C.byref(cs), buf.ctypes.data_as(C.c_void_p), 4,
                                C.c_void_p(m.data_ptr()), 1, 0, None, None)
    assert st == L.TKV_INVALID_ARGUMENT
    hm = np.zeros((1, 2), np.int32)                         # pageable mapping
    st = L.lib().tkv_copy_pages(C.byref(cs), hm.ctypes.data_as(C.c_void_p), 1, None, None)
    assert st == L.TKV_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        ops.swap_pages(c, torch.zeros((4, 1, fmt.page_bytes), dtype=torch.uint8), m, 0)
    with pytest.raises(ValueError):                         # wrong image row shape
        ops.swap_pages(c, torch.zeros((4, 2, 16), dtype=torch.uint8, pin_memory=True), m, 0)


class Loop:
    """Token histories per (layer, sequence) and the GPU state under test."""

    def __init__(self, ops, O, wl, cuda, fmt, Hq, layers, num_pages, max_seqs, width, seed):
        self.ops, self.O, self.wl, self.cuda = ops, O, wl, cuda
        self.fmt, self.Hq, self.layers = fmt, Hq, layers
        self.alloc = A.KiviCacheAllocator(fmt, layers, max_seqs, width, num_pages=num_pages,
                                          device=cuda)
        self.rng = np.random.default_rng(seed)
        self.hist = {}        # seq -> list over layers of (k bits list, v bits list)
        self.err = torch.zeros(1, dtype=torch.int32, device=cuda)

    def tokens(self, n):
        f = self.fmt
        k = self.rng.standard_normal((n, f.n_kv_heads, f.head_dim)).astype(np.float32)
        k[:, :, 3] *= 8.0
        v = self.rng.standard_normal((n, f.n_kv_heads, f.head_dim)).astype(np.float32)
        return self.wl.to_bits(k, "bf16"), self.wl.to_bits(v, "bf16")

    def add(self, sid, n):
        """A new sequence: its prompt appended, then its prefill attention
        (every prompt row over the cache) checked against the oracle."""
        assert self.alloc.allocate_sequence(sid, 0)
        self.hist[sid] = [([], []) for _ in range(self.layers)]
        self.append({sid: n})
        self.check_prefill(sid, n)

    def check_prefill(self, sid, n):
        f = self.fmt
        bt_h, lens, rows = self.alloc.pages.block_tables([sid])
        bt, lens_d, rows_d = self.alloc.get_device_block_tables([sid])
        scale = 1 / math.sqrt(f.head_dim)
        cu_q = torch.tensor([0, n], dtype=torch.int32, device=self.cuda)
        for layer in range(self.layers):
            q = torch.from_numpy(self.wl.f32_to_bf16_bits(
                self.rng.standard_normal((n, self.Hq, f.head_dim))).view(np.int16)).view(
                torch.bfloat16).to(self.cuda)
            out = self.ops.paged_prefill(self.alloc.caches[layer], q, cu_q, bt, lens_d,
                                         max_q_tokens=n, scale=scale, seq_slots=rows_d,
                                         out_dtype=torch.float32, err=self.err)
            kb = np.concatenate(self.hist[sid][layer][0])
            vb = np.concatenate(self.hist[sid][layer][1])
            npg = (len(kb) + 15) // 16 + 1
            st = self.O.PagedState(f.head_dim, f.group_size, f.residual, f.bits, f.n_kv_heads,
                                   npg, 1)
            tbl = np.arange(npg, dtype=np.int32)[None, :]
            st.append(kb, vb, True, np.array([0, len(kb)], np.int32), np.zeros(1, np.int32), tbl)
            ref = st.prefill(q.float().cpu().numpy(), np.array([0, n], np.int32), tbl,
                             np.array([len(kb)], np.int32), scale)
            check_close(out.cpu().numpy(), ref)

    def append(self, counts):
        ids = sorted(counts)
        old = [self.alloc.pages.sequence(s)["len"] for s in ids]
        for s, o in zip(ids, old):
            assert self.alloc.extend_sequence(s, o + counts[s]) >= 0
        bt, _, rows = self.alloc.get_device_block_tables(ids)
        cu = np.concatenate([[0], np.cumsum([counts[s] for s in ids])]).astype(np.int32)
        for layer in range(self.layers):
            ks, vs = zip(*(self.tokens(counts[s]) for s in ids))
            for s, kb, vb in zip(ids, ks, vs):
                self.hist[s][layer][0].append(kb)
                self.hist[s][layer][1].append(vb)
            kt = torch.from_numpy(np.concatenate(ks).view(np.int16)).view(torch.bfloat16)
            vt = torch.from_numpy(np.concatenate(vs).view(np.int16)).view(torch.bfloat16)
            self.ops.paged_append(self.alloc.caches[layer], kt.to(self.cuda), vt.to(self.cuda),
                                  torch.from_numpy(cu).to(self.cuda),
                                  torch.tensor(old, dtype=torch.int32, device=self.cuda), bt,
                                  seq_slots=rows, max_new_tokens=int(max(counts.values())),
                                  err=self.err)

    def fork(self, src, dst):
        assert self.alloc.copy_sequence(src, dst)
        self.hist[dst] = [(list(k), list(v)) for k, v in self.hist[src]]

    def check(self):
        """Pages and ring tokens vs the oracle; decode vs the oracle."""
        torch.cuda.synchronize()
        assert int(self.err.item()) == 0
        f = self.fmt
        ids = sorted(s for s in self.hist if not self.alloc.pages.sequence(s)["evicted"])
        bt_h, lens, rows = self.alloc.pages.block_tables(ids)
        bt, lens_d, rows_d = self.alloc.get_device_block_tables(ids)
        for layer in range(self.layers):
            cache = self.alloc.caches[layer]
            pool = cache.pool.cpu().numpy()
            ring = cache.ring.cpu().numpy().view(np.uint16)
            q = torch.from_numpy(self.wl.f32_to_bf16_bits(
                self.rng.standard_normal((len(ids), self.Hq, f.head_dim))).view(np.int16)).view(
                torch.bfloat16).to(self.cuda)
            scale = 1 / math.sqrt(f.head_dim)
            out = self.ops.paged_decode(cache, q, bt, lens_d, int(lens.max()), scale=scale,
                                        seq_slots=rows_d, out_dtype=torch.float32, err=self.err)
            out = out.cpu().numpy()
            qf = q.float().cpu().numpy()
            for i, s in enumerate(ids):
                kb = np.concatenate(self.hist[s][layer][0])
                vb = np.concatenate(self.hist[s][layer][1])
                n = len(kb)
                assert n == lens[i]
                npg = (n + 15) // 16 + 1
                st = self.O.PagedState(f.head_dim, f.group_size, f.residual, f.bits,
                                       f.n_kv_heads, npg, 1)
                tbl = np.arange(npg, dtype=np.int32)[None, :]
                st.append(kb, vb, True, np.array([0, n], np.int32), np.zeros(1, np.int32), tbl)
                nqp = st.nq(n) // 16
                assert np.array_equal(pool[bt_h[i, :nqp]], st.pool[:nqp]), (layer, s)
                assert np.array_equal(live_ring_values(ring[[rows[i]]], st, [n]),
                                      live_ring_values(st.ring, st, [n])), (layer, s)
                ref = st.decode(qf[[i]], tbl, np.array([n], np.int32), scale)
                check_close(out[[i]], ref)
        torch.cuda.synchronize()
        assert int(self.err.item()) == 0


def test_serving_loop_with_fork_evict_reload(ops, O, wl, cuda):
    fmt = ops.KiviFormat(128, 32, 32, 4, 2)
    lp = Loop(ops, O, wl, cuda, fmt, Hq=8, layers=2, num_pages=160, max_seqs=8, width=64,
              seed=11)
    for sid, n in ((0, 70), (1, 200), (2, 33), (3, 128), (4, 300)):
        lp.add(sid, n)
    lp.check()
    used0 = lp.alloc.stats()["blocks_used"]
    for step in range(48):
        live = [s for s in lp.hist if not lp.alloc.pages.sequence(s)["evicted"]]
        lp.append({s: 1 for s in live})
        if step == 5:
            lp.fork(1, 10)                                  # shares 1's pages
            assert lp.alloc.stats()["blocks_shared"] > 0
        if step == 9:
            lp.check()
            assert lp.alloc.evict_sequence(3)
            assert lp.alloc.evicted_image_bytes(3) > 0
        if step == 15:
            lp.alloc.free_sequence(2)
            del lp.hist[2]
            lp.add(11, 150)                                 # reuses 2's pages and row
        if step == 20:
            assert lp.alloc.reload_sequence(3)
        if step == 30:
            lp.append({4: 40, 10: 17})                      # multi-token appends mid-stream
        if step in (21, 47):
            lp.check()
    assert lp.alloc.stats()["blocks_used"] > used0
    for s in list(lp.hist):
        lp.alloc.free_sequence(s)
    torch.cuda.synchronize()
    st = lp.alloc.stats()
    assert st["blocks_used"] == 0 and st["rows_free"] == st["rows_total"]
