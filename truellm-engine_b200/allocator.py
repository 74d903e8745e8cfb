"""Page allocator of the paged KIVI cache: the reference's CudaAllocator
(src/inference/backends/cuda/cuda_allocator.{h,cpp}) for KIVI pages.

* `PageAllocator` -- the bookkeeping, over the native allocator
  (tkv_allocator_* in include/truellm_kivi.h): free list (lowest page id
  first), reference-counted page sharing, block tables with -1 padding,
  eviction records.  Host only; usable without a GPU.
* `KiviCacheAllocator` -- owns the per-layer device caches (the reference's
  single VRAM pool, auto-sized from free memory like cuda_allocator.cpp:52-73)
  and does the device half of copy_sequence / evict_sequence /
  reload_sequence with the page and ring-row move kernels.

KIVI differences from the fp16 pool: a sequence of length L holds
n_q(L) / 16 pages (whole key groups; the newest tokens live in its fp16 ring
row, also handed out here), pages are written once (when their key group is
flushed) so shared pages need no copy-on-write, and the table width is a
parameter instead of the reference's 2048-block cap (cuda_allocator.cpp:76).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L


class PageAllocator:
    """CudaAllocator's block bookkeeping (cuda_allocator.h:38-160) for KIVI pages."""

    def __init__(self, fmt, num_pages: int, max_seqs: int, max_blocks_per_seq: int):
        self.fmt = fmt
        self._cfmt = fmt.c_struct()
        self._h = C.c_void_p()
        L.check("tkv_allocator_create", L.lib().tkv_allocator_create(
            C.byref(self._cfmt), int(num_pages), int(max_seqs), int(max_blocks_per_seq),
            C.byref(self._h)))
        self._num_pages = int(num_pages)
        self.max_seqs = int(max_seqs)
        self._max_blocks = int(max_blocks_per_seq)

    def close(self) -> None:
        if self._h:
            L.lib().tkv_allocator_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- queries
    def pages_for(self, length: int) -> int:
        """Block-table entries a sequence of `length` tokens uses: n_q / 16."""
        return int(L.lib().tkv_allocator_pages_for(self._h, int(length)))

    def num_free_blocks(self) -> int:
        return self.stats()["blocks_free"]

    def num_total_blocks(self) -> int:
        return self._num_pages

    def block_size(self) -> int:
        return L.TKV_PAGE_SIZE

    def max_blocks_per_seq(self) -> int:
        return self._max_blocks

    def stats(self) -> dict:
        """KvCacheStats (cuda_allocator.cpp:292-306) plus shared pages and ring rows."""
        s = L.TkvAllocatorStats()
        L.check("tkv_allocator_stats", L.lib().tkv_allocator_stats(self._h, C.byref(s)))
        return {"block_size_tokens": L.TKV_PAGE_SIZE, "blocks_total": s.pages_total,
                "blocks_used": s.pages_used, "blocks_free": s.pages_free,
                "blocks_shared": s.pages_shared, "utilization_pct": s.utilization_pct,
                "rows_total": s.rows_total, "rows_free": s.rows_free,
                "sequences": s.sequences, "evicted": s.evicted}

    def sequence(self, seq_id: int) -> dict:
        n, p, r, e = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        L.check("tkv_allocator_sequence", L.lib().tkv_allocator_sequence(
            self._h, int(seq_id), C.byref(n), C.byref(p), C.byref(r), C.byref(e)))
        return {"len": n.value, "n_pages": p.value, "ring_row": r.value, "evicted": bool(e.value)}

    # -------------------------------------------------------------- lifecycle
    def allocate_sequence(self, seq_id: int, num_prompt_tokens: int) -> bool:
        """cuda_allocator.cpp:129-158: False when the id exists, the length
        does not fit the table, or pages / ring rows are short (nothing changes)."""
        return L.lib().tkv_allocator_add_sequence(
            self._h, int(seq_id), int(num_prompt_tokens), None) == L.TKV_OK

    def extend_sequence(self, seq_id: int, new_len: int) -> int:
        """cuda_allocator.cpp:160-171 by length: pages added so the table
        covers `new_len` tokens, or -1 (unknown / evicted id, shorter length,
        out of pages; nothing changes)."""
        added = C.c_int()
        st = L.lib().tkv_allocator_extend(self._h, int(seq_id), int(new_len), C.byref(added))
        return added.value if st == L.TKV_OK else -1

    def free_sequence(self, seq_id: int) -> None:
        L.check("tkv_allocator_free_sequence",
                L.lib().tkv_allocator_free_sequence(self._h, int(seq_id)))

    def fork(self, src_id: int, dst_id: int) -> Tuple[int, int]:
        """copy_sequence bookkeeping: dst shares src's pages and length and gets
        its own ring row.  Returns (src_row, dst_row); the caller copies the
        ring row on the device before either sequence appends again."""
        s, d = C.c_int(), C.c_int()
        L.check("tkv_allocator_fork", L.lib().tkv_allocator_fork(
            self._h, int(src_id), int(dst_id), C.byref(s), C.byref(d)))
        return s.value, d.value

    def copy_sequence(self, src_id: int, dst_id: int) -> bool:
        """cuda_allocator.cpp:187-203 (bookkeeping only; see fork)."""
        try:
            self.fork(src_id, dst_id)
            return True
        except L.TkvError:
            return False

    def block_tables(self, seq_ids: Sequence[int]) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Batched get_device_block_table, on the host: ([n, max_blocks] int32
        -1 padded, seq_lens [n] int32, ring rows [n] int32)."""
        ids = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.uint64))
        n = len(ids)
        bt = np.empty((n, self._max_blocks), np.int32)
        lens = np.empty(n, np.int32)
        rows = np.empty(n, np.int32)
        L.check("tkv_allocator_tables", L.lib().tkv_allocator_tables(
            self._h, ids.ctypes.data_as(C.c_void_p), n, bt.ctypes.data_as(C.c_void_p),
            lens.ctypes.data_as(C.c_void_p), rows.ctypes.data_as(C.c_void_p)))
        return bt, lens, rows

    def evict(self, seq_id: int) -> Tuple[np.ndarray, int]:
        """evict_sequence bookkeeping: (pages in table order, ring row), both released."""
        pages = np.empty(self._max_blocks, np.int32)
        n, r = C.c_int(), C.c_int()
        L.check("tkv_allocator_evict", L.lib().tkv_allocator_evict(
            self._h, int(seq_id), pages.ctypes.data_as(C.c_void_p), C.byref(n), C.byref(r)))
        return pages[:n.value].copy(), r.value

    def reload(self, seq_id: int) -> Tuple[np.ndarray, int]:
        """reload_sequence bookkeeping: fresh (pages, ring row); TkvError with
        TKV_OUT_OF_MEMORY leaves the sequence evicted."""
        pages = np.empty(self._max_blocks, np.int32)
        n, r = C.c_int(), C.c_int()
        L.check("tkv_allocator_reload", L.lib().tkv_allocator_reload(
            self._h, int(seq_id), pages.ctypes.data_as(C.c_void_p), C.byref(n), C.byref(r)))
        return pages[:n.value].copy(), r.value


class KiviCacheAllocator:
    """CudaAllocator for the paged KIVI cache: per-layer device caches plus
    the page bookkeeping, with the device moves of fork / evict / reload.

    All device work goes on the stream passed in (default: the current
    stream); use one stream for the moves and the appends / decodes that
    follow them, so a released page is read before it is rewritten.
    """

    def __init__(self, fmt, num_layers: int, max_seqs: int, max_blocks_per_seq: int,
                 num_pages: int = 0, device="cuda", gpu_memory_utilization: float = 0.90):
        import torch
        from . import ops
        self.torch, self.ops = torch, ops
        self.device = torch.device(device)
        self.fmt = fmt
        self.num_layers = int(num_layers)
        if num_pages <= 0:  # auto-size (cuda_allocator.cpp:52-73)
            free, _ = torch.cuda.mem_get_info(self.device)
            util = gpu_memory_utilization if gpu_memory_utilization > 0 else 0.90
            cf = fmt.c_struct()
            ring = L.lib().tkv_ring_bytes(C.byref(cf), int(max_seqs)) * self.num_layers
            per_page = int(cf.page_bytes) * fmt.n_kv_heads * self.num_layers
            num_pages = int((free * util - ring) // per_page)
            if num_pages <= 0:
                raise MemoryError("no device memory left for the KIVI page pool")
        self.caches: List = [ops.KiviPagedCache(fmt, num_pages, max_seqs, self.device)
                             for _ in range(self.num_layers)]
        self.pages = PageAllocator(fmt, num_pages, max_seqs, max_blocks_per_seq)
        self._images: Dict[int, Tuple[list, list]] = {}
        self._in_flight: list = []  # (event, tensors) kept alive until the event completes

    def kv_layer_cache(self, layer: int):
        return self.caches[layer]

    # lifecycle (host only)
    def allocate_sequence(self, seq_id: int, num_prompt_tokens: int) -> bool:
        return self.pages.allocate_sequence(seq_id, num_prompt_tokens)

    def extend_sequence(self, seq_id: int, new_len: int) -> int:
        return self.pages.extend_sequence(seq_id, new_len)

    def free_sequence(self, seq_id: int) -> None:
        self.pages.free_sequence(seq_id)
        imgs = self._images.pop(seq_id, None)
        if imgs is not None:  # an eviction copy may still be writing them
            self._retire(self._stream(None), imgs[0] + imgs[1])

    def num_free_blocks(self) -> int:
        return self.pages.num_free_blocks()

    def stats(self) -> dict:
        return self.pages.stats()

    # device side
    def _stream(self, stream):
        return stream if stream is not None else self.torch.cuda.current_stream(self.device)

    def _to_device(self, arr: np.ndarray, stream):
        torch = self.torch
        host = torch.from_numpy(np.ascontiguousarray(arr)).pin_memory()
        with torch.cuda.stream(stream):
            return host.to(self.device, non_blocking=True)

    def _retire(self, stream, tensors) -> None:
        ev = self.torch.cuda.Event()
        ev.record(stream)
        self._in_flight = [(e, t) for e, t in self._in_flight if not e.query()]
        self._in_flight.append((ev, tensors))

    def get_device_block_tables(self, seq_ids: Sequence[int], stream=None):
        """Batched get_device_block_table (cuda_allocator.cpp:231-253): device
        int32 (block_tables [n, max_blocks], seq_lens [n], ring rows [n]),
        copied from pinned staging on `stream` without a host sync."""
        stream = self._stream(stream)
        bt, lens, rows = self.pages.block_tables(seq_ids)
        return (self._to_device(bt, stream), self._to_device(lens, stream),
                self._to_device(rows, stream))

    def copy_sequence(self, src_id: int, dst_id: int, stream=None) -> bool:
        """Fork: shared pages plus a device copy of the ring row in every layer."""
        try:
            s, d = self.pages.fork(src_id, dst_id)
        except L.TkvError:
            return False
        stream = self._stream(stream)
        m = self._to_device(np.array([[s, d]], np.int32), stream)
        for c in self.caches:
            self.ops.copy_ring_rows(c, m, stream=stream)
        self._retire(stream, [m])
        return True

    def evict_sequence(self, seq_id: int, stream=None) -> bool:
        """evict_sequence (cuda_allocator.cpp:318-350): the sequence's pages and
        ring row of every layer go to pinned host images; pages and row are released."""
        torch = self.torch
        try:
            pages, row = self.pages.evict(seq_id)
        except L.TkvError:
            return False
        stream = self._stream(stream)
        n = len(pages)
        pm = self._to_device(np.stack([pages, np.arange(n, dtype=np.int32)], 1), stream)
        rm = self._to_device(np.array([[row, 0]], np.int32), stream)
        page_imgs, ring_imgs = [], []
        for c in self.caches:
            pi = torch.empty((max(n, 1),) + tuple(c.pool.shape[1:]), dtype=torch.uint8,
                             pin_memory=True)
            ri = torch.empty((1,) + tuple(c.ring.shape[1:]), dtype=torch.float16,
                             pin_memory=True)
            if n:
                self.ops.swap_pages(c, pi, pm, 0, stream=stream)
            self.ops.swap_ring_rows(c, ri, rm, 0, stream=stream)
            page_imgs.append(pi)
            ring_imgs.append(ri)
        self._images[seq_id] = (page_imgs, ring_imgs)
        self._retire(stream, [pm, rm])
        return True

    def reload_sequence(self, seq_id: int, stream=None) -> bool:
        """reload_sequence (cuda_allocator.cpp:352-378): fresh pages and ring row,
        filled from the saved images.  False (sequence stays evicted) when
        pages or rows are short."""
        if seq_id not in self._images:
            return False
        try:
            pages, row = self.pages.reload(seq_id)
        except L.TkvError:
            return False
        stream = self._stream(stream)
        page_imgs, ring_imgs = self._images.pop(seq_id)
        n = len(pages)
        pm = self._to_device(np.stack([np.arange(n, dtype=np.int32), pages], 1), stream)
        rm = self._to_device(np.array([[0, row]], np.int32), stream)
        for c, pi, ri in zip(self.caches, page_imgs, ring_imgs):
            if n:
                self.ops.swap_pages(c, pi, pm, 1, stream=stream)
            self.ops.swap_ring_rows(c, ri, rm, 1, stream=stream)
        self._retire(stream, [pm, rm] + page_imgs + ring_imgs)
        return True

    def evicted_image_bytes(self, seq_id: int) -> int:
        """Host bytes held for an evicted sequence (all layers)."""
        if seq_id not in self._images:
            return 0
        p, r = self._images[seq_id]
        return sum(t.numel() * t.element_size() for t in p + r)
