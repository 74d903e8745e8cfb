"""Torch-facing wrappers of the C ABI: the reference's kernel entry points.

Mirrors, with the same argument meaning:
  kivi_compressed_bytes / kivi_params_supported / kivi_compress / kivi_decompress
      src/inference/backends/cuda/compression/kivi_cache.cuh:32-84
  reshape_and_cache  -> paged_append    (cuda_engine.cpp:48-50, cache_kernels.cu:202-232)
  paged_attention_v1/v2 -> paged_decode (cuda_engine.cpp:51-62)
Every call goes to the sm_100a library; tensors must be CUDA tensors.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L

_DT = {torch.float16: L.TKV_F16, torch.bfloat16: L.TKV_BF16, torch.float32: L.TKV_F32}


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _ptr(t: Optional[torch.Tensor]):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("KIVI kernels take CUDA tensors")


# ---------------------------------------------------------------------------
# reference-format KIVI (kivi_cache.cuh)
# ---------------------------------------------------------------------------
KIVI_MAX_HEAD_DIM = 128  # kivi_cache.cuh:27
KIVI_MAX_OUTLIERS = 64  # kivi_cache.cuh:28


def kivi_compressed_bytes(head_dim: int, n_outliers: int, group_size: int) -> int:
    """Bytes of one compressed vector (kivi_cache.cuh:32-43)."""
    return int(L.lib().tkv_kivi_compressed_bytes(head_dim, n_outliers, group_size))


def kivi_params_supported(head_dim: int, n_outliers: int, group_size: int) -> bool:
    """kivi_cache.cu:205-211."""
    return bool(L.lib().tkv_kivi_params_supported(head_dim, n_outliers, group_size))


def kivi_compress(d_kv_in: torch.Tensor, d_out: torch.Tensor, n_vecs: int, head_dim: int,
                  n_outliers: int, group_size: int, stream=None) -> None:
    """truellm::kivi_compress: a no-op when kivi_params_supported() is false or
    n_vecs <= 0, as in the reference wrapper (kivi_cache.cu:213-225)."""
    if n_vecs <= 0 or not kivi_params_supported(head_dim, n_outliers, group_size):
        return
    _need_cuda(d_kv_in, d_out)
    L.check("tkv_kivi_compress", L.lib().tkv_kivi_compress(
        _ptr(d_kv_in), _ptr(d_out), n_vecs, head_dim, n_outliers, group_size,
        C.c_void_p(_stream(stream))))


def kivi_decompress(d_in: torch.Tensor, d_kv_out: torch.Tensor, n_vecs: int, head_dim: int,
                    n_outliers: int, group_size: int, stream=None) -> None:
    """truellm::kivi_decompress (kivi_cache.cu:227-239)."""
    if n_vecs <= 0 or not kivi_params_supported(head_dim, n_outliers, group_size):
        return
    _need_cuda(d_in, d_kv_out)
    L.check("tkv_kivi_decompress", L.lib().tkv_kivi_decompress(
        _ptr(d_in), _ptr(d_kv_out), n_vecs, head_dim, n_outliers, group_size,
        C.c_void_p(_stream(stream))))


def kivi_roundtrip_inplace(d_kv: torch.Tensor, n_vecs: int, head_dim: int, n_outliers: int,
                           group_size: int, stream=None) -> None:
    """compress + decompress in place in one launch (KvCompressionPass::run_kivi)."""
    if n_vecs <= 0 or not kivi_params_supported(head_dim, n_outliers, group_size):
        return
    _need_cuda(d_kv)
    L.check("tkv_kivi_roundtrip_inplace", L.lib().tkv_kivi_roundtrip_inplace(
        _ptr(d_kv), n_vecs, head_dim, n_outliers, group_size, C.c_void_p(_stream(stream))))


# ---------------------------------------------------------------------------
# paged KIVI cache
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class KiviFormat:
    head_dim: int
    group_size: int
    residual: int
    bits: int
    n_kv_heads: int

    def c_struct(self) -> L.TkvFormat:
        f = L.TkvFormat()
        L.check("tkv_format_init", L.lib().tkv_format_init(
            C.byref(f), self.head_dim, self.group_size, self.residual, self.bits,
            self.n_kv_heads))
        return f

    @property
    def page_bytes(self) -> int:
        return int(self.c_struct().page_bytes)

    @property
    def ring_cap(self) -> int:
        return int(self.c_struct().ring_cap)

    def quantized_len(self, length: int) -> int:
        x = length - self.residual
        return self.group_size * (x // self.group_size) if x > 0 else 0


class KiviPagedCache:
    """Device buffers of one layer's paged KIVI cache.

    pool: [num_pages, n_kv_heads, page_bytes] uint8 (block-major like the
    reference pool, cuda_allocator.h:9-12); ring: [max_seqs, n_kv_heads,
    ring_cap/16, 2, 16*D] fp16 residual window.  Both zero-initialised.
    """

    def __init__(self, fmt: KiviFormat, num_pages: int, max_seqs: int, device="cuda"):
        self.fmt = fmt
        cf = fmt.c_struct()
        self.num_pages = int(num_pages)
        self.max_seqs = int(max_seqs)
        self.pool = torch.zeros((num_pages, fmt.n_kv_heads, int(cf.page_bytes)),
                                dtype=torch.uint8, device=device)
        self.ring = torch.zeros((max_seqs, fmt.n_kv_heads, int(cf.ring_cap) // 16, 2,
                                 16 * fmt.head_dim), dtype=torch.float16, device=device)

    def c_struct(self) -> L.TkvCache:
        c = L.TkvCache()
        c.pool = self.pool.data_ptr()
        c.ring = self.ring.data_ptr()
        c.num_pages = self.num_pages
        c.max_seqs = self.max_seqs
        c.fmt = self.fmt.c_struct()
        return c


def paged_append(cache: KiviPagedCache, k_new: torch.Tensor, v_new: torch.Tensor,
                 cu_new: torch.Tensor, seq_lens_old: torch.Tensor, block_tables: torch.Tensor,
                 seq_slots: Optional[torch.Tensor] = None, max_new_tokens: Optional[int] = None,
                 err: Optional[torch.Tensor] = None, stream=None) -> None:
    """Quantize-on-append (the KIVI reshape_and_cache).

    k_new, v_new: [T_total, n_kv_heads, D] fp16/bf16; cu_new: [B+1] int32 token
    offsets; seq_lens_old: [B] int32; block_tables: [B, max_blocks] int32.
    max_new_tokens bounds the per-sequence token count (defaults to T_total).
    """
    _need_cuda(k_new, v_new, cu_new, seq_lens_old, block_tables)
    if k_new.dtype not in (torch.float16, torch.bfloat16) or v_new.dtype != k_new.dtype:
        raise ValueError("k_new/v_new must both be fp16 or bf16")
    B = int(seq_lens_old.numel())
    mnt = int(k_new.shape[0]) if max_new_tokens is None else int(max_new_tokens)
    c = cache.c_struct()
    L.check("tkv_paged_append", L.lib().tkv_paged_append(
        C.byref(c), _ptr(k_new.contiguous()), _ptr(v_new.contiguous()), _DT[k_new.dtype],
        _ptr(cu_new), _ptr(seq_lens_old), _ptr(block_tables), int(block_tables.shape[1]),
        _ptr(seq_slots), B, int(k_new.shape[0]), mnt, _ptr(err), C.c_void_p(_stream(stream))))


def decode_workspace_bytes(num_seqs: int, num_q_heads: int, head_dim: int,
                           max_context_len: int) -> int:
    return int(L.lib().tkv_decode_workspace_bytes(num_seqs, num_q_heads, head_dim,
                                                  max_context_len))


def decode_range_workspace_bytes(num_seqs: int, num_q_heads: int, head_dim: int,
                                 split_lo: int, split_hi: int) -> int:
    return int(L.lib().tkv_decode_range_workspace_bytes(num_seqs, num_q_heads, head_dim,
                                                        split_lo, split_hi))


def decode_launches(num_seqs: int, num_q_heads: int, num_kv_heads: int,
                    max_context_len: int) -> int:
    """Kernel launches one paged_decode call makes on the current device: 1
    (merge fused into the decode kernel), or 2 when there is less than one
    (sequence, kv head) pair per 16 resident warps (a separate merge kernel
    spreads the merge of pairs that span many warps over the GPU)."""
    return int(L.lib().tkv_decode_launches(num_seqs, num_q_heads, num_kv_heads,
                                           max_context_len))


def decode_num_splits(max_context_len: int) -> int:
    return int(L.lib().tkv_decode_num_splits(max_context_len))


def paged_decode(cache: KiviPagedCache, q: torch.Tensor, block_tables: torch.Tensor,
                 seq_lens: torch.Tensor, max_context_len: int, scale: Optional[float] = None,
                 out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                 workspace: Optional[torch.Tensor] = None,
                 seq_slots: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
    """Decode attention over the KIVI cache (the paged_attention_v1/v2 slot).

    q: [B, Hq, D] fp16/bf16.  Returns out [B, Hq, D] (dtype of q unless
    out/out_dtype say otherwise).  scale defaults to 1/sqrt(D) (cuda_engine.cpp:1140).
    """
    _need_cuda(q, block_tables, seq_lens)
    B, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=out_dtype or q.dtype, device=q.device)
    ws_bytes = decode_workspace_bytes(B, Hq, D, max_context_len)
    if workspace is None:  # work counters at its start must be zero: allocate zeroed
        workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=q.device)
    c = cache.c_struct()
    L.check("tkv_paged_decode", L.lib().tkv_paged_decode(
        C.byref(c), _ptr(q.contiguous()), _DT[q.dtype], _ptr(out), _DT[out.dtype],
        _ptr(block_tables), int(block_tables.shape[1]), _ptr(seq_lens), _ptr(seq_slots), B, Hq,
        float(scale), int(max_context_len), _ptr(workspace), int(workspace.numel()),
        _ptr(err), C.c_void_p(_stream(stream))))
    return out


class PreparedDecode:
    """tkv_paged_decode with its arguments bound once to fixed buffers: each
    call is one ctypes call, for decode loops where the wrapper's per-call
    work (argument conversion, the format struct) would show beside a
    ~0.1 ms kernel.  The buffers must stay alive and keep their addresses."""

    def __init__(self, cache: KiviPagedCache, q: torch.Tensor, block_tables: torch.Tensor,
                 seq_lens: torch.Tensor, max_context_len: int, out: torch.Tensor,
                 workspace: torch.Tensor, scale: Optional[float] = None,
                 seq_slots: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None,
                 stream=None):
        _need_cuda(q, block_tables, seq_lens, out, workspace)
        if not q.is_contiguous():
            raise ValueError("q must be contiguous")
        B, Hq, D = q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        self._keep = (q, block_tables, seq_lens, out, workspace, seq_slots, err)
        self._c = cache.c_struct()
        self._fn = L.lib().tkv_paged_decode
        self._args = (C.byref(self._c), _ptr(q), _DT[q.dtype], _ptr(out), _DT[out.dtype],
                      _ptr(block_tables), int(block_tables.shape[1]), _ptr(seq_lens),
                      _ptr(seq_slots), B, Hq, float(scale), int(max_context_len),
                      _ptr(workspace), int(workspace.numel() * workspace.element_size()),
                      _ptr(err), C.c_void_p(_stream(stream)))

    def __call__(self) -> None:
        st = self._fn(*self._args)
        if st != L.TKV_OK:
            raise L.TkvError("tkv_paged_decode", st)


def paged_decode_partials(cache: KiviPagedCache, q: torch.Tensor, block_tables: torch.Tensor,
                          seq_lens: torch.Tensor, split_lo: int, split_hi: int,
                          include_residual: bool, part_ml: torch.Tensor, part_o: torch.Tensor,
                          scale: Optional[float] = None,
                          seq_slots: Optional[torch.Tensor] = None,
                          err: Optional[torch.Tensor] = None,
                          work: Optional[torch.Tensor] = None, stream=None) -> None:
    """Split-KV partials (m, l, o) of quantised splits [split_lo, split_hi)
    (+ the residual split) for sequences split across GPUs.  work: >= 8 bytes
    of zeroed device memory reused across calls (allocated when omitted)."""
    _need_cuda(q, block_tables, seq_lens, part_ml, part_o)
    if work is None:
        work = torch.zeros(2, dtype=torch.int32, device=q.device)
    B, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    c = cache.c_struct()
    L.check("tkv_paged_decode_partials", L.lib().tkv_paged_decode_partials(
        C.byref(c), _ptr(q.contiguous()), _DT[q.dtype], _ptr(block_tables),
        int(block_tables.shape[1]), _ptr(seq_lens), _ptr(seq_slots), B, Hq, float(scale),
        int(split_lo), int(split_hi), int(bool(include_residual)), _ptr(part_ml), _ptr(part_o),
        _ptr(work), _ptr(err), C.c_void_p(_stream(stream))))


def paged_decode_range(cache: KiviPagedCache, q: torch.Tensor, block_tables: torch.Tensor,
                       seq_lens: torch.Tensor, split_lo: int, split_hi: int,
                       include_residual: bool, out_ml: torch.Tensor, out_o: torch.Tensor,
                       workspace: torch.Tensor, scale: Optional[float] = None,
                       seq_slots: Optional[torch.Tensor] = None,
                       err: Optional[torch.Tensor] = None, stream=None) -> None:
    """One GPU's share of a token-split decode: quantised splits [split_lo,
    split_hi) (+ the residual split) reduced in the launch to one partial per
    (sequence, q head): out_ml [B, Hq, 2], out_o [B, Hq, D] fp32.  workspace:
    zeroed uint8 device tensor of decode_range_workspace_bytes(B, Hq, D,
    split_lo, split_hi) bytes, reused across calls."""
    _need_cuda(q, block_tables, seq_lens, out_ml, out_o, workspace)
    B, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    c = cache.c_struct()
    L.check("tkv_paged_decode_range", L.lib().tkv_paged_decode_range(
        C.byref(c), _ptr(q.contiguous()), _DT[q.dtype], _ptr(block_tables),
        int(block_tables.shape[1]), _ptr(seq_lens), _ptr(seq_slots), B, Hq, float(scale),
        int(split_lo), int(split_hi), int(bool(include_residual)), _ptr(out_ml), _ptr(out_o),
        _ptr(workspace), int(workspace.numel() * workspace.element_size()), _ptr(err),
        C.c_void_p(_stream(stream))))


def paged_prefill(cache: KiviPagedCache, q: torch.Tensor, cu_q: torch.Tensor,
                  block_tables: torch.Tensor, seq_lens: torch.Tensor,
                  max_q_tokens: Optional[int] = None, scale: Optional[float] = None,
                  out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                  seq_slots: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None,
                  stream=None) -> torch.Tensor:
    """Causal chunked-prefill attention over the KIVI cache: q [T, Hq, D]
    holds, per sequence, its last cu_q[s+1]-cu_q[s] tokens (already appended);
    seq_lens are the lengths after the append.  Returns out [T, Hq, D]."""
    _need_cuda(q, cu_q, block_tables, seq_lens)
    T, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((T, Hq, D), dtype=out_dtype or q.dtype, device=q.device)
    mq = T if max_q_tokens is None else int(max_q_tokens)
    c = cache.c_struct()
    L.check("tkv_paged_prefill", L.lib().tkv_paged_prefill(
        C.byref(c), _ptr(q.contiguous()), _DT[q.dtype], _ptr(out), _DT[out.dtype], _ptr(cu_q),
        _ptr(block_tables), int(block_tables.shape[1]), _ptr(seq_lens), _ptr(seq_slots),
        int(seq_lens.numel()), Hq, T, mq, float(scale), _ptr(err), C.c_void_p(_stream(stream))))
    return out


def merge_partials(part_ml: torch.Tensor, part_o: torch.Tensor, out: torch.Tensor,
                   stream=None) -> torch.Tensor:
    """LSE merge (paged_attention_v2.cu:132-170).  part_ml: [S, B, Hq, 2],
    part_o: [S, B, Hq, D] fp32; out: [B, Hq, D]."""
    _need_cuda(part_ml, part_o, out)
    S, B, Hq, D = part_o.shape
    L.check("tkv_merge_partials", L.lib().tkv_merge_partials(
        _ptr(part_ml), _ptr(part_o), S, B, Hq, D, _ptr(out), _DT[out.dtype],
        C.c_void_p(_stream(stream))))
    return out


# ---------------------------------------------------------------------------
# token split over peer memory (tkv_exchange_*)
# ---------------------------------------------------------------------------
def exchange_buffer_bytes(world: int, num_seqs: int, num_q_heads: int, head_dim: int) -> int:
    return int(L.lib().tkv_exchange_buffer_bytes(world, num_seqs, num_q_heads, head_dim))


class DeviceBuffer:
    """Zeroed device memory from tkv_device_alloc (shareable over CUDA IPC) on
    the current device; freed by close()."""

    def __init__(self, nbytes: int):
        p = C.c_void_p()
        L.check("tkv_device_alloc", L.lib().tkv_device_alloc(int(nbytes), C.byref(p)))
        self.ptr, self.nbytes = int(p.value), int(nbytes)

    def close(self) -> None:
        if self.ptr:
            L.check("tkv_device_free", L.lib().tkv_device_free(C.c_void_p(self.ptr)))
            self.ptr = 0


def ipc_handle(ptr: int) -> bytes:
    h = (C.c_char * L.TKV_IPC_HANDLE_BYTES)()
    L.check("tkv_ipc_get_handle", L.lib().tkv_ipc_get_handle(C.c_void_p(ptr), h))
    return bytes(h)


def ipc_open(handle: bytes) -> int:
    h = (C.c_char * L.TKV_IPC_HANDLE_BYTES).from_buffer_copy(handle)
    p = C.c_void_p()
    L.check("tkv_ipc_open_handle", L.lib().tkv_ipc_open_handle(h, C.byref(p)))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    L.check("tkv_ipc_close_handle", L.lib().tkv_ipc_close_handle(C.c_void_p(ptr)))


def exchange_struct(world: int, rank: int, buffers) -> L.TkvExchange:
    ex = L.TkvExchange()
    ex.world, ex.rank = int(world), int(rank)
    for r, b in enumerate(buffers):
        ex.buffers[r] = int(b)
    return ex


def exchange_decode_range(cache: KiviPagedCache, q: torch.Tensor, block_tables: torch.Tensor,
                          seq_lens: torch.Tensor, split_lo: int, split_hi: int,
                          include_residual: bool, ex: L.TkvExchange,
                          workspace: Optional[torch.Tensor], scale: Optional[float] = None,
                          seq_slots: Optional[torch.Tensor] = None,
                          err: Optional[torch.Tensor] = None, stream=None) -> None:
    """This GPU's range of a token split (see paged_decode_range), reduced and
    stored into every GPU's exchange buffer, flag raised."""
    _need_cuda(q, block_tables, seq_lens)
    B, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    c = cache.c_struct()
    ws_bytes = 0 if workspace is None else int(workspace.numel() * workspace.element_size())
    L.check("tkv_exchange_decode_range", L.lib().tkv_exchange_decode_range(
        C.byref(c), _ptr(q.contiguous()), _DT[q.dtype], _ptr(block_tables),
        int(block_tables.shape[1]), _ptr(seq_lens), _ptr(seq_slots), B, Hq, float(scale),
        int(split_lo), int(split_hi), int(bool(include_residual)), C.byref(ex), _ptr(workspace),
        ws_bytes, _ptr(err), C.c_void_p(_stream(stream))))


def exchange_merge(ex: L.TkvExchange, out: torch.Tensor, err: Optional[torch.Tensor] = None,
                   stream=None) -> torch.Tensor:
    """Waits for every GPU's partials of this step and merges them into out
    [B, Hq, D] (f32, f16 or bf16)."""
    _need_cuda(out)
    B, Hq, D = out.shape
    L.check("tkv_exchange_merge", L.lib().tkv_exchange_merge(
        C.byref(ex), B, Hq, D, _ptr(out), _DT[out.dtype], _ptr(err), C.c_void_p(_stream(stream))))
    return out


# ---------------------------------------------------------------------------
# page and ring-row moves (copy_blocks / swap_blocks, cache_kernels.cu:107-168)
# ---------------------------------------------------------------------------
def _mapping(mapping: torch.Tensor) -> int:
    if mapping.dtype != torch.int32 or mapping.dim() != 2 or mapping.shape[1] != 2:
        raise ValueError("mapping must be an int32 [n, 2] tensor of (src, dst) pairs")
    if not (mapping.is_cuda or mapping.is_pinned()):
        raise ValueError("mapping must be a CUDA or pinned host tensor")
    return int(mapping.shape[0])


def _images(images: torch.Tensor, like: torch.Tensor) -> None:
    """images must be [capacity, *like.shape[1:]] of like's dtype, contiguous,
    in CUDA or pinned host memory: the kernel addresses whole rows of it."""
    if not (images.is_cuda or images.is_pinned()) or not images.is_contiguous():
        raise ValueError("images must be a contiguous CUDA or pinned host tensor")
    if images.dtype != like.dtype or tuple(images.shape[1:]) != tuple(like.shape[1:]):
        raise ValueError(f"images must be [capacity, {', '.join(map(str, like.shape[1:]))}] "
                         f"{like.dtype}")


def copy_pages(cache: KiviPagedCache, mapping: torch.Tensor, err: Optional[torch.Tensor] = None,
               stream=None) -> None:
    """copy_blocks for KIVI pages: pool page mapping[i,0] -> mapping[i,1]."""
    n = _mapping(mapping)
    c = cache.c_struct()
    L.check("tkv_copy_pages", L.lib().tkv_copy_pages(
        C.byref(c), _ptr(mapping), n, _ptr(err), C.c_void_p(_stream(stream))))


def swap_pages(cache: KiviPagedCache, images: torch.Tensor, mapping: torch.Tensor,
               direction: int, err: Optional[torch.Tensor] = None, stream=None) -> None:
    """swap_blocks for KIVI pages.  images: [capacity, n_kv_heads, page_bytes]
    uint8, pinned host (or CUDA); direction 0 = pool -> images, 1 = images -> pool."""
    n = _mapping(mapping)
    _images(images, cache.pool)
    c = cache.c_struct()
    cap = int(images.shape[0])
    L.check("tkv_swap_pages", L.lib().tkv_swap_pages(
        C.byref(c), _ptr(images), cap, _ptr(mapping), n, int(direction), _ptr(err),
        C.c_void_p(_stream(stream))))


def copy_ring_rows(cache: KiviPagedCache, mapping: torch.Tensor,
                   err: Optional[torch.Tensor] = None, stream=None) -> None:
    """Ring row mapping[i,0] -> mapping[i,1] (the device half of a fork)."""
    n = _mapping(mapping)
    c = cache.c_struct()
    L.check("tkv_copy_ring_rows", L.lib().tkv_copy_ring_rows(
        C.byref(c), _ptr(mapping), n, _ptr(err), C.c_void_p(_stream(stream))))


def swap_ring_rows(cache: KiviPagedCache, images: torch.Tensor, mapping: torch.Tensor,
                   direction: int, err: Optional[torch.Tensor] = None, stream=None) -> None:
    """Ring rows to / from images [capacity, *ring row shape] fp16 (pinned host or CUDA)."""
    n = _mapping(mapping)
    _images(images, cache.ring)
    c = cache.c_struct()
    L.check("tkv_swap_ring_rows", L.lib().tkv_swap_ring_rows(
        C.byref(c), _ptr(images), int(images.shape[0]), _ptr(mapping), n, int(direction),
        _ptr(err), C.c_void_p(_stream(stream))))
