"""Chunked-prefill attention (tkv_paged_prefill) against the oracle.

Each case appends a history and then a chunk per sequence to the GPU cache
and to the oracle in lock step, then runs the chunk's query rows through the
prefill kernel: every row (token i of the chunk, q head) attends causally to
the cached tokens up to its position, wherever they live (pages or ring).
Covers D 64/128, INT4/INT2, G 16..128, R = 0, GQA 1..16, empty and whole-
sequence chunks, chunks spanning many key groups, permuted ring rows, and the
length check.
"""
import math

import numpy as np
import pytest
import torch

from kivi_helpers import Twin, bits_to_torch, check_close, i32

pytestmark = pytest.mark.gpu


def _run(ops, O, wl, cuda, D, G, R, bits, Hkv, Hq, hist, chunk, seed, dtype="bf16",
         slots=None):
    rng = np.random.default_rng(seed)
    hist, chunk = np.asarray(hist, np.int32), np.asarray(chunk, np.int32)
    lens = hist + chunk
    need = int(sum((int(L) + 15) // 16 for L in lens))
    num_pages = need + 9
    bt = wl.random_block_tables(lens, num_pages, rng)
    tw = Twin(ops, O, D, G, R, bits, Hkv, num_pages, len(lens) + 2, cuda)
    for part, old in ((hist, np.zeros_like(hist)), (chunk, hist)):
        T = int(part.sum())
        if T == 0:
            continue
        k, v = wl.kv_tokens(rng, T, Hkv, D, np.array([1, 5]), 8.0)
        cu = np.concatenate([[0], np.cumsum(part)]).astype(np.int32)
        tw.append(wl.to_bits(k, dtype), wl.to_bits(v, dtype), dtype, cu, old, bt, seq_slots=slots)
    T = int(chunk.sum())
    q = rng.standard_normal((T, Hq, D)).astype(np.float32)
    qb = wl.to_bits(q, dtype)
    qt = bits_to_torch(qb, dtype, cuda)
    cu_q = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    scale = 1 / math.sqrt(D)
    out = ops.paged_prefill(tw.gpu, qt, i32(cu_q, cuda), i32(bt, cuda), i32(lens, cuda),
                            max_q_tokens=int(chunk.max()), scale=scale, out_dtype=torch.float32,
                            seq_slots=None if slots is None else i32(slots, cuda), err=tw.err)
    torch.cuda.synchronize()
    assert int(tw.err.item()) == 0
    ref = tw.cpu.prefill(qt.float().cpu().numpy(), cu_q, bt, lens, scale, n_threads=8)
    check_close(out.float().cpu().numpy(), ref)
    return {"tw": tw, "bt": bt, "lens": lens, "q": qt, "cu_q": cu_q, "out": out}


@pytest.mark.parametrize("D,G,R,bits,Hkv,Hq", [
    (128, 128, 128, 4, 2, 8),    # the config-2 format, GQA 4
    (128, 32, 32, 2, 2, 4),
    (64, 16, 16, 4, 2, 2),
    (64, 64, 0, 2, 1, 8),        # no residual window
    (128, 16, 16, 4, 1, 16),     # GQA 16: one token per 16-row tile
    (128, 64, 32, 4, 4, 4),      # MHA
])
def test_prefill_matches_oracle(ops, O, wl, cuda, D, G, R, bits, Hkv, Hq):
    _run(ops, O, wl, cuda, D, G, R, bits, Hkv, Hq, hist=[0, 300, 700], chunk=[130, 37, 200],
         seed=D + G + R + bits + Hq)


def test_prefill_edge_chunks(ops, O, wl, cuda):
    """An empty chunk, a one-token chunk (= decode), a whole sequence from an
    empty cache, and a chunk that spans several key groups and the ring."""
    _run(ops, O, wl, cuda, 128, 128, 128, 4, 2, 8, hist=[500, 0, 129, 40], chunk=[0, 777, 1, 600],
         seed=3)


def test_prefill_fp16_inputs_permuted_ring_rows_and_output_dtypes(ops, O, wl, cuda):
    """fp16 K/V/q, ring rows given by seq_slots; bf16 and fp16 outputs are the
    f32 output rounded (the f32 one is checked against the oracle)."""
    slots = np.array([3, 0, 4], np.int32)
    r = _run(ops, O, wl, cuda, 128, 32, 64, 4, 2, 8, hist=[64, 250, 31], chunk=[20, 90, 100],
             seed=4, dtype="f16", slots=slots)
    for dt in (torch.bfloat16, torch.float16):
        out = ops.paged_prefill(r["tw"].gpu, r["q"], i32(r["cu_q"], cuda), i32(r["bt"], cuda),
                                i32(r["lens"], cuda), max_q_tokens=100, out_dtype=dt,
                                seq_slots=i32(slots, cuda))
        torch.cuda.synchronize()
        assert torch.equal(out, r["out"].to(dt))


def test_prefill_last_row_equals_decode(ops, O, wl, cuda):
    """The chunk's last row attends to the whole context: the decode kernel's
    answer for the same cache and query."""
    r = _run(ops, O, wl, cuda, 128, 128, 128, 4, 2, 8, hist=[900, 40], chunk=[61, 300], seed=5)
    last = torch.tensor(r["cu_q"][1:] - 1, dtype=torch.long, device=cuda)
    dec = ops.paged_decode(r["tw"].gpu, r["q"][last].contiguous(), i32(r["bt"], cuda),
                           i32(r["lens"], cuda), int(r["lens"].max()), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.allclose(r["out"][last], dec, atol=2e-3, rtol=2e-3)


def test_prefill_rejects_chunks_longer_than_the_sequence(ops, wl, cuda):
    fmt = ops.KiviFormat(128, 128, 128, 4, 2)
    cache = ops.KiviPagedCache(fmt, 16, 2, cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q = torch.zeros((10, 8, 128), dtype=torch.bfloat16, device=cuda)
    bt = torch.zeros((2, 8), dtype=torch.int32, device=cuda)
    out = torch.full((10, 8, 128), 7.0, dtype=torch.float32, device=cuda)
    ops.paged_prefill(cache, q, torch.tensor([0, 4, 10], dtype=torch.int32, device=cuda), bt,
                      torch.tensor([4, 5], dtype=torch.int32, device=cuda), max_q_tokens=6,
                      out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 0x4
    assert torch.all(out[4:] == 7.0)     # the bad sequence's rows are untouched


def test_prefill_flags_chunks_longer_than_max_q_tokens(ops, wl, cuda):
    """max_q_tokens sizes the grid: a chunk longer than it is flagged and its
    rows left untouched instead of being partly computed."""
    fmt = ops.KiviFormat(128, 128, 128, 4, 2)
    cache = ops.KiviPagedCache(fmt, 16, 2, cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q = torch.zeros((12, 8, 128), dtype=torch.bfloat16, device=cuda)
    bt = torch.zeros((2, 8), dtype=torch.int32, device=cuda)
    out = torch.full((12, 8, 128), 7.0, dtype=torch.float32, device=cuda)
    ops.paged_prefill(cache, q, torch.tensor([0, 3, 12], dtype=torch.int32, device=cuda), bt,
                      torch.tensor([3, 40], dtype=torch.int32, device=cuda), max_q_tokens=4,
                      out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 0x4
    assert torch.all(out[3:] == 7.0)     # the 9-token chunk's rows are untouched
    assert torch.all(out[:3] != 7.0)     # the 3-token chunk was computed
