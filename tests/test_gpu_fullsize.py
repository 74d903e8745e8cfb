"""Parity at BASELINE's full sizes (configs 2-5), where the CPU oracle
cannot redo everything: sampled sequences against the oracle, plus properties
that hold at any size.

* config 2 decode (B=64, contexts U[1024, 8192]): the GPU-built cache copied to
  the oracle gives the same attention for sampled sequences (2e-3); split
  partials of a sequence do not depend on the batch it is decoded in
  (bit-exact between the full batch and a sub-batch).
* config 3 append (64 x 2048 bf16 tokens): sampled sequences' pages and live
  ring tokens equal the oracle's bytes; appending the chunk in two halves
  gives the same pool and ring bytes as one call (chunking invariance).
* config 4 decode (B=8, 131072 tokens, Hq=64): two sampled sequences against
  the oracle; two token ranges merged equal the one-call decode.
* config 5 decode (B=256 continuous batch, INT4 and INT2 halves): the longest
  and shortest sequence of each half against the oracle.
"""
import importlib
import math

import numpy as np
import pytest
import torch

from kivi_helpers import check_close, live_ring_values

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bench():
    return importlib.import_module("bench")


def test_config2_full_batch(ops, O, wl, cuda, bench):
    w = wl.config2(seed=1000)
    cache, bt = bench.build_gpu_cache(ops, w, cuda, torch)
    lens = torch.from_numpy(w.lengths).to(cuda)
    rng = np.random.default_rng(w.seed + 1)
    q = torch.from_numpy(wl.f32_to_bf16_bits(rng.standard_normal((w.B, w.Hq, w.D))).view(
        np.int16)).view(torch.bfloat16).to(cuda)
    scale = 1 / math.sqrt(w.D)
    max_ctx = int(w.lengths.max())
    out = ops.paged_decode(cache, q, bt, lens, max_ctx, scale=scale, out_dtype=torch.float32)

    # oracle on sampled sequences of the GPU-built cache (ring rows = batch rows)
    sample = [0, 1, 2, 3]
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, len(sample))
    st.pool = cache.pool.cpu().numpy()
    st.ring = np.ascontiguousarray(cache.ring.cpu().numpy().view(np.uint16)[sample])
    ref = st.decode(q.float().cpu().numpy()[sample], w.block_tables[sample], w.lengths[sample],
                    scale, n_threads=8)
    check_close(out.cpu().numpy()[sample], ref)

    # batch independence of the split partials: full batch vs sequences 5, 17, 40
    S = ops.decode_num_splits(max_ctx)
    ml = torch.empty((S, w.B, w.Hq, 2), dtype=torch.float32, device=cuda)
    o = torch.empty((S, w.B, w.Hq, w.D), dtype=torch.float32, device=cuda)
    ops.paged_decode_partials(cache, q, bt, lens, 0, S - 1, True, ml, o, scale=scale)
    sub = torch.tensor([5, 17, 40], dtype=torch.long, device=cuda)
    ml_s = torch.empty((S, 3, w.Hq, 2), dtype=torch.float32, device=cuda)
    o_s = torch.empty((S, 3, w.Hq, w.D), dtype=torch.float32, device=cuda)
    ops.paged_decode_partials(cache, q[sub].contiguous(), bt[sub].contiguous(),
                              lens[sub].contiguous(), 0, S - 1, True, ml_s, o_s, scale=scale,
                              seq_slots=sub.to(torch.int32))
    torch.cuda.synchronize()
    assert torch.equal(ml_s, ml[:, sub])
    written = torch.isfinite(ml_s[..., 0])  # empty split slots leave o unwritten
    assert torch.equal(o_s[written], o[:, sub][written])


def _append(ops, cache, k, v, T, B, bt, cu_lo, cu_hi, lens_old, cuda):
    """Appends tokens [cu_lo, cu_hi) of every sequence's T-token chunk."""
    n = cu_hi - cu_lo
    idx = (torch.arange(B, device=cuda)[:, None] * T + cu_lo +
           torch.arange(n, device=cuda)[None, :]).reshape(-1)
    cu = (torch.arange(B + 1, dtype=torch.int32) * n).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_append(cache, k[idx].contiguous(), v[idx].contiguous(), cu,
                     torch.full((B,), lens_old, dtype=torch.int32, device=cuda), bt,
                     max_new_tokens=n, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def test_config3_full_append(ops, O, wl, cuda, bench):
    w = wl.config3(seed=3000)
    k, v = bench.append_inputs(wl, w, torch, cuda)
    fmt = ops.KiviFormat(w.D, w.group, w.residual, w.bits, w.Hkv)
    bt = torch.from_numpy(w.block_tables).to(cuda)
    one = ops.KiviPagedCache(fmt, w.num_pages, w.B, cuda)
    _append(ops, one, k, v, w.T, w.B, bt, 0, w.T, 0, cuda)
    two = ops.KiviPagedCache(fmt, w.num_pages, w.B, cuda)
    _append(ops, two, k, v, w.T, w.B, bt, 0, w.T // 2, 0, cuda)
    _append(ops, two, k, v, w.T, w.B, bt, w.T // 2, w.T, w.T // 2, cuda)
    lengths = np.full(w.B, w.T, np.int32)

    # oracle bytes of sampled sequences
    sample = [0, 31, 63]
    kb = k.view(torch.int16).cpu().numpy().view(np.uint16).reshape(w.B, w.T, w.Hkv, w.D)
    vb = v.view(torch.int16).cpu().numpy().view(np.uint16).reshape(w.B, w.T, w.Hkv, w.D)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, len(sample))
    cu = (np.arange(len(sample) + 1) * w.T).astype(np.int32)
    st.append(kb[sample].reshape(-1, w.Hkv, w.D), vb[sample].reshape(-1, w.Hkv, w.D), True, cu,
              np.zeros(len(sample), np.int32), w.block_tables[sample])
    pool = one.pool.cpu().numpy()
    pages = w.block_tables[sample][:, :st.nq(w.T) // 16].reshape(-1)
    assert np.array_equal(pool[pages], st.pool[pages])
    ring = one.ring.cpu().numpy().view(np.uint16)
    assert np.array_equal(live_ring_values(ring[sample], st, lengths[sample]),
                          live_ring_values(st.ring, st, lengths[sample]))

    # chunking invariance over the whole batch
    assert torch.equal(one.pool, two.pool)
    ring2 = two.ring.cpu().numpy().view(np.uint16)
    assert np.array_equal(live_ring_values(ring, st, lengths), live_ring_values(ring2, st, lengths))


def _oracle_of(O, cache, w, sample, bits=None):
    """The oracle state of sampled sequences of a GPU-built cache: their pages
    gathered into a compact pool (block tables renumbered), their ring rows
    (ring rows of the GPU cache = batch rows) in sample order."""
    bits = w.bits if bits is None else bits
    bt = w.block_tables[sample]
    used = [bt[i, bt[i] >= 0] for i in range(len(sample))]
    pages = np.unique(np.concatenate(used))
    remap = np.full(w.num_pages, -1, np.int32)
    remap[pages] = np.arange(len(pages), dtype=np.int32)
    bt_c = np.where(bt >= 0, remap[np.maximum(bt, 0)], -1).astype(np.int32)
    st = O.PagedState(w.D, w.group, w.residual, bits, w.Hkv, len(pages), len(sample))
    idx = torch.from_numpy(pages.astype(np.int64)).to(cache.pool.device)
    st.pool = np.ascontiguousarray(cache.pool[idx].cpu().numpy())
    rows = torch.tensor(sample, dtype=torch.long, device=cache.ring.device)
    st.ring = np.ascontiguousarray(cache.ring[rows].cpu().numpy().view(np.uint16))
    return st, bt_c


def _q(wl, w, cuda, seed_add=1):
    rng = np.random.default_rng(w.seed + seed_add)
    return torch.from_numpy(wl.f32_to_bf16_bits(rng.standard_normal((w.B, w.Hq, w.D))).view(
        np.int16)).view(torch.bfloat16).to(cuda)


def test_config4_full_batch(ops, O, wl, cuda, bench):
    """Config 4 (B=8, 131072-token contexts, Hq=64, Hkv=8): every pair spans
    hundreds of warps and merges in the slot-parallel merge kernel; two
    sampled sequences against the oracle, and the token-split layout (two
    ranges plus the residual, merged) against the one-call decode."""
    w = wl.config4(seed=4000)
    cache, bt = bench.build_gpu_cache(ops, w, cuda, torch)
    lens = torch.from_numpy(w.lengths).to(cuda)
    q = _q(wl, w, cuda)
    scale = 1 / math.sqrt(w.D)
    max_ctx = int(w.lengths.max())
    assert ops.decode_launches(w.B, w.Hq, w.Hkv, max_ctx) == 2
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_decode(cache, q, bt, lens, max_ctx, scale=scale, out_dtype=torch.float32,
                           err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    sample = [0, 5]
    st, bt_c = _oracle_of(O, cache, w, sample)
    ref = st.decode(q.float().cpu().numpy()[sample], bt_c, w.lengths[sample], scale, n_threads=16)
    check_close(out.cpu().numpy()[sample], ref)

    # token split as the multi-GPU layout runs it: ranges [0, 100), [100, n)
    # of the 512-token splits, the second with the residual
    n = (O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, 1, 1).nq(max_ctx) + 511) // 512
    ml = torch.empty((2, w.B, w.Hq, 2), dtype=torch.float32, device=cuda)
    o = torch.empty((2, w.B, w.Hq, w.D), dtype=torch.float32, device=cuda)
    for r, (lo, hi) in enumerate(((0, 100), (100, n))):
        ws = torch.zeros(ops.decode_range_workspace_bytes(w.B, w.Hq, w.D, lo, hi),
                         dtype=torch.uint8, device=cuda)
        ops.paged_decode_range(cache, q, bt, lens, lo, hi, r == 1, ml[r], o[r], ws, scale=scale,
                               err=err)
    merged = ops.merge_partials(ml, o, torch.empty_like(out))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.allclose(merged, out, atol=2e-3, rtol=2e-3)


def test_config5_full_batch(ops, O, wl, cuda, bench):
    """Config 5 (B=256, log-uniform 128-32768 contexts; sequences 0-127 INT4,
    128-255 INT2, each half one call with the merge fused): the longest and
    the shortest sequence of each half against the oracle."""
    w = wl.config5(seed=5000)
    scale = 1 / math.sqrt(w.D)
    for bits, seqs in ((4, np.arange(0, w.B // 2)), (2, np.arange(w.B // 2, w.B))):
        sub = wl.subset(w, seqs, bits=bits)
        cache, bt = bench.build_gpu_cache(ops, sub, cuda, torch)
        lens = torch.from_numpy(sub.lengths).to(cuda)
        q = _q(wl, sub, cuda)
        max_ctx = int(sub.lengths.max())
        assert ops.decode_launches(sub.B, sub.Hq, sub.Hkv, max_ctx) == 1
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = ops.paged_decode(cache, q, bt, lens, max_ctx, scale=scale,
                               out_dtype=torch.float32, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        sample = [int(np.argmax(sub.lengths)), int(np.argmin(sub.lengths))]
        st, bt_c = _oracle_of(O, cache, sub, sample, bits)
        ref = st.decode(q.float().cpu().numpy()[sample], bt_c, sub.lengths[sample], scale,
                        n_threads=16)
        check_close(out.cpu().numpy()[sample], ref)
        del cache
        torch.cuda.empty_cache()
