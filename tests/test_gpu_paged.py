"""GPU parity of the paged KIVI path through the C ABI:
  * quantize-on-append: pool bytes and live residual ring bit-exact against
    the CPU oracle (same seeded inputs, same chunking);
  * decode attention: within 2e-3 absolute + 2e-3 relative of the oracle's
    fp64 attention over the fp16-rounded dequantised cache;
  * split partials + merge equal the full decode; bounds errors are reported
    through the device error word.
"""
import math

import numpy as np
import pytest
import torch

from kivi_helpers import Twin, bits_to_torch, check_close, i32

pytestmark = pytest.mark.gpu

ATOL = 2e-3
RTOL = 2e-3


def _build(ops, O, wl, cuda, D, G, R, bits, Hkv, lengths, dtype, chunks=(10 ** 6,), seed=0,
           outliers=(1, 7), num_pages=None):
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, np.int32)
    need = int(sum((int(L) + 15) // 16 for L in lengths))
    num_pages = num_pages or need + 7
    bt = wl.random_block_tables(lengths, num_pages, rng)
    T = int(lengths.sum())
    k, v = wl.kv_tokens(rng, T, Hkv, D, np.array(outliers), 8.0)
    kb, vb = wl.to_bits(k, dtype), wl.to_bits(v, dtype)
    tw = Twin(ops, O, D, G, R, bits, Hkv, num_pages, len(lengths), cuda)
    starts = np.concatenate([[0], np.cumsum(lengths)])
    done = np.zeros(len(lengths), np.int64)
    step = 0
    while (done < lengths).any():
        cu, ks, vs, old = [0], [], [], []
        for b in range(len(lengths)):
            n = int(min(chunks[(step + b) % len(chunks)], lengths[b] - done[b]))
            old.append(int(done[b]))
            s = int(starts[b] + done[b])
            ks.append(kb[s:s + n]); vs.append(vb[s:s + n])
            cu.append(cu[-1] + n)
            done[b] += n
        tw.append(np.concatenate(ks), np.concatenate(vs), dtype, np.array(cu, np.int32),
                  np.array(old, np.int32), bt)
        step += 1
    return tw, bt, lengths, rng


def _decode_check(ops, tw, bt, lengths, rng, Hq, q_dtype, cuda, out_dtype=torch.float32):
    B = len(lengths)
    D = tw.fmt.head_dim
    q = rng.standard_normal((B, Hq, D)).astype(np.float32)
    qb = (q.astype(np.float16).view(np.uint16) if q_dtype == "f16" else
          __import__("importlib").import_module("truellm-engine_b200.workloads").f32_to_bf16_bits(q))
    qt = bits_to_torch(qb, q_dtype, cuda)
    qf = qt.float().cpu().numpy()
    scale = 1.0 / math.sqrt(D)
    out = ops.paged_decode(tw.gpu, qt, i32(bt, cuda), i32(lengths, cuda),
                           max_context_len=int(lengths.max()), scale=scale, out_dtype=out_dtype,
                           err=tw.err)
    torch.cuda.synchronize()
    assert int(tw.err.item()) == 0
    ref = tw.cpu.decode(qf, bt, lengths, scale, n_threads=8)
    return check_close(out.float().cpu().numpy(), ref, ATOL, RTOL), out, qt


def test_config1_append_and_decode(ops, O, wl, cuda):
    """B=1, Hq=Hkv=8, D=64, L=512, G=32, R=32, fp16,
    4 of 64 key channels x10, block table = permutation of a 64-page pool."""
    w = wl.config1()
    rng = np.random.default_rng(w.seed)
    L = int(w.lengths[0])
    k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
    tw = Twin(ops, O, w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1, cuda)
    tw.append(wl.to_bits(k, "f16"), wl.to_bits(v, "f16"), "f16", np.array([0, L], np.int32),
              np.array([0], np.int32), w.block_tables)
    tw.assert_same_state(w.lengths)
    err, _, _ = _decode_check(ops, tw, w.block_tables, w.lengths, rng, w.Hq, "f16", cuda)
    assert err < ATOL


@pytest.mark.parametrize("D,G,R,bits,dtype", [
    (128, 128, 128, 4, "bf16"), (128, 128, 128, 2, "bf16"), (64, 32, 32, 4, "f16"),
    (128, 64, 40, 4, "f16"), (128, 32, 16, 2, "bf16"), (128, 16, 0, 4, "bf16"),
    (64, 16, 7, 2, "f16"), (64, 128, 128, 4, "bf16")])
def test_append_bitexact_one_shot(ops, O, wl, cuda, D, G, R, bits, dtype):
    lengths = [1000, 1, 0, 129, G + R, 517, 2 * G + R - 1]
    tw, bt, lengths, _ = _build(ops, O, wl, cuda, D, G, R, bits, 4, lengths, dtype, seed=D + G)
    tw.assert_same_state(lengths)


@pytest.mark.parametrize("chunks", [(1,), (7, 1, 33), (16,), (130, 2), (15, 2)])
def test_append_bitexact_chunked(ops, O, wl, cuda, chunks):
    lengths = [300, 45, 161, 700]
    tw, bt, lengths, _ = _build(ops, O, wl, cuda, 128, 128, 128, 4, 2, lengths, "bf16",
                                chunks=chunks, seed=5)
    tw.assert_same_state(lengths)


@pytest.mark.parametrize("D,G,R,bits,Hq,Hkv,q_dtype", [
    (128, 128, 128, 4, 32, 8, "bf16"),   # Llama-3-8B shape, GQA 4
    (128, 128, 128, 4, 64, 8, "bf16"),   # Llama-3-70B shape, GQA 8
    (128, 128, 128, 2, 32, 8, "bf16"),   # INT2
    (64, 32, 32, 4, 8, 8, "f16"),        # GQA 1
    (128, 64, 40, 4, 16, 4, "f16"),
    (128, 32, 16, 2, 12, 4, "bf16"),     # GQA 3
    (128, 16, 0, 4, 8, 2, "bf16"),
    (64, 16, 7, 2, 16, 2, "f16"),
])
def test_decode_parity(ops, O, wl, cuda, D, G, R, bits, Hq, Hkv, q_dtype):
    lengths = [1500, 1, 0, 129, 512 + R, 1023 + R, 2 * G + R - 1, 3000]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, D, G, R, bits, Hkv, lengths, "bf16",
                                  seed=17 + D + G + bits)
    _decode_check(ops, tw, bt, lengths, rng, Hq, q_dtype, cuda)


def test_decode_after_token_by_token_appends(ops, O, wl, cuda):
    """Decode-style growth: a prompt, then single-token appends crossing group
    flushes, checking state and attention along the way."""
    lengths0 = np.array([250, 129, 383], np.int32)
    tw, bt_full, _, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths0 + 140, "bf16",
                                 seed=9)
    # rebuild from scratch with a prompt then 1-token steps on a fresh twin
    tw = Twin(ops, O, 128, 128, 128, 4, 8, tw.cpu.num_pages, 3, cuda)
    lens = np.zeros(3, np.int32)
    steps = [lengths0] + [np.ones(3, np.int32)] * 140
    for i, inc in enumerate(steps):
        T = int(inc.sum())
        k, v = wl.kv_tokens(rng, T, 8, 128, np.array([1, 7]), 8.0)
        cu = np.concatenate([[0], np.cumsum(inc)]).astype(np.int32)
        tw.append(wl.to_bits(k, "bf16"), wl.to_bits(v, "bf16"), "bf16", cu, lens, bt_full)
        lens = lens + inc
        if i in (0, 6, 70, 140):
            tw.assert_same_state(lens)
            _decode_check(ops, tw, bt_full, lens, rng, 32, "bf16", cuda)


def test_long_context_split_partials_merge(ops, O, wl, cuda):
    """One long sequence: 512-token splits computed in separate calls (as when
    a sequence is split across GPUs) and merged agree with the single-call
    decode (which picks 128-token splits for so few work items) and both with
    the oracle."""
    lengths = [4 * 512 * 2 + 300]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16",
                                  seed=21)
    B, Hq, D = 1, 64, 128
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((B, Hq, D))), "bf16", cuda)
    scale = 1 / math.sqrt(D)
    full = ops.paged_decode(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), int(lengths.max()),
                            scale=scale, out_dtype=torch.float32)
    nq = tw.fmt.quantized_len(int(lengths[0]))
    n_split = (nq + 511) // 512
    cuts = [0, 3, 5, n_split]
    mls, os_ = [], []
    for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
        last = i == len(cuts) - 2
        S = (b - a) + (1 if last else 0)
        ml = torch.empty((S, B, Hq, 2), dtype=torch.float32, device=cuda)
        o = torch.empty((S, B, Hq, D), dtype=torch.float32, device=cuda)
        ops.paged_decode_partials(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), a, b, last, ml,
                                  o, scale=scale)
        mls.append(ml); os_.append(o)
    merged = ops.merge_partials(torch.cat(mls), torch.cat(os_),
                                torch.empty((B, Hq, D), dtype=torch.float32, device=cuda))
    torch.cuda.synchronize()
    assert torch.allclose(merged, full, atol=ATOL, rtol=RTOL)
    ref = tw.cpu.decode(q.float().cpu().numpy(), bt, lengths, scale, n_threads=8)
    check_close(full.cpu().numpy(), ref)
    check_close(merged.cpu().numpy(), ref)


def test_range_decode_reduces_to_one_slot_per_rank(ops, O, wl, cuda):
    """Token split over three emulated ranks: each range is computed and
    reduced in one launch to one partial per (sequence, q head)
    (tkv_paged_decode_range); the three one-slot partials merged with
    tkv_merge_partials equal the single-call decode.  The 1-token sequence has
    no quantised split, so its first two ranges are empty (m = -inf)."""
    lengths = [4 * 512 * 2 + 300, 1, 900]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16",
                                  seed=23)
    B, Hq, D = len(lengths), 64, 128
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((B, Hq, D))), "bf16", cuda)
    scale = 1 / math.sqrt(D)
    bt_d, lens_d = i32(bt, cuda), i32(lengths, cuda)
    max_ctx = int(lengths.max())
    full = ops.paged_decode(tw.gpu, q, bt_d, lens_d, max_ctx, scale=scale,
                            out_dtype=torch.float32)
    n_split = (tw.fmt.quantized_len(max_ctx) + 511) // 512
    cuts = [0, 3, 5, n_split]
    ml = torch.empty((3, B, Hq, 2), dtype=torch.float32, device=cuda)
    o = torch.empty((3, B, Hq, D), dtype=torch.float32, device=cuda)
    wss = [torch.zeros(ops.decode_range_workspace_bytes(B, Hq, D, a, b), dtype=torch.uint8,
                       device=cuda) for a, b in zip(cuts[:-1], cuts[1:])]
    for _ in range(2):  # the second call reuses the workspaces (counters reset)
        for r, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
            ops.paged_decode_range(tw.gpu, q, bt_d, lens_d, a, b, r == 2, ml[r], o[r], wss[r],
                                   scale=scale, err=tw.err)
        merged = ops.merge_partials(ml, o, torch.empty((B, Hq, D), dtype=torch.float32,
                                                       device=cuda))
        torch.cuda.synchronize()
        assert int(tw.err.item()) == 0
        assert torch.isinf(ml[0, 1, :, 0]).all() and torch.isinf(ml[1, 1, :, 0]).all()
        assert torch.allclose(merged, full, atol=ATOL, rtol=RTOL)
    check_close(merged.cpu().numpy(), tw.cpu.decode(q.float().cpu().numpy(), bt, lengths, scale,
                                                    n_threads=8))


@pytest.mark.parametrize("lengths,Hq", [
    ([20000, 1, 700, 4100, 16], 40),   # 157 128-token slots: split kernel + slot-parallel merge
    ([3000, 1, 700, 129, 2048], 40),   # few slots: merge fused into the decode launch
])
def test_decode_equals_split_kernel_plus_merge_kernel(ops, O, wl, cuda, lengths, Hq):
    """tkv_paged_decode (merge fused into the launch, or for long contexts a
    second slot-parallel merge; 128-token splits when the batch has few work
    items) and the 512-token split kernel + the standalone merge both match the
    oracle, also with a GQA group of 5 (not a multiple of the fused merge's
    4-head pass); repeated calls sharing one workspace give identical outputs
    (its counters return to zero after every call)."""
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16",
                                  seed=41)
    B, D = len(lengths), 128
    max_ctx = int(lengths.max())
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((B, Hq, D))), "bf16", cuda)
    scale = 1 / math.sqrt(D)
    bt_d, lens_d = i32(bt, cuda), i32(lengths, cuda)
    S = ops.decode_num_splits(max_ctx)
    ws = torch.zeros(ops.decode_workspace_bytes(B, Hq, D, max_ctx), dtype=torch.uint8,
                     device=cuda)
    outs = [ops.paged_decode(tw.gpu, q, bt_d, lens_d, max_ctx, scale=scale,
                             out_dtype=torch.float32, workspace=ws, err=tw.err)
            for _ in range(3)]
    ml = torch.empty((S, B, Hq, 2), dtype=torch.float32, device=cuda)
    o = torch.empty((S, B, Hq, D), dtype=torch.float32, device=cuda)
    ops.paged_decode_partials(tw.gpu, q, bt_d, lens_d, 0, S - 1, True, ml, o, scale=scale,
                              err=tw.err)
    merged = ops.merge_partials(ml, o, torch.empty((B, Hq, D), dtype=torch.float32,
                                                   device=cuda))
    torch.cuda.synchronize()
    assert int(tw.err.item()) == 0
    for out in outs:
        assert torch.equal(out, outs[0])
    assert torch.allclose(outs[0], merged, atol=ATOL, rtol=RTOL)
    ref = tw.cpu.decode(q.float().cpu().numpy(), bt, lengths, scale, n_threads=8)
    check_close(outs[0].cpu().numpy(), ref)
    check_close(merged.cpu().numpy(), ref)


def test_bf16_and_fp16_outputs(ops, O, wl, cuda):
    lengths = [700, 300]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16", seed=3)
    _, out32, q = _decode_check(ops, tw, bt, lengths, rng, 32, "bf16", cuda)
    for dt in (torch.bfloat16, torch.float16):
        out = ops.paged_decode(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), 700, out_dtype=dt)
        torch.cuda.synchronize()
        assert torch.equal(out, out32.to(dt))


def test_bad_page_id_sets_error_flag(ops, O, wl, cuda):
    """A block-table entry outside the pool is skipped and reported, not read."""
    lengths = [600]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16", seed=4)
    bad = bt.copy()
    bad[0, 3] = tw.gpu.num_pages + 5
    q = torch.zeros((1, 32, 128), dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_decode(tw.gpu, q, i32(bad, cuda), i32(lengths, cuda), 600, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 0x1
    # the context is still usable
    _decode_check(ops, tw, bt, lengths, rng, 32, "bf16", cuda)


def test_seq_slots_indirection(ops, O, wl, cuda):
    """Ring rows chosen through seq_slots give the same attention."""
    lengths = np.array([300, 200], np.int32)
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16", seed=8)
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((2, 32, 128))), "bf16", cuda)
    base = ops.paged_decode(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), 300)
    # swap the two ring rows and decode with seq_slots = [1, 0]
    tw.gpu.ring.copy_(tw.gpu.ring.flip(0))
    swapped = ops.paged_decode(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), 300,
                               seq_slots=i32([1, 0], cuda))
    torch.cuda.synchronize()
    assert torch.equal(base, swapped)


def test_sequence_longer_than_max_context_len_is_flagged(ops, O, wl, cuda):
    """max_context_len bounds seq_lens: a longer sequence is reported with
    TKV_ERR_BAD_LENGTH and gets a zero output instead of a silently truncated
    one; the other sequences of the call are unaffected."""
    lengths = [900, 300, 2000]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16",
                                  seed=12)
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((3, 32, 128))), "bf16", cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    scale = 1 / math.sqrt(128)
    out = ops.paged_decode(tw.gpu, q, i32(bt, cuda), i32(lengths, cuda), 1000, scale=scale,
                           out_dtype=torch.float32, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 0x4
    assert torch.all(out[2] == 0)
    ref = tw.cpu.decode(q.float().cpu().numpy()[:2], bt[:2], lengths[:2], scale, n_threads=8)
    check_close(out[:2].cpu().numpy(), ref)


def test_prepared_decode_equals_paged_decode(ops, O, wl, cuda):
    """PreparedDecode (arguments bound once) launches the same decode."""
    lengths = [700, 1300, 90]
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 128, 128, 4, 8, lengths, "bf16",
                                  seed=13)
    q = bits_to_torch(wl.f32_to_bf16_bits(rng.standard_normal((3, 32, 128))), "bf16", cuda)
    bt_d, lens_d = i32(bt, cuda), i32(lengths, cuda)
    want = ops.paged_decode(tw.gpu, q, bt_d, lens_d, 1300, out_dtype=torch.float32)
    out = torch.empty_like(want)
    ws = torch.zeros(ops.decode_workspace_bytes(3, 32, 128, 1300), dtype=torch.uint8,
                     device=cuda)
    call = ops.PreparedDecode(tw.gpu, q, bt_d, lens_d, 1300, out, ws, err=tw.err)
    for _ in range(2):
        call()
        torch.cuda.synchronize()
        assert int(tw.err.item()) == 0
        assert torch.equal(out, want)
