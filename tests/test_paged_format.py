"""CPU checks of the paged KIVI format: layout math shared by the library and
the oracle, append chunking invariance, the link between the paged quantizer
and the reference-format quantizer, and the fp64 decode / merge oracle."""
import itertools

import numpy as np
import pytest

COMBOS = [(d, g, b) for d in (64, 128) for g in (16, 32, 64, 128) for b in (4, 2)]


@pytest.mark.parametrize("D,G,bits", COMBOS)
def test_layout_math_library_vs_oracle(O, ops, D, G, bits):
    lf = ops.KiviFormat(D, G, 37, bits, 3).c_struct()
    st = O.PagedState(D, G, 37, bits, 3, 4, 2)
    for name in ("head_dim", "residual", "bits", "n_kv_heads", "ring_cap", "n_vgroups",
                 "k_codes_off", "v_codes_off", "v_meta_off", "k_meta_off", "k_meta_slice",
                 "page_bytes"):
        assert getattr(lf, name) == getattr(st.fmt, name), name
    assert lf.group_size == st.fmt.group


def test_documented_page_sizes(ops):
    assert ops.KiviFormat(128, 128, 128, 4, 8).page_bytes == 2176
    assert ops.KiviFormat(128, 128, 128, 2, 8).page_bytes == 1152


def _seq_inputs(wl, rng, lengths, Hkv, D, dtype="f16"):
    T = int(sum(lengths))
    k, v = wl.kv_tokens(rng, T, Hkv, D, np.array([1, 5]), 8.0)
    return wl.to_bits(k, dtype), wl.to_bits(v, dtype)


def _append_chunked(O, fmt_args, lengths, kb, vb, bt, chunks, in_bf16, num_pages):
    """Append each sequence's tokens in the given chunk sizes (round robin)."""
    st = O.PagedState(*fmt_args, num_pages, len(lengths))
    B = len(lengths)
    starts = np.concatenate([[0], np.cumsum(lengths)])
    done = [0] * B
    step = 0
    while any(done[b] < lengths[b] for b in range(B)):
        cu = [0]
        ks, vs = [], []
        lens_old = []
        for b in range(B):
            n = min(chunks[(step + b) % len(chunks)], lengths[b] - done[b])
            lens_old.append(done[b])
            s = starts[b] + done[b]
            ks.append(kb[s:s + n]); vs.append(vb[s:s + n])
            cu.append(cu[-1] + n)
            done[b] += n
        st.append(np.concatenate(ks), np.concatenate(vs), in_bf16, np.array(cu, np.int32),
                  np.array(lens_old, np.int32), bt)
        step += 1
    return st


def _live_ring(st, lengths):
    out = []
    for b, L in enumerate(lengths):
        for h in range(st.fmt.n_kv_heads):
            for t in range(st.nq(L), L):
                for kv in (0, 1):
                    out.append([O_ring(st, b, h, t, kv, c) for c in range(st.fmt.head_dim)])
    return np.array(out)


def O_ring(st, b, h, t, kv, c):
    from oracle import oracle as mod
    return mod.lib().or_ring_get(mod.C.byref(st.fmt), st.ring, b, h, t, kv, c)


@pytest.mark.parametrize("D,G,R,bits,dtype", [(64, 32, 32, 4, "f16"), (128, 128, 128, 4, "bf16"),
                                              (64, 16, 5, 2, "bf16"), (128, 64, 0, 2, "f16")])
def test_append_chunking_invariance(O, wl, D, G, R, bits, dtype):
    rng = np.random.default_rng(7)
    lengths = [300, 45, 161]
    Hkv = 2
    kb, vb = _seq_inputs(wl, rng, lengths, Hkv, D, dtype)
    num_pages = 64
    bt = wl.random_block_tables(np.array(lengths), num_pages, rng)
    args = (D, G, R, bits, Hkv)
    ref = _append_chunked(O, args, lengths, kb, vb, bt, [10 ** 6], dtype == "bf16", num_pages)
    for chunks in ([1], [7, 1, 33], [16], [G + 3, 2]):
        st = _append_chunked(O, args, lengths, kb, vb, bt, chunks, dtype == "bf16", num_pages)
        assert np.array_equal(st.pool, ref.pool), chunks
        assert np.array_equal(_live_ring(st, lengths), _live_ring(ref, lengths)), chunks


@pytest.mark.parametrize("D,G", [(64, 32), (128, 128), (128, 16)])
def test_paged_codes_equal_reference_quantizer(O, wl, D, G):
    """Keys: the per-channel group over G tokens equals the reference
    kivi_compress (0 outliers, group G) of the transposed [D, G] tile; values:
    each token equals kivi_compress of the vector with group G."""
    rng = np.random.default_rng(11)
    L = 3 * G + G // 2 + 40
    R = 40
    Hkv = 1
    kb, vb = _seq_inputs(wl, rng, [L], Hkv, D, "f16")
    bt = wl.random_block_tables(np.array([L]), 64, rng)
    st = O.PagedState(D, G, R, 4, Hkv, 64, 1)
    st.append(kb, vb, False, np.array([0, L], np.int32), np.array([0], np.int32), bt)
    nq = st.nq(L)
    assert nq == 3 * G
    kx = kb[:, 0, :]
    vx = vb[:, 0, :]
    for g0 in range(0, nq, G):
        tile = np.ascontiguousarray(kx[g0:g0 + G].T)            # [D, G]
        rec = O.kivi_compress(tile, 0, G)                        # [D, G/2 + 4]
        for t in range(g0, g0 + G):
            kc, ks, kz, vc, vs, vz = st.unpack_token(bt[0], 0, t)
            i = t - g0
            codes = (rec[:, i // 2] >> (4 * (i % 2))) & 15
            assert np.array_equal(kc, codes)
            assert np.array_equal(ks, rec[:, G // 2:G // 2 + 2].copy().view(np.uint16)[:, 0])
            assert np.array_equal(kz, rec[:, G // 2 + 2:G // 2 + 4].copy().view(np.uint16)[:, 0])
            vrec = O.kivi_compress(vx[t:t + 1], 0, G)[0]
            nvg = -(-D // G)
            for gi in range(nvg):
                base = gi * (G // 2 + 4)
                n = min(G, D - gi * G)
                cb = vrec[base:base + (n + 1) // 2]
                vcodes = np.stack([cb & 15, cb >> 4], 1).reshape(-1)[:n]
                assert np.array_equal(vc[gi * G:gi * G + n], vcodes)
                assert vs[gi] == vrec[base + n // 2:base + n // 2 + 2].view(np.uint16)[0]
                assert vz[gi] == vrec[base + n // 2 + 2:base + n // 2 + 4].view(np.uint16)[0]


def _dequant_numpy(O, st, bt_row, h, L):
    """Independent numpy dequantisation of a sequence: fp32(code*step + zero)
    (the sum is exact in fp64 for these inputs, so this is fmaf) rounded to
    fp16, as the reference decompress writes __half."""
    D, G = st.fmt.head_dim, st.fmt.group
    nq = st.nq(L)
    K = np.zeros((L, D)); V = np.zeros((L, D))
    vg = np.arange(D) // G
    for t in range(L):
        if t < nq:
            kc, ks, kz, vc, vs, vz = st.unpack_token(bt_row, h, t)
            f = lambda u: u.view(np.float16).astype(np.float64)
            K[t] = (kc * f(ks) + f(kz)).astype(np.float32).astype(np.float16)
            V[t] = (vc * f(vs)[vg] + f(vz)[vg]).astype(np.float32).astype(np.float16)
        else:
            for c in range(D):
                K[t, c] = np.uint16(O_ring(st, 0, h, t, 0, c)).view(np.float16)
                V[t, c] = np.uint16(O_ring(st, 0, h, t, 1, c)).view(np.float16)
    return K, V


def test_decode_oracle_against_numpy_attention(O, wl):
    w = wl.config1()
    rng = np.random.default_rng(w.seed)
    L = int(w.lengths[0])
    k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
    st.append(wl.to_bits(k, "f16"), wl.to_bits(v, "f16"), False, np.array([0, L], np.int32),
              np.array([0], np.int32), w.block_tables)
    q = rng.standard_normal((1, w.Hq, w.D)).astype(np.float16).astype(np.float32)
    scale = 1 / np.sqrt(w.D)
    out = st.decode(q, w.block_tables, w.lengths, scale)
    for h in range(w.Hkv):
        K, V = _dequant_numpy(O, st, w.block_tables[0], h, L)
        s = (K @ q[0, h].astype(np.float64)) * scale
        p = np.exp(s - s.max())
        ref = (p @ V) / p.sum()
        assert np.allclose(out[0, h], ref, atol=1e-6, rtol=1e-6)


def test_partial_merge_equals_full(O, wl):
    w = wl.config1()
    rng = np.random.default_rng(3)
    L = int(w.lengths[0])
    k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
    st.append(wl.to_bits(k, "f16"), wl.to_bits(v, "f16"), False, np.array([0, L], np.int32),
              np.array([0], np.int32), w.block_tables)
    q = rng.standard_normal((1, w.Hq, w.D)).astype(np.float32)
    full = st.decode(q, w.block_tables, w.lengths, 0.125)
    cuts = [0, 100, 256, 257, 480, L]
    ms, ls, os_ = [], [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        m, l, o = st.decode_partial(q, w.block_tables, w.lengths, 0.125, a, b)
        ms.append(m.reshape(-1)); ls.append(l.reshape(-1)); os_.append(o.reshape(-1, w.D))
    merged = O.merge(np.array(ms), np.array(ls), np.array(os_))
    assert np.allclose(merged.reshape(full.shape), full, atol=1e-12, rtol=1e-10)


def test_prefill_oracle_against_numpy_causal_attention(O, wl):
    """The chunked-prefill restatement: each of the last n tokens attends to
    the cached tokens up to its own position (GQA 2)."""
    w = wl.config1()
    rng = np.random.default_rng(5)
    L, n, Hq = int(w.lengths[0]), 100, 2 * w.Hkv
    k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
    st.append(wl.to_bits(k, "f16"), wl.to_bits(v, "f16"), False, np.array([0, L], np.int32),
              np.array([0], np.int32), w.block_tables)
    q = rng.standard_normal((n, Hq, w.D)).astype(np.float16).astype(np.float32)
    scale = 1 / np.sqrt(w.D)
    out = st.prefill(q, np.array([0, n], np.int32), w.block_tables, w.lengths, scale)
    for h in range(w.Hkv):
        K, V = _dequant_numpy(O, st, w.block_tables[0], h, L)
        for i in range(0, n, 7):
            p = L - n + i
            for j in range(2):
                s = (K[:p + 1] @ q[i, 2 * h + j].astype(np.float64)) * scale
                e = np.exp(s - s.max())
                ref = (e @ V[:p + 1]) / e.sum()
                assert np.allclose(out[i, 2 * h + j], ref, atol=1e-6, rtol=1e-6)


def test_prefill_oracle_last_row_equals_decode(O, wl):
    w = wl.config1()
    rng = np.random.default_rng(6)
    L = int(w.lengths[0])
    k, v = wl.kv_tokens(rng, L, w.Hkv, w.D, w.outlier_channels, w.outlier_scale)
    st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
    st.append(wl.to_bits(k, "f16"), wl.to_bits(v, "f16"), False, np.array([0, L], np.int32),
              np.array([0], np.int32), w.block_tables)
    q = rng.standard_normal((3, w.Hq, w.D)).astype(np.float32)
    pre = st.prefill(q, np.array([0, 3], np.int32), w.block_tables, w.lengths, 0.125)
    dec = st.decode(q[2:], w.block_tables, w.lengths, 0.125)
    assert np.array_equal(pre[2], dec[0])
