"""Multi-GPU host logic on CPU: the sharding plans, and the three layouts run
as world-size-2 gloo process groups with the CPU oracle standing in for the
per-rank kernels.

* token split (one long sequence over ranks): each rank computes the partial
  (m, l, o) of its split range (the last rank adds the fp16 residual), the
  slot blocks are exchanged with `gather_slots`, and the log-sum-exp merge of
  the gathered slots equals the single-process decode;
* sequence sharding: ranks decode their `balance_sequences` share, the
  gathered outputs in sequence order equal the full batch decode;
* kv-head sharding: each rank keeps only its kv heads' cache, the gathered
  head slices equal the full decode.
"""
import importlib
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SH = importlib.import_module("truellm-engine_b200.sharding")


# ---------------------------------------------------------------- planning
def test_split_ranges_cover_contiguously():
    for n in range(0, 40):
        for world in (1, 2, 3, 4, 8):
            rs = SH.split_ranges(n, world)
            assert len(rs) == world and rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [hi - lo for lo, hi in rs]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)


def test_balance_sequences_is_greedy_and_deterministic():
    lens = [100, 5000, 300, 300, 7000, 20, 2500, 2500]
    parts = SH.balance_sequences(lens, 3)
    # longest first to the lightest rank (ties to the lower rank):
    # 7000->0, 5000->1, 2500->2, 2500->2, 300->1, 300->2, 100->1, 20->2
    assert [p.tolist() for p in parts] == [[4], [0, 1, 2], [3, 5, 6, 7]]
    assert [int(np.asarray(lens)[p].sum()) for p in parts] == [7000, 5400, 5320]
    assert SH.balance_sequences(lens, 1)[0].tolist() == list(range(len(lens)))
    assert [p.tolist() for p in SH.balance_sequences([5, 5], 4)] == [[0], [1], [], []]


def test_head_shard():
    kv, qh = SH.head_shard(8, 64, 8, 3)
    assert list(kv) == [3] and list(qh) == list(range(24, 32))
    kv, qh = SH.head_shard(8, 32, 2, 1)
    assert list(kv) == [4, 5, 6, 7] and list(qh) == list(range(16, 32))
    with pytest.raises(ValueError):
        SH.head_shard(8, 32, 3, 0)


def test_quantized_splits():
    assert SH.quantized_splits(131072, 128, 128) == 256      # config 4: 130944 quantised tokens
    assert SH.quantized_splits(128, 128, 128) == 0
    assert SH.quantized_splits(255 + 128, 128, 128) == 1


# ---------------------------------------------------------------- gloo ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cache(O, wl, D, G, R, Hkv, lengths, seed):
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, np.int32)
    num_pages = int(sum((int(L) + 15) // 16 for L in lengths)) + 3
    bt = wl.random_block_tables(lengths, num_pages, rng)
    k, v = wl.kv_tokens(rng, int(lengths.sum()), Hkv, D, np.array([1, 5]), 8.0)
    st = O.PagedState(D, G, R, 4, Hkv, num_pages, len(lengths))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    st.append(wl.to_bits(k, "bf16"), wl.to_bits(v, "bf16"), True, cu,
              np.zeros(len(lengths), np.int32), bt)
    return st, bt, lengths, k, v, rng


def _token_split_rank(rank, world, port, L, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        wl = importlib.import_module("truellm-engine_b200.workloads")
        D, G, R, Hkv, Hq = 64, 32, 32, 2, 8
        st, bt, lengths, _, _, rng = _cache(O, wl, D, G, R, Hkv, [L], seed=7)
        q = rng.standard_normal((1, Hq, D)).astype(np.float32)
        scale = 1 / math.sqrt(D)
        n = SH.quantized_splits(L, R, G)
        ranges = SH.split_ranges(n, world)
        lo, hi = ranges[rank]
        last = rank == world - 1
        slots = max(b - a for a, b in ranges) + 1
        # this rank's slot block: one oracle partial over its token range, the
        # other slots empty (m = -inf, l = 0, o = 0)
        ml = torch.zeros((slots, 1, Hq, 2), dtype=torch.float64)
        ml[..., 0] = float("-inf")
        o = torch.zeros((slots, 1, Hq, D), dtype=torch.float64)
        tok_lo, tok_hi = lo * SH.SPLIT_TOKENS, (L if last else hi * SH.SPLIT_TOKENS)
        if tok_hi > tok_lo:
            m, l, oo = st.decode_partial(q, bt, lengths, scale, tok_lo, tok_hi)
            ml[0, ..., 0] = torch.from_numpy(m)
            ml[0, ..., 1] = torch.from_numpy(l)
            o[0] = torch.from_numpy(oo)
        all_ml, all_o = SH.gather_slots(ml, o)
        assert all_ml.shape[0] == world * slots
        P = all_ml.shape[0]
        merged = O.merge(all_ml[..., 0].reshape(P, -1).numpy(), all_ml[..., 1].reshape(P, -1).numpy(),
                         all_o.reshape(P, Hq, D).numpy()).reshape(1, Hq, D)
        full = st.decode(q, bt, lengths, scale)
        out_q.put((rank, float(np.abs(merged - full).max()), (lo, hi)))
    finally:
        dist.destroy_process_group()


def _run(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res)


@pytest.mark.parametrize("L", [1500 + 32 + 5, 300])
def test_token_split_gather_merge_equals_full_decode(L):
    """L=300: one quantised split, so rank 1 owns only the residual window."""
    res = _run(_token_split_rank, 2, L)
    for rank, err, _ in res:
        assert err < 1e-9, (rank, err)


def _seq_shard_rank(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        wl = importlib.import_module("truellm-engine_b200.workloads")
        D, G, R, Hkv, Hq = 64, 32, 32, 2, 4
        lengths = [700, 33, 1200, 64, 400, 999]
        st, bt, lengths, _, _, rng = _cache(O, wl, D, G, R, Hkv, lengths, seed=11)
        q = rng.standard_normal((len(lengths), Hq, D)).astype(np.float32)
        scale = 1 / math.sqrt(D)
        parts = SH.balance_sequences(lengths, world)
        mine = parts[rank]
        # each rank decodes its sequences; ring rows follow the batch index, so
        # the rank keeps the full cache here and passes its rows' tables only
        sub = O.PagedState(D, G, R, 4, Hkv, st.num_pages, len(mine))
        sub.pool[:] = st.pool
        sub.ring[:] = st.ring[mine]
        out = torch.from_numpy(sub.decode(q[mine], bt[mine], lengths[mine], scale))
        # gather variable-size shares: pad to the largest share
        n_max = max(len(p) for p in parts)
        pad = torch.zeros((n_max, Hq, D), dtype=torch.float64)
        pad[:len(mine)] = out
        got = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(got, pad)
        full_out = torch.empty((len(lengths), Hq, D), dtype=torch.float64)
        for r, p in enumerate(parts):
            full_out[torch.from_numpy(p)] = got[r][:len(p)]
        full = st.decode(q, bt, lengths, scale)
        out_q.put((rank, float(np.abs(full_out.numpy() - full).max()), len(mine)))
    finally:
        dist.destroy_process_group()


def test_sequence_sharding_gather_equals_full_decode():
    res = _run(_seq_shard_rank, 2)
    assert sum(n for _, _, n in res) == 6
    for rank, err, _ in res:
        assert err < 1e-12, (rank, err)


def _head_shard_rank(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        wl = importlib.import_module("truellm-engine_b200.workloads")
        D, G, R, Hkv, Hq = 64, 32, 32, 4, 8
        lengths = [900, 150]
        st, bt, lengths, k, v, rng = _cache(O, wl, D, G, R, Hkv, lengths, seed=13)
        q = rng.standard_normal((len(lengths), Hq, D)).astype(np.float32)
        scale = 1 / math.sqrt(D)
        kvh, qh = SH.head_shard(Hkv, Hq, world, rank)
        # this rank's cache holds only its kv heads (same pages, same tables)
        mine = O.PagedState(D, G, R, 4, len(kvh), st.num_pages, len(lengths))
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        ks = np.ascontiguousarray(k[:, kvh.start:kvh.stop])
        vs = np.ascontiguousarray(v[:, kvh.start:kvh.stop])
        mine.append(wl.to_bits(ks, "bf16"), wl.to_bits(vs, "bf16"), True, cu,
                    np.zeros(len(lengths), np.int32), bt)
        out = torch.from_numpy(
            mine.decode(np.ascontiguousarray(q[:, qh.start:qh.stop]), bt, lengths, scale))
        got = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(got, out)
        full_out = torch.cat(got, dim=1).numpy()
        full = st.decode(q, bt, lengths, scale)
        out_q.put((rank, float(np.abs(full_out - full).max()), list(kvh)))
    finally:
        dist.destroy_process_group()


def test_kv_head_sharding_gather_equals_full_decode():
    res = _run(_head_shard_rank, 2)
    for rank, err, heads in res:
        assert err < 1e-12, (rank, err)
    assert [h for _, _, h in res] == [[0, 1], [2, 3]]
