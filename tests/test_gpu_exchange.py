"""Token-split decode over peer memory (tkv_exchange_decode_range +
tkv_exchange_merge).

* One process plays every rank on one GPU (each rank's publish runs before
  any rank's merge, so no kernel waits on one that has not run): for 1-4
  ranks, including ranks whose range is empty, every rank's merged output
  equals the one-call decode (and the oracle), on consecutive steps (the two
  parity sets of the exchange buffer).
* A rank whose peer never publishes: the merge's bounded wait gives up,
  reports TKV_ERR_TIMEOUT and writes zeros; the GPU stays usable.
* Two processes on two GPUs (skipped with fewer): `TokenSplitDecoder` over a
  gloo group that only swaps the IPC handles.
"""
import importlib
import math
import os
import time

import numpy as np
import pytest
import torch

from kivi_helpers import check_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def SH():
    return importlib.import_module("truellm-engine_b200.sharding")


@pytest.fixture(scope="module")
def bench():
    return importlib.import_module("bench")


def _case(wl, ops, bench, cuda, L, B=2, seed=4100):
    """Config-4 shapes (Hq=64, Hkv=8, D=128, G=R=128) at context L."""
    w = wl.config4(seed=seed, B=B, L=L)
    cache, bt = bench.build_gpu_cache(ops, w, cuda, torch)
    lens = torch.from_numpy(w.lengths).to(cuda)
    rng = np.random.default_rng(seed + 1)
    q = torch.from_numpy(wl.f32_to_bf16_bits(rng.standard_normal((w.B, w.Hq, w.D))).view(
        np.int16)).view(torch.bfloat16).to(cuda)
    return w, cache, bt, lens, q


@pytest.mark.parametrize("L,world", [(9216, 1), (9216, 2), (9216, 3), (9216, 4), (608, 4)])
def test_emulated_ranks_equal_one_call_decode(ops, O, wl, cuda, bench, SH, L, world):
    w, cache, bt, lens, q = _case(wl, ops, bench, cuda, L)
    scale = 1 / math.sqrt(w.D)
    want = ops.paged_decode(cache, q, bt, lens, L, scale=scale, out_dtype=torch.float32)
    n = SH.quantized_splits(L, w.residual, w.group)
    ranges = SH.split_ranges(n, world)
    exs, bufs = SH.local_exchanges(world, w.B, w.Hq, w.D)
    ws = [torch.zeros(ops.decode_range_workspace_bytes(w.B, w.Hq, w.D, lo, hi),
                      dtype=torch.uint8, device=cuda) for lo, hi in ranges]
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for step in range(3):
            outs = [torch.full((w.B, w.Hq, w.D), float("nan"), device=cuda)
                    for _ in range(world)]
            for r, (lo, hi) in enumerate(ranges):
                ops.exchange_decode_range(cache, q, bt, lens, lo, hi, r == world - 1, exs[r],
                                          ws[r], scale=scale, err=err)
            for r in range(world):
                ops.exchange_merge(exs[r], outs[r], err=err)
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            for r in range(world):
                assert torch.equal(outs[r], outs[0]), (step, r)
            # another split of the tokens: another fp16 rounding of the weights
            assert torch.allclose(outs[0], want, atol=1e-3, rtol=1e-3)
        # the oracle on sequence 0
        st = O.PagedState(w.D, w.group, w.residual, w.bits, w.Hkv, w.num_pages, 1)
        st.pool = cache.pool.cpu().numpy()
        st.ring = np.ascontiguousarray(cache.ring.cpu().numpy().view(np.uint16)[:1])
        ref = st.decode(q.float().cpu().numpy()[:1], w.block_tables[:1], w.lengths[:1], scale,
                        n_threads=8)
        check_close(outs[0].cpu().numpy()[:1], ref)
    finally:
        for b in bufs:
            b.close()


def test_missing_peer_times_out_and_gpu_stays_usable(ops, wl, cuda, bench, SH):
    w, cache, bt, lens, q = _case(wl, ops, bench, cuda, 3008, B=1)
    exs, bufs = SH.local_exchanges(2, w.B, w.Hq, w.D)
    ws = torch.zeros(ops.decode_range_workspace_bytes(w.B, w.Hq, w.D, 0, 100),
                     dtype=torch.uint8, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.full((w.B, w.Hq, w.D), float("nan"), device=cuda)
    try:
        # rank 0 publishes everything; rank 1 (a flag nothing sets) never does
        ops.exchange_decode_range(cache, q, bt, lens, 0, 100, True, exs[0], ws, err=err)
        t0 = time.time()
        ops.exchange_merge(exs[0], out, err=err)
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert int(err.item()) & 0x8  # TKV_ERR_TIMEOUT
        assert torch.all(out == 0)
        assert 1.0 < waited < 30.0
        # the context is fine: an ordinary decode afterwards
        err.zero_()
        got = ops.paged_decode(cache, q, bt, lens, 3008, out_dtype=torch.float32, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and torch.isfinite(got).all()
    finally:
        for b in bufs:
            b.close()


def _two_gpu_worker(rank, port, result):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        ops = importlib.import_module("truellm-engine_b200.ops")
        wl = importlib.import_module("truellm-engine_b200.workloads")
        SH = importlib.import_module("truellm-engine_b200.sharding")
        bench = importlib.import_module("bench")
        w, cache, bt, lens, q = _case(wl, ops, bench, dev, 20000, B=1)
        want = ops.paged_decode(cache, q, bt, lens, 20000, out_dtype=torch.float32)
        dec = SH.TokenSplitDecoder(w.B, w.Hq, w.D, 20000, w.residual, w.group, dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        worst = 0.0
        for _ in range(3):
            out = torch.empty((w.B, w.Hq, w.D), device=dev)
            dec(cache, q, bt, lens, out, err=err)
            torch.cuda.synchronize()
            worst = max(worst, float((out - want).abs().max()))
        dec.close()
        result[rank] = (int(err.item()), worst)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_processes_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = 29600 + os.getpid() % 300
    mp.spawn(_two_gpu_worker, args=(port, result), nprocs=2, join=True)
    for rank in range(2):
        err, worst = result[rank]
        assert err == 0 and worst < 1e-3, (rank, err, worst)
