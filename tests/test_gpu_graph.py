"""tkv_paged_decode inside a CUDA graph (GPU).

A serving loop (and bench.py above one GPU) records a decode step once and
replays it: here an INT4 and an INT2 cache are decoded by two calls on two
streams, captured into one graph with the streams forked from and joined to
the capture stream.  The replayed outputs must equal the outputs of the same
calls made directly, and the device error word must stay clear.
"""
import math

import numpy as np
import pytest
import torch

from kivi_helpers import i32
from test_gpu_paged import _build

pytestmark = pytest.mark.gpu


def _part(ops, O, wl, cuda, bits, lengths, seed):
    tw, bt, lengths, rng = _build(ops, O, wl, cuda, 128, 32, 32, bits, 2, lengths, "bf16",
                                  chunks=(97, 16, 1), seed=seed)
    Hq = 8
    q = torch.from_numpy(wl.f32_to_bf16_bits(rng.standard_normal((len(lengths), Hq, 128)))
                         .view(np.int16)).view(torch.bfloat16).to(cuda)
    max_ctx = int(lengths.max())
    return {
        "tw": tw, "q": q, "bt": i32(bt, cuda), "lens": i32(lengths, cuda), "max_ctx": max_ctx,
        "out": torch.empty_like(q),
        "ws": torch.zeros(ops.decode_workspace_bytes(len(lengths), Hq, 128, max_ctx),
                          dtype=torch.uint8, device=cuda),
    }


def _call(ops, p, stream):
    return ops.PreparedDecode(p["tw"].gpu, p["q"], p["bt"], p["lens"], p["max_ctx"], p["out"],
                              p["ws"], scale=1.0 / math.sqrt(128), err=p["tw"].err,
                              stream=stream)


def test_two_stream_decode_step_replays_as_one_graph(ops, O, wl, cuda):
    parts = [_part(ops, O, wl, cuda, 4, [300, 517, 40, 129], seed=11),
             _part(ops, O, wl, cuda, 2, [1000, 33, 250], seed=12)]
    side = torch.cuda.Stream()

    def step(calls):
        cur = torch.cuda.current_stream()
        side.wait_stream(cur)
        calls[0]()
        with torch.cuda.stream(side):
            calls[1]()
        cur.wait_stream(side)

    direct = [_call(ops, parts[0], torch.cuda.current_stream()), _call(ops, parts[1], side)]
    step(direct)
    torch.cuda.synchronize()
    want = [p["out"].clone() for p in parts]
    for p in parts:
        assert int(p["tw"].err.item()) == 0

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = [_call(ops, parts[0], torch.cuda.current_stream()), _call(ops, parts[1], side)]
        step(captured)
    for p in parts:
        p["out"].zero_()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    for p, w in zip(parts, want):
        assert int(p["tw"].err.item()) == 0
        assert torch.equal(p["out"], w)
    del graph
