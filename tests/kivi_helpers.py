"""Shared helpers for the GPU parity tests: build the same paged KIVI cache on
the GPU (through the C ABI) and in the CPU oracle from identical seeded
inputs, then compare."""
from __future__ import annotations

import numpy as np
import torch


def bits_to_torch(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy())
    return t.view(torch.float16 if dtype == "f16" else torch.bfloat16).to(device)


def i32(a, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(device)


class Twin:
    """A GPU cache and its CPU oracle twin, appended in lock step."""

    def __init__(self, ops, O, D, G, R, bits, Hkv, num_pages, max_seqs, device):
        self.ops, self.O = ops, O
        self.fmt = ops.KiviFormat(D, G, R, bits, Hkv)
        self.gpu = ops.KiviPagedCache(self.fmt, num_pages, max_seqs, device)
        self.cpu = O.PagedState(D, G, R, bits, Hkv, num_pages, max_seqs)
        self.device = device
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def append(self, kb, vb, dtype, cu, lens_old, bt, seq_slots=None):
        d = self.device
        self.ops.paged_append(self.gpu, bits_to_torch(kb, dtype, d), bits_to_torch(vb, dtype, d),
                              i32(cu, d), i32(lens_old, d), i32(bt, d),
                              None if seq_slots is None else i32(seq_slots, d),
                              max_new_tokens=int(np.max(np.diff(cu))) if len(cu) > 1 else 0,
                              err=self.err)
        self.cpu.append(kb, vb, dtype == "bf16", cu, lens_old, bt)

    def assert_same_state(self, lengths):
        torch.cuda.synchronize()
        assert int(self.err.item()) == 0, f"device error flag {int(self.err.item()):#x}"
        gp = self.gpu.pool.cpu().numpy()
        assert np.array_equal(gp, self.cpu.pool), _first_diff(gp, self.cpu.pool)
        # the ring holds stale values in slots of flushed tokens: compare live tokens
        gr = self.gpu.ring.cpu().numpy().view(np.uint16)
        assert np.array_equal(live_ring_values(gr, self.cpu, lengths),
                              live_ring_values(self.cpu.ring, self.cpu, lengths))


def _ring_offsets(D: int, t: int):
    """Half offsets of (token t % 16, channel 0..D-1) inside a chunk's K and V
    blocks (layout in include/truellm_kivi.h)."""
    c = np.arange(D)
    cc = c % 16
    tt = t % 16
    k_lane = 4 * (tt % 8) + (cc % 8) // 2
    k_r = 2 * (cc // 8) + tt // 8
    koff = ((c // 16) * 32 + k_lane) * 8 + 2 * k_r + cc % 2
    v_lane = 4 * (cc % 8) + (tt % 8) // 2
    v_r = 2 * (tt // 8) + cc // 8
    voff = ((c // 16) * 32 + v_lane) * 8 + 2 * v_r + tt % 2
    return koff, voff


def live_ring_values(ring: np.ndarray, st, lengths) -> np.ndarray:
    """[n_live_tokens, H, 2, D] fp16 bits of every sequence's residual tokens."""
    f = st.fmt
    out = []
    for b, L in enumerate(lengths):
        for t in range(st.nq(int(L)), int(L)):
            slot = t % f.ring_cap
            koff, voff = _ring_offsets(f.head_dim, t)
            chunk = ring[b, :, slot // 16]          # [H, 2, 16*D]
            out.append(np.stack([chunk[:, 0, koff], chunk[:, 1, voff]], 1))
    return np.array(out)


def _first_diff(a, b):
    idx = np.argwhere(a != b)
    if len(idx) == 0:
        return "equal"
    i = tuple(idx[0])
    return f"{len(idx)} bytes differ; first at {i}: gpu={a[i]} cpu={b[i]}"


def check_close(got: np.ndarray, ref: np.ndarray, atol=2e-3, rtol=2e-3):
    """Attention parity bar: |got - ref| <= atol + rtol * |ref| elementwise."""
    err = np.abs(got.astype(np.float64) - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (f"{bad.sum()} of {bad.size} outside {atol}+{rtol}|ref|; "
                           f"max abs err {err.max():.3e}")
    return float(err.max())
