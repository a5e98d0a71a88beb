"""Out-of-bounds write checks: every output is written only inside its own extent.

The reference's output invariants (``code/tests/golden/generate_golden.py:509-580``)
check shapes and finiteness; on a GPU the stronger question is whether a store
ever lands outside the tensor it targets.  Each output here is a strided view
into a larger buffer filled with a sentinel bit pattern: guard elements before
and after the tensor, and guard columns between rows (the view's row stride is
wider than its last dimension).  After a launch every guard element must still
hold the sentinel, and the view must equal the result of the same call on
plainly allocated outputs.

Covered: both kernels, both arithmetic modes, partial-chunk varlen batches
(lengths 1, 5, 63, 65, 129), head widths that run in a zero-filled K tile or a
clipped V tile, and the entry point that allocates nothing.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import helpers as H

pytestmark = pytest.mark.gpu

cg = pytest.importorskip("cann_operator_challenge_august_b200")
from cann_operator_challenge_august_b200 import _lib  # noqa: E402

SENTINEL_BF16 = 0x7FA5          # a quiet NaN no kernel produces
SENTINEL_F32 = 0x7FC0A5A5
GUARD = 1024                    # guard elements before and after each output
COL_PAD = 8                     # guard columns after each row (keeps 16-byte row strides)
LENS = [1, 5, 63, 65, 129]


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


class Guarded:
    """A tensor view of `shape` inside a sentinel-filled buffer with guard
    elements around it and guard columns after each row."""

    def __init__(self, shape, dtype, dev):
        self.shape = tuple(shape)
        rows = int(np.prod(shape[:-1]))
        pitch = shape[-1] + COL_PAD
        n = 2 * GUARD + rows * pitch
        idt = torch.int16 if dtype == torch.bfloat16 else torch.int32
        self.sent = SENTINEL_BF16 if dtype == torch.bfloat16 else SENTINEL_F32
        self.raw = torch.full((n,), self.sent, dtype=idt, device=dev)
        strides = [0] * len(shape)
        strides[-1] = 1
        acc = pitch
        for i in range(len(shape) - 2, -1, -1):
            strides[i] = acc
            acc *= shape[i]
        self.view = self.raw.view(dtype).as_strided(self.shape, tuple(strides), GUARD)

    def guards_intact(self):
        """(number of guard elements overwritten, raw index of the first)."""
        mask = torch.ones(self.raw.numel(), dtype=torch.bool, device=self.raw.device)
        idx = torch.arange(self.raw.numel(), device=self.raw.device).as_strided(
            self.shape, self.view.stride(), GUARD)
        mask[idx.reshape(-1)] = False
        bad = (mask & (self.raw != self.sent)).nonzero()
        return int(bad.numel()), (int(bad[0]) if bad.numel() else None)


def _inputs(K, V, dev, seed):
    cu = [0]
    for L in LENS:
        cu.append(cu[-1] + L)
    inp = H.make_inputs(1, cu[-1], 4, K, V, HK=2, seed=seed, cu_seqlens=cu)
    return {n: (x.to(dev) if isinstance(x, torch.Tensor) else x) for n, x in inp.items()}


def _shapes(t):
    B, T, HK, K = t["k"].shape
    H_, V = t["u"].shape[2], t["u"].shape[3]
    ci = cg.prepare_chunk_indices(t["cu_seqlens"])
    N, NT = t["cu_seqlens"].numel() - 1, ci.shape[0]
    return ci, (B, NT, H_, K, V), (B, T, H_, V), (N, H_, K, V)


def _launch(t, ci, h, v, f, numerics, kernel, no_alloc=False, v_tile=0, chains=0):
    op = cg.ChunkGatedDeltaRuleFwdH(t["k"], t["w"], t["u"], t["g"], t["initial_state"], t["cu_seqlens"], ci, 64,
                                    h, v, f, layout="token_major", numerics=numerics, force_kernel=kernel,
                                    v_tile=v_tile, chains=chains)
    if no_alloc:
        ex, op._ex = op._ex, None
        status = ctypes.c_int32(-1)
        st = _lib.load().cgdrChunkGatedDeltaRuleFwdHNoAlloc(
            ex, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(status))
        _lib.check(st, "cgdrChunkGatedDeltaRuleFwdHNoAlloc")
        assert status.value == 0
    else:
        ws = torch.zeros(max(op.workspace_size, 256), dtype=torch.uint8, device=t["k"].device)
        op(ws)
        assert cg.read_device_status(ws) == 0


@pytest.mark.parametrize("K,V,v_tile,chains", [(128, 128, 0, 0), (64, 64, 0, 0), (32, 32, 0, 0), (96, 96, 0, 0),
                                                (256, 256, 0, 0), (64, 96, 0, 0), (128, 128, 32, 2), (96, 48, 32, 2),
                                                (128, 192, 128, 2)])
@pytest.mark.parametrize("kernel", [1, 2])
@pytest.mark.parametrize("numerics", ["fp32_state", "reference"])
def test_outputs_stay_inside_their_extent(K, V, v_tile, chains, kernel, numerics):
    """Two chains per CTA run on the tensor-core kernel only; with V = 48 (32-column
    tiles) and V = 192 (128-column tiles) the last CTA's second chain lies wholly
    past V."""
    if chains and kernel != 1:
        pytest.skip("the V tile and chain options apply to the tensor-core kernel")
    dev = _cuda()
    t = _inputs(K, V, dev, seed=K + 3 * V)
    ci, hs, vs, fs = _shapes(t)
    fdt = torch.float32 if numerics == "fp32_state" else torch.bfloat16
    if numerics == "reference":
        t["initial_state"] = t["initial_state"].to(torch.bfloat16)
    gh, gv, gf = Guarded(hs, torch.bfloat16, dev), Guarded(vs, torch.bfloat16, dev), Guarded(fs, fdt, dev)
    _launch(t, ci, gh.view, gv.view, gf.view, numerics, kernel, v_tile=v_tile, chains=chains)
    torch.cuda.synchronize()
    for name, gd in (("h", gh), ("v_new", gv), ("final_state", gf)):
        n_bad, first = gd.guards_intact()
        assert n_bad == 0, f"{name}: {n_bad} guard elements overwritten (first at raw index {first})"
    # the same call on plainly allocated outputs gives the same values
    h = torch.empty(hs, dtype=torch.bfloat16, device=dev)
    v = torch.empty(vs, dtype=torch.bfloat16, device=dev)
    f = torch.empty(fs, dtype=fdt, device=dev)
    _launch(t, ci, h, v, f, numerics, kernel, v_tile=v_tile, chains=chains)
    torch.cuda.synchronize()
    for name, a, b in (("h", gh.view, h), ("v_new", gv.view, v), ("final_state", gf.view, f)):
        assert torch.equal(a, b), f"{name}: strided outputs differ from contiguous ones"


def test_no_alloc_entry_stays_inside_its_outputs():
    dev = _cuda()
    t = _inputs(128, 128, dev, seed=5)
    ci, hs, vs, fs = _shapes(t)
    gh, gv, gf = (Guarded(hs, torch.bfloat16, dev), Guarded(vs, torch.bfloat16, dev),
                  Guarded(fs, torch.float32, dev))
    for _ in range(2):
        _launch(t, ci, gh.view, gv.view, gf.view, "fp32_state", 0, no_alloc=True)
        torch.cuda.synchronize()
        for name, gd in (("h", gh), ("v_new", gv), ("final_state", gf)):
            n_bad, first = gd.guards_intact()
            assert n_bad == 0, f"{name}: {n_bad} guard elements overwritten (first at raw index {first})"
