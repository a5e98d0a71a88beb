"""The entry point that allocates nothing (cgdrChunkGatedDeltaRuleFwdHNoAlloc).

Some callers of this library cannot call cudaMalloc: a plugin host that only
receives input/output pointers and a stream while its framework's memory
pool owns the device memory, or a latency-critical path that must not take
cudaMalloc's implicit device synchronisation.  For them the library runs
the op on a 64 KiB scratch buffer compiled into it instead of a caller
workspace.  These tests call that entry point through the C ABI and check
it against the ordinary workspace entry point and the CPU oracle, in both
arithmetic modes, on calls in a row whose plans differ (the buffer is shared
by every call and keeps the previous call's contents).

This file is collected last so that a run stopping at its first failure has
already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import helpers as H

pytestmark = pytest.mark.gpu

cg = pytest.importorskip("cann_operator_challenge_august_b200")
from cann_operator_challenge_august_b200 import _lib  # noqa: E402

TOL = 2e-2


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _outputs(t, cu):
    B, T, HK, K = t["k"].shape
    H_, V = t["u"].shape[2], t["u"].shape[3]
    if cu is None:
        N, NT = B, (T + 63) // 64
        ci = None
    else:
        ci = cg.prepare_chunk_indices(cu)
        N, NT = cu.numel() - 1, ci.shape[0]
    h = torch.full((B, NT, H_, K, V), float("nan"), dtype=torch.bfloat16, device=t["k"].device)
    v = torch.full_like(t["u"], float("nan"))
    f = torch.full((N, H_, K, V), float("nan"), dtype=torch.float32, device=t["k"].device)
    return ci, h, v, f


def _plan(t, cu, ci, h, v, f, numerics):
    return cg.ChunkGatedDeltaRuleFwdH(t["k"], t["w"], t["u"], t["g"], t["initial_state"], cu, ci, 64, h, v, f,
                                      layout="token_major", numerics=numerics)


def _run_workspace(t, cu, numerics):
    ci, h, v, f = _outputs(t, cu)
    op = _plan(t, cu, ci, h, v, f, numerics)
    ws = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=t["k"].device)
    op(ws)
    return h, v, f


def _run_no_alloc(t, cu, numerics):
    lib = _lib.load()
    ci, h, v, f = _outputs(t, cu)
    op = _plan(t, cu, ci, h, v, f, numerics)
    assert op.workspace_size <= _lib.NOALLOC_SCRATCH_BYTES
    ex, op._ex = op._ex, None  # the entry point consumes the executor
    status = ctypes.c_int32(-1)
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.cgdrChunkGatedDeltaRuleFwdHNoAlloc(ex, ctypes.c_void_p(stream), ctypes.byref(status))
    _lib.check(st, "cgdrChunkGatedDeltaRuleFwdHNoAlloc")
    assert status.value == 0
    return h, v, f


def _case(which, dev):
    if which == "varlen4":
        inp = H.make_inputs(1, 700, 4, 128, 128, seed=21, cu_seqlens=[0, 5, 200, 333, 700])
    elif which == "varlen2":
        inp = H.make_inputs(1, 400, 4, 64, 64, seed=22, cu_seqlens=[0, 129, 400])
    else:
        inp = H.make_inputs(2, 300, 4, 128, 128, seed=23)
    return inp, {n: (x.to(dev) if isinstance(x, torch.Tensor) else x) for n, x in inp.items()}


@pytest.mark.parametrize("numerics", ["fp32_state", "reference"])
def test_no_alloc_entry_matches_workspace_entry(numerics):
    """Calls in a row with plans that leave different metadata in the shared
    buffer (4 sequences, fixed length, 2 sequences, then 4 again): each result
    equals the workspace entry's bit for bit and is within the north-star
    tolerance of the CPU oracle."""
    dev = _cuda()
    for which in ("varlen4", "fixed", "varlen2", "varlen4"):
        inp, t = _case(which, dev)
        cu = t.get("cu_seqlens")
        ref = _run_workspace(t, cu, numerics)
        got = _run_no_alloc(t, cu, numerics)
        torch.cuda.synchronize()
        oh, ov, of = H.oracle_run(inp, numerics, final_dtype="f32")
        for name, a, b, o in zip(("h", "v_new", "final_state"), got, ref, (oh, ov, of)):
            assert torch.isfinite(a.float()).all(), f"{which}/{name}"
            assert torch.equal(a, b), f"{which}/{name}: no-alloc entry differs from the workspace entry"
            H.assert_close(a, o, TOL, TOL, f"{which}/{name} vs oracle")


def test_no_alloc_rejects_plans_beyond_the_scratch_limit():
    """More sequences than the built-in buffer can index: refused before any
    device work, with a clear error (no tensor is touched)."""
    _cuda()
    n_seq = 9000  # workspace 256 + 4*(N+1) + 4*N rounded > 64 KiB
    base = torch.empty(128, dtype=torch.bfloat16)
    k = base.as_strided((1, n_seq, 1, 64), (0, 0, 0, 1))
    u = base.as_strided((1, n_seq, 1, 64), (0, 0, 0, 1))
    g = torch.empty(1).as_strided((1, n_seq, 1), (0, 0, 0))
    cu = torch.zeros(n_seq + 1, dtype=torch.int64)
    h = base.as_strided((1, n_seq, 1, 64, 64), (0, 0, 0, 0, 1))
    op = cg.ChunkGatedDeltaRuleFwdH(k, k, u, g, None, cu, None, 64, h, None, None, layout="token_major",
                                    numerics="fp32_state", chunk_offsets=None)
    assert op.workspace_size > _lib.NOALLOC_SCRATCH_BYTES
    ex, op._ex = op._ex, None
    st = _lib.load().cgdrChunkGatedDeltaRuleFwdHNoAlloc(ex, ctypes.c_void_p(0), None)
    assert _lib.STATUS_NAMES[st] == "WORKSPACE_TOO_SMALL"
    assert "scratch" in _lib.last_error()
