"""The host-memory front end (cann_operator_challenge_august_b200/host.py): batch rows
pipelined over three streams, copies in and out overlapped with the kernels.  Each row
runs the same kernels as the device API, so the outputs are bit-identical to it."""

from __future__ import annotations

import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu

cg = pytest.importorskip("cann_operator_challenge_august_b200")
host_mod = pytest.importorskip("cann_operator_challenge_august_b200.host")


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


@pytest.mark.parametrize("numerics", ["fp32_state", "reference"])
@pytest.mark.parametrize("piece_bytes", [None, 1 << 16])
@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("B,T,H,K,V", [(3, 333, 4, 128, 128), (5, 128, 2, 64, 64), (1, 1000, 2, 128, 64)])
def test_host_api_matches_device_api(pinned, B, T, H, K, V, piece_bytes, numerics, monkeypatch):
    """Whole rows, and rows split into ranges of chunks (64 KB pieces: several per row)
    that continue from the previous range's final state."""
    dev = _cuda()
    if piece_bytes is not None:
        monkeypatch.setattr(host_mod, "_PIECE_BYTES", piece_bytes)
    inp = helpers.make_inputs(B, T, H, K, V, seed=B * 100 + T)
    host = {n: (x.pin_memory() if pinned else x) for n, x in inp.items() if x is not None}
    h, v, f = cg.chunk_gated_delta_rule_fwd_h_host(host["k"], host["w"], host["u"], host["g"],
                                                   host["initial_state"], device=dev, numerics=numerics)
    torch.cuda.synchronize()
    d = {n: x.to(dev) for n, x in host.items()}
    h2, v2, f2 = cg.chunk_gated_delta_rule_fwd_h(d["k"], d["w"], d["u"], d["g"], d["initial_state"],
                                                 check_device_status=True, numerics=numerics)
    torch.cuda.synchronize()
    assert not h.is_cuda and h.is_pinned() == pinned
    assert torch.equal(h, h2.cpu()) and torch.equal(v, v2.cpu()) and torch.equal(f, f2.cpu())


def test_host_api_into_given_outputs_twice():
    """Two calls in a row into caller-owned pinned outputs; the second overwrites the first."""
    dev = _cuda()
    B, T, H_, K, V = 4, 256, 4, 128, 128
    a = helpers.make_inputs(B, T, H_, K, V, seed=1)
    b = helpers.make_inputs(B, T, H_, K, V, seed=2)
    pa = {n: x.pin_memory() for n, x in a.items() if x is not None}
    pb = {n: x.pin_memory() for n, x in b.items() if x is not None}
    out = (torch.empty(B, T // 64, H_, K, V, dtype=torch.bfloat16, pin_memory=True),
           torch.empty(B, T, H_, V, dtype=torch.bfloat16, pin_memory=True),
           torch.empty(B, H_, K, V, dtype=torch.float32, pin_memory=True))
    cg.chunk_gated_delta_rule_fwd_h_host(pa["k"], pa["w"], pa["u"], pa["g"], pa["initial_state"], device=dev, out=out)
    torch.cuda.synchronize()
    first = [t.clone() for t in out]
    cg.chunk_gated_delta_rule_fwd_h_host(pb["k"], pb["w"], pb["u"], pb["g"], pb["initial_state"], device=dev, out=out)
    torch.cuda.synchronize()
    d = {n: x.to(dev) for n, x in pb.items()}
    ref = cg.chunk_gated_delta_rule_fwd_h(d["k"], d["w"], d["u"], d["g"], d["initial_state"])
    torch.cuda.synchronize()
    for got, want, old in zip(out, ref, first):
        assert torch.equal(got, want.cpu())
        assert not torch.equal(got, old)


def test_host_api_rejects_device_tensors():
    dev = _cuda()
    inp = helpers.make_inputs(1, 64, 1, 64, 64, seed=3, device=dev)
    with pytest.raises(ValueError):
        cg.chunk_gated_delta_rule_fwd_h_host(inp["k"], inp["w"], inp["u"], inp["g"], inp["initial_state"])


@pytest.mark.parametrize("piece_bytes", [None, 1 << 16])
@pytest.mark.parametrize("numerics", ["fp32_state", "reference"])
def test_host_api_varlen(piece_bytes, numerics, monkeypatch):
    """Packed varlen batch with an empty sequence, a one-token sequence and long
    sequences split into several pieces."""
    dev = _cuda()
    if piece_bytes is not None:
        monkeypatch.setattr(host_mod, "_PIECE_BYTES", piece_bytes)
    cu = [0, 300, 300, 301, 1000, 1130]
    inp = helpers.make_inputs(1, 1130, 4, 128, 128, seed=9, cu_seqlens=cu)
    host = {n: x.pin_memory() for n, x in inp.items() if x is not None}
    h, v, f = cg.chunk_gated_delta_rule_fwd_h_host(host["k"], host["w"], host["u"], host["g"], host["initial_state"],
                                                   host["cu_seqlens"], device=dev, numerics=numerics)
    torch.cuda.synchronize()
    d = {n: x.to(dev) for n, x in host.items()}
    h2, v2, f2 = cg.chunk_gated_delta_rule_fwd_h(d["k"], d["w"], d["u"], d["g"], d["initial_state"],
                                                 cu_seqlens=d["cu_seqlens"], check_device_status=True,
                                                 numerics=numerics)
    torch.cuda.synchronize()
    assert h.shape == h2.shape
    assert torch.equal(h, h2.cpu()) and torch.equal(v, v2.cpu()) and torch.equal(f, f2.cpu())
