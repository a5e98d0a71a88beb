"""Chunk output (include/cgdr_chunk_o.h) on the GPU against the oracle
(oracle/gdr_stages.py, pinned to the reference in test_gdr_oracle.py) and
against the reference's own outputs.

Tolerance: the kernel sums q'h and P v_new in one fp32 accumulator and
rounds once, where the reference rounds each product to bf16 and then their
sum.  The bound is |ours - ref| <= 1e-2 |ref| + 2**-7 max|ref| (about one
bf16 ulp relative plus one ulp at the top of the output's range, which
covers the reference's extra roundings of the two terms).  On the
reference's fixtures the output must also pass the reference's own
three-party check (tests/assets/impl/compare.py) against its fp32 golden.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import helpers as H
from oracle import gdr_stages as G

pytestmark = pytest.mark.gpu

cg = pytest.importorskip("cann_operator_challenge_august_b200")

MANIFEST = json.loads((H.ROOT / "tests" / "golden" / "gdr_manifest.json").read_text())


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def assert_o_close(got, ref, what="o"):
    got = H.as_f32(got)
    ref = np.asarray(ref, np.float32)
    bound = 1e-2 * np.abs(ref) + 2.0 ** -7 * float(np.abs(ref).max(initial=0.0))
    err = np.abs(got - ref)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside; max err {err.max():.3e}, "
                           f"max|ref| {np.abs(ref).max():.3e}")


def seg_chunk_cumsum(x, bounds):
    """Chunk-local cumsum over T restarted per sequence; x [B, T, H]."""
    return H.chunk_local_cumsum(x, bounds)


def make_inputs(B, T, H_, HK, K, V, *, seed, cu=None, with_g=True, h_scale=0.3):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HK, K, generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)
    k = torch.randn(B, T, HK, K, generator=gen)
    k = (k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)
    v = (0.5 * torch.randn(B, T, H_, V, generator=gen)).to(torch.bfloat16)
    if cu is None:
        NT = (T + 63) // 64
        bounds = [(0, T)]
    else:
        NT = sum((cu[i + 1] - cu[i] + 63) // 64 for i in range(len(cu) - 1))
        bounds = list(zip(cu[:-1], cu[1:]))
    h = (h_scale * torch.randn(B, NT, H_, K, V, generator=gen)).to(torch.bfloat16)
    g = None
    if with_g:
        g = seg_chunk_cumsum(torch.nn.functional.logsigmoid(torch.randn(B, T, H_, generator=gen) + 2.0), bounds)
    return q, k, v, h, g


def run_case(q, k, v, h, g, scale=None, cu=None):
    dev = _cuda()
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.int64, device=dev)
    o = cg.chunk_fwd_o(q.to(dev), k.to(dev), v.to(dev), h.to(dev), None if g is None else g.to(dev), scale,
                       cu_seqlens=cu_t, check_device_status=True)
    torch.cuda.synchronize()
    ref = G.chunk_o(H.as_f32(q), H.as_f32(k), H.as_f32(v), H.as_f32(h), None if g is None else g.numpy(), scale,
                    None if cu is None else np.asarray(cu))
    return o, ref


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_chunk_o_on_reference_intermediates(name):
    """The reference's own q, k, v_new, per-chunk states and gates in; its
    output out -- within the tolerance, and the reference's cross-check
    against its fp32 golden passes."""
    dev = _cuda()
    m = MANIFEST[name]
    z = np.load(H.ROOT / "tests" / "golden" / f"gdr_{name}.npz")
    bf = lambda a: H.from_bits(a, dev)  # noqa: E731
    lens = z["seq_lens"].astype(np.int64)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64, device=dev)
    o = cg.chunk_fwd_o(bf(z["q"])[None], bf(z["k"])[None], bf(z["v_new"]), bf(z["h"]),
                       torch.from_numpy(z["g_cum"]).to(dev), m["scale"], cu_seqlens=cu, check_device_status=True)
    torch.cuda.synchronize()
    ours = H.as_f32(o)[0]
    assert_o_close(ours, H.as_f32(z["bench_out"]), f"{name} vs reference output")
    r = G.cross_check(ours, H.as_f32(z["golden_out"]), H.as_f32(z["bench_out"]))
    assert r["pass"], r


@pytest.mark.parametrize("B,T,H_,HK,K,V", [
    (2, 300, 4, 2, 128, 128),   # GQA, partial last chunk, two batch rows
    (1, 130, 2, 1, 64, 64),     # K = V = 64
    (1, 200, 2, 2, 128, 256),   # two 128-column V tiles
    (1, 64, 1, 1, 128, 192),    # three 64-column V tiles
    (3, 64, 3, 3, 64, 128),     # exactly one chunk per row
])
def test_chunk_o_fixed_length(B, T, H_, HK, K, V):
    q, k, v, h, g = make_inputs(B, T, H_, HK, K, V, seed=B * 1000 + T + K + V)
    o, ref = run_case(q, k, v, h, g)
    assert_o_close(o, ref)


@pytest.mark.parametrize("cu", [
    [0, 1, 64, 129, 129, 300],      # lengths 1, 63, 65, 0 (empty), 171
    [0, 64, 128, 192],              # whole chunks only
    [0, 5],                         # one short sequence
])
def test_chunk_o_varlen(cu):
    q, k, v, h, g = make_inputs(1, cu[-1], 4, 2, 128, 128, seed=len(cu) * 7 + cu[-1], cu=cu)
    o, ref = run_case(q, k, v, h, g, cu=cu)
    assert_o_close(o, ref)


def test_chunk_o_without_gate_and_custom_scale():
    q, k, v, h, _ = make_inputs(1, 150, 2, 1, 128, 128, seed=5, with_g=False)
    o, ref = run_case(q, k, v, h, None, scale=0.5)
    assert_o_close(o, ref)


def test_pipeline_recurrence_then_chunk_output():
    """fwd_h (fp32 state) then chunk output, all on the GPU, against the two
    oracles chained on the CPU."""
    dev = _cuda()
    B, T, H_, HK, K, V = 2, 257, 4, 2, 128, 128
    inp = H.make_inputs(B, T, H_, K, V, HK=HK, seed=77)
    t = {n: (x.to(dev) if isinstance(x, torch.Tensor) else x) for n, x in inp.items()}
    gen = torch.Generator().manual_seed(78)
    q = torch.randn(B, T, HK, K, generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    h, v_new, _ = cg.chunk_gated_delta_rule_fwd_h(t["k"], t["w"], t["u"], t["g"], t["initial_state"])
    o = cg.chunk_fwd_o(q.to(dev), t["k"], v_new, h, t["g"], check_device_status=True)
    torch.cuda.synchronize()
    oh, ov, _ = H.oracle_run(inp, "fp32_state")
    ref = G.chunk_o(H.as_f32(q), H.as_f32(inp["k"]), H.as_f32(ov), H.as_f32(oh), inp["g"].numpy(), None)
    assert_o_close(o, ref, "pipeline")


def test_chunk_o_flags_bad_chunk_indices():
    """A chunk_indices row naming a sequence that does not exist: that CTA
    touches nothing and the status word records bad metadata (0x2)."""
    dev = _cuda()
    cu = [0, 100, 200]
    q, k, v, h, g = make_inputs(1, 200, 2, 2, 128, 128, seed=9, cu=cu)
    ci = cg.prepare_chunk_indices(torch.tensor(cu, dtype=torch.int64)).clone()
    ci[1, 0] = 7  # no sequence 7
    o = torch.zeros(1, 200, 2, 128, dtype=torch.bfloat16, device=dev)
    op = cg.ChunkGatedDeltaRuleFwdO(q.to(dev), k.to(dev), v.to(dev), h.to(dev), g.to(dev),
                                    torch.tensor(cu, device=dev), ci.to(dev), None, 64, o)
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    op(ws)
    assert cg.read_device_status(ws) & 0x2
    # the chunk with the bad row was not written; the others were
    assert torch.count_nonzero(o[0, 64:100]) == 0
    assert torch.count_nonzero(o[0, 0:64]) > 0
