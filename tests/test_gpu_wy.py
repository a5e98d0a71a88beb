"""WY representation (include/cgdr_wy.h) on the GPU against the oracle
(oracle/gdr_stages.py, pinned to the reference in test_gdr_oracle.py) and the
reference's own stage-1 outputs; then the whole chunked Gated DeltaNet
forward chained on the GPU (WY -> recurrence -> chunk output) against the
reference operator and its fp32 golden.

Tolerance for w and u: |ours - ref| <= 1e-2 |ref| + 2**-7 max|ref|.  The
kernel forms (I + A)^-1 by blocked forward substitution in fp32 where the
reference calls a LAPACK triangular solve, so a few entries of the bf16 T
differ by one rounding; the bound is one bf16 ulp relative plus one ulp at
the top of the tensor's range.  The cumulative gate is compared at 1e-6
relative to its range.  The chained operator must pass the reference's own
three-party check (tests/assets/impl/compare.py) against its fp32 golden,
for the output and the final state.
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


def assert_close(got, ref, what):
    got = H.as_f32(got)
    ref = np.asarray(ref, np.float32)
    bound = 1e-2 * np.abs(ref) + 2.0 ** -7 * float(np.abs(ref).max(initial=0.0))
    err = np.abs(got - ref)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside; max err {err.max():.3e}, "
                           f"max|ref| {np.abs(ref).max():.3e}")


def assert_gcum(got, ref):
    got, ref = H.as_f32(got), np.asarray(ref, np.float32)
    assert np.abs(got - ref).max(initial=0.0) <= 1e-6 * max(1.0, float(np.abs(ref).max(initial=0.0)))


def make_inputs(B, T, H_, HK, K, V, *, seed, with_g=True):
    gen = torch.Generator().manual_seed(seed)
    k = torch.nn.functional.normalize(torch.randn(B, T, HK, K, generator=gen), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, H_, V, generator=gen).to(torch.bfloat16)
    beta = torch.rand(B, T, H_, generator=gen).clamp(1e-6, 1 - 1e-6).to(torch.bfloat16)
    g = (-torch.rand(B, T, H_, generator=gen)) if with_g else None
    return k, v, beta, g


def run_wy(k, v, beta, g, cu=None):
    dev = _cuda()
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.int64, device=dev)
    w, u, gc = cg.chunk_wy_fwd(k.to(dev), v.to(dev), beta.to(dev), None if g is None else g.to(dev), cu_seqlens=cu_t,
                               check_device_status=True)
    torch.cuda.synchronize()
    rw, ru, rg = G.wy(H.as_f32(k), H.as_f32(v), H.as_f32(beta), None if g is None else g.numpy(),
                      None if cu is None else np.asarray(cu))
    return (w, u, gc), (rw, ru, rg)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_wy_on_reference_inputs(name):
    dev = _cuda()
    z = np.load(H.ROOT / "tests" / "golden" / f"gdr_{name}.npz")
    bf = lambda a: H.from_bits(a, dev)  # noqa: E731
    cu = torch.tensor(np.concatenate([[0], np.cumsum(z["seq_lens"].astype(np.int64))]), device=dev)
    g = torch.from_numpy(z["g"])[None].to(dev) if "g" in z.files else None
    w, u, gc = cg.chunk_wy_fwd(bf(z["k"])[None], bf(z["v"])[None], bf(z["beta"])[None], g, cu_seqlens=cu,
                               check_device_status=True)
    torch.cuda.synchronize()
    assert_close(w, H.as_f32(z["w"]), f"{name} w vs reference")
    assert_close(u, H.as_f32(z["u"]), f"{name} u vs reference")
    assert_gcum(gc, z["g_cum"])


@pytest.mark.parametrize("B,T,H_,HK,K,V", [
    (2, 300, 4, 2, 128, 128),   # GQA, partial last chunk
    (1, 130, 2, 1, 64, 64),
    (1, 256, 3, 3, 128, 64),
    (3, 64, 2, 2, 64, 128),
])
def test_wy_fixed_length(B, T, H_, HK, K, V):
    k, v, beta, g = make_inputs(B, T, H_, HK, K, V, seed=T + K + V + B)
    (w, u, gc), (rw, ru, rg) = run_wy(k, v, beta, g)
    assert_close(w, rw, "w")
    assert_close(u, ru, "u")
    assert_gcum(gc, rg)


@pytest.mark.parametrize("cu", [[0, 1, 64, 129, 129, 300], [0, 5], [0, 64, 128]])
def test_wy_varlen(cu):
    k, v, beta, g = make_inputs(1, cu[-1], 4, 2, 128, 128, seed=len(cu) + cu[-1])
    (w, u, gc), (rw, ru, rg) = run_wy(k, v, beta, g, cu)
    assert_close(w, rw, "w")
    assert_close(u, ru, "u")
    assert_gcum(gc, rg)


def test_wy_without_gate():
    k, v, beta, _ = make_inputs(1, 200, 2, 2, 128, 128, seed=3, with_g=False)
    (w, u, gc), (rw, ru, rg) = run_wy(k, v, beta, None)
    assert_close(w, rw, "w")
    assert_close(u, ru, "u")
    assert float(gc.abs().max()) == 0.0


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_chained_operator_passes_the_reference_check(name):
    """WY -> recurrence (fp32 state) -> chunk output on the reference's inputs:
    the output and the final state pass the reference's cross-check against
    its fp32 golden, with its bf16 operator as the benchmark."""
    dev = _cuda()
    m = MANIFEST[name]
    z = np.load(H.ROOT / "tests" / "golden" / f"gdr_{name}.npz")
    bf = lambda a: H.from_bits(a, dev)  # noqa: E731
    q, k, v, beta = bf(z["q"])[None], bf(z["k"])[None], bf(z["v"])[None], bf(z["beta"])[None]
    g = torch.from_numpy(z["g"])[None].to(dev) if "g" in z.files else None
    h0 = H.from_bits(z["h0"], dev)
    h0 = h0.float().transpose(-1, -2).contiguous()  # [N, H, Dv, Dk] -> [N, H, K, V]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(z["seq_lens"].astype(np.int64))]), device=dev)
    w, u, gc = cg.chunk_wy_fwd(k, v, beta, g, cu_seqlens=cu, check_device_status=True)
    h, v_new, fin = cg.chunk_gated_delta_rule_fwd_h(k, w, u, gc, h0, cu_seqlens=cu, check_device_status=True)
    o = cg.chunk_fwd_o(q, k, v_new, h, gc, m["scale"], cu_seqlens=cu, check_device_status=True)
    torch.cuda.synchronize()
    out = H.as_f32(o)[0]
    r = G.cross_check(out, H.as_f32(z["golden_out"]), H.as_f32(z["bench_out"]))
    assert r["pass"], ("out", r)
    fin_ref_layout = fin.transpose(-1, -2).contiguous().cpu().numpy()
    r = G.cross_check(fin_ref_layout, H.as_f32(z["golden_final"]), H.as_f32(z["bench_final"]))
    assert r["pass"], ("final_state", r)
