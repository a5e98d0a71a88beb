"""The numpy restatement of the chunked Gated DeltaNet stages (oracle/gdr_stages.py)
pinned against fixtures produced by the reference's own Python code
(tests/golden/make_gdr_golden.py): the bf16 operator
(ref/chunk_gated_delta_rule/tests/pytest/chunk_gated_delta_rule_benchmark.py),
its stages, and the fp32 golden (chunk_gated_delta_rule_golden.py).  CPU only.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

import helpers as H
from oracle import gdr_stages as G

MANIFEST = json.loads((H.ROOT / "tests" / "golden" / "gdr_manifest.json").read_text())
CASES = sorted(MANIFEST)


def load(name):
    z = np.load(H.ROOT / "tests" / "golden" / f"gdr_{name}.npz")
    return {n: z[n] for n in z.files}


def f32(a):
    return H.as_f32(a)


def inputs(z):
    g = f32(z["g"]) if "g" in z else None
    return f32(z["q"]), f32(z["k"]), f32(z["v"]), f32(z["beta"]), g, f32(z["h0"]), z["seq_lens"]


def agreement(ours, ref):
    """(fraction bit-equal, max |error| / max |ref|).  The second figure is
    normwise: 2**-7 is one bf16 ulp at the top of the tensor's range, so a
    one-ulp difference in an intermediate product that later cancels stays
    within it."""
    ours, ref = np.asarray(ours, np.float32), np.asarray(ref, np.float32)
    scale = max(float(np.abs(ref).max(initial=0.0)), 1e-30)
    return float(np.mean(ours == ref)), float(np.abs(ours - ref).max(initial=0.0)) / scale


ULP = 2.0 ** -7


@pytest.mark.parametrize("name", CASES)
def test_fixture_digests(name):
    z = load(name)
    for arr, meta in MANIFEST[name]["arrays"].items():
        a = z[arr]
        assert list(a.shape) == meta["shape"] and str(a.dtype) == meta["dtype"], arr
        assert hashlib.sha256(a.tobytes()).hexdigest() == meta["sha256"], arr


@pytest.mark.parametrize("name", CASES)
def test_benchmark_operator_restatement(name):
    """benchmark_op vs chunk_gdn_benchmark_opt: bit-equal up to fp32 summation order."""
    z = load(name)
    q, k, v, beta, g, h0, lens = inputs(z)
    out, fin, _ = G.benchmark_op(q, k, v, beta, MANIFEST[name]["scale"], h0, lens, g)
    eq, mx = agreement(out, f32(z["bench_out"]))
    assert eq >= 0.998 and mx <= ULP, (eq, mx)
    eq, mx = agreement(fin, f32(z["bench_final"]))
    assert eq >= 0.998 and mx <= ULP, (eq, mx)


@pytest.mark.parametrize("name", CASES)
def test_stage1_restatement(name):
    """w = -k_cumdecay, u = v_inner and the chunk-local cumulative gate."""
    z = load(name)
    q, k, v, beta, g, h0, lens = inputs(z)
    T, Nk, Dk = q.shape
    Nv = v.shape[1]
    if g is None:
        g = np.zeros((T, Nv), np.float32)
    start = 0
    for S in lens:
        S = int(S)
        rep = Nv // Nk
        s1 = G.stage1(np.repeat(q[start:start + S], rep, 1), np.repeat(k[start:start + S], rep, 1),
                      v[start:start + S], g[start:start + S], beta[start:start + S], MANIFEST[name]["scale"])
        sl = slice(start, start + S)
        eq, mx = agreement(s1["g_cum"][:, :S].T, f32(z["g_cum"])[0, sl])
        assert eq >= 0.999 and mx <= 1e-6, ("g_cum", eq, mx)
        eq, mx = agreement(-s1["k_cumdecay"][:, :S].transpose(1, 0, 2), f32(z["w"])[0, sl])
        assert eq >= 0.995 and mx <= ULP, ("w", eq, mx)
        eq, mx = agreement(s1["v_inner"][:, :S].transpose(1, 0, 2), f32(z["u"])[0, sl])
        assert eq >= 0.995 and mx <= ULP, ("u", eq, mx)
        start += S


@pytest.mark.parametrize("name", CASES)
def test_golden_restatement(name):
    """golden_op vs the fp32 golden through the reference adapter."""
    z = load(name)
    q, k, v, beta, g, h0, lens = inputs(z)
    out, fin = G.golden_op(q, k, v, beta, h0, lens, g, state_bf16=MANIFEST[name]["h0_dtype"] == "bf16")
    eq, mx = agreement(out, f32(z["golden_out"]))
    assert eq >= 0.998 and mx <= ULP, (eq, mx)
    assert np.allclose(fin, f32(z["golden_final"]), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("name", CASES)
def test_chunk_output_restatement(name):
    """chunk_o (the chunk-output kernel's specification) on the reference's
    own intermediates reproduces the reference output.  The fixture's h is
    bf16, so for an fp32 initial state the first chunk's inter-chunk term
    differs by that rounding."""
    z = load(name)
    lens = z["seq_lens"]
    cu = np.concatenate([[0], np.cumsum(lens)])
    o = G.chunk_o(f32(z["q"])[None], f32(z["k"])[None], f32(z["v_new"]), f32(z["h"]), f32(z["g_cum"]),
                  MANIFEST[name]["scale"], cu)[0]
    eq, mx = agreement(o, f32(z["bench_out"]))
    if MANIFEST[name]["h0_dtype"] == "bf16":
        assert eq >= 0.998 and mx <= ULP, (eq, mx)
    else:
        assert eq >= 0.95 and mx <= ULP, (eq, mx)


@pytest.mark.parametrize("name", CASES)
def test_cross_check_restatement(name):
    """compare.py's criterion: the benchmark against itself passes with all
    ratios 1; an output with a planted error of 5% fails."""
    z = load(name)
    bench, golden = f32(z["bench_out"]), f32(z["golden_out"])
    r = G.cross_check(bench, golden, bench)
    assert r["pass"] and r["mare_ratio"] == pytest.approx(1.0)
    rng = np.random.default_rng(0)
    bad = bench + 0.05 * np.abs(bench).max() * rng.standard_normal(bench.shape).astype(np.float32)
    assert not G.cross_check(bad, golden, bench)["pass"]


@pytest.mark.parametrize("name", CASES)
def test_wy_fla_layout_restatement(name):
    """The fla-layout WY wrapper (the WY kernel's specification) reproduces the
    reference's stage-1 outputs on its own inputs."""
    z = load(name)
    lens = z["seq_lens"]
    cu = np.concatenate([[0], np.cumsum(lens)])
    g = f32(z["g"])[None] if "g" in z else None
    w, u, gc = G.wy(f32(z["k"])[None], f32(z["v"])[None], f32(z["beta"])[None], g, cu)
    for got, ref, what in ((w, z["w"], "w"), (u, z["u"], "u"), (gc, z["g_cum"], "g_cum")):
        eq, mx = agreement(got, f32(ref))
        assert eq >= 0.995 and mx <= ULP, (what, eq, mx)
