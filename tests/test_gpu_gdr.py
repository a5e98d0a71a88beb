"""The composed chunked Gated DeltaNet forward (include/cgdr_gdr.h), called
the way the reference's operator is called, against the reference:

* on the reference's own fixtures (inputs drawn with its recipe, outputs of
  its bf16 operator and fp32 golden, tests/golden/make_gdr_golden.py), the
  output and final state pass the reference's three-party check
  (ref/chunk_gated_delta_rule/tests/assets/impl/compare.py);
* on larger ragged batches, the same check against the oracle's
  restatements of the reference operator and golden (oracle/gdr_stages.py,
  pinned in test_gdr_oracle.py);
* lengths that do not sum to T set the device status bit instead of
  reading or writing out of bounds.
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


def check(out, fin, golden_out, golden_fin, bench_out, bench_fin):
    r = G.cross_check(H.as_f32(out), golden_out, bench_out)
    assert r["pass"], ("out", r)
    r = G.cross_check(H.as_f32(fin), golden_fin, bench_fin)
    assert r["pass"], ("final_state", r)


PATHS = ["fused", "three_kernels"]


def _path_applies(path, dk):
    """The fused recurrence + output kernel runs Dk in (64, 128]."""
    if path == "fused" and dk <= 64:
        pytest.skip("the fused kernel runs Dk in (64, 128]")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_operator_on_reference_fixtures(name, path):
    dev = _cuda()
    m = MANIFEST[name]
    z = np.load(H.ROOT / "tests" / "golden" / f"gdr_{name}.npz")
    _path_applies(path, z["q"].shape[-1])
    bf = lambda a: H.from_bits(a, dev)  # noqa: E731
    h0 = bf(z["h0"]) if z["h0"].dtype == np.uint16 else torch.from_numpy(z["h0"]).to(dev)
    g = torch.from_numpy(z["g"]).to(dev) if "g" in z.files else None
    asl = torch.from_numpy(z["seq_lens"]).to(dev)
    out, fin = cg.chunk_gated_delta_rule(bf(z["q"]), bf(z["k"]), bf(z["v"]), bf(z["beta"]), h0, asl, m["scale"], g,
                                         check_device_status=True, path=path)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and fin.dtype == h0.dtype
    check(out, fin, H.as_f32(z["golden_out"]), H.as_f32(z["golden_final"]), H.as_f32(z["bench_out"]),
          H.as_f32(z["bench_final"]))


def make_case(lens, nk, nv, dk, dv, state_dtype, seed, with_g=True):
    gen = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.nn.functional.normalize(torch.randn(T, nk, dk, generator=gen), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(T, nk, dk, generator=gen), dim=-1).to(torch.bfloat16)
    v = torch.randn(T, nv, dv, generator=gen).to(torch.bfloat16)
    beta = torch.rand(T, nv, generator=gen).clamp(1e-6, 1 - 1e-6).to(torch.bfloat16)
    g = (-torch.rand(T, nv, generator=gen)) if with_g else None
    h0 = (0.1 * torch.randn(len(lens), nv, dv, dk, generator=gen)).to(state_dtype)
    return q, k, v, beta, g, h0, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("lens,nk,nv,dk,dv,state", [
    ([200, 64, 1000], 2, 4, 128, 128, torch.float32),
    ([1, 63, 65, 130], 1, 2, 64, 128, torch.bfloat16),
    ([512], 4, 4, 128, 64, torch.bfloat16),
    # head widths outside {64, 128}: zero-padded copies in the workspace
    ([100, 37], 2, 4, 32, 32, torch.float32),
    ([150], 1, 2, 96, 48, torch.bfloat16),
    ([64, 65], 2, 2, 128, 80, torch.float32),
    # several sequences of several chunks, partial last chunks
    ([1000, 300, 64, 700], 2, 8, 128, 128, torch.float32),
])
@pytest.mark.parametrize("path", PATHS)
def test_operator_on_ragged_batches(lens, nk, nv, dk, dv, state, path):
    dev = _cuda()
    _path_applies(path, dk)
    q, k, v, beta, g, h0, asl = make_case(lens, nk, nv, dk, dv, state, seed=sum(lens) + nv)
    scale = dk ** -0.5
    out, fin = cg.chunk_gated_delta_rule(q.to(dev), k.to(dev), v.to(dev), beta.to(dev), h0.to(dev), asl.to(dev), scale,
                                         g.to(dev), check_device_status=True, path=path)
    torch.cuda.synchronize()
    f = H.as_f32
    bout, bfin, _ = G.benchmark_op(f(q), f(k), f(v), f(beta), scale, f(h0), lens, g.numpy())
    gout, gfin = G.golden_op(f(q), f(k), f(v), f(beta), f(h0), lens, g.numpy(), state_bf16=state == torch.bfloat16)
    check(out, fin, gout, gfin, bout, bfin)


@pytest.mark.parametrize("path", PATHS)
def test_operator_without_gate(path):
    dev = _cuda()
    lens = [100, 37]
    q, k, v, beta, _, h0, asl = make_case(lens, 2, 2, 128, 128, torch.bfloat16, seed=5, with_g=False)
    out, fin = cg.chunk_gated_delta_rule(q.to(dev), k.to(dev), v.to(dev), beta.to(dev), h0.to(dev), asl.to(dev), None,
                                         None, check_device_status=True, path=path)
    torch.cuda.synchronize()
    f = H.as_f32
    bout, bfin, _ = G.benchmark_op(f(q), f(k), f(v), f(beta), 128 ** -0.5, f(h0), lens, None)
    gout, gfin = G.golden_op(f(q), f(k), f(v), f(beta), f(h0), lens, None)
    check(out, fin, gout, gfin, bout, bfin)


def test_lengths_not_summing_to_t_are_flagged():
    dev = _cuda()
    q, k, v, beta, g, h0, _ = make_case([64, 64], 1, 1, 64, 64, torch.bfloat16, seed=7)
    asl = torch.tensor([64, 100], dtype=torch.int32, device=dev)  # 164 != T = 128
    out = torch.zeros_like(v, device=dev)
    fin = torch.zeros_like(h0, device=dev)
    op = cg.ChunkGatedDeltaRule(q.to(dev), k.to(dev), v.to(dev), beta.to(dev), h0.to(dev), asl, g.to(dev), None, out,
                                fin)
    ws = torch.zeros(op.workspace_size, dtype=torch.uint8, device=dev)
    op(ws)
    assert cg.read_device_status(ws) & 0x2


@pytest.mark.parametrize("lens,nk,nv,dv,state", [
    ([4096, 4096], 8, 64, 128, torch.float32),           # the auto path's fused regime: B * Nv = 128
    ([77, 0, 2000, 1, 640], 4, 8, 64, torch.bfloat16),   # V = 64, ragged, an empty sequence
])
def test_fused_matches_three_kernels(lens, nk, nv, dv, state):
    """The two paths compute the same products; they differ only in how the
    output's two fp32 terms are summed (one fma against an MMA accumulation),
    so the bf16 outputs agree to the last bit nearly everywhere and the final
    states (the same recurrence) exactly."""
    dev = _cuda()
    q, k, v, beta, g, h0, asl = make_case(lens, nk, nv, 128, dv, state, seed=11)
    args = [x.to(dev) for x in (q, k, v, beta, h0, asl)]
    o1, f1 = cg.chunk_gated_delta_rule(*args, None, g.to(dev), check_device_status=True, path="fused")
    o2, f2 = cg.chunk_gated_delta_rule(*args, None, g.to(dev), check_device_status=True, path="three_kernels")
    torch.cuda.synchronize()
    assert torch.equal(f1, f2)
    a, b = o1.float(), o2.float()
    assert torch.isfinite(a).all()
    assert (a == b).float().mean().item() >= 0.99
    assert ((a - b).abs() <= 2 ** -7 * b.abs() + 1e-6).all()
