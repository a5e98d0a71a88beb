"""The CPU oracle pinned against the reference's own golden vectors (CPU only).

The fixtures under tests/golden/ were produced by the reference's
run_reference (code/tests/golden/generate_golden.py:350-440) on its 24 named
cases, 12 stress samples and the kernel-UT case; see make_golden.py.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
import helpers as H
from oracle import oracle

MAN = cases.load_manifest()
GOLDEN = list(MAN["cases"])


def _oracle_outputs(inp, mode):
    w, u, g = H.hm_to_tm_inputs(inp["w"], inp["u"], inp["g"])
    h, v, f = oracle.fwd_h(inp["k"], w, u, g, inp.get("initial_state"), inp["cu_seqlens"], mode=mode,
                           final_dtype="bf16")
    hh, vv = H.tm_to_hm_outputs(h, v)
    return {"h": hh, "v": vv, "final_state": f}


def _against_gold(arr, gold, name):
    a = np.ascontiguousarray(arr).reshape(-1)
    if "samples" in gold:
        idx, ref = gold["samples"][name]
        return a[idx], ref
    return a, gold[name].reshape(-1)


@pytest.mark.parametrize("case", GOLDEN)
def test_oracle_reference_mode_matches_golden(case):
    """Bit-exact for most cases; elsewhere the only differences are fp32
    summation-order flips of a bf16 rounding (torch's GEMM vs a double sum)."""
    spec, inp, gold = cases.load_case(case)
    out = _oracle_outputs(inp, "reference")
    for n in ("h", "v", "final_state"):
        assert list(out[n].shape) == gold["shapes"][n]
        got, ref = _against_gold(out[n], gold, n)
        exact = float(np.mean(got == ref))
        st = H.close_stats(got, ref, 2e-2, 2e-2)
        assert exact >= 0.99, f"{case}/{n}: {exact:.4%} bit-equal"
        assert st["bad"] <= max(1, int(1e-4 * st["n"])), f"{case}/{n}: {st}"
        assert st["max_abs"] <= 0.125, f"{case}/{n}: {st}"


def test_oracle_bit_exact_on_small_cases():
    """Where the reference's GEMMs are short, the restatement is bit-exact."""
    exact_cases = ["smoke_single_partial", "two_chunk_single", "single_token", "ut_kernel_varlen_t5",
                   "two_v_tiles", "four_v_tiles", "official_example", "varlen_many"]
    for case in exact_cases:
        spec, inp, gold = cases.load_case(case)
        out = _oracle_outputs(inp, "reference")
        for n in ("h", "v", "final_state"):
            assert cases.sha256(np.ascontiguousarray(out[n])) == gold["sha256"][n], f"{case}/{n}"


def test_restated_input_generator_matches_reference_digests():
    """cases.build_case regenerates the reference's inputs bit for bit."""
    for case in ("long_1024_heads", "varlen_eval_style", "stress_008"):
        spec = MAN["cases"][case]["spec"]
        t = cases.build_case(spec)
        for n, digest in MAN["cases"][case]["input_sha256"].items():
            assert cases.sha256(cases.storage(t[n])) == digest, (case, n)


def test_oracle_deterministic():
    spec, inp, gold = cases.load_case("grouped_heads_packed")
    a = _oracle_outputs(inp, "reference")
    b = _oracle_outputs(inp, "reference")
    for n in a:
        assert np.array_equal(a[n], b[n])


def test_fp32_state_semantics_close_to_reference_on_baseline_recipe():
    """On the benchmark input recipe the Triton (fp32 state) arithmetic stays
    within the north-star 2e-2 of the reference rounding chain."""
    import torch
    inp = H.make_inputs(1, 1024, 4, 128, 128, seed=0)
    r = H.oracle_run(inp, "reference", final_dtype="f32")
    f = H.oracle_run(inp, "fp32_state")
    for a, b in zip(f, r):
        H.assert_close(a, b, 2e-2, 2e-2)
    assert isinstance(inp["k"], torch.Tensor)


def test_oracle_edge_semantics():
    """Partial chunks use g_last = g[len-1]; h[:, first chunk] = initial state;
    an empty sequence leaves final_state = initial state."""
    import torch
    inp = H.make_inputs(1, 70, 2, 32, 32, seed=3, cu_seqlens=[0, 5, 5, 70])
    h, v, f = H.oracle_run(inp, "fp32_state")
    h0 = inp["initial_state"].numpy()
    # sequence 1 is empty: final == h0 (fp32 state keeps it exactly)
    assert np.array_equal(f[1], h0[1])
    # first chunk of sequence 0 stores bf16(h0)
    assert np.array_equal(H.as_f32(h[0, 0]), H.as_f32(H.oracle.f32_to_bf16_bits(h0[0])))
    assert h.shape[1] == 1 + 0 + 2
    assert isinstance(inp["k"], torch.Tensor)


def test_parity_budget_covers_every_golden_case():
    """The per-case budgets the GPU parity tests enforce (written from a B200 run
    by tests/golden/make_parity_budget.py) cover every golden case, both
    kernels and both arithmetic modes; the reference rounding chain stays
    within a handful of elements per case."""
    import json
    budget = json.loads((cases.GOLDEN_DIR / "parity_budget.json").read_text())
    for numerics in ("reference", "fp32_state"):
        for kernel in ("tc", "general"):
            table = budget[numerics][kernel]
            assert set(table) == set(GOLDEN), (numerics, kernel)
            for case, outs in table.items():
                assert set(outs) == {"h", "v", "final_state"}
                for name, (bad, mx) in outs.items():
                    assert 0 <= bad and 0.0 <= mx <= 0.0625, (numerics, kernel, case, name)
                    if numerics == "reference":
                        assert bad <= 2, (kernel, case, name, bad)
