"""The golden-case runner (runner/cgdr_fwd_h_case): the counterpart of the
reference's example program ``code/examples/test_aclnn_chunk_gated_delta_rule_fwd_h.cpp``.

A case directory holds manifest.json and the input_*.bin files in the
reference's layout; the runner writes actual_h.bin, actual_v.bin and
actual_final_state.bin.  The CPU tests cover the command line and the input
checks (all raised before any device call); the GPU tests write committed
golden fixtures as case directories and compare the runner's outputs with
the Python API (bit-identical: the same library call) and with the goldens
(the tolerance of the golden parity tests: >= 97 % bit-equal, >= 99.9 %
within rtol/atol 2e-2).
"""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import helpers as H

PKG = Path(__file__).resolve().parent.parent / "cann_operator_challenge_august_b200"
RUNNER = PKG / "runner" / "cgdr_fwd_h_case"
BF_TOL = 2e-2


def _runner() -> Path:
    if not RUNNER.exists():
        pytest.skip("case runner not built (python -m cann_operator_challenge_august_b200.build)")
    return RUNNER


def _run(*args, timeout=120):
    return subprocess.run([str(_runner()), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def write_case_dir(path: Path, spec: dict, inp: dict) -> None:
    """The reference's case-directory format: manifest + raw little-endian storage."""
    path.mkdir(parents=True, exist_ok=True)
    man = {"total_tokens": int(inp["k"].shape[1]), "total_chunks": int(inp["chunk_indices"].shape[0]),
           "hv": int(spec["hv"]), "hk": int(spec["hk"]), "dim": int(spec["dim"])}
    (path / "manifest.json").write_text(json.dumps(man, indent=2))
    for name in ("k", "w", "u", "g", "cu_seqlens", "chunk_indices", "initial_state"):
        if name in inp:
            np.ascontiguousarray(inp[name]).tofile(path / f"input_{name}.bin")


# ---------------------------------------------------------------- CPU: command line and input checks

def test_usage_exit_code():
    r = _run()
    assert r.returncode == 2 and "CASE_DIR" in r.stderr


def test_missing_manifest_is_reported(tmp_path):
    r = _run(tmp_path)
    assert r.returncode == 1 and "manifest.json" in r.stderr


def test_manifest_without_a_key_is_reported(tmp_path):
    (tmp_path / "manifest.json").write_text(json.dumps({"total_tokens": 5, "hv": 1, "hk": 1, "dim": 32}))
    r = _run(tmp_path)
    assert r.returncode == 1 and "total_chunks" in r.stderr


def test_short_cu_seqlens_is_reported(tmp_path):
    (tmp_path / "manifest.json").write_text(
        json.dumps({"total_tokens": 5, "total_chunks": 1, "hv": 1, "hk": 1, "dim": 32}))
    np.array([0], dtype=np.int64).tofile(tmp_path / "input_cu_seqlens.bin")
    r = _run(tmp_path)
    assert r.returncode == 1 and "input_cu_seqlens.bin" in r.stderr


def test_case_dir_matches_the_reference_format(tmp_path):
    """Sizes of the written files follow the manifest's shapes."""
    spec, inp, _ = cases.load_case("grouped_heads_packed")
    write_case_dir(tmp_path, spec, inp)
    man = json.loads((tmp_path / "manifest.json").read_text())
    T, NT, HV, HK, D = (man[k] for k in ("total_tokens", "total_chunks", "hv", "hk", "dim"))
    N = len(spec["seq_lens"])
    sizes = {"k": T * HK * D * 2, "w": HV * T * D * 2, "u": HV * T * D * 2, "g": HV * T * 4,
             "cu_seqlens": (N + 1) * 8, "chunk_indices": NT * 2 * 8, "initial_state": N * HV * D * D * 2}
    for name, n in sizes.items():
        assert (tmp_path / f"input_{name}.bin").stat().st_size == n, name


# ---------------------------------------------------------------- GPU: golden cases through the runner

RUNNER_CASES = ["smoke_single_partial", "boundary_63_64_65", "grouped_heads_packed", "without_initial_state",
                "two_v_tiles", "four_v_tiles", "official_example", "varlen_eval_style", "stress_007",
                "heads_equal_hk_hv", "no_state_long"]


def _read_bits(path: Path, shape) -> np.ndarray:
    a = np.fromfile(path, dtype=np.uint16)
    assert a.size == int(np.prod(shape)), f"{path.name}: {a.size} values, expected shape {shape}"
    return a


@pytest.mark.gpu
@pytest.mark.parametrize("case", RUNNER_CASES)
def test_runner_matches_api_and_goldens(case, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import cann_operator_challenge_august_b200 as cg

    spec, inp, gold = cases.load_case(case)
    write_case_dir(tmp_path, spec, inp)
    r = _run(tmp_path, 0)
    assert r.returncode == 0, r.stdout + r.stderr
    got = {n: _read_bits(tmp_path / f"actual_{n}.bin", gold["shapes"][n]) for n in ("h", "v", "final_state")}

    dev = torch.device("cuda")
    t = {n: H.from_bits(a, dev) if a.dtype == np.uint16 else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
         for n, a in inp.items()}
    h, v, f = cg.run(t["k"], t["w"], t["u"], t["g"], t.get("initial_state"), t["cu_seqlens"], t["chunk_indices"], 64,
                     check_device_status=True)
    torch.cuda.synchronize()
    for n, out in (("h", h), ("v", v), ("final_state", f)):
        api = H.to_bits(out).reshape(-1)
        assert np.array_equal(got[n], api), f"{case}/{n}: runner and Python API differ"
        bits = got[n]
        if "samples" in gold:
            idx, ref = gold["samples"][n]
            bits = bits[idx]
        else:
            ref = gold[n].reshape(-1)
        exact = float(np.mean(bits == ref)) if bits.size else 1.0
        st = H.close_stats(bits, ref, BF_TOL, BF_TOL)
        assert exact >= 0.97, f"{case}/{n}: only {exact:.4%} bit-equal; {st}"
        assert st["bad"] <= int(1e-3 * st["n"]), f"{case}/{n}: {st}"
