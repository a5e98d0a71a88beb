#!/usr/bin/env python3
"""Writes tests/golden/parity_budget.json: for every golden case, kernel and
arithmetic mode, how many elements of each output lie beyond rtol = atol =
2e-2 of the reference's golden, and the largest absolute difference.

Run on a B200 (it calls the CUDA library through the C ABI):

    python tests/golden/make_parity_budget.py

The GPU parity tests (tests/test_gpu_parity.py) fail when a case exceeds its
recorded count or maximum, so an arithmetic change that moves even one more
element past the tolerance shows up as a test failure; re-run this script
only after such a change has been reviewed.  The goldens themselves come from
the reference's run_reference (make_golden.py); the kernels are
deterministic, so the counts repeat exactly from run to run.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (ROOT, ROOT / "tests", HERE):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import cases  # noqa: E402
import helpers as H  # noqa: E402

import cann_operator_challenge_august_b200 as cg  # noqa: E402

TOL = 2e-2
KERNELS = {"tc": 1, "general": 2}


def to_dev(inp, dev):
    return {n: (H.from_bits(a, dev) if a.dtype == np.uint16 else torch.from_numpy(np.ascontiguousarray(a)).to(dev))
            for n, a in inp.items()}


def measure(gold, name, bits):
    """(elements beyond 2e-2 of the golden, max |difference|) of one output."""
    a = np.ascontiguousarray(bits).reshape(-1)
    if "samples" in gold:
        idx, ref = gold["samples"][name]
        a = a[idx]
    else:
        ref = gold[name].reshape(-1)
    st = H.close_stats(a, ref, TOL, TOL)
    return st["bad"], st["max_abs"]


def run_case(case, kernel, numerics, dev):
    """Outputs of one golden case in the reference's (head-major) layout, as bf16 bits."""
    spec, inp, gold = cases.load_case(case)
    t = to_dev(inp, dev)
    fk = KERNELS[kernel]
    if numerics == "reference":
        h, v, f = cg.run(t["k"], t["w"], t["u"], t["g"], t.get("initial_state"), t["cu_seqlens"], t["chunk_indices"],
                         64, force_kernel=fk, check_device_status=True)
        return gold, {"h": H.to_bits(h), "v": H.to_bits(v), "final_state": H.to_bits(f)}
    w, u, g = (t[n].transpose(1, 2).contiguous() for n in ("w", "u", "g"))
    h, v, f = cg.chunk_gated_delta_rule_fwd_h(t["k"], w, u, g, t.get("initial_state"), cu_seqlens=t["cu_seqlens"],
                                              chunk_indices=t["chunk_indices"], force_kernel=fk,
                                              final_state_dtype=torch.bfloat16, check_device_status=True)
    hh, vv = H.tm_to_hm_outputs(H.to_bits(h), H.to_bits(v))
    return gold, {"h": hh, "v": vv, "final_state": H.to_bits(f)}


def main() -> int:
    dev = torch.device("cuda")
    out = {"tolerance": "rtol = atol = 2e-2 against the reference's goldens",
           "entries": "[elements beyond the tolerance, max |difference|] per output"}
    for numerics in ("reference", "fp32_state"):
        out[numerics] = {}
        for kernel in KERNELS:
            table = {}
            for case in cases.load_manifest()["cases"]:
                gold, got = run_case(case, kernel, numerics, dev)
                table[case] = {n: list(measure(gold, n, got[n])) for n in ("h", "v", "final_state")}
            out[numerics][kernel] = table
            print(numerics, kernel, sum(x["h"][0] + x["v"][0] + x["final_state"][0] for x in table.values()),
                  flush=True)
    (HERE / "parity_budget.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
