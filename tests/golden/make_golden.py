#!/usr/bin/env python3
"""Generate the committed golden fixtures from the reference's own oracle.

Run in a container where the reference tree is mounted (it is never read at
test time):

    python tests/golden/make_golden.py --reference-root <path-to-reference>

It imports ``generate_golden`` from
``<root>/ChunkGatedDeltaRuleFwdH_problem_290_template/code/tests/golden/``
and, for each of its 24 named cases (``CASES``, generate_golden.py:37-257),
a deterministic sample of its stress sampler (``build_stress_specs``,
:663-710, seed 20260817), and the kernel-UT case of
``code/tests/ut/op_kernel/chunk_gated_delta_rule_fwd_h_data/gen_data.py:175-191``:

* builds the inputs with the reference's ``build_case`` (or the UT recipe),
* runs the reference's ``run_reference`` (generate_golden.py:350-440),
* runs the reference's ``validate_outputs`` invariants (:526-580),
* writes ``<case>.npz`` plus an entry in ``manifest.json``.

Small cases store every input and output array.  Big cases store the
sha256 of each input and output storage (the same digests the reference's
own manifests record, generate_golden.py:589-600) and a seeded sample of
output elements; tests regenerate their inputs with ``cases.build_case``
and check the input digests first.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases as cases_mod  # noqa: E402

FULL_LIMIT_BYTES = 1_300_000     # inputs + outputs stored whole below this
SAMPLES_PER_OUTPUT = 4096
N_STRESS = 12


def import_reference(root: Path):
    path = root / "ChunkGatedDeltaRuleFwdH_problem_290_template/code/tests/golden/generate_golden.py"
    spec = importlib.util.spec_from_file_location("ref_generate_golden", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_generate_golden"] = mod
    spec.loader.exec_module(mod)
    return mod


def ut_case_inputs():
    """gen_data.py:175-191: seeded numpy draws rounded to bf16 via ml_dtypes."""
    from ml_dtypes import bfloat16
    rng = np.random.default_rng(290)
    k = rng.uniform(-0.125, 0.125, (1, 5, 1, 32)).astype(bfloat16)
    w = rng.uniform(-0.125, 0.125, (1, 1, 5, 32)).astype(bfloat16)
    u = rng.uniform(-0.25, 0.25, (1, 1, 5, 32)).astype(bfloat16)
    g = -0.05 * np.arange(1, 6, dtype=np.float32).reshape(1, 1, 5)
    h0 = rng.uniform(-0.0625, 0.0625, (1, 1, 32, 32)).astype(bfloat16)

    def t(a):
        return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)

    return {"k": t(k), "w": t(w), "u": t(u), "g": torch.from_numpy(g), "initial_state": t(h0),
            "cu_seqlens": torch.tensor([0, 5], dtype=torch.int64),
            "chunk_indices": torch.tensor([[0, 0]], dtype=torch.int64)}


def write_case(name, spec, inputs, outputs, manifest, full_override=None):
    st = cases_mod.storage
    in_arrays = {n: st(t) for n, t in inputs.items() if t is not None}
    out_arrays = {n: st(t) for n, t in zip(("h", "v", "final_state"), outputs)}
    nbytes = sum(a.nbytes for a in in_arrays.values()) + sum(a.nbytes for a in out_arrays.values())
    full = nbytes <= FULL_LIMIT_BYTES if full_override is None else full_override
    payload = {}
    if full:
        payload.update({"in_" + n: a for n, a in in_arrays.items()})
        payload.update({"out_" + n: a for n, a in out_arrays.items()})
    else:
        rng = np.random.default_rng(spec["seed"] & 0xFFFFFFFF)
        for n, a in out_arrays.items():
            flat = a.reshape(-1)
            cnt = min(SAMPLES_PER_OUTPUT, flat.size)
            idx = np.sort(rng.choice(flat.size, size=cnt, replace=False)).astype(np.int64)
            payload["idx_" + n] = idx
            payload["val_" + n] = flat[idx]
    fname = f"{name}.npz"
    np.savez_compressed(HERE / fname, **payload)
    manifest["cases"][name] = {
        "file": fname,
        "spec": spec,
        "full": bool(full),
        "inputs": sorted(in_arrays),
        "input_sha256": {n: cases_mod.sha256(a) for n, a in in_arrays.items()},
        "output_sha256": {n: cases_mod.sha256(a) for n, a in out_arrays.items()},
        "output_shapes": {n: list(a.shape) for n, a in out_arrays.items()},
    }
    return full, nbytes


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference-root", type=Path, required=True)
    args = ap.parse_args()
    ref = import_reference(args.reference_root)
    manifest = {"generator": "tests/golden/make_golden.py", "chunk_size": ref.CHUNK_SIZE,
                "source": "reference generate_golden.run_reference", "cases": {}}

    specs = [asdict(s) for s in ref.CASES]
    stress = [asdict(s) for s in ref.build_stress_specs(N_STRESS, 20260817)]
    for spec in specs + stress:
        spec["seq_lens"] = list(spec["seq_lens"])
        ref_spec = ref.CaseSpec(**{**spec, "seq_lens": tuple(spec["seq_lens"])})
        inputs = ref.build_case(ref_spec)
        mine = cases_mod.build_case(spec)
        for n, t in inputs.items():
            if t is None:
                assert mine[n] is None, (spec["name"], n)
            else:
                assert torch.equal(t, mine[n]), f"{spec['name']}: restated generator differs on {n}"
        outputs = ref.run_reference(**inputs, chunk_size=ref.CHUNK_SIZE)
        ref.validate_outputs(ref_spec, inputs, outputs)
        full, nbytes = write_case(spec["name"], spec, inputs, outputs, manifest)
        print(f"{spec['name']}: {'full' if full else 'sampled'} ({nbytes} B)")

    # Kernel UT case of the reference (gen_data.py), run through run_reference.
    ut = ut_case_inputs()
    outputs = ref.run_reference(**ut, chunk_size=ref.CHUNK_SIZE)
    spec = {"name": "ut_kernel_varlen_t5", "seq_lens": [5], "hv": 1, "hk": 1, "dim": 32,
            "seed": 290, "description": "gen_data.py kernel-UT case", "with_initial_state": True}
    write_case(spec["name"], spec, ut, outputs, manifest, full_override=True)
    print(f"{spec['name']}: full")

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
