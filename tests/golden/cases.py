"""Input generators for the reference's golden cases, restated.

The reference builds its named golden cases with ``build_case`` /
``build_gate`` (``code/tests/golden/generate_golden.py:443-506``) from a
seeded ``torch.Generator`` and samples stress shapes with
``build_stress_specs`` (``:663-710``).  This module regenerates the same
inputs without the reference tree, so the GPU box (where the reference is
absent) can rebuild the big cases whose arrays are not committed.  The
regenerated inputs are pinned by the sha256 digests that
``make_golden.py`` recorded from the reference's own generator.

Everything is in the reference's layout: k ``[1,T,HK,D]``, w/u
``[1,HV,T,D]``, g ``[1,HV,T]`` fp32, initial_state ``[N,HV,D,D]`` bf16.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

CHUNK = 64
GOLDEN_DIR = Path(__file__).resolve().parent


def build_gate(seq_lens, hv):
    """Chunk-local, strictly decreasing negative gates (generate_golden.py:443-459)."""
    total = sum(seq_lens)
    gate = torch.empty((1, hv, total), dtype=torch.float32)
    base = 0
    for L in seq_lens:
        for c0 in range(0, L, CHUNK):
            n = min(CHUNK, L - c0)
            pos = torch.arange(1, n + 1, dtype=torch.float32)
            for h in range(hv):
                rate = 0.01 + 0.0025 * (h % 5)
                gate[0, h, base + c0: base + c0 + n] = -rate * pos
        base += L
    return gate


def build_case(spec: dict) -> dict:
    """Same draws, in the same order, as generate_golden.py:462-506."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(spec["seed"])
    T = sum(spec["seq_lens"])
    hv, hk, dim = spec["hv"], spec["hk"], spec["dim"]

    def uniform(shape):
        return torch.rand(shape, generator=gen, dtype=torch.float32) * 2.0 - 1.0

    k = uniform((1, T, hk, dim)).to(torch.bfloat16)
    w = (uniform((1, hv, T, dim)) / dim).to(torch.bfloat16)
    u = uniform((1, hv, T, dim)).to(torch.bfloat16)
    g = build_gate(spec["seq_lens"], hv)
    h0 = None
    if spec.get("with_initial_state", True):
        h0 = (torch.randn((len(spec["seq_lens"]), hv, dim, dim), generator=gen,
                          dtype=torch.float32) * 0.25).to(torch.bfloat16)
    cu = [0]
    for L in spec["seq_lens"]:
        cu.append(cu[-1] + L)
    cu = torch.tensor(cu, dtype=torch.int64)
    rows = [(s, c) for s in range(len(spec["seq_lens"]))
            for c in range((spec["seq_lens"][s] + CHUNK - 1) // CHUNK)]
    ci = torch.tensor(rows, dtype=torch.int64).reshape(-1, 2)
    return {"k": k, "w": w, "u": u, "g": g, "initial_state": h0,
            "cu_seqlens": cu, "chunk_indices": ci}


def storage(t: torch.Tensor) -> np.ndarray:
    """Raw storage as the reference writes it (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy() if hasattr(torch, "uint16") else \
            t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def sha256(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes(order="C")).hexdigest()


def load_manifest() -> dict:
    return json.loads((GOLDEN_DIR / "manifest.json").read_text())


def load_case(name: str) -> tuple[dict, dict, dict]:
    """Return (spec, inputs, golden) for one committed case.

    ``inputs`` maps names to numpy storage arrays (reference layout).
    ``golden`` holds either full arrays (``h``, ``v``, ``final_state``) or,
    for big cases, ``samples`` -- ``{name: (flat_indices, values)}`` -- plus
    the sha256 of each full output.
    """
    man = load_manifest()["cases"][name]
    spec = man["spec"]
    path = GOLDEN_DIR / man["file"]
    data = np.load(path)
    if man["full"]:
        inputs = {n: data["in_" + n] for n in man["inputs"]}
        golden = {n: data["out_" + n] for n in ("h", "v", "final_state")}
    else:
        t = build_case(spec)
        inputs = {n: storage(t[n]) for n in man["inputs"]}
        for n, digest in man["input_sha256"].items():
            if sha256(inputs[n]) != digest:
                raise AssertionError(f"{name}: regenerated input {n} does not match the reference")
        golden = {"samples": {n: (data["idx_" + n], data["val_" + n]) for n in ("h", "v", "final_state")}}
    golden["sha256"] = man["output_sha256"]
    golden["shapes"] = man["output_shapes"]
    return spec, inputs, golden
