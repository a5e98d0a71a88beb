#!/usr/bin/env python3
"""Generate the committed fixtures of the chunked Gated DeltaNet operator
(the stages around the recurrence) from the reference's own Python code.

Run where the reference tree is mounted (it is never read at test time):

    python tests/golden/make_gdr_golden.py --reference-root <path-to-reference>

It imports, from
``<root>/ChunkGatedDeltaRuleFwdH_problem_290_template/ref/chunk_gated_delta_rule/tests/pytest/``,
the bf16 operator ``chunk_gated_delta_rule_benchmark.py`` (stage1_opt,
stage2_opt, stage3_opt, chunk_gdn_benchmark_opt) and the fp32 golden
``chunk_gated_delta_rule_golden.py`` (chunk_gated_delta_rule_npu), and for
each case below:

* draws inputs with the reference's input recipe (tests/assets/impl/inputs.py:
  q, k L2-normalised, g clipped to [-1, 0], beta clipped to (0, 1)),
* runs the golden through the reference adapter's conventions
  (tests/assets/impl/golden.py:106-150) and the bf16 operator end to end,
* runs the operator's stages one chunk at a time to record the intermediate
  tensors in the fla layout the stage kernels use: the chunk-local
  cumulative gate, w = -k_cumdecay, u = v_inner, the state before every chunk
  (transposed to [Dk, Dv], bf16), v_new and the output,
* writes ``gdr_<case>.npz`` (bf16 tensors as uint16 bits) and
  ``gdr_manifest.json`` (shapes and sha256 of every array).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
PYTEST_DIR = "ChunkGatedDeltaRuleFwdH_problem_290_template/ref/chunk_gated_delta_rule/tests/pytest"

# name: (sequence lengths, Nk, Nv, Dk, Dv, h0 dtype, has g, seed)
CASES = {
    "single_chunk": ([64], 1, 1, 64, 64, "bf16", True, 11),
    "ragged_two": ([100, 37], 1, 2, 128, 128, "f32", True, 12),
    "gqa_partial": ([130], 1, 2, 128, 64, "bf16", True, 13),
    "multi_chunk_no_g": ([192, 128, 65], 1, 2, 128, 128, "bf16", False, 14),
    "tiny_lengths": ([1, 5, 63, 64, 65], 1, 1, 64, 64, "f32", True, 15),
    "wide_heads": ([256], 2, 4, 128, 128, "bf16", True, 16),
}


def load(root: Path, name: str):
    path = root / PYTEST_DIR / f"{name}.py"
    spec = importlib.util.spec_from_file_location(f"ref_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_inputs(lens, nk, nv, dk, dv, h0_dtype, has_g, seed):
    """The reference's input recipe (inputs.py:62-81) on seeded draws."""
    gen = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = F.normalize(torch.randn(T, nk, dk, generator=gen), p=2, dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(T, nk, dk, generator=gen), p=2, dim=-1).to(torch.bfloat16)
    v = torch.randn(T, nv, dv, generator=gen).to(torch.bfloat16)
    beta = torch.rand(T, nv, generator=gen).clamp(1e-6, 1 - 1e-6).to(torch.bfloat16)
    g = (-torch.rand(T, nv, generator=gen)).clamp(-1.0, 0.0) if has_g else None
    h0 = 0.1 * torch.randn(len(lens), nv, dv, dk, generator=gen)
    h0 = h0.to(torch.bfloat16) if h0_dtype == "bf16" else h0.float()
    asl = torch.tensor(lens, dtype=torch.int32)
    return q, k, v, beta, g, h0, asl


def run_golden(gold, q, k, v, beta, g, h0, asl, scale):
    """golden.py:106-150: the fp32 native golden through the adapter."""
    qf, kf, vf = (x.unsqueeze(0).float() for x in (q, k, v))
    bt = beta.unsqueeze(0).float()
    if g is None:
        g = torch.zeros(v.shape[0], v.shape[1])
    gt = g.unsqueeze(0).float()
    cu = F.pad(asl, (1, 0)).cumsum(0).to(torch.int64)
    st = h0.transpose(-1, -2).clone().float()
    o, s = gold.chunk_gated_delta_rule_npu(qf, kf, vf, gt, bt, scale=scale, initial_state=st, cu_seqlens=cu,
                                           chunk_size=64)
    return o[0].to(q.dtype), s.transpose(-1, -2).to(h0.dtype)


def run_stages(bench, q, k, v, beta, g, h0, asl, scale):
    """The bf16 operator's stages per sequence (benchmark.py:178-224), with
    stage 2 stepped one chunk at a time to record the state before each
    chunk.  Returns fla-layout intermediates."""
    T, nk, dk = q.shape
    nv, dv = v.shape[1], v.shape[2]
    if g is None:
        g = torch.zeros(T, nv)
    rep = nv // nk
    gcum = torch.zeros(1, T, nv)
    w = torch.zeros(1, T, nv, dk, dtype=torch.bfloat16)
    u = torch.zeros(1, T, nv, dv, dtype=torch.bfloat16)
    vnew = torch.zeros(1, T, nv, dv, dtype=torch.bfloat16)
    states = []
    out = torch.zeros(T, nv, dv, dtype=torch.bfloat16)
    final = torch.zeros_like(h0, dtype=torch.bfloat16)
    start = 0
    for b, S in enumerate(asl.tolist()):
        end = start + S
        qs, ks = q[start:end], k[start:end]
        g_cum, kcd, v_inner, q_prime, kg, qkt = bench.stage1_opt(qs, ks, v[start:end], g[start:end],
                                                                 beta[start:end], scale, 64)
        cur = h0[b].clone()
        nc = (S + 63) // 64
        ai_all, vn_all = [], []
        for c in range(nc):
            sl = slice(64 * c, 64 * c + 64)
            # [nv, dk, dv] in bf16, the dtype the recurrence writes h in (an fp32
            # initial state is rounded here; the reference multiplies with it unrounded)
            states.append(cur.float().transpose(-1, -2).to(torch.bfloat16))
            cur, ai, vn = bench.stage2_opt(q_prime[:, sl], v_inner[:, sl], g_cum[:, sl], kcd[:, sl], cur, kg[:, sl],
                                           64)
            ai_all.append(ai)
            vn_all.append(vn)
        ai_all = torch.cat(ai_all, 1)
        vn_all = torch.cat(vn_all, 1)
        final[b] = cur.to(torch.bfloat16)
        o = bench.stage3_opt(qkt, scale, g_cum, ai_all, vn_all, 64)
        out[start:end] = o[:S]
        gcum[0, start:end] = g_cum[:, :S].T
        w[0, start:end] = (-kcd[:, :S]).transpose(0, 1)
        u[0, start:end] = v_inner[:, :S].transpose(0, 1)
        vnew[0, start:end] = vn_all[:, :S].transpose(0, 1)
        start = end
    h = torch.stack(states, 0).unsqueeze(0)  # [1, NT, nv, dk, dv]
    del rep
    return dict(g_cum=gcum, w=w, u=u, h=h, v_new=vnew, o_stages=out, final_stages=final)


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True, type=Path)
    args = ap.parse_args()
    bench = load(args.reference_root, "chunk_gated_delta_rule_benchmark")
    gold = load(args.reference_root, "chunk_gated_delta_rule_golden")
    torch.set_num_threads(1)  # one summation order for the CPU matmuls
    manifest = {}
    for name, (lens, nk, nv, dk, dv, h0_dtype, has_g, seed) in CASES.items():
        q, k, v, beta, g, h0, asl = make_inputs(lens, nk, nv, dk, dv, h0_dtype, has_g, seed)
        scale = 1.0 / dk ** 0.5
        g_out, g_fin = run_golden(gold, q, k, v, beta, g, h0, asl, scale)
        b_out, b_fin = bench.chunk_gdn_benchmark_opt(q, k, v, beta, scale, h0, asl.tolist(), g=g, chunk_size=64)
        st = run_stages(bench, q, k, v, beta, g, h0, asl, scale)
        assert torch.equal(st["o_stages"], b_out), name
        assert torch.equal(st["final_stages"], b_fin.to(torch.bfloat16)), name
        arrays = dict(q=q, k=k, v=v, beta=beta, h0=h0, seq_lens=asl, golden_out=g_out, golden_final=g_fin,
                      bench_out=b_out, bench_final=b_fin, g_cum=st["g_cum"], w=st["w"], u=st["u"], h=st["h"],
                      v_new=st["v_new"])
        if g is not None:
            arrays["g"] = g
        np_arrays = {n: bits(t) for n, t in arrays.items()}
        np.savez_compressed(HERE / f"gdr_{name}.npz", **np_arrays)
        manifest[name] = dict(
            seq_lens=lens, nk=nk, nv=nv, dk=dk, dv=dv, h0_dtype=h0_dtype, has_g=has_g, seed=seed, scale=scale,
            arrays={n: dict(shape=list(a.shape), dtype=str(a.dtype), sha256=hashlib.sha256(a.tobytes()).hexdigest())
                    for n, a in np_arrays.items()})
        print(name, {n: a.shape for n, a in np_arrays.items()})
    (HERE / "gdr_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
