"""Shared test helpers: seeded inputs of the benchmark configurations, layout
adapters between the reference (head-major) and fla (token-major) layouts,
and comparison statistics."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from oracle import oracle  # noqa: E402  (checker only)

CHUNK = 64


# ---- bf16 bit helpers -----------------------------------------------------------

def to_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 numpy bits; fp32 stays fp32."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(a).to(device)


def as_f32(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        return a.detach().float().cpu().numpy()
    a = np.asarray(a)
    return oracle.bf16_bits_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


def bf16_ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two bf16 bit arrays (sign-magnitude order)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))


def close_stats(got, ref, rtol, atol):
    g, r = as_f32(got).reshape(-1), as_f32(ref).reshape(-1)
    err = np.abs(g - r)
    bad = ~(err <= atol + rtol * np.abs(r))
    bad &= ~(np.isnan(g) & np.isnan(r))
    return {
        "n": g.size,
        "bad": int(bad.sum()),
        "max_abs": float(err.max(initial=0.0)),
        "max_rel": float((err / np.maximum(np.abs(r), 1e-6)).max(initial=0.0)),
        "first_bad": None if not bad.any() else int(np.flatnonzero(bad)[0]),
    }


def assert_close(got, ref, rtol, atol, what=""):
    s = close_stats(got, ref, rtol, atol)
    assert s["bad"] == 0, f"{what}: {s['bad']}/{s['n']} outside rtol={rtol} atol={atol}; {s}"
    return s


# ---- layout adapters (head-major <-> token-major) -----------------------------------

def hm_to_tm_inputs(w, u, g):
    """Reference layout w/u [B,HV,T,*], g [B,HV,T] -> fla layout."""
    return (np.ascontiguousarray(np.swapaxes(w, 1, 2)), np.ascontiguousarray(np.swapaxes(u, 1, 2)),
            np.ascontiguousarray(np.swapaxes(g, 1, 2)))


def tm_to_hm_outputs(h, v):
    """fla layout h [B,NT,H,K,V], v [B,T,H,V] -> reference layout."""
    return np.ascontiguousarray(np.swapaxes(h, 1, 2)), np.ascontiguousarray(np.swapaxes(v, 1, 2))


# ---- synthetic inputs of the benchmark configurations -------------------------------

def chunk_local_cumsum(x: torch.Tensor, seq_bounds) -> torch.Tensor:
    """Cumulative sum over T restarted at every 64-token chunk of every sequence.
    x: [B, T, H]."""
    out = torch.empty_like(x)
    for b in range(x.shape[0]):
        for bos, eos in seq_bounds:
            for c0 in range(bos, eos, CHUNK):
                c1 = min(c0 + CHUNK, eos)
                out[b, c0:c1] = torch.cumsum(x[b, c0:c1], dim=0)
    return out


def make_inputs(B, T, H, K, V, *, HK=None, seed=0, dtype=torch.bfloat16, gate_shift=2.0, h0="randn",
                cu_seqlens=None, device="cpu"):
    """Seeded inputs in the fla layout, following the benchmark recipes:
    k ~ randn L2-normalised over K; w = beta * k (beta = sigmoid(randn) per
    (t, h)); u ~ 0.5 randn; g = chunk-local cumsum of logsigmoid(randn +
    gate_shift); h0 ~ 0.1 randn (fp32), zeros, or None."""
    HK = H if HK is None else HK
    gen = torch.Generator(device="cpu").manual_seed(seed)
    k = torch.randn(B, T, HK, K, generator=gen)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    w = beta[..., None] * k.repeat_interleave(H // HK, dim=2)
    u = 0.5 * torch.randn(B, T, H, V, generator=gen)
    if cu_seqlens is None:
        bounds = [(0, T)]
    else:
        cu = [int(x) for x in cu_seqlens]
        bounds = list(zip(cu[:-1], cu[1:]))
    g = chunk_local_cumsum(torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen) + gate_shift), bounds)
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    if h0 == "randn":
        init = 0.1 * torch.randn(N, H, K, V, generator=gen)
    elif h0 == "zeros":
        init = torch.zeros(N, H, K, V)
    else:
        init = None
    cast = (lambda x: x.to(dtype)) if dtype != torch.float32 else (lambda x: x)
    out = {"k": cast(k), "w": cast(w), "u": cast(u), "g": g.float(), "initial_state": init}
    if cu_seqlens is not None:
        out["cu_seqlens"] = torch.tensor(cu_seqlens, dtype=torch.int64)
    return {n: (x.to(device) if isinstance(x, torch.Tensor) else x) for n, x in out.items()}


def varlen_lengths(n_seq, total, lo=64, hi=4096, seed=0):
    """Lengths uniform in [lo, hi], multiples of 64, rescaled to sum to `total`
    (the benchmark's varlen recipe: 16 sequences packed into T_total)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n_seq)
    lens = np.maximum(64, (lens // 64) * 64)
    # rescale to the requested total (kept multiples of 64)
    scale = total / lens.sum()
    lens = np.maximum(64, np.round(lens * scale / 64).astype(int) * 64)
    lens[-1] += total - lens.sum()
    assert lens.min() > 0 and lens.sum() == total
    return [int(x) for x in lens]


def oracle_run(inp, mode, *, store_final=True, save_new_value=True, use_g=True, final_dtype=None, h0_bf16=False):
    """Run the CPU oracle on fla-layout torch inputs; returns numpy outputs."""
    def np_of(t):
        if t is None:
            return None
        return to_bits(t) if t.dtype == torch.bfloat16 else t.detach().cpu().float().numpy()
    h0 = inp.get("initial_state")
    if h0 is not None and h0_bf16:
        h0 = h0.to(torch.bfloat16)
    cu = inp.get("cu_seqlens")
    return oracle.fwd_h(np_of(inp["k"]), np_of(inp["w"]), np_of(inp["u"]),
                        None if (inp.get("g") is None or not use_g) else np_of(inp["g"]),
                        np_of(h0), None if cu is None else cu.cpu().numpy(), mode=mode,
                        store_final=store_final, save_new_value=save_new_value, use_g=use_g,
                        final_dtype=final_dtype)
