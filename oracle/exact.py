"""The recurrence in float64 with no intermediate rounding -- TEST
INFRASTRUCTURE ONLY (a measuring stick, never the product).

Only ``tests/`` use this module.  Given the same inputs (bf16 values widened
exactly, fp32 gates), it evaluates the op's mathematics up to float64
rounding:

    h[c]   = S
    v_new  = u_c - w_c S
    S      = S exp(g_last) + k_c^T (v_new * exp(g_last - g_c))
    final  = S after the sequence's last chunk

(``docs/problem.txt:81-167`` without its fp16/bf16 rounding points; the
Triton kernel ``docs/problem.txt:353-422`` without its fp32 state and bf16
operand casts).  It answers which of two arithmetic modes is closer to the
mathematics on the reference's own golden inputs; neither mode is expected to
match it bit for bit.

Arrays use the fla layout: k ``[B,T,HK,K]``, w ``[B,T,H,K]``, u
``[B,T,H,V]``, g ``[B,T,H]``, h0 ``[N,H,K,V]``.  bf16 arrays arrive as
``numpy.uint16`` bit patterns.
"""

from __future__ import annotations

import numpy as np

CHUNK = 64


def _f64(a):
    if a is None:
        return None
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return a.astype(np.float64)


def fwd_h(k, w, u, g, h0=None, cu_seqlens=None):
    """Returns float64 ``(h [B,NT,H,K,V], v_new [B,T,H,V], final [N,H,K,V])``."""
    k, w, u, g, h0 = _f64(k), _f64(w), _f64(u), _f64(g), _f64(h0)
    B, T, HK, K = k.shape
    H, V = u.shape[2], u.shape[3]
    rep = H // HK
    if cu_seqlens is None:
        seqs = [(b, 0, T) for b in range(B)]
        NT = (T + CHUNK - 1) // CHUNK
    else:
        cu = [int(x) for x in np.asarray(cu_seqlens)]
        seqs = [(0, cu[i], cu[i + 1]) for i in range(len(cu) - 1)]
        NT = sum((e - s + CHUNK - 1) // CHUNK for _, s, e in seqs)
    N = len(seqs)
    h = np.zeros((B, NT, H, K, V))
    v_new = np.zeros((B, T, H, V))
    fin = np.zeros((N, H, K, V))
    boh = 0
    for n, (b, bos, eos) in enumerate(seqs):
        S = np.zeros((H, K, V)) if h0 is None else h0[n].copy()
        nc = (eos - bos + CHUNK - 1) // CHUNK
        for c in range(nc):
            t0, t1 = bos + c * CHUNK, min(bos + (c + 1) * CHUNK, eos)
            ci = (boh + c) if cu_seqlens is not None else c
            h[b, ci] = S
            kc = np.repeat(k[b, t0:t1], rep, axis=1)           # [t, H, K]
            wc, uc, gc = w[b, t0:t1], u[b, t0:t1], g[b, t0:t1]  # [t, H, *]
            vn = uc - np.einsum("thk,hkv->thv", wc, S)
            v_new[b, t0:t1] = vn
            gl = gc[-1]                                          # [H]
            vd = vn * np.exp(gl[None, :] - gc)[:, :, None]
            S = S * np.exp(gl)[:, None, None] + np.einsum("thk,thv->hkv", kc, vd)
        fin[n] = S
        boh += nc
    return h, v_new, fin
