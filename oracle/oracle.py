"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module.  It is the checker; the product never routes through it.

The C restatement lives in ``cgdr_oracle.c`` (see its header for the
reference lines it follows).  Two semantics are exposed:

* ``mode="reference"``: the contest's normative PyTorch reference
  (``docs/problem.txt:81-167``, ``code/tests/golden/generate_golden.py:350-440``)
  with every fp16/bf16 rounding point and a bf16 state between chunks.
* ``mode="fp32_state"``: the Triton kernel's semantics
  (``docs/problem.txt:272-432``): fp32 state, bf16 MMA operands for bf16 I/O,
  ``safe_exp`` gating.

Arrays use the fla layout: k ``[B,T,HK,K]``, w ``[B,T,H,K]``, u/v_new
``[B,T,H,V]``, g ``[B,T,H]`` fp32, h0/final ``[N,H,K,V]``, h ``[B,NT,H,K,V]``.
bf16 arrays are carried as ``numpy.uint16`` bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle_cgdr.so"
_lib = None

DT_BF16 = 1
DT_F32 = 2
MODES = {"reference": 0, "fp32_state": 1}


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc only; no GPU needed)."""
    src = _HERE / "cgdr_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE), "liboracle_cgdr.so"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.cgdr_oracle_fwd_h.argtypes = [i64] * 6 + [vp] * 6 + [i64] + [vp] * 3 + [ctypes.c_int] * 6
        lib.cgdr_oracle_fwd_h.restype = ctypes.c_int
        lib.cgdr_oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().cgdr_oracle_max_threads())


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _dt(a):
    if a.dtype == np.uint16:
        return DT_BF16
    if a.dtype == np.float32:
        return DT_F32
    raise TypeError(f"oracle arrays must be uint16 (bf16 bits) or float32, got {a.dtype}")


def fwd_h(k, w, u, g, h0=None, cu_seqlens=None, *, mode="reference", store_final=True,
          final_dtype=None, save_new_value=True, use_g=True, n_threads=0):
    """Run the oracle; returns ``(h, v_new, final_state)`` as numpy arrays.

    ``h``/``v_new`` have the dtype of the inputs; ``final_state`` is bf16 bits
    in reference mode and fp32 in fp32_state mode unless ``final_dtype`` says
    otherwise ("bf16" or "f32").
    """
    k, w, u = (np.ascontiguousarray(x) for x in (k, w, u))
    io = _dt(k)
    if _dt(w) != io or _dt(u) != io:
        raise TypeError("k, w and u must share a dtype")
    B, T, HK, K = k.shape
    H, V = u.shape[2], u.shape[3]
    if w.shape != (B, T, H, K) or u.shape[:2] != (B, T):
        raise ValueError("w must be [B,T,H,K] and u [B,T,H,V]")
    if g is not None:
        g = np.ascontiguousarray(g, dtype=np.float32)
        if g.shape != (B, T, H):
            raise ValueError("g must be [B,T,H]")
    if cu_seqlens is not None:
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int64)
        N = cu.shape[0] - 1
        lens = np.diff(cu)
        NT = int(((lens + 63) // 64).sum())
    else:
        cu = None
        N = B
        NT = (T + 63) // 64
    h0c = None if h0 is None else np.ascontiguousarray(h0)
    h = np.zeros((B, NT, H, K, V), dtype=k.dtype)
    v_new = np.zeros((B, T, H, V), dtype=k.dtype) if save_new_value else None
    if final_dtype is None:
        final_dtype = "bf16" if mode == "reference" else "f32"
    fin = None
    if store_final:
        fin = np.zeros((N, H, K, V), dtype=np.uint16 if final_dtype == "bf16" else np.float32)
    rc = _load().cgdr_oracle_fwd_h(
        B, T, HK, H, K, V,
        _ptr(k), _ptr(w), _ptr(u), _ptr(g), _ptr(h0c), _ptr(cu), N,
        _ptr(h), _ptr(v_new), _ptr(fin),
        io, 0 if h0c is None else _dt(h0c), 0 if fin is None else _dt(fin),
        MODES[mode], int(bool(use_g)), int(n_threads),
    )
    if rc != 0:
        raise ValueError("oracle rejected the shapes")
    return h, v_new, fin


# ---- bf16 helpers (numpy has no bfloat16) ---------------------------------

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (uint16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def default_threads() -> int:
    return os.cpu_count() or 1
