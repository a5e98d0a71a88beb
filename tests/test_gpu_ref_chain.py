"""The packed (f16x2 / bf16x2) form of the reference rounding chain used by the
tensor-core epilogues gives the same bits as the scalar form for finite
operands (the kernels route any warp holding another value through the scalar
form).  The test compiles tests/cuda/ref_chain_pairs.cu with nvcc and compares
both forms element by element on random and edge-case inputs."""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = tmp_path_factory.mktemp("refchain") / "libref_chain_pairs.so"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                    "-shared", "-o", str(out), str(HERE / "cuda" / "ref_chain_pairs.cu")], check=True)
    lib = ctypes.CDLL(str(out))
    lib.run_pairs.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    return lib


def _round_bf16(x):
    return torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def _round_f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def _inputs(rng, n):
    """Mixtures of scales: ordinary values, values near the f16 range limit, values
    in the f16 subnormal range, and exact cancellations."""
    scale = rng.choice([1e-6, 1e-4, 1e-2, 1.0, 30.0, 3000.0, 30000.0, 60000.0], size=(n, 1))
    x = (rng.standard_normal((n, 5)) * scale).astype(np.float32)
    return x


def _run(lib, which, x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((x.shape[0], 4), np.uint32)
    rc = lib.run_pairs(which, x.ctypes.data, out.ctypes.data, x.shape[0])
    assert rc == 0
    return out


def test_epilogue1_pair_bits_equal(lib):
    rng = np.random.default_rng(0)
    x = _inputs(rng, 200_000)
    x[:, 0:2] = _round_bf16(x[:, 0:2])                                   # u is bf16
    x[:, 4] = _round_f16(np.abs(np.tanh(x[:, 4])))                       # gate: an f16 value in [0, 1]
    x[::7, 2] = x[::7, 0]                                                # exact cancellation u - w.S
    keep = np.all(np.abs(x[:, :4]) < 65000.0, axis=1)                    # the packed domain
    out = _run(lib, 1, x[keep])
    assert np.array_equal(out[:, 0], out[:, 2]), "v_new bits differ"
    assert np.array_equal(out[:, 1], out[:, 3]), "v_decay bits differ"


def test_epilogue2_pair_bits_equal(lib):
    rng = np.random.default_rng(1)
    x = _inputs(rng, 200_000)
    x[:, 0:2] = _round_bf16(x[:, 0:2] * 2.0)                             # state is bf16, may exceed 65504
    x[:, 4] = _round_f16(np.exp(-np.abs(x[:, 4]) / 1000.0))              # alpha: f16 value in (0, 1]
    x[::5, 2] = 1.0e6                                                    # update beyond the f16 range (inf)
    out = _run(lib, 2, x)
    assert np.array_equal(out[:, 0], out[:, 2]), "state bits differ (first element)"
    assert np.array_equal(out[:, 1], out[:, 3]), "state bits differ (second element)"


def test_epilogue1_fast_pair_bits_equal(lib):
    """The chain without saturations, on its domain (|u|, |acc| < 16384, gate in [0, 1])."""
    rng = np.random.default_rng(2)
    x = _inputs(rng, 200_000)
    x[:, 0:2] = _round_bf16(x[:, 0:2])
    x[:, 4] = _round_f16(np.abs(np.tanh(x[:, 4])))
    x[::7, 2] = x[::7, 0]
    keep = np.all(np.abs(x[:, :4]) < 16384.0, axis=1)
    out = _run(lib, 3, x[keep])
    assert keep.sum() > 100_000
    assert np.array_equal(out[:, 0], out[:, 2]), "v_new bits differ"
    assert np.array_equal(out[:, 1], out[:, 3]), "v_decay bits differ"


def test_epilogue2_fast_pair_bits_equal(lib):
    """The state update without saturation, on its domain (finite state, |acc| < 32768,
    alpha in [0, 1]); the state may exceed the f16 range (the conversion saturates it,
    as the reference's cast does)."""
    rng = np.random.default_rng(3)
    x = _inputs(rng, 200_000)
    x[:, 0:2] = _round_bf16(x[:, 0:2] * 2.0)
    x[:, 4] = _round_f16(np.exp(-np.abs(x[:, 4]) / 1000.0))
    keep = np.all(np.abs(x[:, 2:4]) < 32768.0, axis=1)
    for which in (4, 5):  # fp32 pair in and out; bf16 pair bits in and out
        out = _run(lib, which, x[keep])
        assert keep.sum() > 100_000
        assert np.array_equal(out[:, 0], out[:, 2]), f"state bits differ (first element, form {which})"
        assert np.array_equal(out[:, 1], out[:, 3]), f"state bits differ (second element, form {which})"
