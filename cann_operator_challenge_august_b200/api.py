"""Python front ends of the op, over the C ABI (include/cgdr_fwd_h.h).

Three entry points mirror the reference's three interfaces:

* :func:`chunk_gated_delta_rule_fwd_h` -- the fla / vLLM Python signature of
  the reference (``docs/problem.txt:436-500``): token-major layout,
  ``(h, v_new, final_state)`` with an fp32 final state.  Default arithmetic
  is the Triton kernel's (fp32 state).
* :func:`run` -- the contest's PyTorch reference signature
  (``docs/problem.txt:81``): head-major layout, bf16 outputs, the reference
  rounding chain.
* :class:`ChunkGatedDeltaRuleFwdH` -- the two-phase ACLNN call
  (``code/examples/test_aclnn_chunk_gated_delta_rule_fwd_h.cpp:297-326``):
  workspace query, then launch on a stream into caller-owned outputs.

PyTorch provides device memory and the current stream only; the compute is
the CUDA library.  Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

CHUNK_SIZE = 64

_DT = {torch.bfloat16: _lib.DT_BF16, torch.float32: _lib.DT_FLOAT32, torch.float16: _lib.DT_FLOAT16,
       torch.int64: _lib.DT_INT64, torch.int32: _lib.DT_INT32}


def _desc(t: torch.Tensor | None) -> _lib.CgdrTensor:
    if t is None:
        return _lib.null_tensor()
    if t.dtype not in _DT:
        return _lib.make_tensor(t.data_ptr(), 0, t.shape, t.stride())
    return _lib.make_tensor(t.data_ptr(), _DT[t.dtype], t.shape, t.stride())


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def prepare_chunk_indices(cu_seqlens: torch.Tensor, chunk_size: int = CHUNK_SIZE,
                          capacity: int | None = None) -> torch.Tensor:
    """Rows of (sequence, chunk within the sequence) -- docs/problem.txt:251-260.

    Without ``capacity`` the list is computed on the host from the sequence
    lengths (one device->host copy of ``cu_seqlens``, the reference's way)
    and has exactly one row per chunk.  With ``capacity`` (at least
    ``ceil(T / chunk_size) + N - 1``) a device kernel fills ``capacity`` rows
    on the current stream, padding with (-1, -1) rows that the kernels skip:
    no host synchronisation (see :func:`chunk_capacity`)."""
    if capacity is not None:
        if not cu_seqlens.is_cuda:
            raise ValueError("the device chunk list needs cu_seqlens on a CUDA device")
        out = torch.empty(int(capacity), 2, dtype=torch.int64, device=cu_seqlens.device)
        cu = cu_seqlens.to(torch.int64).contiguous()
        st = _lib.load().cgdrPrepareChunkIndices(ctypes.byref(_desc(cu)), int(chunk_size), ctypes.byref(_desc(out)),
                                                 ctypes.byref(_lib.null_tensor()),
                                                 ctypes.c_void_p(_stream_handle(cu.device)))
        _lib.check(st, "cgdrPrepareChunkIndices")
        return out
    lens = (cu_seqlens[1:] - cu_seqlens[:-1]).tolist()
    rows = [(s, c) for s, L in enumerate(lens) for c in range(math.ceil(L / chunk_size))]
    out = torch.tensor(rows, dtype=torch.int64).reshape(-1, 2)
    return out.to(cu_seqlens.device)


def chunk_capacity(total_tokens: int, n_sequences: int, chunk_size: int = CHUNK_SIZE) -> int:
    """Rows that always hold the chunk list of ``n_sequences`` packed into
    ``total_tokens``: ceil(T / chunk) + N - 1 (each sequence boundary can
    split one chunk)."""
    return (int(total_tokens) + chunk_size - 1) // chunk_size + int(n_sequences) - 1


def prepare_chunk_offsets(cu_seqlens: torch.Tensor, chunk_size: int = CHUNK_SIZE) -> torch.Tensor:
    """Cumulative chunk count per sequence -- docs/problem.txt:262-270 (on device)."""
    lens = cu_seqlens[1:] - cu_seqlens[:-1]
    counts = (lens + chunk_size - 1) // chunk_size
    return torch.cat([counts.new_zeros(1), counts.cumsum(0)])


class ChunkGatedDeltaRuleFwdH:
    """Two-phase call, the ACLNN pattern of the reference.

    ``op = ChunkGatedDeltaRuleFwdH(k, w, u, g, initial_state, cu_seqlens,
    chunk_indices, chunk_size, h, v, final_state, **options)`` validates and
    plans (phase 1; no device work); ``op.workspace_size`` is the byte count
    phase 2 needs; ``op(workspace, stream)`` enqueues the kernels (phase 2).
    An object is launched at most once, like an aclOpExecutor.
    """

    def __init__(self, k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_size, h, v, final_state,
                 *, chunk_offsets=None, layout="head_major", numerics="reference",
                 strict_reference_limits=False, force_kernel=0, v_tile=0, wait_timeout_ms=0, fault_inject=0,
                 chains=0, extended=True):
        lib = _lib.load()
        self._keep = (k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_offsets, h, v, final_state)
        ws = ctypes.c_uint64(0)
        ex = ctypes.c_void_p(None)
        descs = [_desc(x) for x in (k, w, u, g, initial_state, cu_seqlens, chunk_indices)]
        outs = [_desc(x) for x in (h, v, final_state)]
        if extended:
            opt = _lib.CgdrFwdHOptions(
                layout=_lib.LAYOUT_HEAD_MAJOR if layout == "head_major" else _lib.LAYOUT_TOKEN_MAJOR,
                numerics=_lib.NUMERICS[numerics], strict_reference_limits=int(strict_reference_limits),
                force_kernel=int(force_kernel), v_tile=int(v_tile), wait_timeout_ms=int(wait_timeout_ms),
                fault_inject=int(fault_inject), chains=int(chains))
            st = lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx(
                *[ctypes.byref(d) for d in descs], ctypes.byref(_desc(chunk_offsets)), int(chunk_size),
                *[ctypes.byref(d) for d in outs], ctypes.byref(opt), ctypes.byref(ws), ctypes.byref(ex))
        else:
            st = lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize(
                *[ctypes.byref(d) for d in descs], int(chunk_size), *[ctypes.byref(d) for d in outs],
                ctypes.byref(ws), ctypes.byref(ex))
        _lib.check(st, "cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize")
        self._ex = ex
        self.workspace_size = int(ws.value)

    @property
    def plan(self) -> dict:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        pl = _lib.CgdrFwdHPlan()
        _lib.check(_lib.load().cgdrGetPlan(self._ex, ctypes.byref(pl)), "cgdrGetPlan")
        return pl.as_dict()

    def __call__(self, workspace: torch.Tensor, stream: int | None = None) -> None:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        ex, self._ex = self._ex, None
        if stream is None:
            stream = _stream_handle(workspace.device)
        st = _lib.load().cgdrChunkGatedDeltaRuleFwdH(
            ctypes.c_void_p(workspace.data_ptr()), workspace.numel() * workspace.element_size(), ex,
            ctypes.c_void_p(stream))
        _lib.check(st, "cgdrChunkGatedDeltaRuleFwdH")

    def __del__(self):
        if getattr(self, "_ex", None) is not None and _lib._lib is not None:
            _lib._lib.cgdrDestroyExecutor(self._ex)
            self._ex = None


def read_device_status(workspace: torch.Tensor, stream: int | None = None) -> int:
    """Synchronise and return the device status word of the last launch."""
    if stream is None:
        stream = _stream_handle(workspace.device)
    out = ctypes.c_int32(0)
    _lib.load().cgdrReadDeviceStatus(ctypes.c_void_p(workspace.data_ptr()), workspace.numel(),
                                     ctypes.c_void_p(stream), ctypes.byref(out))
    return int(out.value)


def _launch(op: ChunkGatedDeltaRuleFwdH, device: torch.device, check_device_status: bool) -> None:
    ws = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=device)
    op(ws)
    if check_device_status:
        status = read_device_status(ws)
        if status:
            raise RuntimeError(f"device status 0x{status:x}: "
                               + ("a bounded wait expired " if status & _lib.DEVICE_WAIT_TIMEOUT else "")
                               + ("inconsistent cu_seqlens" if status & _lib.DEVICE_BAD_VARLEN else ""))


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors (there is no CPU implementation)")


def chunk_gated_delta_rule_fwd_h(
    k: torch.Tensor,
    w: torch.Tensor,
    u: torch.Tensor,
    g: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    chunk_size: int = CHUNK_SIZE,
    save_new_value: bool = True,
    cu_seqlens: torch.LongTensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    chunk_offsets: torch.Tensor | None = None,
    *,
    output_final_state: bool = True,
    numerics: str = "fp32_state",
    final_state_dtype: torch.dtype = torch.float32,
    check_device_status: bool = False,
    **plan_options,
) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """fla / vLLM signature (docs/problem.txt:436-500), token-major layout.

    k ``[B,T,Hg,K]``, w ``[B,T,H,K]``, u ``[B,T,H,V]``, g ``[B,T,H]`` fp32,
    initial_state ``[N,H,K,V]``.  Returns h ``[B,NT,H,K,V]``, v_new
    ``[B,T,H,V]`` (``None`` if ``save_new_value`` is False) and final_state
    ``[N,H,K,V]`` (fp32 by default, as in the reference wrapper).

    ``numerics="fp32_state"`` (default) follows the Triton kernel;
    ``"reference"`` follows the contest's PyTorch reference bit for bit up to
    fp32 summation order.  With cu_seqlens and neither chunk_indices nor
    chunk_offsets, the chunk count is derived on the host (one sync), like
    the reference wrapper (problem.txt:455-460).
    """
    _require_cuda(k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_offsets)
    B, T, Hg, K = k.shape
    H, V = u.shape[-2], u.shape[-1]
    if cu_seqlens is None:
        N, NT = B, (T + chunk_size - 1) // chunk_size
    else:
        N = cu_seqlens.numel() - 1
        if chunk_indices is not None:
            NT = chunk_indices.shape[0]
        elif chunk_offsets is not None:
            NT = int(chunk_offsets[-1].item())
        else:
            chunk_indices = prepare_chunk_indices(cu_seqlens, chunk_size)
            NT = chunk_indices.shape[0]
    h = k.new_empty(B, NT, H, K, V)
    v_new = torch.empty_like(u) if save_new_value else None
    final_state = k.new_empty(N, H, K, V, dtype=final_state_dtype) if output_final_state else None
    op = ChunkGatedDeltaRuleFwdH(
        k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_size, h, v_new, final_state,
        chunk_offsets=chunk_offsets, layout="token_major", numerics=numerics, **plan_options)
    _launch(op, k.device, check_device_status)
    return h, v_new, final_state


def run(k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_size=CHUNK_SIZE, *,
        check_device_status: bool = False, **plan_options):
    """The contest reference signature (docs/problem.txt:81): head-major layout.

    k ``[B,T,HK,K]``, w ``[B,HV,T,K]``, u ``[B,HV,T,V]``, g ``[B,HV,T]``,
    initial_state ``[N,HV,K,V]``; returns h ``[B,HV,NT,K,V]``, v
    ``[B,HV,T,V]`` and final_state ``[N,HV,K,V]``, all bf16, computed with the
    reference's rounding chain.  Fixed-length batches (cu_seqlens None) treat
    every batch row as its own sequence.
    """
    _require_cuda(k, w, u, g, initial_state, cu_seqlens, chunk_indices)
    B, T, HK, K = k.shape
    HV, V = u.shape[1], u.shape[3]
    if cu_seqlens is None:
        N, NT = B, (T + chunk_size - 1) // chunk_size
    else:
        N, NT = cu_seqlens.numel() - 1, chunk_indices.shape[0]
    h = k.new_empty(B, HV, NT, K, V)
    v = torch.empty((B, HV, T, V), dtype=u.dtype, device=u.device)
    final_state = torch.empty((N, HV, K, V), dtype=u.dtype, device=u.device)
    op = ChunkGatedDeltaRuleFwdH(k, w, u, g, initial_state, cu_seqlens, chunk_indices, chunk_size, h, v,
                                 final_state, layout="head_major", numerics="reference", **plan_options)
    _launch(op, k.device, check_device_status)
    return h, v, final_state
