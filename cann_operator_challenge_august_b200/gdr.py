"""Python front ends of the stages around the hidden-state recurrence, over
the C ABI in include/cgdr_chunk_o.h and include/cgdr_wy.h.

* :class:`ChunkGatedDeltaRuleFwdO` -- two-phase call of the chunk output
  (workspace query, then launch into a caller-owned ``o``).
* :func:`chunk_fwd_o` -- allocate-and-call form with the argument set of the
  fla ``chunk_fwd_o`` wrapper.
* :class:`ChunkGatedDeltaRuleWY` / :func:`chunk_wy_fwd` -- the WY
  representation that produces the recurrence's w, u and chunk-local
  cumulative gate from k, v, beta and the per-token gate (the reference's
  stage 1, ref/chunk_gated_delta_rule/tests/pytest/
  chunk_gated_delta_rule_benchmark.py:55-83).
* :class:`ChunkGatedDeltaRule` / :func:`chunk_gated_delta_rule` -- the whole
  chunked Gated DeltaNet forward (WY, recurrence, chunk output) with the
  arguments of the reference's operator: aclnnChunkGatedDeltaRule
  (ref/chunk_gated_delta_rule/op_host/op_api/aclnn_chunk_gated_delta_rule.cpp:125)
  and its torch_npu form npu_chunk_gated_delta_rule (argument order of
  ref/chunk_gated_delta_rule/tests/assets/impl/golden.py:88-94).

The chunk output is the consumer of ``chunk_gated_delta_rule_fwd_h``'s ``h``
and ``v_new``: per 64-token chunk, ``o = q' h[c] + P v_new`` with
``q' = bf16(q * scale * exp(g))`` and ``P = bf16(bf16(q k^T) * scale *
exp(g_i - g_j))`` on and below the diagonal (the reference's stage 2
inter-chunk term and stage 3, ref/chunk_gated_delta_rule/tests/pytest/
chunk_gated_delta_rule_benchmark.py:77-79, :129, :145-175).

Nothing here computes on the CPU: the CUDA library does the work and raises
if it is missing.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .api import CHUNK_SIZE, _desc, _require_cuda, _stream_handle, prepare_chunk_indices, read_device_status


class ChunkGatedDeltaRuleFwdO:
    """Two-phase chunk output: ``op = ChunkGatedDeltaRuleFwdO(q, k, v_new, h,
    g, cu_seqlens, chunk_indices, scale, chunk_size, o)`` validates and plans;
    ``op(workspace)`` enqueues the kernel on the current stream.  Launched at
    most once."""

    def __init__(self, q, k, v_new, h, g, cu_seqlens, chunk_indices, scale, chunk_size, o, *, wait_timeout_ms=0):
        lib = _lib.load()
        self._keep = (q, k, v_new, h, g, cu_seqlens, chunk_indices, o)
        ws = ctypes.c_uint64(0)
        ex = ctypes.c_void_p(None)
        opt = _lib.CgdrChunkOOptions(wait_timeout_ms=int(wait_timeout_ms))
        descs = [_desc(x) for x in (q, k, v_new, h, g, cu_seqlens, chunk_indices)]
        st = lib.cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize(
            *[ctypes.byref(d) for d in descs], float(scale if scale is not None else 0.0), int(chunk_size),
            ctypes.byref(_desc(o)), ctypes.byref(opt), ctypes.byref(ws), ctypes.byref(ex))
        _lib.check(st, "cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize")
        self._ex = ex
        self.workspace_size = int(ws.value)

    @property
    def grid(self) -> int:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        return int(_lib.load().cgdrChunkOGridSize(self._ex))

    def __call__(self, workspace: torch.Tensor, stream: int | None = None) -> None:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        ex, self._ex = self._ex, None
        if stream is None:
            stream = _stream_handle(workspace.device)
        st = _lib.load().cgdrChunkGatedDeltaRuleFwdO(
            ctypes.c_void_p(workspace.data_ptr()), workspace.numel() * workspace.element_size(), ex,
            ctypes.c_void_p(stream))
        _lib.check(st, "cgdrChunkGatedDeltaRuleFwdO")

    def __del__(self):
        if getattr(self, "_ex", None) is not None and _lib._lib is not None:
            _lib._lib.cgdrDestroyChunkOExecutor(self._ex)
            self._ex = None


def chunk_fwd_o(
    q: torch.Tensor,
    k: torch.Tensor,
    v_new: torch.Tensor,
    h: torch.Tensor,
    g: torch.Tensor | None = None,
    scale: float | None = None,
    cu_seqlens: torch.LongTensor | None = None,
    chunk_size: int = CHUNK_SIZE,
    chunk_indices: torch.Tensor | None = None,
    *,
    check_device_status: bool = False,
) -> torch.Tensor:
    """Chunk output ``o [B,T,H,V]`` (bf16) from q, k ``[B,T,Hg,K]``, v_new
    ``[B,T,H,V]``, h ``[B,NT,H,K,V]`` and the chunk-local cumulative gate g
    ``[B,T,H]``.  ``scale`` defaults to ``K ** -0.5``.  With cu_seqlens and no
    chunk_indices the chunk list is derived on the host (one sync)."""
    _require_cuda(q, k, v_new, h, g, cu_seqlens, chunk_indices)
    if cu_seqlens is not None and chunk_indices is None:
        chunk_indices = prepare_chunk_indices(cu_seqlens, chunk_size)
    o = torch.empty_like(v_new)
    op = ChunkGatedDeltaRuleFwdO(q, k, v_new, h, g, cu_seqlens, chunk_indices, scale, chunk_size, o)
    ws = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=q.device)
    op(ws)
    if check_device_status:
        status = read_device_status(ws)
        if status:
            raise RuntimeError(f"device status 0x{status:x}")
    return o


class ChunkGatedDeltaRuleWY:
    """Two-phase WY representation: ``op = ChunkGatedDeltaRuleWY(k, v, beta,
    g, cu_seqlens, chunk_indices, chunk_size, w, u, g_cum)`` validates and
    plans; ``op(workspace)`` enqueues the kernel on the current stream."""

    def __init__(self, k, v, beta, g, cu_seqlens, chunk_indices, chunk_size, w, u, g_cum, *, wait_timeout_ms=0):
        lib = _lib.load()
        self._keep = (k, v, beta, g, cu_seqlens, chunk_indices, w, u, g_cum)
        ws = ctypes.c_uint64(0)
        ex = ctypes.c_void_p(None)
        opt = _lib.CgdrWyOptions(wait_timeout_ms=int(wait_timeout_ms))
        descs = [_desc(x) for x in (k, v, beta, g, cu_seqlens, chunk_indices)]
        outs = [_desc(x) for x in (w, u, g_cum)]
        st = lib.cgdrChunkGatedDeltaRuleWYGetWorkspaceSize(
            *[ctypes.byref(d) for d in descs], int(chunk_size), *[ctypes.byref(d) for d in outs], ctypes.byref(opt),
            ctypes.byref(ws), ctypes.byref(ex))
        _lib.check(st, "cgdrChunkGatedDeltaRuleWYGetWorkspaceSize")
        self._ex = ex
        self.workspace_size = int(ws.value)

    def __call__(self, workspace: torch.Tensor, stream: int | None = None) -> None:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        ex, self._ex = self._ex, None
        if stream is None:
            stream = _stream_handle(workspace.device)
        st = _lib.load().cgdrChunkGatedDeltaRuleWY(
            ctypes.c_void_p(workspace.data_ptr()), workspace.numel() * workspace.element_size(), ex,
            ctypes.c_void_p(stream))
        _lib.check(st, "cgdrChunkGatedDeltaRuleWY")

    def __del__(self):
        if getattr(self, "_ex", None) is not None and _lib._lib is not None:
            _lib._lib.cgdrDestroyWyExecutor(self._ex)
            self._ex = None


def chunk_wy_fwd(
    k: torch.Tensor,
    v: torch.Tensor,
    beta: torch.Tensor,
    g: torch.Tensor | None = None,
    cu_seqlens: torch.LongTensor | None = None,
    chunk_size: int = CHUNK_SIZE,
    chunk_indices: torch.Tensor | None = None,
    *,
    check_device_status: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """WY representation: returns ``(w [B,T,H,K], u [B,T,H,V], g_cum [B,T,H])``
    from k ``[B,T,Hg,K]``, v ``[B,T,H,V]``, beta ``[B,T,H]`` (bf16) and the
    per-token log gate g ``[B,T,H]`` (fp32, optional).  ``g_cum`` is the
    chunk-local cumulative gate that the recurrence and the chunk output take
    as their ``g``."""
    _require_cuda(k, v, beta, g, cu_seqlens, chunk_indices)
    if cu_seqlens is not None and chunk_indices is None:
        chunk_indices = prepare_chunk_indices(cu_seqlens, chunk_size)
    B, T, H = v.shape[0], v.shape[1], v.shape[2]
    w = k.new_empty(B, T, H, k.shape[3])
    u = torch.empty_like(v)
    g_cum = torch.empty(B, T, H, dtype=torch.float32, device=v.device)
    op = ChunkGatedDeltaRuleWY(k, v, beta, g, cu_seqlens, chunk_indices, chunk_size, w, u, g_cum)
    ws = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=v.device)
    op(ws)
    if check_device_status:
        status = read_device_status(ws)
        if status:
            raise RuntimeError(f"device status 0x{status:x}")
    return w, u, g_cum


class ChunkGatedDeltaRule:
    """Two-phase call of the whole operator, the aclnnChunkGatedDeltaRule
    pattern: ``op = ChunkGatedDeltaRule(query, key, value, beta,
    initial_state, actual_seq_lengths, g, scale, out, final_state)``
    validates (the reference's checks) and sizes the workspace;
    ``op(workspace)`` enqueues the metadata, WY, recurrence and chunk-output
    kernels on the current stream.  ``path`` selects the recurrence and
    output kernels: ``"fused"`` (one kernel; h and v_new stay on chip),
    ``"three_kernels"`` (recurrence then chunk output) or ``"auto"``."""

    def __init__(self, query, key, value, beta, initial_state, actual_seq_lengths, g, scale, out, final_state,
                 *, path: str = "auto"):
        lib = _lib.load()
        self._keep = (query, key, value, beta, initial_state, actual_seq_lengths, g, out, final_state)
        ws = ctypes.c_uint64(0)
        ex = ctypes.c_void_p(None)
        descs = [_desc(x) for x in (query, key, value, beta, initial_state, actual_seq_lengths, g)]
        if path not in _lib.GDR_PATHS:
            raise ValueError(f"path must be one of {sorted(_lib.GDR_PATHS)}")
        opt = _lib.CgdrGdrOptions(path=_lib.GDR_PATHS[path])
        st = lib.cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx(
            *[ctypes.byref(d) for d in descs], float(scale if scale is not None else 0.0), ctypes.byref(_desc(out)),
            ctypes.byref(_desc(final_state)), ctypes.byref(opt), ctypes.byref(ws), ctypes.byref(ex))
        _lib.check(st, "cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx")
        self._ex = ex
        self.workspace_size = int(ws.value)

    @property
    def path(self) -> str:
        """``"fused"`` or ``"three_kernels"``: the kernels this plan runs."""
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        out = ctypes.c_int32(0)
        _lib.check(_lib.load().cgdrGetGdrPath(self._ex, ctypes.byref(out)), "cgdrGetGdrPath")
        return {v: k for k, v in _lib.GDR_PATHS.items()}[int(out.value)]

    def __call__(self, workspace: torch.Tensor, stream: int | None = None) -> None:
        if self._ex is None:
            raise RuntimeError("executor already consumed")
        ex, self._ex = self._ex, None
        if stream is None:
            stream = _stream_handle(workspace.device)
        st = _lib.load().cgdrChunkGatedDeltaRule(
            ctypes.c_void_p(workspace.data_ptr()), workspace.numel() * workspace.element_size(), ex,
            ctypes.c_void_p(stream))
        _lib.check(st, "cgdrChunkGatedDeltaRule")

    def __del__(self):
        if getattr(self, "_ex", None) is not None and _lib._lib is not None:
            _lib._lib.cgdrDestroyGdrExecutor(self._ex)
            self._ex = None


def chunk_gated_delta_rule(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    beta: torch.Tensor,
    initial_state: torch.Tensor,
    actual_seq_lengths: torch.Tensor,
    scale: float | None = None,
    g: torch.Tensor | None = None,
    *,
    workspace: torch.Tensor | None = None,
    check_device_status: bool = False,
    path: str = "auto",
) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference operator's Python form (torch_npu.npu_chunk_gated_delta_rule):
    query, key ``[T, Nk, Dk]``, value ``[T, Nv, Dv]``, beta ``[T, Nv]`` (bf16),
    initial_state ``[B, Nv, Dv, Dk]`` (bf16 or fp32), actual_seq_lengths
    ``[B]`` int32 (summing to T), scale (default ``Dk ** -0.5``), g ``[T, Nv]``
    fp32 per-token log gate (optional).  Returns ``out [T, Nv, Dv]`` (bf16)
    and ``final_state`` (the dtype of initial_state).  ``workspace`` may be a
    caller-owned uint8 buffer of at least the planned size.  ``path``: see
    :class:`ChunkGatedDeltaRule`."""
    _require_cuda(query, key, value, beta, initial_state, actual_seq_lengths, g)
    out = torch.empty_like(value)
    final_state = torch.empty_like(initial_state)
    op = ChunkGatedDeltaRule(query, key, value, beta, initial_state, actual_seq_lengths, g, scale, out, final_state,
                             path=path)
    if workspace is None or workspace.numel() * workspace.element_size() < op.workspace_size:
        workspace = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=value.device)
    op(workspace)
    if check_device_status:
        status = read_device_status(workspace)
        if status:
            raise RuntimeError(f"device status 0x{status:x}")
    return out, final_state
