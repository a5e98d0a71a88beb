"""Host-memory front end of the recurrence: inputs and outputs in (pinned) CPU
memory, the copies overlapped with the kernels.

A caller whose tensors live in host memory would otherwise copy every input to
the device, run the op and copy every output back, one after the other: on the
north-star workload that is 0.82 GB in and 0.81 GB out around a 0.27 ms
kernel, so the PCIe copies are the whole cost.  PCIe carries both directions at
once, so this front end pipelines pieces of the batch: each sequence (a batch
row, or a sequence of a packed varlen batch), split along T at chunk boundaries
into ranges of about 48 MB of input, a range continuing from the previous
range's final state.  Piece i+1 is
copied in on one stream while piece i computes on a second stream and piece i-1
is copied out on a third. Two device slots per tensor are
recycled, and each stream waits on CUDA events. The caller's current stream
waits on all of it before the function returns, so the outputs are ready for
work queued on that stream, and a synchronize makes them ready on the host.

The kernels are the same as chunk_gated_delta_rule_fwd_h's, piece by piece (a
row is an independent problem: its own sequence, initial and final state; a
range of chunks starts from the state the kernel carries across the chunk
boundary, fp32, or bf16-valued in the reference arithmetic, which fp32 holds
exactly), so the outputs are bit-identical to the device API's.
"""

from __future__ import annotations

import torch

from .api import CHUNK_SIZE, ChunkGatedDeltaRuleFwdH

_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream, torch.cuda.Stream]] = {}
# input bytes per pipelined piece: small enough that filling and draining the
# pipeline costs little, large enough that a piece's kernel launch is negligible
_PIECE_BYTES = 48 << 20


def _streams(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        _STREAMS[idx] = tuple(torch.cuda.Stream(device=idx) for _ in range(3))
    return _STREAMS[idx]


def plan_pieces(seqs, tok_bytes: int, piece_bytes: int):
    """Pipeline pieces of the problems ``seqs`` = [(batch row, first token, tokens,
    first chunk in h, state row)]: each non-empty sequence split at chunk boundaries
    into balanced ranges of about ``piece_bytes`` of input (``tok_bytes`` per token).
    Returns [(batch row, first token, end token, first chunk in h, state row, first
    range of its sequence, last range of its sequence)]."""
    pieces = []
    for (b, a, L, c, n) in seqs:
        if L <= 0:
            continue
        nch = (L + CHUNK_SIZE - 1) // CHUNK_SIZE
        parts = max(1, min(nch, round(L * tok_bytes / piece_bytes)))
        per_s = (nch + parts - 1) // parts * CHUNK_SIZE  # tokens per range, balanced
        ranges = [(t0, min(L, t0 + per_s)) for t0 in range(0, L, per_s)]
        for j, (t0, t1) in enumerate(ranges):
            pieces.append((b, a + t0, a + t1, c + t0 // CHUNK_SIZE, n, j == 0, j == len(ranges) - 1))
    return pieces


def _host_empty(shape, dtype, pin: bool):
    return torch.empty(shape, dtype=dtype, pin_memory=pin)


def chunk_gated_delta_rule_fwd_h_host(
    k: torch.Tensor,
    w: torch.Tensor,
    u: torch.Tensor,
    g: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    cu_seqlens: torch.Tensor | None = None,
    *,
    device: torch.device | str = "cuda",
    save_new_value: bool = True,
    output_final_state: bool = True,
    numerics: str = "fp32_state",
    final_state_dtype: torch.dtype = torch.float32,
    out: tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None] | None = None,
    **plan_options,
) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """chunk_gated_delta_rule_fwd_h on host tensors.

    k ``[B,T,Hg,K]``, w ``[B,T,H,K]``, u ``[B,T,H,V]``, g ``[B,T,H]`` fp32 and
    initial_state ``[N,H,K,V]`` are CPU tensors with contiguous rows; they must
    be pinned for the copies to overlap (pageable memory still works, without
    overlap).  With ``cu_seqlens`` (a CPU int64 tensor ``[N+1]``, B = 1) the
    batch is packed varlen, as for chunk_gated_delta_rule_fwd_h.  Returns CPU
    tensors h ``[B,NT,H,K,V]`` (NT summed over the sequences when varlen),
    v_new ``[B,T,H,V]`` (``None`` if ``save_new_value`` is False) and
    final_state ``[N,H,K,V]`` (``None`` if ``output_final_state`` is False),
    pinned, or written into ``out``.  The caller's current stream on ``device`` waits for the whole
    pipeline; synchronize it before reading the outputs on the host.
    ``plan_options`` (``v_tile``, ``force_kernel``, ...) pass through to
    :class:`ChunkGatedDeltaRuleFwdH`.
    """
    for t in (k, w, u, g, initial_state, cu_seqlens):
        if t is not None and t.is_cuda:
            raise ValueError("chunk_gated_delta_rule_fwd_h_host takes host (CPU) tensors")
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("device must be a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    B, T, _, K = k.shape
    H, V = u.shape[-2], u.shape[-1]
    # the problems: (batch row, first token, tokens, first chunk in h, state row)
    if cu_seqlens is None:
        NT = (T + CHUNK_SIZE - 1) // CHUNK_SIZE
        seqs = [(b, 0, T, 0, b) for b in range(B)]
    else:
        if B != 1:
            raise ValueError("a varlen batch (cu_seqlens) has B = 1")
        cu = [int(x) for x in cu_seqlens.tolist()]
        if len(cu) < 2 or cu[0] != 0 or cu[-1] != T or any(b < a for a, b in zip(cu, cu[1:])):
            raise ValueError("cu_seqlens must rise from 0 to T")
        seqs, c = [], 0
        for n, (a, b) in enumerate(zip(cu, cu[1:])):
            seqs.append((0, a, b - a, c, n))
            c += (b - a + CHUNK_SIZE - 1) // CHUNK_SIZE
        NT = c
    N = len(seqs)
    pin = k.is_pinned()
    if out is None:
        h_out = _host_empty((B, NT, H, K, V), k.dtype, pin)
        v_out = _host_empty((B, T, H, V), u.dtype, pin) if save_new_value else None
        f_out = _host_empty((N, H, K, V), final_state_dtype, pin) if output_final_state else None
    else:
        h_out, v_out, f_out = out
    for t in [x for x in (k, w, u, g, h_out, v_out) if x is not None]:
        if t.shape[0] != B or not t[0].is_contiguous():
            raise ValueError("k, w, u, g, h and v_new need B rows of contiguous memory")
    for t in [x for x in (initial_state, f_out) if x is not None]:
        if t.shape[0] != N or not t[0].is_contiguous():
            raise ValueError("initial_state and final_state need one contiguous row per sequence")
    # an empty sequence's final state is its initial state, as the kernel loads it (the
    # reference arithmetic keeps the state in bf16)
    for (_, _, L, _, n) in seqs:
        if L == 0 and f_out is not None:
            if initial_state is None:
                f_out[n].zero_()
            elif numerics == "reference":
                f_out[n].copy_(initial_state[n].to(torch.bfloat16))
            else:
                f_out[n].copy_(initial_state[n])

    # pieces: the rows, each split along T at chunk boundaries into ranges of about
    # kPieceBytes of input; a range continues from the previous range's final state (the
    # fp32 state the kernel would carry across that chunk boundary)
    tok_bytes = sum(x[0, 0].numel() * x.element_size() for x in (k, w, u) + ((g,) if g is not None else ()))
    pieces = plan_pieces(seqs, tok_bytes, _PIECE_BYTES)
    if not pieces:
        return h_out, v_out, f_out
    per = max(t1 - t0 for (_, t0, t1, _, _, _, _) in pieces)
    per = (per + CHUNK_SIZE - 1) // CHUNK_SIZE * CHUNK_SIZE

    caller = torch.cuda.current_stream(dev)
    s_in, s_comp, s_out = _streams(dev)
    for s in (s_in, s_comp, s_out):
        s.wait_stream(caller)
    tin = [k, w, u] + ([g] if g is not None else [])       # split along T
    with torch.cuda.device(dev):
        # two device slots per tensor, one piece each (allocated on the caller's stream,
        # which waits for every use below before it can reuse them)
        def slot(x, rows):
            return torch.empty((1, rows) + tuple(x.shape[2:]), dtype=x.dtype, device=dev)
        n_per = per // CHUNK_SIZE
        slot_in = [[slot(x, per) for x in tin] for _ in range(2)]
        slot_h = [torch.empty((1, n_per, H, K, V), dtype=h_out.dtype, device=dev) for _ in range(2)]
        slot_v = [slot(v_out, per) if v_out is not None else None for _ in range(2)]
        h0_dev = [torch.empty((1, H, K, V), dtype=initial_state.dtype, device=dev) if initial_state is not None
                  else None for _ in range(2)]
        # the state between ranges (fp32) and the final state of each row
        carry = [torch.empty((1, H, K, V), dtype=torch.float32, device=dev) for _ in range(2)]
        fin_dtype = f_out.dtype if f_out is not None else torch.float32
        slot_f = [torch.empty((1, H, K, V), dtype=fin_dtype, device=dev) for _ in range(2)]
        copied_in = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]
        copied_out = [torch.cuda.Event() for _ in range(2)]
        for i, (b, t0, t1, c0, srow, first, last) in enumerate(pieces):
            s = i % 2
            n = t1 - t0
            c1 = c0 + (n + CHUNK_SIZE - 1) // CHUNK_SIZE
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(computed[s])  # piece i-2 has read this input slot
                for dst, src in zip(slot_in[s], tin):
                    dst[:, :n].copy_(src[b:b + 1, t0:t1], non_blocking=True)
                if first and initial_state is not None:
                    h0_dev[s].copy_(initial_state[srow:srow + 1], non_blocking=True)
                copied_in[s].record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(copied_in[s])
                if i >= 2:
                    s_comp.wait_event(copied_out[s])  # piece i-2's outputs have left this slot
                it = iter(slot_in[s])
                kd, wd, ud = (next(it)[:, :n] for _ in range(3))
                gd = next(it)[:, :n] if g is not None else None
                if first:
                    h0d = h0_dev[s]
                else:
                    h0d = carry[(i - 1) % 2]
                hd = slot_h[s][:, :c1 - c0]
                vd = slot_v[s][:, :n] if v_out is not None else None
                fd = slot_f[s] if last else carry[i % 2]
                if last and f_out is None:
                    fd = None
                op = ChunkGatedDeltaRuleFwdH(kd, wd, ud, gd, h0d, None, None, CHUNK_SIZE, hd, vd, fd,
                                             layout="token_major", numerics=numerics, **plan_options)
                ws = torch.empty(max(op.workspace_size, 256), dtype=torch.uint8, device=dev)
                op(ws, s_comp.cuda_stream)
                computed[s].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[s])
                h_out[b:b + 1, c0:c1].copy_(slot_h[s][:, :c1 - c0], non_blocking=True)
                if v_out is not None:
                    v_out[b:b + 1, t0:t1].copy_(slot_v[s][:, :n], non_blocking=True)
                if last and f_out is not None:
                    f_out[srow:srow + 1].copy_(slot_f[s], non_blocking=True)
                copied_out[s].record(s_out)
        caller.wait_stream(s_out)
        caller.wait_stream(s_comp)
        caller.wait_stream(s_in)
        # the slot tensors were used on the side streams (each workspace was allocated on
        # the compute stream itself)
        used = [x for row in slot_in for x in row] + slot_h + [x for x in slot_v + h0_dev if x is not None]
        for t in used + carry + slot_f:
            t.record_stream(s_in)
            t.record_stream(s_comp)
            t.record_stream(s_out)
    return h_out, v_out, f_out
