"""C-ABI surface on CPU (no kernel is launched): the library loads, exports
every symbol include/cgdr_fwd_h.h declares, and phase 1 validates and plans
exactly as the reference's host code does.

The accept/reject cases port the reference's InferShape unit tests
(code/tests/ut/op_host/test_chunk_gated_delta_rule_fwd_h_infershape.cpp:113-222)
and the plan checks port its tiling tests
(code/tests/ut/op_host/test_chunk_gated_delta_rule_fwd_h_tiling.cpp:39-162).
Phase 1 only reads shapes, strides and dtypes, so host tensors stand in for
device buffers here.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import cann_operator_challenge_august_b200 as cg
from cann_operator_challenge_august_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
BF, F32, I64 = torch.bfloat16, torch.float32, torch.int64


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    headers = sorted((ROOT / "include").glob("*.h"))
    assert {h.name for h in headers} == set(_lib.EXPORTS_BY_HEADER)
    for hdr in headers:
        declared = set(re.findall(r"^(?:cgdrStatus|void|int32_t|int64_t|const char\*)\s+(cgdr\w+)\(",
                                  hdr.read_text(), re.MULTILINE))
        expected = set(_lib.EXPORTS_BY_HEADER[hdr.name])
        assert declared == expected, (hdr.name, declared ^ expected)
        for sym in declared:
            assert hasattr(lib, sym), sym
    assert lib.cgdrGetAbiVersion() == 1


def e(shape, dtype=BF):
    return torch.empty(shape, dtype=dtype)


def varlen_case(with_state=True, with_final=True, chunk=64):
    """MakeVarlenCase of the reference UT: T=10016, N=2, NT=158, HV=8, HK=2, D=128."""
    d = dict(k=e((1, 10016, 2, 128)), w=e((1, 8, 10016, 128)), u=e((1, 8, 10016, 128)),
             g=e((1, 8, 10016), F32), initial_state=e((2, 8, 128, 128)) if with_state else None,
             cu_seqlens=e((3,), I64), chunk_indices=e((158, 2), I64), chunk_size=chunk,
             h=e((1, 8, 158, 128, 128)), v=e((1, 8, 10016, 128)),
             final_state=e((2, 8, 128, 128)) if with_final else None)
    return d


def fixed_case():
    """MakeFixedLengthCase: T=65, HV=4, HK=2, D=64."""
    return dict(k=e((1, 65, 2, 64)), w=e((1, 4, 65, 64)), u=e((1, 4, 65, 64)), g=e((1, 4, 65), F32),
                initial_state=e((1, 4, 64, 64)), cu_seqlens=None, chunk_indices=None, chunk_size=64,
                h=e((1, 4, 2, 64, 64)), v=e((1, 4, 65, 64)), final_state=e((1, 4, 64, 64)))


def phase1(d, strict=True, **kw):
    return cg.ChunkGatedDeltaRuleFwdH(d["k"], d["w"], d["u"], d["g"], d["initial_state"], d["cu_seqlens"],
                                      d["chunk_indices"], d["chunk_size"], d["h"], d["v"], d["final_state"],
                                      strict_reference_limits=strict, **kw)


def reject(d, status, strict=True, **kw):
    with pytest.raises(cg.CgdrValueError) as ei:
        phase1(d, strict=strict, **kw)
    assert ei.value.status_name == status, str(ei.value)


# ---- InferShape UT ports --------------------------------------------------------

def test_varlen_success():
    op = phase1(varlen_case())
    pl = op.plan
    assert (pl["batch"], pl["value_heads"], pl["chunk_count"], pl["key_dim"], pl["value_dim"]) == (1, 8, 158, 128, 128)
    assert pl["sequence_count"] == 2


def test_optional_initial_state_and_final_state():
    op = phase1(varlen_case(False, False))
    assert op.plan["has_initial_state"] == 0 and op.plan["store_final_state"] == 0


def test_fixed_length_success():
    op = phase1(fixed_case())
    assert op.plan["chunk_count"] == 2 and op.plan["sequence_count"] == 1


def test_rejects_invalid_batch():
    d = varlen_case()
    d["k"] = e((2, 10016, 2, 128))
    with pytest.raises(cg.CgdrValueError):
        phase1(d)


def test_rejects_invalid_rank():
    d = varlen_case()
    d["g"] = e((1, 8, 10016, 1), F32)
    reject(d, "BAD_RANK")


def test_rejects_mismatched_key_and_value_dimensions():
    d = varlen_case()
    d["u"] = e((1, 8, 10016, 64))
    with pytest.raises(cg.CgdrValueError):
        phase1(d)


def test_rejects_out_of_range_head_dimension():
    d = varlen_case()
    d["k"], d["w"], d["u"] = e((1, 10016, 2, 16)), e((1, 8, 10016, 16)), e((1, 8, 10016, 16))
    d["initial_state"] = e((2, 8, 16, 16))
    d["h"], d["v"], d["final_state"] = e((1, 8, 158, 16, 16)), e((1, 8, 10016, 16)), e((2, 8, 16, 16))
    reject(d, "BAD_SHAPE")
    # outside the reference's limits this build still accepts K = V = 16 (tensor cores,
    # K tile 64 with the columns past K zero-filled by the tensor maps)
    pl = phase1(d, strict=False).plan
    assert pl["kernel"] == 1 and pl["v_tile"] == 64 and pl["v_tile_count"] == 1


def test_rejects_non_divisible_head_ratio():
    d = varlen_case()
    d["w"], d["u"], d["g"] = e((1, 7, 10016, 128)), e((1, 7, 10016, 128)), e((1, 7, 10016), F32)
    d["initial_state"] = e((2, 7, 128, 128))
    d["h"], d["v"], d["final_state"] = e((1, 7, 158, 128, 128)), e((1, 7, 10016, 128)), e((2, 7, 128, 128))
    reject(d, "BAD_SHAPE")


def test_rejects_mismatched_token_dimension():
    d = varlen_case()
    d["w"] = e((1, 8, 10015, 128))
    reject(d, "BAD_SHAPE")


def test_rejects_invalid_initial_state():
    d = varlen_case()
    d["initial_state"] = e((1, 8, 128, 128))
    reject(d, "BAD_SHAPE")


def test_rejects_invalid_chunk_indices_shape():
    d = varlen_case()
    d["chunk_indices"] = e((158, 3), I64)
    reject(d, "BAD_VARLEN")


def test_rejects_impossible_chunk_count():
    d = varlen_case()
    d["chunk_indices"] = e((160, 2), I64)
    d["h"] = e((1, 8, 160, 128, 128))
    reject(d, "BAD_VARLEN")


def test_rejects_half_input():
    d = varlen_case()
    d["k"] = e((1, 10016, 2, 128), torch.float16)
    reject(d, "BAD_DTYPE")


def test_rejects_unsupported_chunk_size():
    reject(varlen_case(chunk=32), "BAD_CHUNK_SIZE")


def test_rejects_only_one_varlen_metadata_input():
    d = varlen_case()
    d["chunk_indices"] = None
    reject(d, "BAD_VARLEN")
    reject(d, "BAD_VARLEN", extended=False)


def test_strict_limits_reject_what_the_reference_rejects():
    d = varlen_case()
    d["cu_seqlens"] = e((6,), I64)  # five sequences > the reference's four
    d["initial_state"] = e((5, 8, 128, 128))
    d["final_state"] = e((5, 8, 128, 128))
    reject(d, "BAD_VARLEN")
    assert phase1(d, strict=False).plan["sequence_count"] == 5


# ---- tiling UT ports ------------------------------------------------------------

def test_plan_varlen_all_optional_paths():
    pl = phase1(varlen_case()).plan
    assert pl["plan_key"] == 7  # has_init | varlen<<1 | store_final<<2 (tiling.cpp:255-259)
    assert (pl["total_tokens"], pl["sequence_count"], pl["chunk_count"]) == (10016, 2, 158)
    assert (pl["value_heads"], pl["key_heads"], pl["head_ratio"]) == (8, 2, 4)
    assert pl["kernel"] == 1 and pl["v_tile"] in (32, 64, 128)
    # the reference arithmetic runs two chains per CTA where the tile is built for them
    assert pl["task_count"] == 2 * 8 * pl["v_tile_count"] * pl["chains"]
    assert pl["grid"] == 2 * 8 * pl["v_tile_count"]
    assert pl["workspace_bytes"] >= 256 + 4 * 3 + 4 * 2


def test_plan_fixed_length_without_optional_state_or_final():
    d = fixed_case()
    d["initial_state"] = None
    d["final_state"] = None
    pl = phase1(d).plan
    assert pl["plan_key"] == 0
    assert (pl["sequence_count"], pl["chunk_count"]) == (1, 2)
    assert pl["task_count"] == 4 * pl["v_tile_count"] * pl["chains"]
    assert pl["workspace_bytes"] == 256


def test_plan_rejects_half_present_varlen_metadata():
    d = dict(k=e((1, 64, 1, 64)), w=e((1, 1, 64, 64)), u=e((1, 1, 64, 64)), g=e((1, 1, 64), F32),
             initial_state=None, cu_seqlens=e((2,), I64), chunk_indices=None, chunk_size=64,
             h=e((1, 1, 1, 64, 64)), v=e((1, 1, 64, 64)), final_state=None)
    reject(d, "BAD_VARLEN", extended=False)


def test_plan_kernel_selection():
    """bf16 with K, V multiples of 8 and K <= 256 -> tensor cores; else general."""
    B, T, H = 4, 8192, 32
    k, w, u, g = e((B, T, H, 128)), e((B, T, H, 128)), e((B, T, H, 128)), e((B, T, H), F32)
    h, v, f = e((B, 128, H, 128, 128)), e((B, T, H, 128)), e((B, H, 128, 128), F32)
    op = cg.ChunkGatedDeltaRuleFwdH(k, w, u, g, None, None, None, 64, h, v, f, layout="token_major",
                                    numerics="fp32_state")
    pl = op.plan
    assert pl["kernel"] == 1 and pl["grid"] == pl["task_count"] == B * H * (128 // pl["v_tile"])
    # fp32 I/O -> general kernel
    k32, w32, u32 = e((1, 256, 2, 64), F32), e((1, 256, 2, 64), F32), e((1, 256, 2, 64), F32)
    op = cg.ChunkGatedDeltaRuleFwdH(k32, w32, u32, e((1, 256, 2), F32), None, None, None, 64,
                                    e((1, 4, 2, 64, 64), F32), e((1, 256, 2, 64), F32), e((1, 2, 64, 64), F32),
                                    layout="token_major", numerics="fp32_state")
    assert op.plan["kernel"] == 2
    # fp32 I/O is not the reference arithmetic
    with pytest.raises(cg.CgdrValueError):
        cg.ChunkGatedDeltaRuleFwdH(k32, w32, u32, e((1, 256, 2), F32), None, None, None, 64,
                                   e((1, 4, 2, 64, 64), F32), e((1, 256, 2, 64), F32), None,
                                   layout="token_major", numerics="reference")


@pytest.mark.parametrize("K,V,vt,tiles,block", [
    (32, 32, 64, 1, 192),     # K tile 64, one partial V tile
    (64, 96, 64, 2, 192),     # K tile 64, partial second V tile
    (96, 96, 32, 3, 192),     # K tile 128, 32-column tiles
    (128, 40, 32, 2, 192),    # V % 32 != 0: partial 32-column tile
    (256, 256, 64, 4, 320),   # K tile 256: two M = 128 halves of MMA2, 8 epilogue warps
    (200, 64, 64, 1, 320),
])
def test_plan_tensor_core_head_widths(K, V, vt, tiles, block):
    """The reference accepts 32 <= K == V <= 256 (infershape.cpp:214-219); every K, V
    that is a multiple of 8 up to 256 runs on the tensor cores, in a K tile of 64,
    128 or 256 and V tiles clipped at V."""
    B, T, H = 1, 200, 2
    op = cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, V)), e((B, T, H), F32), None,
                                    None, None, 64, e((B, 4, H, K, V)), e((B, T, H, V)), e((B, H, K, V), F32),
                                    layout="token_major", numerics="fp32_state")
    pl = op.plan
    assert pl["kernel"] == 1, pl
    assert (pl["v_tile"], pl["v_tile_count"], pl["block"]) == (vt, tiles, block)
    assert pl["task_count"] == B * H * tiles
    # widths that are not multiples of 8 stay on the general kernel
    if K == 32:
        op = cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, 36)), e((B, T, H, 36)), e((B, T, H, 36)), e((B, T, H), F32),
                                        None, None, None, 64, e((B, 4, H, 36, 36)), e((B, T, H, 36)),
                                        e((B, H, 36, 36), F32), layout="token_major", numerics="fp32_state")
        assert op.plan["kernel"] == 2


def test_plan_rejects_unbuilt_tile_choices():
    B, T, H = 1, 128, 2
    args = lambda K, V: (e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, V)), e((B, T, H), F32), None, None,  # noqa: E731
                         None, 64, e((B, 2, H, K, V)), e((B, T, H, V)), None)
    for K, vt in ((256, 128), (64, 32)):
        with pytest.raises(cg.CgdrError, match="UNSUPPORTED"):
            cg.ChunkGatedDeltaRuleFwdH(*args(K, K), layout="token_major", numerics="fp32_state", v_tile=vt)


def test_executor_lifecycle_and_errors():
    lib = _lib.load()
    op = phase1(fixed_case())
    ex = op._ex
    op._ex = None
    lib.cgdrDestroyExecutor(ex)
    st = lib.cgdrChunkGatedDeltaRuleFwdH(ctypes.c_void_p(1 << 20), 256, ctypes.c_void_p(0), ctypes.c_void_p(0))
    assert _lib.STATUS_NAMES[st] == "BAD_EXECUTOR"
    # a too-small workspace is refused before any device work
    op = phase1(varlen_case())
    ex = op._ex
    op._ex = None
    st = lib.cgdrChunkGatedDeltaRuleFwdH(ctypes.c_void_p(1 << 20), 16, ex, ctypes.c_void_p(0))
    assert _lib.STATUS_NAMES[st] == "WORKSPACE_TOO_SMALL"


def test_python_front_end_refuses_cpu_tensors():
    k = torch.zeros(1, 64, 1, 64, dtype=BF)
    with pytest.raises(ValueError, match="CUDA"):
        cg.chunk_gated_delta_rule_fwd_h(k, k, k, torch.zeros(1, 64, 1))


@pytest.mark.parametrize("B,H,K,V,expected", [
    (2, 16, 128, 128, 32),   # 32 pairs: 128 tasks of 32 columns fit one CTA per SM
    (1, 32, 128, 128, 32),
    (2, 32, 128, 128, 64),   # 64 pairs: 32-column tiles would need 256 CTAs
    (4, 32, 128, 128, 128),  # 128 pairs: 64-column tiles would put two CTAs on an SM
    (2, 16, 64, 64, 64),     # K = 64 runs 64- or 128-column tiles only
    (4, 32, 128, 96, 32),    # V % 64 != 0 (K = 128): 32-column tiles whatever the task count
])
def test_plan_v_tile_choice(B, H, K, V, expected):
    """The planner takes the narrowest V tile that keeps one CTA per SM (148 SMs),
    one chain per CTA for the fp32-state arithmetic and two for the reference
    arithmetic where the tile is built for them (32 and 128 columns, K tile 128)."""
    T = 256
    op = cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, V)), e((B, T, H), F32), None,
                                    None, None, 64, e((B, T // 64, H, K, V)), e((B, T, H, V)), e((B, H, K, V), F32),
                                    layout="token_major", numerics="fp32_state")
    assert (op.plan["v_tile"], op.plan["chains"]) == (expected, 1)
    op = cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, V)), e((B, T, H), F32), None,
                                    None, None, 64, e((B, T // 64, H, K, V)), e((B, T, H, V)), e((B, H, K, V), BF),
                                    layout="token_major", numerics="reference")
    assert (op.plan["v_tile"], op.plan["chains"]) == (expected, 2 if K == 128 and expected in (32, 128) else 1)


@pytest.mark.parametrize("K,vt,chains", [(64, 32, 0), (64, 32, 2), (64, 128, 2), (128, 64, 2), (256, 64, 2),
                                         (128, 128, 3)])
def test_plan_rejects_unbuilt_tile_and_chain_choices(K, vt, chains):
    B, T, H = 1, 128, 2
    with pytest.raises(cg.CgdrError) as ei:
        cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, K)), e((B, T, H), F32), None,
                                   None, None, 64, e((B, 2, H, K, K)), e((B, T, H, K)), None,
                                   layout="token_major", numerics="fp32_state", v_tile=vt, chains=chains)
    assert ei.value.status_name == "UNSUPPORTED"


@pytest.mark.parametrize("vt,V", [(32, 128), (32, 48), (128, 256), (128, 192)])
def test_plan_two_chains_per_cta(vt, V):
    """chains 2: each V tile's two column halves are chains of their own in one CTA
    (eight epilogue warps, a producer and one MMA issuer per chain); task_count
    counts chains, grid CTAs."""
    B, T, H, K = 2, 256, 4, 128
    op = cg.ChunkGatedDeltaRuleFwdH(e((B, T, H, K)), e((B, T, H, K)), e((B, T, H, V)), e((B, T, H), F32), None,
                                    None, None, 64, e((B, T // 64, H, K, V)), e((B, T, H, V)), e((B, H, K, V), F32),
                                    layout="token_major", numerics="fp32_state", v_tile=vt, chains=2)
    pl = op.plan
    assert (pl["kernel"], pl["v_tile"], pl["chains"], pl["block"]) == (1, vt, 2, 32 * 11)
    assert pl["v_tile_count"] == (V + vt - 1) // vt and pl["grid"] == B * H * pl["v_tile_count"]
    assert pl["task_count"] == 2 * pl["grid"]


# ---- host-memory front end: the pipeline's pieces (pure host logic) -------------

def test_host_pieces_cover_every_chunk_once():
    from cann_operator_challenge_august_b200.host import plan_pieces
    # a packed varlen batch: empty, one-token, ragged and long sequences
    lens = [0, 1, 300, 0, 4096, 63, 65]
    seqs, a, c = [], 0, 0
    for n, L in enumerate(lens):
        seqs.append((0, a, L, c, n))
        a += L
        c += (L + 63) // 64
    for piece_bytes in (1 << 10, 1 << 16, 1 << 30):
        pieces = plan_pieces(seqs, tok_bytes=1000, piece_bytes=piece_bytes)
        tokens = sorted((t0, t1) for (_, t0, t1, *_rest) in pieces)
        covered = [t for (t0, t1) in tokens for t in range(t0, t1)]
        assert covered == list(range(sum(lens)))  # every token once, in order
        for (b, t0, t1, c0, n, first, last) in pieces:
            s0 = seqs[n][1]
            assert (t0 - s0) % 64 == 0 and c0 == seqs[n][3] + (t0 - s0) // 64  # chunk-aligned starts
        for n, L in enumerate(lens):
            mine = [p for p in pieces if p[4] == n]
            assert len(mine) == (0 if L == 0 else len(mine))
            if L:
                assert mine[0][5] and mine[-1][6] and sum(p[5] for p in mine) == 1 and sum(p[6] for p in mine) == 1


def test_host_pieces_are_balanced():
    from cann_operator_challenge_august_b200.host import plan_pieces
    # one 8192-token row at ~24.7 KB per token: four ranges of 2048 tokens
    pieces = plan_pieces([(0, 0, 8192, 0, 0)], tok_bytes=24704, piece_bytes=48 << 20)
    assert [(t0, t1) for (_, t0, t1, *_r) in pieces] == [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192)]
