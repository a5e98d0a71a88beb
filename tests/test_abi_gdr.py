"""Phase 1 of the composed operator (include/cgdr_gdr.h) on CPU: the argument
checks of the reference's aclnnChunkGatedDeltaRule.  The cases port the
reference's tiling unit tests
(ref/chunk_gated_delta_rule/tests/ut/op_host/test_chunk_gated_delta_rule_tiling.cpp:70-842)
and its ACLNN dtype checks (op_host/op_api/aclnn_chunk_gated_delta_rule.cpp:54-95).
Phase 1 only reads shapes, strides and dtypes, so host tensors stand in for
device buffers; no kernel is launched.
"""

from __future__ import annotations

import pytest
import torch

import cann_operator_challenge_august_b200 as cg

BF, F32, F16, I32, I64 = torch.bfloat16, torch.float32, torch.float16, torch.int32, torch.int64


def case(bs, seq_len, nk, nv, dk, dv, *, state=BF, with_g=True, out_dtype=BF, fin_dtype=None, asl=I32, g_dtype=F32):
    t = bs * seq_len
    fin_dtype = state if fin_dtype is None else fin_dtype
    return dict(query=torch.empty(t, nk, dk, dtype=BF), key=torch.empty(t, nk, dk, dtype=BF),
                value=torch.empty(t, nv, dv, dtype=BF), beta=torch.empty(t, nv, dtype=BF),
                initial_state=torch.empty(bs, nv, dv, dk, dtype=state),
                actual_seq_lengths=torch.empty(bs, dtype=asl),
                g=torch.empty(t, nv, dtype=g_dtype) if with_g else None, scale=None,
                out=torch.empty(t, nv, dv, dtype=out_dtype), final_state=torch.empty(bs, nv, dv, dk, dtype=fin_dtype))


def plan(d):
    return cg.ChunkGatedDeltaRule(d["query"], d["key"], d["value"], d["beta"], d["initial_state"],
                                  d["actual_seq_lengths"], d["g"], d["scale"], d["out"], d["final_state"])


def rejected(d, status):
    with pytest.raises(cg.CgdrError) as ei:
        plan(d)
    assert ei.value.status_name == status, str(ei.value)


@pytest.mark.parametrize("name,args,kw", [
    ("BasicWithGamma", (2, 100, 4, 8, 128, 128), {}),
    ("BasicWithoutGamma", (2, 100, 4, 8, 128, 128), dict(with_g=False)),
    ("BasicFp32StateWithoutGamma", (2, 100, 4, 8, 128, 128), dict(state=F32, with_g=False)),
    ("BasicFp32StateWithGamma", (2, 100, 4, 8, 128, 128), dict(state=F32)),
    ("SingleBatch", (1, 64, 4, 4, 64, 64), {}),
    ("MaxBatch8", (8, 32, 4, 4, 64, 64), {}),
    ("GQA_2x", (2, 64, 4, 8, 64, 64), {}),
    ("GQA_4x", (2, 64, 2, 8, 64, 64), {}),
    ("Dim128", (2, 64, 4, 4, 128, 128), {}),
    ("DifferentDKDV", (2, 64, 4, 4, 64, 128), {}),
    ("ScaleInvSqrt", (2, 64, 4, 4, 64, 64), {}),
    ("MaxHeads48", (2, 64, 48, 48, 32, 32), {}),
])
def test_accepts_the_reference_valid_cases(name, args, kw):
    op = plan(case(*args, **kw))
    bs, seq_len, nk, nv, dk, dv = args
    t = bs * seq_len
    nt_max = (t + 63) // 64 + bs - 1
    # the workspace holds g_c, w, u, v_new and one state per chunk slot
    assert op.workspace_size >= 2 * nt_max * nv * dk * dv + 2 * t * nv * (dk + 2 * dv) + 4 * t * nv


@pytest.mark.parametrize("dk,dv", [(32, 32), (96, 48), (128, 80), (1, 128)])
def test_head_dims_outside_64_128_are_padded(dk, dv):
    """MaxHeads48 (dk = dv = 32) and other widths the reference accepts run
    through zero-padded copies at the next of 64 / 128; the workspace holds
    them."""
    bs, seq_len, nk, nv = 2, 64, 4, 8
    op = plan(case(bs, seq_len, nk, nv, dk, dv))
    t = bs * seq_len
    kp, vp = (64 if dk <= 64 else 128), (64 if dv <= 64 else 128)
    nt_max = (t + 63) // 64 + bs - 1
    padded = 2 * 2 * t * nk * kp * (kp != dk) + 2 * 2 * t * nv * vp * (vp != dv) + 2 * 4 * bs * nv * kp * vp
    assert op.workspace_size >= 2 * nt_max * nv * kp * vp + 2 * t * nv * (kp + 2 * vp) + padded


@pytest.mark.parametrize("nk,nv", [(4, 3), (4, 5), (8, 7)])
def test_rejects_nv_not_multiple_of_nk(nk, nv):
    rejected(case(2, 64, nk, nv, 64, 64), "BAD_SHAPE")


def test_rejects_fp16_out():
    rejected(case(2, 64, 4, 8, 64, 64, out_dtype=F16), "BAD_DTYPE")


def test_rejects_fp16_final_state():
    rejected(case(2, 64, 4, 8, 64, 64, fin_dtype=F16), "BAD_DTYPE")


def test_rejects_int64_actual_seq_lengths():
    rejected(case(2, 64, 4, 8, 64, 64, asl=I64), "BAD_DTYPE")


def test_rejects_bf16_gamma():
    rejected(case(2, 64, 4, 8, 64, 64, g_dtype=BF), "BAD_DTYPE")


def test_rejects_query_rank_2():
    d = case(2, 64, 4, 8, 64, 64)
    d["query"] = torch.empty(128, 4 * 64, dtype=BF)
    rejected(d, "BAD_RANK")


def test_rejects_query_key_head_mismatch():
    d = case(2, 64, 4, 8, 64, 64)
    d["key"] = torch.empty(128, 2, 64, dtype=BF)
    rejected(d, "BAD_SHAPE")


def test_rejects_final_state_with_t_instead_of_b():
    d = case(2, 64, 4, 8, 64, 64)
    d["final_state"] = torch.empty(128, 8, 64, 64, dtype=BF)
    rejected(d, "BAD_SHAPE")


def test_rejects_more_than_64_heads_and_dims_above_128():
    rejected(case(1, 64, 80, 80, 64, 64), "BAD_SHAPE")
    rejected(case(1, 64, 4, 4, 64, 256), "BAD_SHAPE")


def test_requires_every_tensor_but_g():
    d = case(2, 64, 4, 8, 64, 64)
    d["beta"] = None
    rejected(d, "NULL_ARGUMENT")


# ---------------------------------------------------------------- recurrence + output path

def plan_path(d, path):
    return cg.ChunkGatedDeltaRule(d["query"], d["key"], d["value"], d["beta"], d["initial_state"],
                                  d["actual_seq_lengths"], d["g"], d["scale"], d["out"], d["final_state"], path=path)


@pytest.mark.parametrize("args,expected", [
    ((8, 64, 4, 16, 128, 128), "fused"),          # B * Nv = 128 >= 74, Dk = 128
    ((2, 64, 16, 64, 96, 64), "fused"),           # Dk 96 runs padded to 128
    ((2, 64, 4, 8, 128, 128), "three_kernels"),   # B * Nv = 16: too few tasks
    ((8, 64, 4, 16, 64, 128), "three_kernels"),   # Dk = 64: the fused kernel runs K = 128 only
])
def test_auto_path(args, expected):
    assert plan_path(case(*args), "auto").path == expected


def test_fused_workspace_has_no_states():
    """The fused plan keeps h and v_new on chip: its workspace is smaller than
    the three-kernel plan's by the per-chunk states and v_new."""
    bs, seq_len, nk, nv, dk, dv = 8, 64, 4, 16, 128, 128
    d = case(bs, seq_len, nk, nv, dk, dv)
    fused, three = plan_path(d, "fused"), plan_path(d, "three_kernels")
    assert (fused.path, three.path) == ("fused", "three_kernels")
    t = bs * seq_len
    nt_max = (t + 63) // 64 + bs - 1
    assert fused.workspace_size < 2 * nt_max * nv * dk * dv
    assert three.workspace_size - fused.workspace_size >= 2 * nt_max * nv * dk * dv + 2 * t * nv * dv


def test_forced_fused_path_on_small_batches():
    assert plan_path(case(1, 64, 4, 4, 128, 64), "fused").path == "fused"


def test_fused_path_rejects_dk_64():
    with pytest.raises(cg.CgdrError) as ei:
        plan_path(case(2, 64, 4, 4, 64, 64), "fused")
    assert ei.value.status_name == "UNSUPPORTED"


def test_unknown_path_name():
    with pytest.raises(ValueError):
        plan_path(case(2, 64, 4, 4, 64, 64), "two_kernels")
