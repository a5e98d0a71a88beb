"""ctypes binding of the C ABI in include/*.h.

The shared library is built in-tree (``python -m
cann_operator_challenge_august_b200.build``).  There is no fallback: if the
library is missing or cannot be loaded, every entry point raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcgdr_fwd_h.so"

MAX_DIMS = 8

# cgdrStatus
STATUS_NAMES = {
    0: "SUCCESS", 1: "NULL_ARGUMENT", 2: "BAD_RANK", 3: "BAD_DTYPE", 4: "BAD_SHAPE",
    5: "BAD_CHUNK_SIZE", 6: "BAD_VARLEN", 7: "BAD_STRIDE", 8: "UNSUPPORTED",
    9: "WORKSPACE_TOO_SMALL", 10: "CUDA_ERROR", 11: "DEVICE_ERROR", 12: "BAD_EXECUTOR",
}
STATUS = {v: k for k, v in STATUS_NAMES.items()}

# cgdrDataType
DT_BF16, DT_FLOAT32, DT_FLOAT16, DT_INT64, DT_INT32 = 1, 2, 3, 4, 5
LAYOUT_HEAD_MAJOR, LAYOUT_TOKEN_MAJOR = 0, 1
NUMERICS = {"reference": 0, "fp32_state": 1}

NOALLOC_SCRATCH_BYTES = 65536  # CGDR_NOALLOC_SCRATCH_BYTES

DEVICE_WAIT_TIMEOUT = 0x1
DEVICE_BAD_VARLEN = 0x2

# Every symbol declared in include/*.h, by header.
EXPORTS_BY_HEADER = {
    "cgdr_fwd_h.h": (
        "cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize",
        "cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx",
        "cgdrChunkGatedDeltaRuleFwdH",
        "cgdrChunkGatedDeltaRuleFwdHNoAlloc",
        "cgdrDestroyExecutor",
        "cgdrGetPlan",
        "cgdrReadDeviceStatus",
        "cgdrGetLastErrorMessage",
        "cgdrGetAbiVersion",
    ),
    "cgdr_chunk_o.h": (
        "cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize",
        "cgdrChunkGatedDeltaRuleFwdO",
        "cgdrDestroyChunkOExecutor",
        "cgdrChunkOGridSize",
    ),
    "cgdr_wy.h": (
        "cgdrChunkGatedDeltaRuleWYGetWorkspaceSize",
        "cgdrChunkGatedDeltaRuleWY",
        "cgdrDestroyWyExecutor",
    ),
    "cgdr_varlen.h": ("cgdrPrepareChunkIndices",),
    "cgdr_gdr.h": (
        "cgdrChunkGatedDeltaRuleGetWorkspaceSize",
        "cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx",
        "cgdrGetGdrPath",
        "cgdrChunkGatedDeltaRule",
        "cgdrDestroyGdrExecutor",
    ),
}
EXPORTS = tuple(sym for syms in EXPORTS_BY_HEADER.values() for sym in syms)


class CgdrTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("strides", ctypes.c_int64 * MAX_DIMS),
    ]


class CgdrFwdHOptions(ctypes.Structure):
    _fields_ = [
        ("layout", ctypes.c_int32),
        ("numerics", ctypes.c_int32),
        ("strict_reference_limits", ctypes.c_int32),
        ("force_kernel", ctypes.c_int32),
        ("v_tile", ctypes.c_int32),
        ("wait_timeout_ms", ctypes.c_int32),
        ("fault_inject", ctypes.c_int32),
        ("chains", ctypes.c_int32),
    ]


class CgdrChunkOOptions(ctypes.Structure):
    _fields_ = [("wait_timeout_ms", ctypes.c_int32), ("reserved", ctypes.c_int32 * 7)]


class CgdrWyOptions(ctypes.Structure):
    _fields_ = [("wait_timeout_ms", ctypes.c_int32), ("reserved", ctypes.c_int32 * 7)]


class CgdrGdrOptions(ctypes.Structure):
    _fields_ = [("path", ctypes.c_int32), ("reserved", ctypes.c_int32 * 7)]


GDR_PATHS = {"auto": 0, "fused": 1, "three_kernels": 2}


class CgdrFwdHPlan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "batch", "total_tokens", "key_heads", "value_heads", "key_dim", "value_dim",
        "sequence_count", "chunk_count", "head_ratio", "v_tile", "v_tile_count", "task_count")] + [
        (n, ctypes.c_int32) for n in (
            "has_initial_state", "is_varlen", "store_final_state", "save_new_value", "plan_key",
            "kernel", "grid", "block", "smem_bytes", "stages", "numerics", "layout")] + [
        ("workspace_bytes", ctypes.c_uint64), ("chains", ctypes.c_int32), ("reserved", ctypes.c_int32)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library; raise if it is absent (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(python -m cann_operator_challenge_august_b200.build)")
    lib = ctypes.CDLL(str(LIB_PATH))
    T = ctypes.POINTER(CgdrTensor)
    u64p = ctypes.POINTER(ctypes.c_uint64)
    exp = ctypes.POINTER(ctypes.c_void_p)
    lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize.argtypes = [T] * 7 + [ctypes.c_int64] + [T] * 3 + [u64p, exp]
    lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx.argtypes = (
        [T] * 8 + [ctypes.c_int64] + [T] * 3 + [ctypes.POINTER(CgdrFwdHOptions), u64p, exp])
    lib.cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSizeEx.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleFwdH.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    lib.cgdrChunkGatedDeltaRuleFwdH.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleFwdHNoAlloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                       ctypes.POINTER(ctypes.c_int32)]
    lib.cgdrChunkGatedDeltaRuleFwdHNoAlloc.restype = ctypes.c_int
    lib.cgdrDestroyExecutor.argtypes = [ctypes.c_void_p]
    lib.cgdrDestroyExecutor.restype = None
    lib.cgdrGetPlan.argtypes = [ctypes.c_void_p, ctypes.POINTER(CgdrFwdHPlan)]
    lib.cgdrGetPlan.restype = ctypes.c_int
    lib.cgdrReadDeviceStatus.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p,
                                         ctypes.POINTER(ctypes.c_int32)]
    lib.cgdrReadDeviceStatus.restype = ctypes.c_int
    lib.cgdrGetLastErrorMessage.argtypes = []
    lib.cgdrGetLastErrorMessage.restype = ctypes.c_char_p
    lib.cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize.argtypes = (
        [T] * 7 + [ctypes.c_double, ctypes.c_int64, T, ctypes.POINTER(CgdrChunkOOptions), u64p, exp])
    lib.cgdrChunkGatedDeltaRuleFwdOGetWorkspaceSize.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleFwdO.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    lib.cgdrChunkGatedDeltaRuleFwdO.restype = ctypes.c_int
    lib.cgdrDestroyChunkOExecutor.argtypes = [ctypes.c_void_p]
    lib.cgdrDestroyChunkOExecutor.restype = None
    lib.cgdrChunkOGridSize.argtypes = [ctypes.c_void_p]
    lib.cgdrChunkOGridSize.restype = ctypes.c_int64
    lib.cgdrChunkGatedDeltaRuleWYGetWorkspaceSize.argtypes = (
        [T] * 6 + [ctypes.c_int64] + [T] * 3 + [ctypes.POINTER(CgdrWyOptions), u64p, exp])
    lib.cgdrChunkGatedDeltaRuleWYGetWorkspaceSize.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleWY.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    lib.cgdrChunkGatedDeltaRuleWY.restype = ctypes.c_int
    lib.cgdrDestroyWyExecutor.argtypes = [ctypes.c_void_p]
    lib.cgdrDestroyWyExecutor.restype = None
    lib.cgdrChunkGatedDeltaRuleGetWorkspaceSize.argtypes = [T] * 7 + [ctypes.c_float, T, T, u64p, exp]
    lib.cgdrChunkGatedDeltaRuleGetWorkspaceSize.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx.argtypes = (
        [T] * 7 + [ctypes.c_float, T, T, ctypes.POINTER(CgdrGdrOptions), u64p, exp])
    lib.cgdrChunkGatedDeltaRuleGetWorkspaceSizeEx.restype = ctypes.c_int
    lib.cgdrGetGdrPath.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
    lib.cgdrGetGdrPath.restype = ctypes.c_int
    lib.cgdrChunkGatedDeltaRule.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    lib.cgdrChunkGatedDeltaRule.restype = ctypes.c_int
    lib.cgdrDestroyGdrExecutor.argtypes = [ctypes.c_void_p]
    lib.cgdrDestroyGdrExecutor.restype = None
    lib.cgdrPrepareChunkIndices.argtypes = [T, ctypes.c_int64, T, T, ctypes.c_void_p]
    lib.cgdrPrepareChunkIndices.restype = ctypes.c_int
    lib.cgdrGetAbiVersion.argtypes = []
    lib.cgdrGetAbiVersion.restype = ctypes.c_int32
    _lib = lib
    return lib


def last_error() -> str:
    return load().cgdrGetLastErrorMessage().decode(errors="replace")


class CgdrError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{where}: {self.status_name}: {last_error()}")


class CgdrValueError(CgdrError, ValueError):
    """Argument validation failures (the reference's GRAPH_FAILED cases)."""


VALIDATION_STATUSES = {1, 2, 3, 4, 5, 6, 7}


def check(status: int, where: str) -> None:
    if status != 0:
        if status in VALIDATION_STATUSES:
            raise CgdrValueError(status, where)
        raise CgdrError(status, where)


def null_tensor() -> CgdrTensor:
    return CgdrTensor()


def make_tensor(data_ptr: int, dtype: int, shape, strides) -> CgdrTensor:
    t = CgdrTensor()
    t.data = data_ptr
    t.dtype = dtype
    t.ndim = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        t.shape[i] = int(s)
        t.strides[i] = int(st)
    return t
