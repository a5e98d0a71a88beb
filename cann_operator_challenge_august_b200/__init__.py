"""B200-native (sm_100a) ChunkGatedDeltaRuleFwdH -- the chunked gated-delta-rule
forward hidden-state recurrence of Gated DeltaNet prefill.

The compute is a CUDA library with a C ABI (include/cgdr_fwd_h.h for the
recurrence, include/cgdr_wy.h for the WY representation that feeds it,
include/cgdr_chunk_o.h for the chunk output that consumes it, and
include/cgdr_gdr.h for the whole chunked Gated DeltaNet forward built from
the three); this package is its Python host side.  See :mod:`.api` and
:mod:`.gdr`.
"""

from .api import (  # noqa: F401
    CHUNK_SIZE,
    ChunkGatedDeltaRuleFwdH,
    chunk_capacity,
    chunk_gated_delta_rule_fwd_h,
    prepare_chunk_indices,
    prepare_chunk_offsets,
    read_device_status,
    run,
)
from .gdr import (  # noqa: F401
    ChunkGatedDeltaRule,
    ChunkGatedDeltaRuleFwdO,
    ChunkGatedDeltaRuleWY,
    chunk_fwd_o,
    chunk_gated_delta_rule,
    chunk_wy_fwd,
)
from .host import chunk_gated_delta_rule_fwd_h_host  # noqa: F401
from ._lib import CgdrError, CgdrValueError  # noqa: F401

__all__ = [
    "CHUNK_SIZE",
    "ChunkGatedDeltaRuleFwdH",
    "chunk_capacity",
    "chunk_gated_delta_rule_fwd_h",
    "chunk_gated_delta_rule_fwd_h_host",
    "prepare_chunk_indices",
    "prepare_chunk_offsets",
    "read_device_status",
    "run",
    "ChunkGatedDeltaRuleFwdO",
    "chunk_fwd_o",
    "ChunkGatedDeltaRuleWY",
    "chunk_wy_fwd",
    "ChunkGatedDeltaRule",
    "chunk_gated_delta_rule",
    "CgdrError",
    "CgdrValueError",
]
