"""B200-native (sm_100a) ChunkGatedDeltaRuleFwdH -- the chunked gated-delta-rule
forward hidden-state recurrence of Gated DeltaNet prefill.

The compute is a CUDA library with a C ABI (include/cgdr_fwd_h.h); this
package is its Python host side.  See :mod:`.api` for the entry points.
"""

from .api import (  # noqa: F401
    CHUNK_SIZE,
    ChunkGatedDeltaRuleFwdH,
    chunk_gated_delta_rule_fwd_h,
    prepare_chunk_indices,
    prepare_chunk_offsets,
    read_device_status,
    run,
)
from ._lib import CgdrError, CgdrValueError  # noqa: F401

__all__ = [
    "CHUNK_SIZE",
    "ChunkGatedDeltaRuleFwdH",
    "chunk_gated_delta_rule_fwd_h",
    "prepare_chunk_indices",
    "prepare_chunk_offsets",
    "read_device_status",
    "run",
    "CgdrError",
    "CgdrValueError",
]
