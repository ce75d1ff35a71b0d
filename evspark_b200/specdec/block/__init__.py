"""Block-verify path on the device (mirror of evspark/specdec/block/__init__.py)."""

from evspark_b200.model import PARAM_KEYS
from evspark_b200.specdec.block.chunk import install_chunk_forward
from evspark_b200.specdec.block.driver import (
    block_forward,
    clone_inference_params,
    collapse_inference_params,
    diff_states,
    expand_inference_params,
    get_seqlen_offset,
    prefill,
    set_seqlen_offsets,
    snapshot_states,
    step_forward_reference,
    step_seqlen_offsets,
)
from evspark_b200.specdec.block.slice import ChunkStash, slice_states_to_accept

__all__ = [
    "PARAM_KEYS", "ChunkStash", "block_forward", "clone_inference_params", "collapse_inference_params",
    "diff_states", "expand_inference_params", "get_seqlen_offset", "install_chunk_forward", "prefill",
    "set_seqlen_offsets", "slice_states_to_accept", "snapshot_states", "step_forward_reference",
    "step_seqlen_offsets",
]
