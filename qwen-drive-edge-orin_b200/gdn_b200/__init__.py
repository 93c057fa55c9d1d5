"""gdn_b200: B200-native (sm_100a) chunked gated-DeltaNet prefill with a fused
gated-RMSNorm epilogue, behind the reference's C ABI and torch-binding
interface.

Public Python surface (mirrors the reference's ``kernels/torch_binding.cpp``
and ``kernels/harness/chunk_delta.py``):

* :func:`chunk_prefill` ``(q, k, v, g, beta, s0=None) -> [o, sf]``
* :func:`chunk_prefill_gated` ``(q, k, v, g, beta, z, w, s0=None, eps=1e-6) -> [y, sf]``
* :func:`chunk_prefill_varlen` ``(q, k, v, g, beta, cu_seqlens, s0=None, z=None, w=None, eps=1e-6)``
* :func:`run_chunk_prefill` (the TRT adapter's fp16 inputs, pre-stage fused)
* :func:`recurrent_decode` (single/few-token recurrent update, state in place)
* :func:`gated_rmsnorm` ``(o, z, w, eps=1e-6) -> y``
* :func:`chunk_gated_delta_rule_fast` (transformers-compatible signature)

Every call goes through the C-ABI shared library ``libgdn_b200.so`` built
from ``csrc/``; there is no CPU or library fallback.
"""
from .binding import (  # noqa: F401
    chunk_prefill,
    chunk_prefill_debug,
    chunk_prefill_debug_native,
    chunk_prefill_gated,
    chunk_prefill_varlen,
    chunk_prefill_segmented,
    segmented_plan,
    segment_bounds,
    segment_entry_states,
    run_chunk_prefill,
    recurrent_decode,
    gated_rmsnorm,
    chunk_gated_delta_rule_fast,
    workspace_size,
    GdnError,
)
from ._lib import load_library, library_path  # noqa: F401
