"""The reference's own CPU implementation of this path, for timing (TEST/BENCH INFRASTRUCTURE ONLY).

The reference's parity harness takes its oracle from transformers
(``kernels/harness/parity_test.py:22-26``): ``torch_chunk_gated_delta_rule``
(bit-identical to the reference's verbatim copy at ``parity_test.py:35-96``,
checked by ``tests/golden/make_golden.py``) followed in the model by
``Qwen3_5RMSNormGated`` (transformers ``modeling_qwen3_5.py:175-190``; the
reference's ``gated_rmsnorm`` plugin reproduces it). ``bench.py`` times this
pair on the host cores as the CPU baseline and as its ``--impl reference`` arm.
Nothing on the product path imports this module.
"""
from __future__ import annotations

import torch
from transformers.models.qwen3_5.modeling_qwen3_5 import (  # noqa: F401
    Qwen3_5RMSNormGated,
    torch_chunk_gated_delta_rule,
)


def reference_gated_prefill(q, k, v, g, beta, z, w, s0, eps: float = 1e-6):
    """q/k [B,T,HQK,D] bf16 (pre-normalised), v/z [B,T,HV,D] bf16, g/beta fp32, w [D], s0 fp32.
    Returns (y bf16 [B,T,HV,D], final state fp32) exactly as the reference computes them on CPU."""
    rep = v.shape[2] // q.shape[2]
    if rep > 1:  # the model's repeat_interleave (modeling_qwen3_5.py:495-496)
        q = q.repeat_interleave(rep, dim=2)
        k = k.repeat_interleave(rep, dim=2)
    with torch.no_grad():
        o, sf = torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=s0,
                                             output_final_state=True, use_qk_l2norm_in_kernel=False)
        norm = Qwen3_5RMSNormGated(o.shape[-1], eps=eps)
        norm.weight.copy_(w.float())
        y = norm(o.reshape(-1, o.shape[-1]), z.reshape(-1, z.shape[-1])).reshape(o.shape)
    return y, sf
