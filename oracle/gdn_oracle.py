"""CPU oracle for the gated-DeltaNet chunked prefill and its gated-RMSNorm stage.

TEST INFRASTRUCTURE ONLY. This module is the checker the parity tests, the
``smoke()`` entry and the ``cpu_baseline`` leg of ``bench.py`` compare the CUDA
path against. Nothing on the product path imports it; the product path has no
CPU fallback and fails loudly when its CUDA library is missing.

It is a numpy restatement, in float32 arithmetic, of the reference's own CPU
algorithm for this path:

* ``chunk_gated_delta_rule`` follows the torch chunked fallback that the
  reference's harness uses as its oracle, ``kernels/harness/parity_test.py:35-96``
  (a verbatim copy of transformers ``modeling_qwen3_5.torch_chunk_gated_delta_rule``,
  pinned by the reference at transformers 5.14.1, ``docs/environment.md:11``).
* ``gated_rmsnorm`` follows the reference's fused norm kernel
  ``export/patches/orin_text_engine/files/cpp/kernels/gatedRmsNorm/gatedRmsNormKernel.cu:21-54``
  (= ``Qwen3_5RMSNormGated.forward`` with the weight held in float32).
* ``recurrent_gated_delta_rule`` follows transformers
  ``modeling_qwen3_5.torch_recurrent_gated_delta_rule`` (the single-token
  decode update the reference leaves to stock Edge-LLM).
* ``gdn_gate`` and ``l2norm`` follow the reference's pre-stage adapter
  ``export/patches/orin_text_engine/files/cpp/kernels/gdnKernels/gdnChunkPrefillSm87.cu:44-125``.

Parity is pinned: ``tests/golden/`` holds vectors produced by the reference's
torch fallback (script ``tests/golden/make_golden.py``), and
``tests/test_oracle.py`` checks this restatement against every one of them.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round",
    "l2norm",
    "chunk_gated_delta_rule",
    "chunk_gated_delta_rule_varlen",
    "gated_rmsnorm",
    "recurrent_gated_delta_rule",
    "gdn_gate",
    "softplus",
    "fp16_round",
    "adapter_prefill",
]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32.

    This is the rounding torch applies in ``tensor.to(torch.bfloat16)``; the
    reference rounds o to the input dtype before its norm
    (``gatedRmsNormKernel.cu:47``) and casts the GDN output to bf16
    (``parity_test.py:95``).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).reshape(x.shape).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The upper 16 bits of bf16-representable float32 values (for bit-exact storage)."""
    x = np.ascontiguousarray(bf16_round(x), dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    """Inverse of :func:`bf16_bits`."""
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Row L2 normalisation in float32, eps inside the rsqrt.

    Follows ``gdnChunkPrefillSm87.cu:52-85`` (fp32 sum of squares,
    ``rsqrtf(total + 1e-6)``) and transformers ``l2norm`` (``parity_test.py:28-30``).
    """
    x = np.asarray(x, dtype=np.float32)
    inv = 1.0 / np.sqrt((x * x).sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
    return (x * inv.astype(np.float32)).astype(np.float32)


def softplus(x: np.ndarray) -> np.ndarray:
    """log(1+e^x) with torch's threshold 20 (``gdnChunkPrefillSm87.cu:44-49``)."""
    x = np.asarray(x, dtype=np.float32)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def gdn_gate(a, b, A_log, dt_bias):
    """g = -exp(A_log[h]) * softplus(a + dt_bias[h]); beta = sigmoid(b).

    Follows ``gdnChunkPrefillSm87.cu:113-125``; ``a``/``b`` are [..., HV].
    """
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    g = (-np.exp(np.asarray(A_log, np.float32)) * softplus(a + np.asarray(dt_bias, np.float32))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)
    return g, beta


def _expand_heads(x: np.ndarray, hv: int) -> np.ndarray:
    """repeat_interleave of the qk heads to the v heads (v-head h reads qk-head h // (HV/HQK)).

    Follows ``kernels/chunk_delta_cuda.h:12-14`` and the model's
    ``repeat_interleave`` (transformers ``modeling_qwen3_5.py:495-496``).
    """
    hqk = x.shape[2]
    if hqk == hv:
        return x
    assert hv % hqk == 0, "HV must be a multiple of HQK"
    return np.repeat(x, hv // hqk, axis=2)


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size: int = 64, initial_state=None,
                           output_final_state: bool = True, return_fp32: bool = False,
                           intermediates: dict | None = None):
    """Chunked gated delta rule, float32 math.

    Inputs (numpy, any float dtype; rounded values are taken as given):
      q, k [B, T, HQK, DK]; v [B, T, HV, DV]; g, beta [B, T, HV];
      initial_state [B, HV, DK, DV] or None (zeros).
    Returns (o [B, T, HV, DV] rounded to bf16 unless ``return_fp32``,
    final_state [B, HV, DK, DV] float32). When ``intermediates`` is a dict it
    is filled with per-chunk arrays [B, HV, NC, ...]: ``c`` (in-chunk cumsum),
    ``T`` ((I+L)^-1), ``W`` (k_cumdecay), ``v_new``, ``o`` (fp32, before
    rounding) and ``S_entry`` (state entering the chunk); and with the views of
    the reference's debug entry (``kernels/torch_binding.cpp:57-84``, filled by
    ``kernels/chunk_delta_cuda.cu``): ``value`` (its ``w`` = T v_beta, :268-282),
    ``decay`` (its ``de``, :284-294), ``eg`` / ``ed`` / ``gl`` (e^c, e^{c_L - c},
    e^{c_L}, :284-291), ``A`` (the assembled strict-lower -(k_beta k^T) decay
    before substitution, :158-175), ``M`` ((q k^T) decay scale, :480-509) and
    ``T_post_leaf`` (T after the 16 x 16 diagonal leaves are inverted, the other
    blocks still holding A, :176-214).

    Step-by-step restatement of ``kernels/harness/parity_test.py:35-96``:
      * transpose to [B, H, T, D] and pad T to a chunk multiple with zeros (:42-53);
      * scale q by 1/sqrt(DK) (:54-55);
      * k_beta, v_beta (:56-57); in-chunk cumsum of g (:63);
      * decay = exp(tril(c_i - c_j)) masked lower-inclusive (:64);
      * attn = -(k_beta k^T * decay) strictly lower (:65), forward substitution (:66-69),
        + I  ->  T = (I + L)^-1;
      * value = T v_beta, k_cumdecay = T (k_beta * e^c) (:71-72);
      * per chunk: v_new = value - k_cumdecay S; o = (q e^c) S + (q k^T * decay) v_new;
        S <- S e^{c_L} + (k e^{c_L - c})^T v_new (:79-89).
    """
    f32 = np.float32
    q = _expand_heads(np.asarray(q, f32), np.asarray(v).shape[2])
    k = _expand_heads(np.asarray(k, f32), np.asarray(v).shape[2])
    v = np.asarray(v, f32)
    g = np.asarray(g, f32)
    beta = np.asarray(beta, f32)
    B, T, H, DK = k.shape
    DV = v.shape[-1]
    C = chunk_size
    # [B, H, T, D]
    q, k, v = (np.ascontiguousarray(x.transpose(0, 2, 1, 3)) for x in (q, k, v))
    g = np.ascontiguousarray(g.transpose(0, 2, 1))
    beta = np.ascontiguousarray(beta.transpose(0, 2, 1))
    pad = (C - T % C) % C
    if pad:
        q = np.pad(q, ((0, 0), (0, 0), (0, pad), (0, 0)))
        k = np.pad(k, ((0, 0), (0, 0), (0, pad), (0, 0)))
        v = np.pad(v, ((0, 0), (0, 0), (0, pad), (0, 0)))
        g = np.pad(g, ((0, 0), (0, 0), (0, pad)))
        beta = np.pad(beta, ((0, 0), (0, 0), (0, pad)))
    Tp = T + pad
    NC = Tp // C
    scale = f32(1.0 / np.sqrt(DK))
    q = q * scale
    v_beta = v * beta[..., None]
    k_beta = k * beta[..., None]
    q, k, v, k_beta, v_beta = (x.reshape(B, H, NC, C, x.shape[-1]) for x in (q, k, v, k_beta, v_beta))
    g = g.reshape(B, H, NC, C)
    c = np.cumsum(g, axis=-1, dtype=f32)
    tri_incl = np.tril(np.ones((C, C), dtype=bool))
    diff = c[..., :, None] - c[..., None, :]
    decay = np.where(tri_incl, np.exp(np.where(tri_incl, diff, 0.0)), 0.0).astype(f32)
    strict = np.tril(np.ones((C, C), dtype=bool), k=-1)
    attn = np.where(strict, -(k_beta @ np.swapaxes(k, -1, -2)) * decay, 0.0).astype(f32)
    if intermediates is not None:
        intermediates["A"] = attn.copy()
        intermediates["decay"] = decay.copy()
        intermediates["M"] = ((q @ np.swapaxes(k, -1, -2)) * decay).astype(f32)  # q already carries the scale
        post = attn.copy()
        eye16 = np.eye(16, dtype=f32)
        for bl in range(C // 16):
            blk = slice(16 * bl, 16 * bl + 16)
            post[..., blk, blk] = np.linalg.inv(eye16 - attn[..., blk, blk]).astype(f32)
        intermediates["T_post_leaf"] = post
    for i in range(1, C):
        row = attn[..., i, :i].copy()
        sub = attn[..., :i, :i].copy()
        attn[..., i, :i] = row + (row[..., :, None] * sub).sum(-2)
    attn = attn + np.eye(C, dtype=f32)
    value = attn @ v_beta
    k_cumdecay = attn @ (k_beta * np.exp(c)[..., None])
    if initial_state is None:
        S = np.zeros((B, H, DK, DV), dtype=f32)
    else:
        S = np.array(initial_state, dtype=f32, copy=True)
    out = np.zeros_like(value)
    if intermediates is not None:
        intermediates["c"] = c.copy()
        intermediates["T"] = attn.copy()
        intermediates["W"] = k_cumdecay.copy()
        intermediates["value"] = value.copy()
        intermediates["eg"] = np.exp(c).astype(f32)
        intermediates["ed"] = np.exp(c[..., -1:] - c).astype(f32)
        intermediates["gl"] = np.exp(c[..., -1]).astype(f32)
        intermediates["v_new"] = np.zeros((B, H, NC, C, DV), f32)
        intermediates["S_entry"] = np.zeros((B, H, NC, DK, DV), f32)
    for n in range(NC):
        q_i, k_i, v_i = q[:, :, n], k[:, :, n], value[:, :, n]
        a_i = (q_i @ np.swapaxes(k_i, -1, -2)) * decay[:, :, n]
        v_new = v_i - k_cumdecay[:, :, n] @ S
        inter = (q_i * np.exp(c[:, :, n])[..., None]) @ S
        out[:, :, n] = inter + a_i @ v_new
        if intermediates is not None:
            intermediates["v_new"][:, :, n] = v_new
            intermediates["S_entry"][:, :, n] = S
        cl = c[:, :, n, -1]
        S = S * np.exp(cl)[..., None, None] + np.swapaxes(
            k_i * np.exp(cl[..., None] - c[:, :, n])[..., None], -1, -2) @ v_new
    if intermediates is not None:
        intermediates["o"] = out.copy()
    o = out.reshape(B, H, Tp, DV)[:, :, :T].transpose(0, 2, 1, 3)
    o = np.ascontiguousarray(o, dtype=f32)
    if not return_fp32:
        o = bf16_round(o)
    return o, (S.astype(f32) if output_final_state else None)


def chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu_seqlens, chunk_size: int = 64,
                                  initial_state=None, return_fp32: bool = False):
    """Packed variable-length form: B must be 1; sequences [cu[i], cu[i+1]) are
    independent, each starting from initial_state[i] (or zeros) and returning
    its own final state. Per-sequence loop over :func:`chunk_gated_delta_rule`."""
    cu = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    assert np.asarray(q).shape[0] == 1
    N = len(cu) - 1
    HV, DK, DV = np.asarray(v).shape[2], np.asarray(k).shape[3], np.asarray(v).shape[3]
    o = np.zeros(np.asarray(v).shape, dtype=np.float32)
    states = np.zeros((N, HV, DK, DV), dtype=np.float32)
    for i in range(N):
        a, b = cu[i], cu[i + 1]
        s0 = None if initial_state is None else np.asarray(initial_state)[i:i + 1]
        if b == a:
            states[i] = 0.0 if s0 is None else s0[0]
            continue
        oi, si = chunk_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                        chunk_size, s0, True, return_fp32)
        o[:, a:b] = oi
        states[i] = si[0]
    return o, states


def fp16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to float16 (nearest, ties to even), returned as float32."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def gated_rmsnorm(o, z, w, eps: float = 1e-6, io_dtype: str = "bf16"):
    """y = bf16( (w * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z) ), float32 math, rows over the last dim.

    Follows ``gatedRmsNormKernel.cu:21-54``: sum of squares in fp32 (:33-41),
    ``rsqrtf(ss/dv + eps)`` (:42), normalised value rounded to the I/O dtype
    before the weight (:47), silu(z) in fp32 (:48), product rounded (:50).
    With bf16 I/O this is ``Qwen3_5RMSNormGated.forward`` with a float32 weight
    holding the bf16 values (transformers ``modeling_qwen3_5.py:181-190``).
    """
    rnd = bf16_round if io_dtype == "bf16" else fp16_round
    o = np.asarray(o, np.float32)
    z = np.asarray(z, np.float32)
    w = np.asarray(w, np.float32)
    var = (o * o).mean(axis=-1, keepdims=True, dtype=np.float32)
    n = rnd(o * (1.0 / np.sqrt(var + np.float32(eps))).astype(np.float32))
    silu = (z / (1.0 + np.exp(-z))).astype(np.float32)
    return rnd((w * n) * silu)


def adapter_prefill(q16, k16, v16, a16, b16, A_log, dt_bias16, h0, z16=None, w16=None, eps: float = 1e-6):
    """The reference's TRT adapter composition (gdnChunkPrefillSm87.cu:186-320): q/k L2-normalised in
    fp32 and rounded to bf16 (:52-85), v rounded to bf16 (:88-98), gates in fp32 (:113-125), the chunked
    rule with h0 as the initial state, o rounded to bf16 then converted to fp16 (:100-110, :300).
    With z/w, the fp16 gated RMSNorm of the plugin follows (gatedRmsNormKernel.cu:21-54).
    Returns (o or y as fp16-valued float32, final state fp32)."""
    q = bf16_round(l2norm(np.asarray(q16, np.float32)))
    k = bf16_round(l2norm(np.asarray(k16, np.float32)))
    v = bf16_round(np.asarray(v16, np.float32))
    g, beta = gdn_gate(a16, b16, A_log, dt_bias16)
    o, sf = chunk_gated_delta_rule(q, k, v, g, beta, 64, h0)
    o16 = fp16_round(o)
    if z16 is not None:
        return gated_rmsnorm(o16, z16, w16, eps, io_dtype="fp16"), sf
    return o16, sf


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None):
    """Token-by-token recurrence (decode form), float32 math.

    Follows transformers ``modeling_qwen3_5.torch_recurrent_gated_delta_rule``:
    S <- S e^{g_t}; kv = S^T k_t; delta = (v_t - kv) beta_t; S <- S + k_t delta^T;
    o_t = S^T (q_t / sqrt(DK)). Returns (o bf16-rounded, final state fp32).
    """
    f32 = np.float32
    q = _expand_heads(np.asarray(q, f32), np.asarray(v).shape[2])
    k = _expand_heads(np.asarray(k, f32), np.asarray(v).shape[2])
    v = np.asarray(v, f32)
    g = np.asarray(g, f32)
    beta = np.asarray(beta, f32)
    B, T, H, DK = k.shape
    DV = v.shape[-1]
    scale = f32(1.0 / np.sqrt(DK))
    S = np.zeros((B, H, DK, DV), f32) if initial_state is None else np.array(initial_state, f32, copy=True)
    o = np.zeros((B, T, H, DV), f32)
    for t in range(T):
        S = S * np.exp(g[:, t])[..., None, None]
        kv = (S * k[:, t, :, :, None]).sum(-2)
        delta = (v[:, t] - kv) * beta[:, t, :, None]
        S = S + k[:, t, :, :, None] * delta[:, :, None, :]
        o[:, t] = (S * (q[:, t] * scale)[:, :, :, None]).sum(-2)
    return bf16_round(o), S
