"""Seeded synthetic inputs for the gated-DeltaNet prefill path.

There is no public dataset on this path and the reference's real-activation
fixtures are not shipped, so every test and benchmark runs on seeded synthetic
tensors with the shapes and value distributions the reference and its
benchmark configurations name:

* ``dist="baseline"``: q, k ~ N(0,1) L2-normalised per head in fp32 then rounded
  to bf16 (the adapter's ``l2normFp16ToBf16``, ``gdnChunkPrefillSm87.cu:52-85``);
  v, z ~ N(0,1); beta = sigmoid(N(0,1)); g = -softplus(N(0,1)); norm weight
  w = 1 + 0.1 N(0,1); initial state ~ N(0, 0.02) (std).
* ``dist="refgrid"``: the reference harness generator ``make_inputs``
  (``kernels/harness/parity_test.py:102-121``): q, k ~ N(0,1)/8 (optionally
  L2-normalised), v ~ N(0,1), g = -U(0, 0.3), beta ~ U(0,1), s0 ~ N(0,1) * 0.5.

Values are drawn with numpy's PCG64 generator so the same seed gives the same
tensors on every machine; bf16 tensors are returned as float32 arrays holding
bf16-representable values (round to nearest even).
"""
from __future__ import annotations

import dataclasses

import numpy as np

__all__ = ["GdnInputs", "make_inputs", "bf16_round_np", "make_cu_seqlens"]


def bf16_round_np(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bf16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).reshape(x.shape).copy()


def _l2n(x: np.ndarray) -> np.ndarray:
    inv = 1.0 / np.sqrt((x * x).sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(1e-6))
    return (x * inv.astype(np.float32)).astype(np.float32)


@dataclasses.dataclass
class GdnInputs:
    q: np.ndarray          # [B, T, HQK, DK]  bf16 values (float32 storage) or fp32
    k: np.ndarray          # [B, T, HQK, DK]
    v: np.ndarray          # [B, T, HV, DV]
    g: np.ndarray          # [B, T, HV] fp32
    beta: np.ndarray       # [B, T, HV] fp32
    z: np.ndarray          # [B, T, HV, DV]
    w: np.ndarray          # [DV]
    s0: np.ndarray | None  # [B, HV, DK, DV] fp32 (or [N, ...] for varlen)
    eps: float = 1e-6


def make_inputs(B: int, T: int, HQK: int, HV: int, D: int = 128, seed: int = 0,
                dist: str = "baseline", with_s0: bool = True, l2: bool = True,
                dtype: str = "bf16", n_states: int | None = None) -> GdnInputs:
    """Seeded inputs. ``dtype`` is "bf16" (q/k/v/z/w rounded to bf16) or "fp32".

    ``n_states`` overrides the leading dimension of the initial state (varlen
    batches carry one state per packed sequence).
    """
    rng = np.random.default_rng(seed)
    f32 = np.float32
    nrm = lambda *s: rng.standard_normal(s, dtype=f32)  # noqa: E731
    if dist == "baseline":
        q = _l2n(nrm(B, T, HQK, D))
        k = _l2n(nrm(B, T, HQK, D))
        v = nrm(B, T, HV, D)
        beta = (1.0 / (1.0 + np.exp(-nrm(B, T, HV)))).astype(f32)
        a = nrm(B, T, HV)
        g = (-np.where(a > 20.0, a, np.log1p(np.exp(np.minimum(a, 20.0))))).astype(f32)
        s_std = 0.02
    elif dist == "refgrid":
        q = nrm(B, T, HQK, D) / f32(8.0)
        k = nrm(B, T, HQK, D) / f32(8.0)
        if dtype == "bf16":
            q, k = bf16_round_np(q), bf16_round_np(k)
        if l2:
            q, k = _l2n(q), _l2n(k)
        v = nrm(B, T, HV, D)
        g = -(rng.random((B, T, HV), dtype=f32) * f32(0.3))
        beta = rng.random((B, T, HV), dtype=f32)
        s_std = 0.5
    else:
        raise ValueError(f"unknown dist {dist!r}")
    z = nrm(B, T, HV, D)
    w = (1.0 + 0.1 * nrm(D)).astype(f32)
    ns = B if n_states is None else n_states
    s0 = (nrm(ns, HV, D, D) * f32(s_std)).astype(f32) if with_s0 else None
    if dtype == "bf16":
        q, k, v, z, w = (bf16_round_np(x) for x in (q, k, v, z, w))
    elif dtype != "fp32":
        raise ValueError(f"unknown dtype {dtype!r}")
    return GdnInputs(q=q.astype(f32), k=k.astype(f32), v=v.astype(f32), g=g.astype(f32),
                     beta=beta.astype(f32), z=z.astype(f32), w=w.astype(f32), s0=s0)


def make_cu_seqlens(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    """int32 cumulative sequence offsets for ``n`` packed sequences with
    lengths uniform in [lo, hi] (inclusive), seeded."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n)
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
