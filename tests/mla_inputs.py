"""Seeded synthetic inputs for the MLA decode-attention parity tests.

A self-contained generator (splitmix64 -> 53-bit uniforms -> Box-Muller normals) so the committed
golden fixtures do not depend on any library's random stream.  Distributions follow the
reference's config 1 (BASELINE config): W_UK, W_UV ~ N(0, 0.02) stored as f16; q and the KV cache
~ N(0, 1), q in f32 and the cache in f16; softmax scale 1/sqrt(nope + rope).

Geometry names follow the reference (engine/m1_layer.h:47-55): H heads, nope, rope, R = latent
(kv_lora_rank), D = R + rope (the KV row), V = value head width.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        idx = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + idx * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, n: int) -> np.ndarray:
    """n standard normals (float64) from a seed, bit-stable across numpy versions."""
    m = (n + 1) // 2
    u = _splitmix64(seed, 2 * m)
    u1 = ((u[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740993.0)
    u2 = (u[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m, np.float64)
    z[0::2] = r * np.cos(2.0 * math.pi * u2)
    z[1::2] = r * np.sin(2.0 * math.pi * u2)
    return z[:n]


def uniform_int(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform on [lo, hi] (inclusive)."""
    u = _splitmix64(seed, n)
    return (lo + (u % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int64)


@dataclass(frozen=True)
class Geometry:
    H: int = 32
    nope: int = 128
    rope: int = 64
    R: int = 512
    V: int = 128

    @property
    def D(self) -> int:
        return self.R + self.rope

    @property
    def dq(self) -> int:
        return self.nope + self.rope

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.nope + self.rope)


BASELINE = Geometry()


def make_layer(seed: int, N: int, g: Geometry = BASELINE):
    """One layer's inputs: q f32 (H, nope+rope), W_UK f16 (H, R, nope), kcache f16 (N, D),
    W_UV f16 (H, V, R).  Each tensor draws from its own sub-seed."""
    q = normal(seed * 8 + 1, g.H * g.dq).astype(np.float32).reshape(g.H, g.dq)
    w_uk = (0.02 * normal(seed * 8 + 2, g.H * g.R * g.nope)).astype(np.float16).reshape(
        g.H, g.R, g.nope)
    kc = normal(seed * 8 + 3, N * g.D).astype(np.float16).reshape(N, g.D)
    w_uv = (0.02 * normal(seed * 8 + 4, g.H * g.V * g.R)).astype(np.float16).reshape(
        g.H, g.V, g.R)
    return q, w_uk, kc, w_uv


def window_mask(N: int, base: int, length: int) -> np.ndarray:
    """The engine's mask: 0 on [base, base+length), -inf elsewhere (m1_layer.cpp:756-773)."""
    m = np.full(N, -np.inf, np.float32)
    lo, hi = max(base, 0), min(base + length, N)
    if hi > lo:
        m[lo:hi] = 0.0
    return m


def ragged_lengths(seed: int, n: int = 16, lo: int = 512, hi: int = 65536) -> np.ndarray:
    """Per-sequence KV lengths of the ragged batched decode (config 5: 16 sequences, lengths
    uniform on [512, 65536] by seed)."""
    return uniform_int(seed, n, lo, hi)


def packed_bases(lengths, gap: int = 0) -> np.ndarray:
    """First cache row of each sequence when the sequences are packed back to back (with
    ``gap`` unused rows after each)."""
    lengths = np.asarray(lengths, np.int64)
    return np.concatenate([[0], np.cumsum(lengths + gap)[:-1]]).astype(np.int64)


# The Mistral-Small-4 geometry (engine/m1_layer.h:47-55): nope 64, rope 64, latent 256, KV row
# 320, Q8_0 W_UK / W_UV.  Weights are drawn like BASELINE's (N(0, 0.02)) and stored as Q8_0 with
# ggml's reference quantizer, so every consumer reads the same bytes.
MISTRAL = Geometry(nope=64, rope=64, R=256, V=128)

# the engine's rope / norm scalars for that geometry (m1_layer.cpp:60-95, m1_layer.h:56-67)
MISTRAL_ROPE = {"freq_base": 10000.0, "freq_scale": 1.0 / 128.0, "ext_factor": 1.0,
                "attn_factor": 1.0 / (1.0 + 0.1 * math.log(128.0)), "beta_fast": 32.0,
                "beta_slow": 1.0, "eps": 9.999999974752427e-07, "n_dims": 64, "n_ctx_orig": 8192}


def make_layer_q8(seed: int, N: int, g: Geometry = MISTRAL):
    """(q f32 (H, dq), W_UK Q8_0 bytes (H, R, nope/32*34), kcache f16 (N, D),
    W_UV Q8_0 bytes (H, V, R/32*34))."""
    from oracle import oracle as O
    q = normal(seed * 8 + 1, g.H * g.dq).astype(np.float32).reshape(g.H, g.dq)
    w_uk = (0.02 * normal(seed * 8 + 2, g.H * g.R * g.nope)).astype(np.float32).reshape(
        g.H, g.R, g.nope)
    kc = normal(seed * 8 + 3, N * g.D).astype(np.float16).reshape(N, g.D)
    w_uv = (0.02 * normal(seed * 8 + 4, g.H * g.V * g.R)).astype(np.float32).reshape(
        g.H, g.V, g.R)
    return q, O.q8_0_quantize(w_uk), kc, O.q8_0_quantize(w_uv)


def make_kvwrite(seed: int, N: int, n_in: int = 4096, g: Geometry = MISTRAL):
    """(cur f32 (n_in,), W_kva Q8_0 bytes (D, n_in/32*34), kv_a_norm f32 (R,), kcache f16 (N, D))."""
    from oracle import oracle as O
    cur = normal(seed * 8 + 5, n_in).astype(np.float32)
    w = (0.02 * normal(seed * 8 + 6, g.D * n_in)).astype(np.float32).reshape(g.D, n_in)
    nw = (1.0 + 0.1 * normal(seed * 8 + 7, g.R)).astype(np.float32)
    kc = normal(seed * 8 + 3, N * g.D).astype(np.float16).reshape(N, g.D)
    return cur, O.q8_0_quantize(w), nw, kc
