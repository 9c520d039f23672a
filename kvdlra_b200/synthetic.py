"""Seeded synthetic KV streams with the shapes of the benchmark workloads.

All generators are numpy-based and deterministic in their seed, so the same
inputs can be rebuilt on any host.  Keys are produced pre-RoPE and rotated with
the model's RoPE (default Llama rotary, ``theta``) before they are handed to a
cache, exactly as a model's attention layer hands post-RoPE keys to
``Cache.update``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def default_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """Default Llama rotary inverse frequencies, fp32 (``1/theta**(2i/D)``)."""
    exps = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(theta) ** exps)).astype(np.float32)


def apply_rope_htd(x: np.ndarray, positions: np.ndarray, inv_freq: np.ndarray,
                   scaling: float = 1.0) -> np.ndarray:
    """Rotate ``(H, T, D)`` fp32 keys at ``positions`` (``x cos + rotate_half(x) sin``)."""
    pos = positions.astype(np.int64).astype(np.float32)
    freqs = (pos[:, None] * inv_freq[None, :]).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=1)
    cos = (np.cos(emb) * np.float32(scaling)).astype(np.float32)
    sin = (np.sin(emb) * np.float32(scaling)).astype(np.float32)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


@dataclass
class LowRankStream:
    """One layer's synthetic stream: post-RoPE keys, values, pre-RoPE keys and
    the planted needle positions.  Arrays are ``(H, T, D)`` fp32."""

    k_post: np.ndarray
    v: np.ndarray
    k_pre: np.ndarray
    needles: np.ndarray


def lowrank_stream(
    num_heads: int = 8,
    head_dim: int = 64,
    t: int = 4096,
    *,
    signal_rank: int = 16,
    noise: float = 0.01,
    n_needles: int = 16,
    needle_norm: float = 5.0,
    theta: float = 500000.0,
    seed: int = 0,
    span_copies: tuple[int, int] | None = None,
) -> LowRankStream:
    """The single-layer stream of the synthetic workload: per head,
    ``K = Q diag(sigma) C + E`` with ``Q`` the QR of an N(0,1) ``D x r`` draw,
    ``sigma_i = 2^(-i/4)``, ``C ~ N(0,1)``, ``E ~ noise * N(0,1)``; values are an
    independent draw of the same form.  ``n_needles`` token positions (uniform,
    distinct, never a sink) get a key that is a unit vector orthogonal to that
    head's ``Q`` scaled to ``needle_norm``.  ``span_copies = (copies, length)``
    plants instead one span of ``length`` such keys verbatim at ``copies``
    random non-overlapping places (the same pre-RoPE content each time)."""
    rng = np.random.default_rng(seed)
    sig = (2.0 ** (-np.arange(signal_rank) / 4.0)).astype(np.float32)

    def draw(h_q: list[np.ndarray] | None) -> tuple[np.ndarray, list[np.ndarray]]:
        out = np.empty((num_heads, t, head_dim), np.float32)
        qs = []
        for h in range(num_heads):
            q, _ = np.linalg.qr(rng.standard_normal((head_dim, signal_rank)))
            c = rng.standard_normal((signal_rank, t))
            e = noise * rng.standard_normal((head_dim, t))
            out[h] = ((q * sig) @ c + e).T.astype(np.float32)
            qs.append(q)
        return out, qs

    k_pre, qk = draw(None)
    v, _ = draw(None)
    if span_copies is not None:
        copies, length = span_copies
        slots = (t - 8) // length
        starts = 8 + length * np.sort(rng.choice(slots, size=copies, replace=False))
        span = np.empty((num_heads, length, head_dim))
        for h in range(num_heads):
            x = rng.standard_normal((length, head_dim))
            x = x - (x @ qk[h]) @ qk[h].T
            span[h] = x / np.linalg.norm(x, axis=1, keepdims=True) * needle_norm
        needles = np.concatenate([st + np.arange(length) for st in starts])
        for st in starts:
            k_pre[:, st : st + length] = span.astype(np.float32)
    else:
        needles = np.sort(rng.choice(np.arange(8, t), size=n_needles, replace=False)) if n_needles else np.zeros(0, np.int64)
        for p in needles:
            for h in range(num_heads):
                x = rng.standard_normal(head_dim)
                x = x - qk[h] @ (qk[h].T @ x)
                x = x / np.linalg.norm(x) * needle_norm
                k_pre[h, p] = x.astype(np.float32)
    inv = default_inv_freq(head_dim, theta)
    k_post = apply_rope_htd(k_pre, np.arange(t), inv)
    return LowRankStream(k_post=k_post, v=v, k_pre=k_pre, needles=needles.astype(np.int64))


def gaussian_kv(num_layers: int, num_heads: int, head_dim: int, t: int, *, theta: float = 500000.0,
                seed: int = 0, scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    """``(layers, H, T, D)`` post-RoPE keys and values from N(0, scale^2) pre-RoPE draws."""
    rng = np.random.default_rng(seed)
    k = (scale * rng.standard_normal((num_layers, num_heads, t, head_dim))).astype(np.float32)
    v = (scale * rng.standard_normal((num_layers, num_heads, t, head_dim))).astype(np.float32)
    inv = default_inv_freq(head_dim, theta)
    for layer in range(num_layers):
        k[layer] = apply_rope_htd(k[layer], np.arange(t), inv)
    return k, v
