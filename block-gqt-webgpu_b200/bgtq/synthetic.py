"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The key profile is the one the configs describe: RoPE frequency pair ``i`` of an
``n_pairs``-pair head is drawn as ``N(0, sigma_i^2)`` with
``sigma_i = 0.5 + 4 * exp(-(n_pairs - 1 - i) / 10)`` (low-frequency pairs dominate),
laid out split-half like HuggingFace RoPE: pair ``i`` occupies dimensions ``i`` and
``i + n_pairs`` (reference: ``vendor/blockgtq-calibration/rope_utils.py:23-32``).
Keys are rounded to FP16 before encoding, as the reference's key stores only accept
FP16 rows (``src/runtime/keys.ts:11-15``).

NumPy's PCG64 generator is used for everything that must be reproducible across
machines (golden vectors, parity tests); large bench inputs are drawn on the GPU.
"""
from __future__ import annotations

import numpy as np


def pair_sigma(n_pairs: int) -> np.ndarray:
    i = np.arange(n_pairs, dtype=np.float64)
    return 0.5 + 4.0 * np.exp(-((n_pairs - 1) - i) / 10.0)


def profiled(rng: np.random.Generator, rows: int, dim: int) -> np.ndarray:
    """``rows`` vectors of width ``dim`` with the pair-energy profile, FP32, split-half layout."""
    if dim % 2:
        raise ValueError("dimension must be even")
    n_pairs = dim // 2
    blocks = rng.standard_normal((rows, n_pairs, 2)) * pair_sigma(n_pairs)[None, :, None]
    out = np.concatenate([blocks[..., 0], blocks[..., 1]], axis=-1)
    return out.astype(np.float32)


def pair_energy_scores(q: np.ndarray, k: np.ndarray) -> np.ndarray:
    """``s_i = (E||q_i||^2 + E||k_i||^2) / 2`` over split-half pairs.

    Restates ``compute_freq_importance_energy`` (``vendor/blockgtq-calibration/freq_analysis.py:18-35``)
    in float32 like the reference (torch float32 mean of squared pair norms).
    """
    def energy(x):
        x = np.asarray(x, dtype=np.float32)
        n = x.shape[-1] // 2
        e = x[:, :n] * x[:, :n] + x[:, n:] * x[:, n:]
        return e.mean(axis=0, dtype=np.float32)
    return ((energy(q) + energy(k)) / np.float32(2)).astype(np.float32)


def decode_workload(seed: int, tokens: int, dim: int, queries: int = 1,
                    v_dtype=np.float16):
    """K (FP16-rounded), Q (FP32) and V for one head, all from one seed."""
    rng = np.random.default_rng(seed)
    k = profiled(rng, tokens, dim).astype(np.float16)
    q = profiled(rng, queries, dim)
    v = rng.standard_normal((tokens, dim)).astype(v_dtype)
    return k, q, v
