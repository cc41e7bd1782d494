"""Seeded synthetic inputs with the shapes and value distributions BASELINE.json names (no public
dataset is involved; the reference's own benchmark workload files are external)."""

from __future__ import annotations

import numpy as np


def sinusoid_noise(series: int, length: int, seed: int = 0) -> np.ndarray:
    """Config 3/5: sinusoids with period ~ U[8, 512] and phase ~ U[0, 2π) plus N(0, 0.1) noise."""
    rng = np.random.default_rng(seed)
    period = rng.uniform(8.0, 512.0, series)
    phase = rng.uniform(0.0, 2 * np.pi, series)
    t = np.arange(length, dtype=np.float64)
    x = np.sin(2 * np.pi * t[None, :] / period[:, None] + phase[:, None])
    x += rng.normal(0.0, 0.1, (series, length))
    return x.astype(np.float32)


def random_walk(series: int, length: int, seed: int = 0) -> np.ndarray:
    """Config 2: x_t = x_{t−1} + N(0, 1), x_0 = 0."""
    rng = np.random.default_rng(seed)
    steps = rng.standard_normal((series, length))
    steps[:, 0] = 0.0
    return np.cumsum(steps, axis=1).astype(np.float32)


def ar2(series: int, length: int, phi1: float = 0.6, phi2: float = 0.3, sigma: float = 1.0, burn_in: int = 200,
        seed: int = 0) -> np.ndarray:
    """Config 4: AR(2) with φ1 = 0.6, φ2 = 0.3, σ = 1 after a 200-step burn-in."""
    rng = np.random.default_rng(seed)
    e = rng.normal(0.0, sigma, (series, length + burn_in))
    x = np.zeros((series, length + burn_in))
    for t in range(2, length + burn_in):
        x[:, t] = phi1 * x[:, t - 1] + phi2 * x[:, t - 2] + e[:, t]
    return x[:, burn_in:].astype(np.float32)


def mixed_batch(series: int, length: int, patch: int, seed: int = 11, covariate_groups: int = 0):
    """A batch in the spirit of the reference's batch-parity tests (TimestralBatchParityAccelTest.java:
    75-116): random walks plus a daily sinusoid, NaN gaps, late starts, some multi-row series.
    Returns (inputs, observed, group, role)."""
    rng = np.random.default_rng(seed)
    rows, groups, roles = [], [], []
    g = 0
    for s in range(series):
        nvar = 1 if s >= covariate_groups else 2 + (s % 2)
        for v in range(nvar):
            x = np.cumsum(rng.standard_normal(length)) + 3 * np.sin(2 * np.pi * np.arange(length) / 24.0)
            obs = np.ones(length, bool)
            if rng.random() < 0.5:
                gap = rng.integers(0, length - patch)
                obs[gap:gap + rng.integers(1, 3 * patch)] = False
            if rng.random() < 0.3:
                obs[:rng.integers(1, length // 2)] = False
            x = np.where(obs, x, 0.0)
            rows.append((x.astype(np.float32), obs))
            groups.append(g)
            roles.append(0 if v == 0 else (1 if v == 1 else 2))
        g += 1
    inputs = np.stack([r[0] for r in rows])
    observed = np.stack([r[1] for r in rows])
    return inputs, observed, np.array(groups, np.int32), np.array(roles, np.int32)
