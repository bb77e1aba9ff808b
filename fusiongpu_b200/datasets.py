"""Seed-deterministic synthetic workloads (Gaussian mixtures) for the five configs.

The reference reads TEXMEX ``.fvecs`` files (utils.h:23-47) and ships no data.
These generators stand in for a dataset: numpy's PCG64 bit generator is
platform independent, so the same seed yields the same vectors on every
machine, and test fixtures can be regenerated instead of stored.

Each config is a mixture of isotropic Gaussians; a point picks its component
uniformly at random.  ``C1``/``C2``/``C5`` are integer valued in ``[0, 255]``
(clamped and rounded), ``C3``/``C4`` are unit-normalised.  C3's centres are
normalised N(0, I) draws; C4's are plain N(0, I) draws (only the sampled
vectors are normalised), as the two configs state.
"""
from __future__ import annotations

import concurrent.futures
import dataclasses
import os

import numpy as np


@dataclasses.dataclass(frozen=True)
class MixtureSpec:
    """Shape of one synthetic workload."""

    name: str
    n_base: int
    n_query: int
    dim: int
    n_centres: int
    sigma: float
    kind: str  # "int255" (uniform centres, clamp+round), "unit" (N(0,I) centres, normalised)
    centre_hi: float = 128.0
    dtype: str = "float32"
    seed: int = 0
    normalise_centres: bool = True  # "unit" kind only


# The five workloads, in BASELINE order.
C1 = MixtureSpec("C1", 100_000, 1_000, 128, 256, 12.0, "int255", 128.0, "float32", 1)
C2 = MixtureSpec("C2", 1_000_000, 10_000, 128, 4_096, 10.0, "int255", 128.0, "float32", 2)
C3 = MixtureSpec("C3", 10_000_000, 10_000, 96, 16_384, 0.05, "unit", 0.0, "float32", 3)
C4 = MixtureSpec("C4", 1_000_000, 10_000, 768, 2_000, 0.3, "unit", 0.0, "float16", 4, normalise_centres=False)
C5 = MixtureSpec("C5", 100_000_000, 10_000, 128, 65_536, 8.0, "int255", 255.0, "uint8", 5)

CONFIGS = {s.name: s for s in (C1, C2, C3, C4, C5)}


def scaled(spec: MixtureSpec, n_base: int, n_query: int, n_centres: int | None = None,
           seed: int | None = None) -> MixtureSpec:
    """A smaller workload with the same generator (used by tests)."""
    return dataclasses.replace(
        spec, name=f"{spec.name}-n{n_base}", n_base=n_base, n_query=n_query,
        n_centres=n_centres if n_centres is not None else spec.n_centres,
        seed=spec.seed if seed is None else seed)


def _centres(spec: MixtureSpec, rng: np.random.Generator) -> np.ndarray:
    if spec.kind == "int255":
        return rng.uniform(0.0, spec.centre_hi, size=(spec.n_centres, spec.dim)).astype(np.float32)
    c = rng.standard_normal(size=(spec.n_centres, spec.dim)).astype(np.float32)
    if spec.normalise_centres:
        c /= np.linalg.norm(c, axis=1, keepdims=True)
    return c


def _draw(spec: MixtureSpec, centres: np.ndarray, n: int, stream: int, chunk: int = 1 << 16) -> np.ndarray:
    """Rows in chunks of ``chunk``; chunk c draws from its own PCG64 stream
    ``[seed, stream, c]``, so the result does not depend on the thread count."""
    out_dtype = np.uint8 if spec.dtype == "uint8" else (np.float16 if spec.dtype == "float16" else np.float32)
    out = np.empty((n, spec.dim), dtype=out_dtype)

    def one(ci: int) -> None:
        s = ci * chunk
        e = min(n, s + chunk)
        rng = np.random.Generator(np.random.PCG64([spec.seed, stream, ci]))
        comp = rng.integers(0, spec.n_centres, size=e - s)
        x = rng.standard_normal(size=(e - s, spec.dim), dtype=np.float32)
        x *= np.float32(spec.sigma)
        x += centres[comp]
        if spec.kind == "int255":
            np.clip(x, 0.0, 255.0, out=x)
            np.rint(x, out=x)
        else:
            x /= np.linalg.norm(x, axis=1, keepdims=True)
        out[s:e] = x.astype(out_dtype)

    nchunks = (n + chunk - 1) // chunk
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(one, range(nchunks)))
    return out


def generate(spec: MixtureSpec) -> tuple[np.ndarray, np.ndarray]:
    """Return ``(base, queries)`` for ``spec``; both C-contiguous, dtype per spec."""
    rng_c = np.random.Generator(np.random.PCG64([spec.seed, 0]))
    centres = _centres(spec, rng_c)
    base = _draw(spec, centres, spec.n_base, 1)
    queries = _draw(spec, centres, spec.n_query, 2)
    return base, queries
