"""Explicit random parameters following the reference distributions.

The reference draws hash parameters and initial weights from rand 0.8.5's
StdRng (ChaCha12) and rand_distr's Normal; neither is available here, so the
engine and the CPU oracle both take these arrays explicitly.  Distributions:

* SimHash planes: ternary {-1: 1/6, 0: 2/3, +1: 1/6}, order table, bit, dim
  (crates/klearu-core/src/hash/simhash.rs:37-71).
* WTA/DWTA windows: the first ``w`` entries of a full shuffle of 0..d, per
  (table, hash fn) (dwta.rs:64-74, wta.rs:65-75).
* MinHash permutations: a full shuffle of 0..d per table (minhash.rs:45-52).
* SRP: each dim is -1 / +1 with probability sparsity/2 each (srp.rs:60-78).
* Weights: N(0, sqrt(2/d)) per row, bias 0 (network/neuron.rs:23-43).
"""

from __future__ import annotations

import numpy as np

from .config import HashFunctionType as HF


def simhash_planes(rng: np.random.Generator, L: int, K: int, d: int) -> np.ndarray:
    r = rng.random((L, K, d))
    out = np.zeros((L, K, d), dtype=np.int8)
    out[r < 1.0 / 6.0] = -1
    out[r >= 1.0 / 6.0 + 2.0 / 3.0] = 1
    return out


def windows(rng: np.random.Generator, L: int, K: int, d: int, w: int) -> np.ndarray:
    out = np.empty((L, K, w), dtype=np.uint32)
    for t in range(L):
        for k in range(K):
            if d <= 4 * w:
                out[t, k] = rng.permutation(d)[:w]
            else:  # first w of a uniform shuffle = w distinct uniform draws in order
                out[t, k] = rng.choice(d, size=w, replace=False)
    return out


def minhash_perms(rng: np.random.Generator, L: int, d: int) -> np.ndarray:
    return np.stack([rng.permutation(d).astype(np.uint32) for _ in range(L)])


def srp_projections(rng: np.random.Generator, L: int, K: int, d: int, sparsity: float = 1.0 / 3.0):
    pneg = sparsity / 2.0
    pzero_end = pneg + (1.0 - sparsity)
    rowptr = [0]
    idx, coef = [], []
    for _ in range(L * K):
        r = rng.random(d)
        neg = r < pneg
        pos = r >= pzero_end
        nz = np.nonzero(neg | pos)[0]
        idx.append(nz.astype(np.uint32))
        coef.append(np.where(neg[nz], -1, 1).astype(np.int8))
        rowptr.append(rowptr[-1] + len(nz))
    return (np.asarray(rowptr, dtype=np.uint32), np.concatenate(idx) if idx else np.zeros(0, np.uint32),
            np.concatenate(coef) if coef else np.zeros(0, np.int8))


def hash_params(kind: int, rng: np.random.Generator, d: int, K: int, L: int, w: int = 8) -> dict:
    """Parameter arrays of one hash family, keyed like kl_hash_params."""
    kind = HF(kind)
    if kind == HF.SimHash:
        return {"planes": simhash_planes(rng, L, K, d)}
    if kind in (HF.WtaHash, HF.DwtaHash):
        return {"windows": windows(rng, L, K, d, min(w, d))}
    if kind == HF.MinHash:
        return {"perms": minhash_perms(rng, L, d)}
    rp, ix, cf = srp_projections(rng, L, K, d)
    return {"srp_rowptr": rp, "srp_idx": ix, "srp_coef": cf}


def init_weights(rng: np.random.Generator, n: int, d: int) -> np.ndarray:
    sd = np.float32(np.sqrt(2.0 / d))
    return (rng.standard_normal((n, d), dtype=np.float32) * sd).astype(np.float32)
