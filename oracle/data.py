"""CPU restatement of klearu-core's LibSVM loader and BatchIterator order
(test infrastructure: the parity checker for klearu_b200/csrc/data.cu).

* parse_libsvm follows crates/klearu-core/src/data/libsvm.rs:39-111
  (load_from_reader) and :127-185 (parse_line), with
  crates/klearu-core/src/tensor/sparse.rs:36-57 (from_pairs);
* batch_order follows crates/klearu-core/src/data/dataset.rs:60-111
  (fisher_yates_shuffle, splitmix64, Iterator::next).
"""

from __future__ import annotations

import re

import numpy as np

M64 = (1 << 64) - 1


def splitmix64(state: int) -> int:  # dataset.rs:82-87
    z = (state + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def shuffled_indices(n: int, seed: int) -> list[int]:  # dataset.rs:71-80
    idx = list(range(n))
    st = seed & M64
    for i in range(n - 1, 0, -1):
        st = splitmix64(st)
        j = st % (i + 1)
        idx[i], idx[j] = idx[j], idx[i]
    return idx


def batch_order(n: int, batch_size: int, seed: int) -> list[list[int]]:  # dataset.rs:94-111
    idx = shuffled_indices(n, seed)
    return [idx[p:p + batch_size] for p in range(0, n, batch_size)]


_U32 = re.compile(r"^\+?[0-9]+$")
_F32 = re.compile(r"^[+-]?(inf|infinity|nan|([0-9]+(\.[0-9]*)?|\.[0-9]+)([eE][+-]?[0-9]+)?)$", re.I)


def _u32(s: str):
    if not _U32.match(s):
        return None
    v = int(s)
    return v if v < 2 ** 32 else None


def _f32(s: str):
    if not _F32.match(s):
        return None
    return np.float32(float(s))


def parse_libsvm(text: str, feature_dim: int, num_labels: int):
    """(examples, feature_dim, num_labels) with examples a list of
    (indices uint32, values float32, labels list); raises ValueError with the
    reference's message on a malformed line."""
    raw = []
    min_idx, has_zero = None, False
    for line_no, line in enumerate(text.split("\n")):
        line = line.strip()
        if not line or line.startswith("#"):
            continue
        toks = line.split()
        labels = []
        for s in toks[0].split(","):
            v = _u32(s)
            if v is None:
                raise ValueError(f"line {line_no + 1}: invalid label '{s}'")
            labels.append(v)
        feats = []
        for t in toks[1:]:
            if t.startswith("#"):
                break
            if ":" not in t:
                raise ValueError(f"line {line_no + 1}: expected 'index:value', got '{t}'")
            a, b = t.split(":", 1)
            ix = _u32(a)
            if ix is None:
                raise ValueError(f"line {line_no + 1}: invalid feature index '{a}'")
            v = _f32(b)
            if v is None:
                raise ValueError(f"line {line_no + 1}: invalid feature value '{b}'")
            has_zero |= ix == 0
            min_idx = ix if min_idx is None else min(min_idx, ix)
            feats.append((ix, v))
        raw.append((labels, feats))
    offset = 1 if (not has_zero and min_idx == 1) else 0
    out = []
    for labels, feats in raw:
        pairs = [(min(ix - offset, feature_dim - 1), v) for ix, v in feats]
        pairs.sort(key=lambda p: p[0])  # stable
        idx, val = [], []
        for i, v in pairs:
            if idx and idx[-1] == i:
                val[-1] = np.float32(val[-1] + v)
                continue
            idx.append(i)
            val.append(np.float32(v))
        out.append((np.asarray(idx, np.uint32), np.asarray(val, np.float32), labels))
    return out, feature_dim, num_labels
