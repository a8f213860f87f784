"""LibSVM loader and batch iterator (klearu_b200/csrc/data.cu) against the
reference's own tests (crates/klearu-core/src/data/libsvm.rs:204-413,
dataset.rs:113-330) and the CPU restatement in oracle/data.py.  Host-only:
runs without a GPU."""

import numpy as np
import pytest

from klearu_b200.data import BatchIterator, DatasetError, Example, LibSvmDataset, SparseVector
from oracle import data as OD


def load(text, dim, nl, threads=0):
    return LibSvmDataset.load_from_str(text, dim, nl, threads)


def both(text, dim, nl, threads=0):
    """The native dataset and the oracle's parse of the same text."""
    return load(text, dim, nl, threads), OD.parse_libsvm(text, dim, nl)[0]


# ---- libsvm.rs tests, each on the native parser and the oracle ------------
def test_single_label_0based():  # libsvm.rs:216-233
    ds, o = both("0 0:1.0 2:3.5\n1 1:2.0\n", 4, 2)
    assert len(ds) == 2 and ds.feature_dim() == 4 and ds.num_labels() == 2
    e0, e1 = ds.get(0), ds.get(1)
    assert e0.labels == [0] and list(e0.features.indices) == [0, 2] and list(e0.features.values) == [1.0, 3.5]
    assert e1.labels == [1] and list(e1.features.indices) == [1] and list(e1.features.values) == [2.0]
    assert [list(x[0]) for x in o] == [[0, 2], [1]]


def test_single_label_1based_autodetect():  # libsvm.rs:235-249
    ds, o = both("0 1:1.0 3:2.0\n1 2:5.0\n", 4, 2)
    assert list(ds.get(0).features.indices) == [0, 2] and list(ds.get(0).features.values) == [1.0, 2.0]
    assert list(ds.get(1).features.indices) == [1]
    assert [list(x[0]) for x in o] == [[0, 2], [1]]


def test_multi_label():  # libsvm.rs:251-257
    ds, o = both("0,3,7 0:1.0 1:2.0\n", 5, 10)
    assert ds.get(0).labels == [0, 3, 7] and o[0][2] == [0, 3, 7]


def test_empty_features():  # libsvm.rs:259-266
    ds, _ = both("5\n", 10, 6)
    assert ds.get(0).labels == [5] and len(ds.get(0).features.indices) == 0


def test_blank_lines_and_comments():  # libsvm.rs:268-273
    ds, o = both("# This is a comment\n\n0 0:1.0\n   \n1 1:2.0\n", 5, 2)
    assert len(ds) == 2 and len(o) == 2


def test_inline_comment():  # libsvm.rs:275-281
    ds, _ = both("0 0:1.0 1:2.0 # this is a comment\n", 5, 2)
    assert len(ds.get(0).features.indices) == 2


def test_empty_file():  # libsvm.rs:283-289
    ds, o = both("", 10, 5)
    assert len(ds) == 0 and ds.is_empty() and o == []


@pytest.mark.parametrize("text,msg", [
    ("abc 0:1.0\n", "invalid label"),                 # libsvm.rs:291-298
    ("0 badformat\n", "expected 'index:value'"),      # libsvm.rs:300-307
    ("0 abc:1.0\n", "invalid feature index"),         # libsvm.rs:309-316
    ("0 0:not_a_number\n", "invalid feature value"),  # libsvm.rs:318-325
])
def test_invalid_lines(text, msg):
    with pytest.raises(DatasetError, match=msg):
        load(text, 10, 5)
    with pytest.raises(ValueError, match=msg):
        OD.parse_libsvm(text, 10, 5)


def test_from_examples():  # libsvm.rs:327-343
    ex = [Example(SparseVector.from_pairs(10, [(0, 1.0)]), [0]), Example(SparseVector.from_pairs(10, [(5, 2.0)]), [1])]
    ds = LibSvmDataset.from_examples(ex, 10, 2)
    assert len(ds) == 2 and ds.feature_dim() == 10 and ds.num_labels() == 2
    assert ds.get(0).labels == [0] and ds.get(1).labels == [1]


def test_dataset_trait_is_empty():  # libsvm.rs:345-349
    assert LibSvmDataset.from_examples([], 10, 5).is_empty()


def test_sparse_vector_dim_matches():  # libsvm.rs:351-356
    assert load("0 0:1.0 3:2.0\n", 100, 1).get(0).features.dim == 100


def test_mixed_0based_keeps_0based():  # libsvm.rs:358-365
    assert list(load("0 0:1.0 5:2.0\n", 10, 1).get(0).features.indices) == [0, 5]


def test_multiple_features_sorted():  # libsvm.rs:367-375
    e = load("0 3:1.0 1:2.0 0:3.0\n", 10, 1).get(0)
    assert list(e.features.indices) == [0, 1, 3] and list(e.features.values) == [3.0, 2.0, 1.0]


def test_large_feature_index_clamped():  # libsvm.rs:377-385
    e = load("0 0:1.0 999:2.0\n", 10, 1).get(0)
    assert list(e.features.indices) == [0, 9]


def test_negative_feature_values():  # libsvm.rs:387-393
    assert list(load("0 0:-1.5 2:3.0\n", 5, 1).get(0).features.values) == [-1.5, 3.0]


def test_many_labels():  # libsvm.rs:395-401
    assert load("0,1,2,3,4,5,6,7,8,9 0:1.0\n", 5, 10).get(0).labels == list(range(10))


# ---- native parser == oracle on generated files -----------------------------
def _gen_text(rng, n, dim, one_based, dups=True, extras=True):
    lines = []
    for i in range(n):
        r = rng.random()
        if extras and r < 0.03:
            lines.append("# comment line")
            continue
        if extras and r < 0.05:
            lines.append("   ")
            continue
        labs = ",".join(str(int(x)) for x in rng.integers(0, 1000, rng.integers(1, 5)))
        if extras and rng.random() < 0.1:
            labs = "+" + labs
        k = int(rng.integers(0, 30))
        ix = rng.integers(1 if one_based else 0, dim + (5 if extras else 0), k)
        if dups and k > 2:
            ix[-1] = ix[0]
        fmt = ["{:.6g}", "{:.3e}", "{}", "{:.9f}"]
        vals = [fmt[int(rng.integers(0, 4))].format(float(v)) for v in rng.standard_normal(k)]
        toks = [f"{a}:{b}" for a, b in zip(ix, vals)]
        tail = " # trailing" if extras and rng.random() < 0.1 else ""
        sep = "\t" if rng.random() < 0.2 else " "
        lines.append(labs + (sep + sep.join(toks) if toks else "") + tail)
    return "\r\n".join(lines) if rng.random() < 0.5 else "\n".join(lines) + "\n"


def _same(ds, o):
    assert len(ds) == len(o)
    for i, (oi, ov, ol) in enumerate(o):
        e = ds.get(i)
        assert e.labels == ol, i
        assert np.array_equal(np.asarray(e.features.indices), oi), i
        assert np.array_equal(np.asarray(e.features.values).view(np.uint32), ov.view(np.uint32)), i


@pytest.mark.parametrize("one_based", [False, True])
@pytest.mark.parametrize("threads", [1, 4])
def test_generated_files_match_oracle(one_based, threads):
    rng = np.random.default_rng(11 + one_based)
    text = _gen_text(rng, 3000, 500, one_based)
    ds, o = both(text, 500, 1000, threads)
    _same(ds, o)


def test_multi_chunk_parse_and_error_line():
    # > 1 MiB per chunk so that several threads parse; the error sits in a later chunk
    rng = np.random.default_rng(5)
    text = _gen_text(rng, 60000, 2000, False, extras=False)
    ds, o = both(text, 2000, 1000, 8)
    _same(ds, o)
    lines = text.split("\n")
    bad = len(lines) * 3 // 4
    lines[bad] = "7 12:0.5 13:oops"
    with pytest.raises(DatasetError, match=rf"^line {bad + 1}: invalid feature value 'oops'"):
        load("\n".join(lines), 2000, 1000, 8)


def test_file_load(tmp_path):
    p = tmp_path / "d.svm"
    p.write_text("1,2 1:0.5 4:1.5\n3 2:2.0\n")
    ds = LibSvmDataset.load(p, 8, 4)
    assert len(ds) == 2 and list(ds.get(0).features.indices) == [0, 3]
    with pytest.raises(DatasetError, match="cannot open"):
        LibSvmDataset.load(tmp_path / "missing.svm", 8, 4)


# ---- BatchIterator (dataset.rs) ---------------------------------------------
def _labelled(n, nl):
    return LibSvmDataset.from_examples([Example(SparseVector.from_pairs(100, [(i % 100, 1.0)]), [i % nl])
                                        for i in range(n)], 100, nl)


def _epoch(it):
    return [BatchIterator.as_host_batch(b) for b in it]


def _first_labels(batches):
    return [int(x) for hb in batches for x in hb.labels[hb.label_ptr[:-1]]]


@pytest.mark.parametrize("prefetch", [True, False])
def test_batch_order_matches_reference_shuffle(prefetch):
    n, bs = 37, 5
    ds = _labelled(n, n)
    for seed in (0, 42, 2 ** 63 + 5):
        got = _epoch(BatchIterator(ds, bs, seed, prefetch))
        want = OD.batch_order(n, bs, seed)
        assert [hb.batch for hb in got] == [len(b) for b in want]
        assert _first_labels(got) == [i for b in want for i in b]


def test_batch_iterator_covers_all_examples():  # dataset.rs:170-189
    b = _epoch(BatchIterator(_labelled(10, 5), 3, 42))
    assert [hb.batch for hb in b] == [3, 3, 3, 1]


def test_batch_iterator_exact_division_and_large_batch():  # dataset.rs:191-210
    assert [hb.batch for hb in _epoch(BatchIterator(_labelled(9, 3), 3, 0))] == [3, 3, 3]
    assert [hb.batch for hb in _epoch(BatchIterator(_labelled(5, 3), 100, 0))] == [5]
    assert _epoch(BatchIterator(_labelled(0, 3), 10, 0)) == []  # dataset.rs:212-218


def test_batch_iterator_reset():  # dataset.rs:253-300
    ds = _labelled(10, 10)
    it = BatchIterator(ds, 3, 42)
    e1 = _first_labels(_epoch(it))
    it.reset(99)
    e2 = _first_labels(_epoch(it))
    it.reset(42)
    e3 = _first_labels(_epoch(it))
    assert e1 != e2 and e1 == e3 and sorted(e1) == list(range(10))


def test_batch_csr_contents():
    rng = np.random.default_rng(3)
    text = _gen_text(rng, 500, 300, False, extras=False)
    ds, o = both(text, 300, 1000)
    for prefetch in (True, False):
        order = OD.batch_order(len(o), 64, 7)
        for hb, idxs in zip(_epoch(BatchIterator(ds, 64, 7, prefetch)), order):
            for s, e in enumerate(idxs):
                a, b = hb.rowptr[s], hb.rowptr[s + 1]
                assert np.array_equal(hb.idx[a:b], o[e][0]) and np.array_equal(hb.val[a:b], o[e][1])
                c, d = hb.label_ptr[s], hb.label_ptr[s + 1]
                assert list(hb.labels[c:d]) == o[e][2]


def test_c1_shaped_text_parses_back_to_the_generator_stream():
    """The loader bench's C1-shaped text (9 significant digits) parses back to
    the example stream it was written from, bit for bit; ids shift down by one
    only where the reference's 1-based detection fires (libsvm.rs:70-75: no
    id 0 and a minimum of 1)."""
    from klearu_b200.bench_loader import synthetic_text
    from klearu_b200.synthetic import XcGenerator

    n = 600
    ds = LibSvmDataset.load_from_str(synthetic_text(n, seed=3), 135909, 670091, 4)
    hb = XcGenerator(135909, 670091, seed=3).batch(n)
    assert len(ds) == n
    off = 1 if int(hb.idx.min()) == 1 else 0
    assert np.array_equal(np.asarray(ds.rowptr), hb.rowptr)
    assert np.array_equal(np.asarray(ds.idx), hb.idx - off)
    assert np.array_equal(np.asarray(ds.val).view(np.uint32), hb.val.view(np.uint32))
    assert np.array_equal(np.asarray(ds.label_ptr), hb.label_ptr)
    assert np.array_equal(np.asarray(ds.labels), hb.labels)
