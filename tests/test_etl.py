"""Native ETL kernels vs their NumPy references (CPU; needs the built extension)."""
import numpy as np
import pytest

etl = pytest.importorskip("flare_b200.data.etl")
try:
    from flare_b200._native import native

    native().etl
except Exception:  # pragma: no cover - extension not built in this environment
    pytest.skip("native extension not built", allow_module_level=True)


def _records(n, rng):
    lines = []
    for i in range(n):
        items = []
        if rng.random() < 0.9:
            items.append(f"7\x03{rng.integers(-5, 10**12)}")
        if rng.random() < 0.8:
            items.append(f"12\x03{rng.random() * 100:.4f}")
        if rng.random() < 0.7:
            k = rng.integers(1, 6)
            items.append("30\x03" + ",".join(str(x) for x in rng.integers(0, 1000, k)))
        items.append("99\x03ignored")
        if rng.random() < 0.1:
            items.append("7\x03notanumber")
        rng.shuffle(items)
        lines.append(f"user{i}\tctx\t" + "\x02".join(items))
    return ("\n".join(lines) + "\n").encode()


def test_scanner_matches_reference():
    rng = np.random.default_rng(0)
    data = _records(500, rng)
    sc = etl.RecordScanner([etl.FieldSpec(7), etl.FieldSpec(12, is_float=True), etl.FieldSpec(30, length=4)],
                           num_columns=3)
    a, va, na = sc.scan(data, 600)
    b, vb, nb = sc.scan_reference(data, 600)
    assert na == nb == 500
    for code in (7, 12, 30):
        np.testing.assert_array_equal(a[code], b[code])
        np.testing.assert_array_equal(va[code], vb[code])


def test_encoders_match_reference():
    rng = np.random.default_rng(1)
    v = rng.integers(-10, 2**62, 1000)
    v[::17] = etl.NULL
    np.testing.assert_array_equal(etl.hash_bucket(v, 1000, default_value=5), etl.hash_bucket_reference(v, 1000, 5))
    off = np.concatenate([[0], np.cumsum(rng.integers(0, 5, 200))])
    vals = rng.integers(-100, 10**9, off[-1])
    np.testing.assert_array_equal(etl.fnv1a_lists(vals, off), etl.fnv1a_lists_reference(vals, off))
    np.testing.assert_array_equal(etl.fnv1a_lists(vals, off, 997), etl.fnv1a_lists_reference(vals, off, 997))
    np.testing.assert_array_equal(etl.fnv1a_seeded(vals[:300], 12345), etl.fnv1a_seeded_reference(vals[:300], 12345))
    f = rng.normal(0, 10, 500).astype(np.float32)
    f[::11] = etl.NULL
    bounds = np.array([-5.0, 0.0, 2.5, 10.0], dtype=np.float32)
    np.testing.assert_array_equal(etl.bucketize(f, bounds), etl.bucketize_reference(f, bounds))
    np.testing.assert_array_equal(etl.pack_fids(v, 3), etl.pack_fids_reference(v, 3))
    ob = np.concatenate([[0], np.cumsum(rng.integers(0, 6, 200))])
    b = rng.integers(0, 50, ob[-1])
    a = rng.integers(0, 50, off[-1])
    np.testing.assert_array_equal(etl.intersect_lists(a, off, b, ob), etl.intersect_lists_reference(a, off, b, ob))


def test_arrow_row_parser_matches_reference():
    pa = pytest.importorskip("pyarrow")
    rng = np.random.default_rng(2)
    vocab = {"red": 1, "green": 2, "blue": 3}
    lines = []
    for i in range(300):
        items = []
        if rng.random() < 0.8:
            items.append(f"5\x03{rng.integers(-3, 10**9)}")
        if rng.random() < 0.8:
            items.append("8\x03" + ",".join(str(x) for x in rng.integers(0, 100, rng.integers(0, 6))))
        if rng.random() < 0.8:
            items.append(f"9\x03{rng.choice(['red', 'green', 'blue', 'mauve'])}")
        if rng.random() < 0.5:
            items.append(f"11\x03{rng.random():.5f},{rng.random():.5f}")
        lines.append(f"{rng.integers(0, 10**6)}\t{rng.choice(['ios', 'android', 'web'])}\t" + "\x02".join(items))
    parser = etl.ArrowRowParser(feature_column=2, fixed={5: (1, False), 11: (2, True)}, lists={8: False},
                                categories={9: (vocab, 0)}, direct={"uid": 0},
                                metadata={"os": (1, {"ios": 1, "android": 2}, 0)})
    col = pa.array(lines, type=pa.string()).slice(7)   # a slice exercises the offset handling
    got = parser.parse(col)
    want = parser.parse_reference(lines[7:])
    for c in (5, 11):
        np.testing.assert_array_equal(got["fixed"][c], want["fixed"][c])
    vals, offs = got["lists"][8]
    assert [list(vals[offs[i]:offs[i + 1]]) for i in range(len(offs) - 1)] == want["lists"][8]
    np.testing.assert_array_equal(got["categories"][9], want["categories"][9])
    np.testing.assert_array_equal(got["direct"]["uid"], want["direct"]["uid"])
    np.testing.assert_array_equal(got["metadata"]["os"], want["metadata"]["os"])
