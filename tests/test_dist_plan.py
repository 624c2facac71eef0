"""Host-side scheduling of the distributed GEMM: tile and chunk orders (CPU)."""
from flare_b200.ops.dist_gemm import BM, BN, chunk_order, tile_order


def _g(nranks, my, S, chunk=128):
    return {"nranks": nranks, "my": my, "rows_per_rank": S, "chunk_rows": chunk}


def test_tile_order_covers_every_tile_once_local_rows_first():
    M, N = 4 * 256, 3 * BN
    ga = _g(4, 2, 256)
    order = tile_order(M, N, ga=ga)
    assert sorted(order) == sorted((mt << 16) | nt for mt in range(M // BM) for nt in range(N // BN))
    first_rows = {(t >> 16) * BM // 256 for t in order[: (256 // BM) * (N // BN)]}
    assert first_rows == {2}  # this rank's rows come first
    owners = [(t >> 16) * BM // 256 for t in order]
    dist = [(o - 2) % 4 for o in owners]
    assert dist == sorted(dist)


def test_tile_order_reduce_scatter_sends_first():
    M, N = 2 * 512, 2 * BN
    rs = {"nranks": 2, "my": 0, "rows_per_rank": 512}
    order = tile_order(M, N, rs=rs)
    owners = [(t >> 16) * BM // 512 for t in order]
    assert owners[: len(order) // 2] == [1] * (len(order) // 2)
    assert owners[len(order) // 2:] == [0] * (len(order) // 2)


def test_chunk_order_only_remote_nearest_first():
    ga = _g(4, 1, 256, 64)
    gb = _g(2, 0, 512, 128)
    gb["pieces"] = 3
    items = [c & 0xFFFFFFFF for c in chunk_order(ga, gb)]
    a = [(c >> 12) & 0x7FFFF for c in items if c >> 31 == 0]
    b = [((c >> 12) & 0x7FFFF, c & 0xFFF) for c in items if c >> 31 == 1]
    per_a = 256 // 64
    assert a == list(range(2 * per_a, 3 * per_a)) + list(range(3 * per_a, 4 * per_a)) + list(range(0, per_a))
    assert b == [(c, k) for c in range(4, 8) for k in range(3)]
    assert chunk_order(None, None) == []


def test_piece_split_covers_chunk():
    from flare_b200.ops.dist_gemm import _pieces

    for rows, cols in ((128, 6669), (64, 512), (128, 4096), (2, 8), (128, 65536)):
        n, per = _pieces(rows, cols)
        assert n <= 4096 and n * per >= rows * ((cols + 7) // 8) > (n - 1) * per
