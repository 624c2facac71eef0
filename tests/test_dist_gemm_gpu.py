"""Numerics of the persistent distributed tcgen05 GEMM (csrc/gemm_dist.cu) on one GPU.

The fused all-gather and reduce-scatter paths are exercised on one GPU by
standing in for the peer with local buffers: a "peer" full buffer holds the
rows the peer owns (the gather copies them like it would over NVLink), and for
the reduce-scatter the peer's partials and flags are written by the host
before the launch, so no launch ever waits for another launch.  The real
multi-GPU path is covered by the DCN-v2 equivalence test on 2 GPUs.
"""
import pytest
import torch

from flare_b200.ops.dist_gemm import BN, DistGemmContext, chunk_order, tile_order
from flare_b200.ops.gemm import gemm_reference

pytestmark = pytest.mark.gpu


class _Heap:
    """Minimal single-rank stand-in for SymmetricHeap (world 1)."""

    def __init__(self, device):
        self.rank, self.world_size, self.device = 0, 1, device
        self._keep = []

    def alloc(self, shape, dtype):
        from flare_b200.parallel.symm import SymBuffer

        t = torch.zeros(*shape, dtype=dtype, device=self.device)
        self._keep.append(t)
        return SymBuffer(t, 0, [t.data_ptr()])


def _rand(rows, cols, device, scale=1.0, ld=None):
    ld = ld or (cols + 7) // 8 * 8
    buf = torch.zeros(rows, ld, device=device)
    buf[:, :cols] = torch.randn(rows, cols, device=device) * scale
    return buf.to(torch.bfloat16)[:, :cols]


def _call(ctx, a, b, out, *, a_t=False, b_t=False, ga=None, gb=None, rs=None, bias=None, relu=False, mask=None,
          colsum=None, accumulate=False, epi=0, aux0=None, aux1=None, zout=None):
    from flare_b200._native import native

    M = a.shape[1] if a_t else a.shape[0]
    K = a.shape[0] if a_t else a.shape[1]
    N = b.shape[1] if b_t else b.shape[0]
    tiles = tile_order(M, N, ga=ga, gb=gb, rs=rs, a_mn=a_t, b_mn=b_t)
    chunks = chunk_order(ga, gb)
    tt = torch.tensor(tiles, dtype=torch.int32, device=out.device)
    ct = torch.tensor(chunks or [0], dtype=torch.int32, device=out.device)
    g = {"A": a.data_ptr(), "lda": a.stride(0), "a_mn": a_t, "B": b.data_ptr(), "ldb": b.stride(0), "b_mn": b_t,
         "M": M, "N": N, "K": K, "C": out.data_ptr(), "ldc": out.stride(0),
         "c_dtype": 0 if out.dtype == torch.float32 else 1, "accumulate": accumulate,
         "bias": bias.data_ptr() if bias is not None else 0, "act": 1 if relu else 0, "alpha": 1.0,
         "mask": mask.data_ptr() if mask is not None else 0, "ldm": mask.stride(0) if mask is not None else 0,
         "colsum": colsum.data_ptr() if colsum is not None else 0, "status": ctx.status.ptr,
         "timeout_ns": 2_000_000_000}
    d = {"g": g, "tiles": tt.data_ptr(), "num_tiles": len(tiles), "chunks": ct.data_ptr(), "num_chunks": len(chunks),
         "ga": ga, "gb": gb, "rs": rs, "epi": epi, **ctx.fields()}
    for name, t in (("aux0", aux0), ("aux1", aux1), ("zout", zout)):
        if t is not None:
            d[name] = t.data_ptr()
            d["ld" + {"aux0": "0", "aux1": "1", "zout": "z"}[name]] = t.stride(0)
    native().gemm_dist(d)
    torch.cuda.synchronize()
    ctx.check()
    return out


@pytest.fixture
def ctx(cuda):
    return DistGemmContext(_Heap(cuda))


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (384, 512, 320), (1000, 600, 336)])
def test_persistent_gemm_majors(ctx, cuda, a_t, b_t, M, N, K):
    torch.manual_seed(0)
    a = _rand(K, M, cuda) if a_t else _rand(M, K, cuda)
    b = _rand(K, N, cuda) if b_t else _rand(N, K, cuda)
    bias = (torch.randn(N, device=cuda)).to(torch.bfloat16)
    out = torch.empty(M, (N + 7) // 8 * 8, dtype=torch.bfloat16, device=cuda)[:, :N]
    _call(ctx, a, b, out, a_t=a_t, b_t=b_t, bias=bias, relu=True)
    ref = gemm_reference(a, b, a_t=a_t, b_t=b_t, bias=bias, relu=True)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=5e-2)


def test_persistent_gemm_epilogues(ctx, cuda):
    torch.manual_seed(1)
    M, N, K = 640, 768, 256
    a, b = _rand(M, K, cuda), _rand(N, K, cuda)
    ref = gemm_reference(a, b)
    mask = _rand(M, N, cuda)
    colsum = torch.zeros(N, device=cuda)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    _call(ctx, a, b, out, mask=mask, colsum=colsum)
    masked = torch.where(mask.float() > 0, ref, torch.zeros_like(ref))
    torch.testing.assert_close(out.float(), masked, rtol=2e-2, atol=5e-2)
    torch.testing.assert_close(colsum, masked.sum(0), rtol=1e-2, atol=0.5)
    acc = torch.full((M, N), 0.5, device=cuda)
    _call(ctx, a, b, acc, accumulate=True)
    torch.testing.assert_close(acc, 0.5 + ref, rtol=1e-3, atol=1e-2)
    # cross layer: z = acc + bias, out = x0 * z + xl
    bias = torch.randn(N, device=cuda).to(torch.bfloat16)
    x0, xl = _rand(M, N, cuda), _rand(M, N, cuda)
    z = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    out2 = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    _call(ctx, a, b, out2, bias=bias, epi=1, aux0=x0, aux1=xl, zout=z)
    zr = ref + bias.float()
    torch.testing.assert_close(z.float(), zr, rtol=2e-2, atol=5e-2)
    torch.testing.assert_close(out2.float(), x0.float() * zr + xl.float(), rtol=2e-2, atol=1e-1)
    # residual into fp32 accumulator
    acc2 = torch.ones(M, N, device=cuda)
    _call(ctx, a, b, acc2, accumulate=True, epi=2, aux1=xl)
    torch.testing.assert_close(acc2, 1 + ref + xl.float(), rtol=1e-3, atol=2e-2)


def _gather_spec(full_local, full_peer, my, S, cols, chunk_rows, ready):
    from flare_b200.ops.dist_gemm import _pieces

    src = [None, None]
    src[my] = full_local.data_ptr()
    src[1 - my] = full_peer.data_ptr()
    done = torch.zeros_like(ready)
    _KEEP.append(done)
    pieces, per = _pieces(chunk_rows, cols)
    return {"nranks": 2, "my": my, "src": src, "dst": full_local.data_ptr(), "ld": full_local.stride(0),
            "rows_per_rank": S, "row_elems": (cols + 7) // 8 * 8, "chunk_rows": chunk_rows,
            "pieces": pieces, "piece_vecs": per, "ready": ready.data_ptr(), "done": done.data_ptr()}


_KEEP = []


def _to_blocks(part, n_tiles):
    """[S, N] partial -> the reduce-scatter receive layout (per tile, quarter, 32-column chunk:
    element (r, 8q+e) of the 32 x 32 block at q*256 + r*8 + e)."""
    S, N = part.shape
    padded = torch.zeros(S, n_tiles * BN, dtype=part.dtype, device=part.device)
    padded[:, :N] = part
    x = padded.view(S // 128, 4, 32, n_tiles, 8, 4, 8)        # mt, quarter, r, nt, chunk, q, e
    x = x.permute(0, 3, 1, 4, 5, 2, 6).contiguous()           # mt, nt, quarter, chunk, q, r, e
    return x.view(-1)


def _from_blocks(flat, S, N, n_tiles):
    x = flat.view(S // 128, n_tiles, 4, 8, 4, 32, 8).permute(0, 2, 5, 1, 3, 4, 6).contiguous()
    return x.view(S, n_tiles * BN)[:, :N]


@pytest.mark.parametrize("my", [0, 1])
def test_gather_a_rows(ctx, cuda, my):
    """All-gather of A's rows (sequence-parallel activations) fused into the GEMM."""
    torch.manual_seed(2)
    S, K, N = 256, 200, 512
    full = _rand(2 * S, K, cuda)
    mine = full.clone()
    mine[(1 - my) * S:(2 - my) * S] = 0  # the peer's rows are not here yet
    peer = full.clone()
    peer[my * S:(my + 1) * S] = 0
    b = _rand(N, K, cuda)
    ready = torch.zeros(2 * S // 64, dtype=torch.int32, device=cuda)
    ga = _gather_spec(mine, peer, my, S, K, 64, ready)
    out = torch.empty(2 * S, N, dtype=torch.bfloat16, device=cuda)
    _call(ctx, mine, b, out, ga=ga)
    torch.testing.assert_close(mine.float(), full.float())
    torch.testing.assert_close(out.float(), gemm_reference(full, b), rtol=2e-2, atol=5e-2)


def test_gather_b_rows_and_mn_major_gather(ctx, cuda):
    """FSDP weight gather (B rows), and a gathered operand read MN-major (weight gradient)."""
    torch.manual_seed(3)
    S, K, M = 384, 136, 256
    wfull = _rand(2 * S, K, cuda)
    mine = wfull.clone()
    mine[S:] = 0
    peer = wfull.clone()
    peer[:S] = 0
    a = _rand(M, K, cuda)
    ready = torch.zeros(2 * S // 128, dtype=torch.int32, device=cuda)
    gb = _gather_spec(mine, peer, 0, S, K, 128, ready)
    out = torch.empty(M, 2 * S, dtype=torch.bfloat16, device=cuda)
    _call(ctx, a, mine, out, gb=gb)
    torch.testing.assert_close(out.float(), gemm_reference(a, wfull), rtol=2e-2, atol=5e-2)
    # dW = G^T X with G gathered by rows (rows are the K dimension here)
    G = _rand(2 * S, 256, cuda)
    X = _rand(2 * S, 192, cuda)
    gm = G.clone()
    gm[:S] = 0
    gp = G.clone()
    gp[S:] = 0
    ready2 = torch.zeros(2 * S // 128, dtype=torch.int32, device=cuda)
    ga = _gather_spec(gm, gp, 1, S, 256, 128, ready2)
    dw = torch.zeros(256, 192, device=cuda)
    _call(ctx, gm, X, dw, a_t=True, b_t=True, ga=ga)
    torch.testing.assert_close(dw, gemm_reference(G, X, a_t=True, b_t=True), rtol=1e-2, atol=0.2)


def test_reduce_scatter_rows(ctx, cuda):
    """GEMM -> reduce-scatter with the peer's partials pre-placed (and flagged) by the host."""
    torch.manual_seed(4)
    S, N, K = 256, 520, 192
    M = 2 * S
    a, b = _rand(M, K, cuda), _rand(N, K, cuda)
    bias = torch.randn(N, device=cuda).to(torch.bfloat16)
    my = 1
    n_tiles = (N + BN - 1) // BN
    tiles_per_rank = (S // 128) * n_tiles
    blk = tiles_per_rank * 4 * 8 * 1024
    recv_local = torch.zeros(2 * blk, dtype=torch.bfloat16, device=cuda)
    recv_peer = torch.zeros(2 * blk, dtype=torch.bfloat16, device=cuda)
    flags_local = torch.zeros(2 * tiles_per_rank * 8, dtype=torch.int32, device=cuda)
    flags_peer = torch.zeros_like(flags_local)
    peer_partial = _rand(S, N, cuda)  # what rank 0 computed for my rows
    recv_local[:blk] = _to_blocks(peer_partial, n_tiles)
    epoch = int(ctx.ctl[0].item()) + 1
    flags_local[:tiles_per_rank * 8] = epoch  # sender 0 -> all my tiles ready
    rs = {"nranks": 2, "my": my, "rows_per_rank": S, "recv_peer": [recv_peer.data_ptr(), recv_local.data_ptr()],
          "recv_local": recv_local.data_ptr(), "flag_peer": [flags_peer.data_ptr(), flags_local.data_ptr()],
          "flag_local": flags_local.data_ptr()}
    out = torch.empty(S, N, dtype=torch.bfloat16, device=cuda)
    _call(ctx, a, b, out, rs=rs, bias=bias, relu=True)
    full = gemm_reference(a, b)
    mine = torch.relu(full[my * S:(my + 1) * S] + peer_partial.float() + bias.float())
    torch.testing.assert_close(out.float(), mine, rtol=2e-2, atol=1e-1)
    # what was sent to rank 0: my partial of rank 0's rows, flagged
    sent_part = _from_blocks(recv_peer[my * blk:(my + 1) * blk], S, N, n_tiles)
    torch.testing.assert_close(sent_part.float(), full[:S], rtol=2e-2, atol=5e-2)
    sent = flags_peer[my * tiles_per_rank * 8:(my + 1) * tiles_per_rank * 8]
    assert bool((sent == epoch).all())


def test_block_layout_roundtrip(cuda):
    x = torch.randn(256, 520, device=cuda)
    assert torch.equal(_from_blocks(_to_blocks(x, 3), 256, 520, 3), x)
