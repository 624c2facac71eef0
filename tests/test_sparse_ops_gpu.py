"""Padded-inverse sparse operator kernels and GPU dedup vs CPU references."""
import pytest
import torch

from flare_b200.ops.sparse import (
    CpuSparseEmbeddingOperator,
    CudaSparseEmbeddingOperator,
    unique_first_occurrence,
    unique_first_occurrence_reference,
)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_padded_gather_scatter(cuda, dtype):
    torch.manual_seed(0)
    rows, dim, B, F, E, pad = 50, 16, 8, 3, 4, 50
    emb = torch.randn(rows, dim).to(dtype)
    inv = torch.randint(0, rows + 1, (B * F * E,), dtype=torch.int32)
    cpu = CpuSparseEmbeddingOperator("float32" if dtype == torch.float32 else "float16")
    gpu = CudaSparseEmbeddingOperator("float32" if dtype == torch.float32 else "float16")
    with gpu.execution_context():
        g1 = gpu.gather(emb.to(cuda), inv.to(cuda), B, dim, pad)
        g2 = gpu.gather_pooled(emb.to(cuda), inv.to(cuda), B, dim, (F, E), pad)
        grad = torch.randn(B * F * E, dim)
        s1 = gpu.scatter(rows, dim, inv.to(cuda), pad, grad.to(cuda))
        pg = torch.randn(B, F, dim)
        s2 = gpu.scatter_pooled(rows, dim, inv.to(cuda), pad, pg.to(cuda), (F, E))
    torch.testing.assert_close(g1.cpu(), cpu.gather(emb, inv, B, dim, pad))
    torch.testing.assert_close(g2.cpu().float(), cpu.gather_pooled(emb, inv, B, dim, (F, E), pad).float(),
                               rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(s1.cpu(), cpu.scatter(rows, dim, inv, pad, grad), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(s2.cpu(), cpu.scatter_pooled(rows, dim, inv, pad, pg, (F, E)), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n", [1, 17, 100000])
def test_unique_first_occurrence(cuda, n):
    torch.manual_seed(1)
    keys = torch.randint(-50, 500, (n,), dtype=torch.int64)
    u, inv, first = unique_first_occurrence(keys.to(cuda))
    ru, rinv, rfirst = unique_first_occurrence_reference(keys)
    assert torch.equal(u.cpu(), ru) and torch.equal(inv.cpu(), rinv) and torch.equal(first.cpu(), rfirst)


def test_unique_first_occurrence_high_bit_keys(cuda):
    """Keys that differ only above bit 32 (a table tag packed into the high bits) hash apart."""
    import time

    keys = (torch.arange(4096, dtype=torch.int64) % 1024) << 32
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    u, inv, first = unique_first_occurrence(keys.to(cuda))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    ru, rinv, rfirst = unique_first_occurrence_reference(keys)
    assert torch.equal(u.cpu(), ru) and torch.equal(inv.cpu(), rinv) and torch.equal(first.cpu(), rfirst)
