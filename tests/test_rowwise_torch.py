"""Plain-PyTorch row-wise Adagrad (the oracle / baseline optimizer) vs the CPU reference collection."""
import torch
import torch.nn as nn

from flare_b200.models.dlrm import RowwiseAdagradTorch
from flare_b200.sparse.config import SparseOptimizerConfig, SparseTableSpec
from flare_b200.sparse.reference import CpuEmbeddingBagCollection


def test_rowwise_adagrad_torch_matches_reference_collection():
    torch.manual_seed(0)
    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05, weight_decay=0.01)
    t = SparseTableSpec("t", 40, 8, optimizer=opt)
    B = 16
    ref = CpuEmbeddingBagCollection([t], B, optimizer=opt, seed=3)
    emb = nn.EmbeddingBag(40, 8, mode="sum", sparse=True)
    with torch.no_grad():
        emb.weight.copy_(ref.weights[0])
    ro = RowwiseAdagradTorch([emb.weight], lr=0.05, eps=opt.eps, weight_decay=0.01)
    for step in range(1, 4):
        lens = torch.randint(0, 5, (B,))
        ids = torch.randint(0, 40, (int(lens.sum()),))
        offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.cumsum(0)])
        ref.set_input(offs.int(), ids.int())
        ref.forward()
        g = torch.randn(B, 8)
        ref.backward(g, step)
        ro.zero_grad()
        out = emb(ids, offs[:-1])
        out.backward(g)
        ro.step()
        torch.testing.assert_close(emb.weight.detach(), ref.weights[0], rtol=1e-5, atol=1e-6)
