"""Dense layer library vs explicit references (CPU); the tcgen05 linear layer on the GPU."""
import pytest
import torch

from flare_b200.models.layers import (CGC, MLP, PLE, UCGC, UPLE, BatchedExpertMoE, CategoricalEmbedding, NamedTokens,
                                      TcLinear, TokenMix, fp32_rms_normalize)


def test_mlp_and_gates_shapes():
    torch.manual_seed(0)
    mlp = MLP(8, [16, 4], last_layer_use_activate=False)
    assert mlp(torch.randn(3, 8)).shape == (3, 4)
    base = [torch.randn(5, 8) for _ in range(3)]
    gate = torch.randn(5, 6)
    assert [o.shape for o in PLE(8, 6, 2, [12, 4], 3)(base, gate)] == [(5, 4)] * 3
    assert [o.shape for o in CGC(8, 6, 2, [12, 4], 3)(base, gate)] == [(5, 4)] * 2
    assert len(UPLE(8, 6, 2, [4], 3)(base, [gate] * 3)) == 3
    assert len(UCGC(8, 6, 2, [4], 3)(base, [gate] * 3)) == 2


def test_token_mix_moe_named_tokens():
    torch.manual_seed(1)
    tm = TokenMix(4, 16, 2, hidden_dims=(32,))
    assert tm(torch.randn(3, 4, 16)).shape == (3, 16)
    for sparse in (False, True):
        moe = BatchedExpertMoE(2, 8, 2, 4, sparse, 2)
        y = moe(torch.randn(2, 5, 8))
        assert y.shape == (2, 5, 8) and torch.isfinite(y).all()
    nt = NamedTokens(["a", "b", "c"])
    assert nt.select(torch.arange(6).view(1, 3, 2), ["c", "a"]).tolist() == [[[4, 5], [0, 1]]]
    x = torch.randn(4, 8)
    assert torch.allclose(fp32_rms_normalize(x).pow(2).mean(-1), torch.ones(4), atol=1e-3)


def test_categorical_embedding_null_and_mean():
    emb = CategoricalEmbedding({"a": (10, 4), "b": (5, 4)}, {"a": (0, 2), "b": (2, 2)}, pooling="mean")
    side = torch.tensor([[1, 0, 3, 4]])  # a = [id 1, null], b = [3, 4]
    out = emb(side)[4]
    t = emb.tables["4"]
    assert out.shape == (1, 2, 4)
    assert torch.allclose(out[0, 0], t[1], atol=1e-6)  # null skipped, mean over one id
    off = emb.vocab_offsets["b"]
    assert torch.allclose(out[0, 1], (t[off + 3] + t[off + 4]) / 2, atol=1e-6)


@pytest.mark.gpu
def test_tclinear_matches_fp32_on_gpu(cuda):
    torch.manual_seed(2)
    lin = TcLinear(64, 128).to(cuda)
    x = torch.randn(256, 64, device=cuda).to(torch.bfloat16).requires_grad_(True)
    y = lin(x)
    y.float().sum().backward()
    xr = x.detach().float().requires_grad_(True)
    yr = torch.nn.functional.linear(xr, lin.weight.detach().to(torch.bfloat16).float(),
                                    lin.bias.detach().to(torch.bfloat16).float())
    yr.sum().backward()
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lin.weight.grad, (torch.ones(256, 128, device=cuda).t() @ xr.detach()), rtol=1e-2,
                               atol=1e-1)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=2e-2, atol=5e-2)


def _loop_mix(x, head_moe, token_moe, H):
    """One head-mix + token-mix layer written with explicit per-head / per-token concatenation."""
    B, T, D = x.shape
    hd = D // H
    heads = torch.stack([torch.cat([x[:, t, h * hd:(h + 1) * hd] for t in range(T)], -1) for h in range(H)])
    y = head_moe(heads)  # [H, B, T*hd]
    toks = torch.stack([torch.cat([y[h, :, t * hd:(t + 1) * hd] for h in range(H)], -1) for t in range(T)])
    return token_moe(toks).transpose(0, 1)  # [B, T, D]


def test_token_mix_large_moe_matches_loop_oracle():
    from flare_b200.models.layers import TokenMixLargeMoe, _head_major, _token_major

    torch.manual_seed(0)
    x = torch.randn(5, 4, 24)
    torch.testing.assert_close(_token_major(_head_major(x, 6), 4).transpose(0, 1), x)  # pure re-layout
    m = TokenMixLargeMoe(2, 4, 24, head_num=6, scale_size=2, num_experts=3, sparse=True, top_k=2)
    out = m(x)
    ref = x
    for i in range(2):
        ref = _loop_mix(ref, m.head_moe[i], m.token_moe[i], 6)
    torch.testing.assert_close(out, ref.mean(1), rtol=1e-5, atol=1e-5)
    out.sum().backward()
    assert all(p.grad is not None for p in m.parameters())


def test_token_mix_pre_gate_no_pool():
    from flare_b200.models.layers import TokenMixLargePreGateNoPool

    torch.manual_seed(1)
    with pytest.raises(ValueError):
        TokenMixLargePreGateNoPool(2, 4, 24, head_num=6, residual_enabled=True, residual_layers=(2,))
    m = TokenMixLargePreGateNoPool(2, 4, 24, head_num=6, scale_size=2, num_experts=2, residual_enabled=True,
                                   residual_layers=(1,))
    x = torch.randn(3, 4, 24)
    y = m(x)
    assert y.shape == x.shape
    torch.testing.assert_close(m(x, torch.ones(3, 48)), y)  # unit gates change nothing
    g = torch.rand(3, 48)
    yg = m(x, g)
    # the first gate scales layer 0's input; gating layer 0 by g0 equals feeding x * g0 ungated
    g2 = torch.cat([torch.ones(3, 24), g[:, 24:]], 1)
    torch.testing.assert_close(m(x * g[:, :24].unsqueeze(1), g2), yg)
    yg.pow(2).sum().backward()
    assert m.block_norms["1"].scale.grad is not None
