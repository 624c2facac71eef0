"""Jagged causal attention (tcgen05) vs the fp32 PyTorch reference, forward and backward."""
import math

import pytest
import torch

from flare_b200.ops.attention import (DMODEL, AttentionBuffers, jagged_attention_backward, jagged_attention_forward,
                                      jagged_attention_reference, pack_offsets)

pytestmark = pytest.mark.gpu


def _setup(cuda, lengths, seed=0):
    torch.manual_seed(seed)
    offs, _ = pack_offsets(lengths)
    T_cap = (int(offs[-1]) + 127) // 128 * 128 + 128
    buf = AttentionBuffers(T_cap, cuda)
    buf.qkv.copy_(torch.randn(T_cap, 3 * DMODEL, device=cuda).to(torch.bfloat16))
    buf.vt.copy_(buf.qkv[:, 2 * DMODEL:].t())
    buf.qt.copy_(buf.qkv[:, :DMODEL].t())
    return buf, offs.to(cuda), offs


def _rows(lengths):
    return torch.nonzero(pack_offsets(lengths)[1]).flatten()


@pytest.mark.parametrize("lengths", [[37, 128, 200, 1, 300, 512], [512] * 3, [129, 255, 384, 64, 8]])
def test_forward_matches_reference(cuda, lengths):
    buf, offs_d, offs = _setup(cuda, lengths)
    jagged_attention_forward(buf, offs_d, len(lengths), 512)
    torch.cuda.synchronize()
    buf.status.check("attention forward")
    ref = jagged_attention_reference(buf.qkv, offs)
    rows = _rows(lengths).to(cuda)
    torch.testing.assert_close(buf.out[rows].float(), ref[rows], rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("lengths", [[37, 128, 200, 1, 300, 512], [129, 255, 384, 64, 8]])
def test_backward_matches_autograd(cuda, lengths):
    buf, offs_d, offs = _setup(cuda, lengths, seed=1)
    jagged_attention_forward(buf, offs_d, len(lengths), 512)
    dout = torch.randn(buf.T_cap, DMODEL, device=cuda).to(torch.bfloat16)
    valid = torch.zeros(buf.T_cap, dtype=torch.bool, device=cuda)
    valid[_rows(lengths).to(cuda)] = True
    dout[~valid] = 0  # padding tokens carry no loss gradient
    buf.dout.copy_(dout)
    buf.dout_t.copy_(dout.t())
    jagged_attention_backward(buf, offs_d, len(lengths), 512)
    torch.cuda.synchronize()
    buf.status.check("attention backward")
    x = buf.qkv.float().clone().requires_grad_(True)
    ref = jagged_attention_reference(x, offs)
    rows = _rows(lengths).to(cuda)
    (ref * dout.float()).sum().backward()
    g = x.grad[rows]
    got = buf.dqkv[rows].float()
    for name, sl in (("dQ", slice(0, DMODEL)), ("dK", slice(DMODEL, 2 * DMODEL)), ("dV", slice(2 * DMODEL, None))):
        err = (got[:, sl] - g[:, sl]).norm() / g[:, sl].norm()
        assert err < 3e-2, f"{name} relative error {err:.3e}"
    assert float(buf.dq_acc.abs().max()) == 0.0  # workspace left zeroed for the next call
