"""Fused multitask-layer kernels against plain PyTorch fp32: gate mixing (forward and backward),
ReLU backward with bias-gradient column sums, and the one-node ReLU MLP on the tcgen05 GEMM."""
import pytest
import torch

from flare_b200.models.layers import MLP
from flare_b200.ops.mixing import gate_mix, gate_mix_supported, relu_bwd_colsum_

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,E,D", [(1, 3, 8), (37, 16, 64), (1000, 24, 128), (257, 64, 512), (64, 5, 1024)])
def test_gate_mix_matches_fp32_autograd(cuda, B, E, D):
    torch.manual_seed(B + E + D)
    logits = (torch.randn(B, E, device=cuda) * 2).to(torch.bfloat16)
    ys = [torch.randn(B, D, device=cuda).to(torch.bfloat16) for _ in range(E)]
    assert gate_mix_supported(logits, ys)
    lg = logits.detach().clone().requires_grad_(True)
    yy = [y.detach().clone().requires_grad_(True) for y in ys]
    out = gate_mix(lg, yy)
    dout = torch.randn(B, D, device=cuda).to(torch.bfloat16)
    out.backward(dout)

    lr = logits.double().requires_grad_(True)
    yr = [y.double().requires_grad_(True) for y in ys]
    ref = (torch.stack(yr, -1) * torch.softmax(lr, -1).unsqueeze(1)).sum(-1)
    ref.backward(dout.double())
    torch.testing.assert_close(out.double(), ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(lg.grad.double(), lr.grad, rtol=2e-2, atol=2e-2)
    for a, b in zip(yy, yr):
        torch.testing.assert_close(a.grad.double(), b.grad, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("rows,cols", [(1000, 136), (4096, 128), (37, 8), (3000, 1040)])
def test_relu_bwd_colsum(cuda, rows, cols):
    torch.manual_seed(0)
    g = torch.randn(rows, cols, device=cuda).to(torch.bfloat16)
    h = torch.relu(torch.randn(rows, cols, device=cuda)).to(torch.bfloat16)
    out = torch.empty_like(g)
    cs = torch.full((cols,), 0.5, device=cuda)
    relu_bwd_colsum_(g, h, out, cs)
    want = torch.where(h > 0, g, torch.zeros_like(g))
    torch.testing.assert_close(out, want, rtol=0, atol=0)
    torch.testing.assert_close(cs, 0.5 + want.float().sum(0), rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("last_act", [True, False])
def test_relu_mlp_one_node_matches_fp32(cuda, last_act):
    """The one-node ReLU MLP against an fp64 reference that rounds activations and hidden gradients
    to bf16 where the kernels store them (so both take the same ReLU masks)."""
    torch.manual_seed(1)
    mlp = MLP(64, [128, 256, 32], activate="relu", last_layer_use_activate=last_act).to(cuda)
    x = torch.randn(300, 64, device=cuda).to(torch.bfloat16).requires_grad_(True)
    y = mlp(x)
    assert y.grad_fn is not None and "TcReluMLP" in type(y.grad_fn).__name__
    gy = torch.randn_like(y)
    y.backward(gy)

    bf = lambda t: t.to(torch.bfloat16).double()  # noqa: E731
    W = [bf(l.weight) for l in mlp.layers]
    b = [bf(l.bias) for l in mlp.layers]
    hs = [x.detach().double()]
    for i in range(3):
        pre = hs[-1] @ W[i].t() + b[i]
        hs.append(bf(torch.relu(pre) if i < 2 or last_act else pre))
    torch.testing.assert_close(y.double(), hs[-1], rtol=2e-2, atol=2e-2)
    g = gy.double()
    if last_act:
        g = bf(g * (hs[3] > 0))
    for i in reversed(range(3)):
        l = mlp.layers[i]
        torch.testing.assert_close(l.weight.grad.double(), g.t() @ hs[i], rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(l.bias.grad.double(), g.sum(0), rtol=1e-2, atol=1e-2)
        dx = g @ W[i]
        if i > 0:
            g = bf(dx * (hs[i] > 0))
        else:
            torch.testing.assert_close(x.grad.double(), dx, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("shared_input", [True, False])
def test_ple_stacked_experts_match_fp64_eager(cuda, shared_input):
    """PLE with single-layer ReLU experts: one stacked GEMM per shared input (+ fused gate mixing) on
    bf16 CUDA inputs against the same module's eager path in fp64 on the CPU."""
    import copy

    from flare_b200.models.layers import PLE

    torch.manual_seed(3)
    ple = PLE(64, 64, 4, [32], 3).to(cuda)
    assert ple.stackable
    ref = copy.deepcopy(ple).cpu().double()
    with torch.no_grad():
        for p, q in zip(ple.parameters(), ref.parameters()):
            q.copy_(p.to(torch.bfloat16).double())
    xs = [torch.randn(200, 64, device=cuda).to(torch.bfloat16) for _ in range(3)]
    if shared_input:
        xs = [xs[0]] * 3
    xs = [x.requires_grad_(True) if i == 0 else x for i, x in enumerate(xs)]
    outs = ple(xs, xs[0])
    gys = [torch.randn_like(o) for o in outs]
    torch.autograd.backward(outs, gys)
    xr = [x.detach().double().cpu().requires_grad_(True) for x in xs]
    if shared_input:
        xr = [xr[0]] * 3
    outs_r = ref(xr, xr[0])
    torch.autograd.backward(outs_r, [g.double().cpu() for g in gys])
    for o, r in zip(outs, outs_r):
        torch.testing.assert_close(o.double().cpu(), r, rtol=3e-2, atol=3e-2)

    def close(a, b, tol=4e-2):
        err = (a.double().cpu() - b).abs() - tol * (1 + b.abs())
        assert (err > 0).double().mean() < 5e-3 and bool((err < 10 * tol * (1 + b.abs())).all()), err.max()

    close(xs[0].grad, xr[0].grad)
    for (n, p), (_, q) in zip(ple.named_parameters(), ref.named_parameters()):
        close(p.grad, q.grad)
