"""Dense-tower kernels (interaction, fused head+BCE, optimizers, helpers) vs fp32 references."""
import pytest
import torch

from flare_b200.ops import dense as D
from flare_b200.training.flat import adam_reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,F,dim", [(64, 26, 128), (37, 4, 64), (16, 8, 256), (1001, 31, 128), (9, 32, 64)])
def test_interaction_fwd_bwd(cuda, B, F, dim):
    torch.manual_seed(0)
    W = D.interaction_out_width(F, dim)
    bot = torch.randn(B, dim).to(torch.bfloat16)
    emb = torch.randn(B, F * dim).to(torch.bfloat16)
    out_ref = torch.zeros(B, W, dtype=torch.bfloat16)
    D.interaction_forward(bot, emb, F, out_ref)
    out = torch.zeros(B, W, dtype=torch.bfloat16, device=cuda)
    D.interaction_forward(bot.to(cuda), emb.to(cuda), F, out)
    torch.testing.assert_close(out.cpu().float(), out_ref.float(), rtol=2e-2, atol=5e-2)
    dout = torch.randn(B, W).to(torch.bfloat16)
    dbot_r, demb_r = torch.empty(B, dim, dtype=torch.bfloat16), torch.empty(B, F * dim, dtype=torch.bfloat16)
    D.interaction_backward(dout, bot, emb, F, dbot_r, demb_r)
    dbot = torch.empty(B, dim, dtype=torch.bfloat16, device=cuda)
    demb = torch.empty(B, F * dim, dtype=torch.bfloat16, device=cuda)
    D.interaction_backward(dout.to(cuda), bot.to(cuda), emb.to(cuda), F, dbot, demb)
    torch.testing.assert_close(dbot.cpu().float(), dbot_r.float(), rtol=2e-2, atol=1e-1)
    torch.testing.assert_close(demb.cpu().float(), demb_r.float(), rtol=2e-2, atol=1e-1)


@pytest.mark.parametrize("B,H,T", [(1000, 256, 1), (64, 128, 3)])
def test_head_bce(cuda, B, H, T):
    torch.manual_seed(1)
    h = torch.relu(torch.randn(B, H)).to(torch.bfloat16)
    w = (torch.randn(T, H) * 0.1).to(torch.bfloat16)
    b = (torch.randn(T) * 0.1).to(torch.bfloat16)
    y = (torch.rand(B, T) < 0.3).float()
    outs = {}
    for dev in ("cpu", cuda):
        logits = torch.zeros(B, T, device=dev)
        loss = torch.zeros(1, device=dev)
        dh = torch.zeros(B, H, dtype=torch.bfloat16, device=dev)
        dw = torch.zeros(T, H, device=dev)
        db = torch.zeros(T, device=dev)
        D.head_bce(h.to(dev), w.to(dev), b.to(dev), y.to(dev), grad_scale=1.0 / B, logits=logits, loss_sum=loss,
                   dh=dh, dw=dw, db=db, valid_count=B - 5)
        outs[str(dev)] = [t.cpu().float() for t in (logits, loss, dh, dw, db)]
    ref, got = outs["cpu"], outs[str(cuda)]
    for r, g in zip(ref, got):
        torch.testing.assert_close(g, r, rtol=2e-2, atol=2e-3)


@pytest.mark.parametrize("kind", ["adam", "adamw", "sgd", "adagrad", "rmsprop"])
def test_dense_optimizer_flat(cuda, kind):
    from flare_b200.training.flat import DenseOptimizerConfig, DenseState, FlatParams

    torch.manual_seed(2)
    fp = FlatParams()
    fp.register("w", (37, 19), "normal", 0.1)
    fp.register("b", (19,), "normal", 0.1)
    cfg = DenseOptimizerConfig(kind=kind, learning_rate=0.01, weight_decay=0.01, momentum=0.9)
    st_gpu = DenseState(fp, cfg, device=cuda, seed=3)
    st_cpu = DenseState(fp, cfg, device=torch.device("cpu"), seed=3)
    for _ in range(3):
        g = torch.randn(st_cpu.n)
        st_cpu.grad.copy_(g)
        st_gpu.grad.copy_(g.to(cuda))
        st_cpu.apply(grad_scale=0.5)
        st_gpu.apply(grad_scale=0.5)
    torch.testing.assert_close(st_gpu.master.cpu(), st_cpu.master, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(st_gpu.compute.cpu().float(), st_cpu.master.to(torch.bfloat16).float())
    assert float(st_gpu.grad.abs().max()) == 0.0


def test_colsum_cast_init(cuda):
    torch.manual_seed(4)
    x = torch.randn(3000, 70).to(torch.bfloat16)
    out = torch.zeros(70, device=cuda)
    D.colsum_(x.to(cuda), out)
    torch.testing.assert_close(out.cpu(), x.float().sum(0), rtol=1e-4, atol=1e-3)
    xf = torch.randn(100, 13)
    y = torch.empty(100, 16, dtype=torch.bfloat16, device=cuda)
    D.cast_pad_bf16(xf.to(cuda), y)
    assert torch.equal(y.cpu()[:, :13], xf.to(torch.bfloat16)) and float(y[:, 13:].abs().max()) == 0
    t = torch.empty(10001, device=cuda)
    D.init_uniform_(t, -0.01, 0.01, seed=7, index_offset=5)
    ref = D.uniform_reference(10001, -0.01, 0.01, 7, 5)
    torch.testing.assert_close(t.cpu(), ref, rtol=0, atol=1e-8)
