"""The generic engine API on the fused path (one GPU): windows of micro-steps with the fused update at
the boundary track the eager fp32 TrainEngine; checkpoints round-trip; the factory picks the engine."""
import copy

import pytest
import torch
import torch.nn as nn

from flare_b200.models.layers import MLP
from flare_b200.training.contracts import TrainingExecutionPlan, ZeroStage
from flare_b200.training.engine import TrainEngine
from flare_b200.training.flat import DenseOptimizerConfig
from flare_b200.training.fused_engine import FusedTrainEngine, make_train_engine

pytestmark = pytest.mark.gpu


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.mlp = MLP(32, [64, 32], activate="relu")
        self.head = nn.Linear(32, 1)          # not a TcLinear: its gradient reaches the flat buffer by hook
        self.scale = nn.Parameter(torch.ones(1))

    def forward(self, x):
        h = self.mlp(x)
        return (self.head(h) * self.scale).squeeze(-1)


def _loss(out, y):
    return nn.functional.binary_cross_entropy_with_logits(out.float(), y)


def test_fused_engine_tracks_eager_engine(cuda):
    torch.manual_seed(0)
    net = Net()
    ref_net = copy.deepcopy(net).to(cuda)
    plan = TrainingExecutionPlan.replicated(micro_steps=2)
    opt = DenseOptimizerConfig(kind="adam", learning_rate=1e-2)
    fused = make_train_engine(net.to(cuda), _loss, plan, opt, device=cuda)
    assert isinstance(fused, FusedTrainEngine)
    ref = TrainEngine(ref_net, _loss, plan, opt, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(1)
    lf, lr = [], []
    for i in range(12):
        x = torch.randn(256, 32, device=cuda, generator=g)
        y = (x[:, 0] > 0).float()
        rf = fused.micro_step_once(x.to(torch.bfloat16), y)
        rr = ref.micro_step_once(x, y)
        assert rf.optimizer_applied == rr.optimizer_applied == (i % 2 == 1)
        lf.append(float(rf.loss))
        lr.append(float(rr.loss))
    assert fused.step == ref.step == 6
    for a, b in zip(lf, lr):
        assert abs(a - b) <= 0.03 * abs(b) + 3e-3, (lf, lr)
    assert sum(lf[-4:]) < sum(lf[:4])
    got = fused.capture_checkpoint_state()["model_state"]
    want = ref.capture_checkpoint_state()["model_state"]
    for n in want:
        diff = (got[n] - want[n]).abs()
        assert float(diff.max()) < 0.05, n  # bf16 compute vs fp32, six Adam steps of 1e-2

    # checkpoint round trip into a fresh engine
    other = FusedTrainEngine(copy.deepcopy(Net()).to(cuda), _loss, plan, opt, device=cuda)
    other.restore_checkpoint_state(fused.capture_checkpoint_state())
    back = other.capture_checkpoint_state()
    for n in got:
        assert torch.equal(back["model_state"][n], got[n])
    assert back["step"] == 6
    # a partial window is applied before a checkpoint
    x = torch.randn(256, 32, device=cuda, generator=g).to(torch.bfloat16)
    fused.micro_step_once(x, (x[:, 0] > 0).float())
    with pytest.raises(RuntimeError, match="boundary"):
        fused.capture_checkpoint_state()
    assert fused.finalize_checkpoint_window() and fused.step == 7


def test_factory_falls_back_to_the_eager_engine(cuda):
    opt = DenseOptimizerConfig(kind="adam", learning_rate=1e-3)
    e = make_train_engine(Net().to(cuda), _loss, TrainingExecutionPlan.sharded(ZeroStage.PARAMETER), opt, device=cuda)
    assert isinstance(e, TrainEngine)
    e = make_train_engine(Net(), _loss, TrainingExecutionPlan.replicated(), opt, device=torch.device("cpu"))
    assert isinstance(e, TrainEngine)
