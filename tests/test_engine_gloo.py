"""ZeRO stages / accumulation modes over 2 gloo ranks equal one rank on the global batch."""
import pytest
import torch
import torch.nn as nn

from flare_b200.testing.gloo import run_ranks
from flare_b200.training.contracts import TrainingExecutionPlan, ZeroStage
from flare_b200.training.engine import TrainEngine
from flare_b200.training.flat import DenseOptimizerConfig


def _model():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(7, 16), nn.ReLU(), nn.Linear(16, 1))


def _data(step, micro):
    g = torch.Generator().manual_seed(100 * step + micro)
    x = torch.randn(8, 7, generator=g)
    y = (torch.rand(8, 1, generator=g) < 0.5).float()
    return x, y


def _train(rank, world, stage, sync_mode, steps=3, micro=2):
    plan = TrainingExecutionPlan.sharded(ZeroStage(stage), micro_steps=micro, sync_mode=sync_mode)
    eng = TrainEngine(_model(), lambda o, y: nn.functional.binary_cross_entropy_with_logits(o, y), plan,
                      DenseOptimizerConfig(kind="adam", learning_rate=0.01), device=torch.device("cpu"))
    for s in range(steps):
        for m in range(micro):
            x, y = _data(s, m)
            n = x.shape[0] // world
            eng.micro_step_once(x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n])
    st = eng.capture_checkpoint_state()
    return {k: v.clone() for k, v in st["model_state"].items()}, st["step"]


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
@pytest.mark.parametrize("sync_mode", ["boundary", "micro"])
def test_zero_stages_match_single_rank(stage, sync_mode):
    ref, ref_step = _train(0, 1, stage, sync_mode)
    outs = run_ranks(_train, 2, stage, sync_mode)
    for params, step in outs:
        assert step == ref_step == 3
        for k in ref:
            torch.testing.assert_close(params[k], ref[k], rtol=1e-5, atol=1e-6)


def _ckpt_roundtrip(rank, world):
    plan = TrainingExecutionPlan.sharded(ZeroStage.GRADIENT, micro_steps=2)
    mk = lambda: TrainEngine(_model(), lambda o, y: nn.functional.binary_cross_entropy_with_logits(o, y), plan,  # noqa: E731
                             DenseOptimizerConfig(learning_rate=0.01), device=torch.device("cpu"))
    a = mk()
    x, y = _data(0, 0)
    a.micro_step_once(x, y)
    assert a.finalize_checkpoint_window()  # partial window applied before capture
    state = a.capture_checkpoint_state()
    b = mk()
    b.restore_checkpoint_state(state)
    for e in (a, b):
        for m in range(2):
            e.micro_step_once(*_data(1, m))
    sa, sb = a.capture_checkpoint_state(), b.capture_checkpoint_state()
    return max((sa["model_state"][k] - sb["model_state"][k]).abs().max().item() for k in sa["model_state"])


def test_checkpoint_roundtrip_sharded():
    diffs = run_ranks(_ckpt_roundtrip, 2)
    assert max(diffs) == 0.0


def _train_node(rank, world, stage, sync_mode, steps=3, micro=2):
    plan = TrainingExecutionPlan.sharded(ZeroStage(stage), micro_steps=micro, sync_mode=sync_mode, shard_scope="node")
    eng = TrainEngine(_model(), lambda o, y: nn.functional.binary_cross_entropy_with_logits(o, y), plan,
                      DenseOptimizerConfig(kind="adam", learning_rate=0.01), device=torch.device("cpu"), node_size=2)
    assert eng.shards == 2 and eng.master.numel() == (eng.padded if stage == 0 else eng.padded // 2)
    for s in range(steps):
        for m in range(micro):
            x, y = _data(s, m)
            n = x.shape[0] // world
            eng.micro_step_once(x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n])
    st = eng.capture_checkpoint_state()
    return {k: v.clone() for k, v in st["model_state"].items()}, st["step"], eng.checkpoint_layout()["shard_scope"]


@pytest.mark.parametrize("stage", [1, 2, 3])
def test_node_scope_zero_matches_single_rank(stage):
    """4 ranks as 2 nodes x 2: shards live inside a node, gradients are summed over all 4 ranks."""
    ref, ref_step = _train(0, 1, stage, "boundary")
    for params, step, scope in run_ranks(_train_node, 4, stage, "boundary"):
        assert step == ref_step == 3 and scope == "node"
        for k in ref:
            torch.testing.assert_close(params[k], ref[k], rtol=1e-5, atol=1e-6)


def _topology(rank, world, stage):
    from flare_b200.benchmarks.zero_topology import run

    return run(rank, world, stage=stage, node_size=2, steps=3, width=32, depth=2, batch=8)


@pytest.mark.parametrize("stage", [2, 3])
def test_zero_topology_benchmark_node_equals_global(stage):
    out = run_ranks(_topology, 4, stage)[0]
    assert out["max_param_diff_global_vs_node"] < 1e-6
    g, n = out["scopes"]["global"], out["scopes"]["node"]
    assert g["shards"] == 4 and n["shards"] == 2
    assert n["intra_node_bytes"] > 0 and g["intra_node_bytes"] == 0
    assert n["cross_node_bytes"] > 0 and g["ms_per_step"] > 0 and n["ms_per_step"] > 0


def _bn_model():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(7, 16), nn.BatchNorm1d(16), nn.ReLU(), nn.Linear(16, 1))


def _train_bn(rank, world, check):
    plan = TrainingExecutionPlan.sharded(ZeroStage(1), micro_steps=1)
    eng = TrainEngine(_bn_model(), lambda o, y: nn.functional.binary_cross_entropy_with_logits(o, y), plan,
                      DenseOptimizerConfig(learning_rate=0.01), device=torch.device("cpu"), check_replication=check)
    losses = []
    for s in range(3):
        x, y = _data(s, 0)
        n = x.shape[0] // world
        losses.append(float(eng.micro_step_once(x[rank * n:(rank + 1) * n], y[rank * n:(rank + 1) * n]).loss))
    st = eng.capture_checkpoint_state()
    bn = eng.model[1]
    return bn.running_mean.clone(), int(bn.num_batches_tracked), losses, st["buffers"]["1.running_mean"]


def test_buffers_are_averaged_and_replicated_and_loss_is_global():
    outs = run_ranks(_train_bn, 2, True)
    (m0, n0, l0, ck0), (m1, n1, l1, ck1) = outs
    torch.testing.assert_close(m0, m1)  # averaged running statistics, identical on both ranks
    assert n0 == n1 == 3 and l0 == l1  # replicated integer buffer (checked), loss reported as the global mean
    torch.testing.assert_close(ck0, m0)  # buffers are checkpoint state


def _sparse_contract(rank, world):
    """Two ranks, each with half the batch: summed normalised input gradients = the global-batch gradient."""
    torch.manual_seed(0)
    model = nn.Linear(4, 1)
    plan = TrainingExecutionPlan.sharded(ZeroStage(0), micro_steps=1)
    eng = TrainEngine(model, lambda o, y: nn.functional.mse_loss(o, y), plan, DenseOptimizerConfig(learning_rate=0.0),
                      device=torch.device("cpu"))
    g = torch.Generator().manual_seed(3)
    x, y = torch.randn(8, 4, generator=g), torch.randn(8, 1, generator=g)
    n = 8 // world
    pooled = x[rank * n:(rank + 1) * n].clone().requires_grad_(True)
    eng.micro_step_once(pooled, y[rank * n:(rank + 1) * n])
    return eng.input_gradients({"pooled": pooled})["pooled"]


def test_input_gradients_follow_the_sample_mean_contract():
    one = _sparse_contract(0, 1)
    parts = run_ranks(_sparse_contract, 2)
    torch.testing.assert_close(torch.cat(parts), one, rtol=1e-6, atol=1e-7)


class _WithConstant(nn.Module):
    def __init__(self, mutate: bool):
        super().__init__()
        from flare_b200.training.precision import register_constant

        self.lin = nn.Linear(7, 1)
        self.mutate = mutate
        register_constant(self, "table", torch.arange(7, dtype=torch.float32))

    def forward(self, x):
        if self.mutate:
            self.table.add_(1.0)
        return self.lin(x * self.table)


def test_constant_buffers_are_checked_and_fp32_islands_stay_fp32():
    from flare_b200.training.precision import Fp32Island, PrecisionPolicy, constant_buffers

    plan = TrainingExecutionPlan.replicated()
    x, y = _data(0, 0)
    for mutate in (False, True):
        m = _WithConstant(mutate)
        assert list(constant_buffers(m)) == ["table"]
        eng = TrainEngine(m, lambda o, t: nn.functional.binary_cross_entropy_with_logits(o, t), plan,
                          DenseOptimizerConfig(learning_rate=0.01), device=torch.device("cpu"), validate_constants=True)
        if mutate:
            with pytest.raises(RuntimeError, match="constant buffer table changed"):
                eng.micro_step_once(x, y)
        else:
            eng.micro_step_once(x, y)
            assert "table" in eng.capture_checkpoint_state()["buffers"]
    lin = nn.Linear(7, 3)
    island = Fp32Island(lin)
    with torch.autocast("cpu", dtype=PrecisionPolicy.bf16().compute_dtype):
        assert lin(x).dtype == torch.bfloat16 and island(x.bfloat16()).dtype == torch.float32
    torch.testing.assert_close(island(x), lin(x))
