"""Training contracts: ZeRO table, execution / input plans, update windows, task and payload schemas (CPU)."""
import pytest

from flare_b200.training.contracts import (
    EvaluationEnvelope,
    OptimizerUpdateWindow,
    PayloadField,
    PayloadSchema,
    TrainingExecutionPlan,
    TrainingStateBlueprint,
    ZeroExecutionPolicy,
    ZeroStage,
    resolve_training_input_plan,
    zero_partition_contract,
)
from flare_b200.training.precision import PrecisionPolicy


def test_zero_contract_table():
    c = zero_partition_contract(ZeroStage.GRADIENT)
    assert (c.parameter_partition, c.optimizer_state_partition, c.gradient_partition) == (
        "replicated", "sharded", "sharded")
    assert (c.gradient_collective, c.parameter_collective) == ("reduce-scatter", "all-gather")
    assert zero_partition_contract(ZeroStage.OPTIMIZER_STATE).gradient_collective == "all-reduce"
    assert zero_partition_contract(ZeroStage.PARAMETER).parameter_partition == "sharded"
    with pytest.raises(TypeError):
        zero_partition_contract(2)
    with pytest.raises(ValueError):
        ZeroExecutionPolicy(ZeroStage.REPLICATED, shard_scope="node")


def test_update_window_roundtrip_and_validation():
    w = OptimizerUpdateWindow(2, 2, True, True, 7)
    assert OptimizerUpdateWindow.decode(w.encode()) == w
    with pytest.raises(ValueError):
        OptimizerUpdateWindow(1, 2, True, False, 0)
    with pytest.raises(ValueError):
        OptimizerUpdateWindow(1, 2, False, True, 0)
    with pytest.raises(ValueError):
        OptimizerUpdateWindow.decode([1, 2, 3])
    with pytest.raises(ValueError):
        OptimizerUpdateWindow.decode([1, 1, 2, 0, 0])


def test_input_plan():
    p = resolve_training_input_plan(reader_repeat_first_batch=False, latest_checkpoint_step=None, run_steps=10,
                                    target_step=10, checkpoint_interval_steps=5)
    assert p.mode == "manifest" and p.checkpoint_enabled and p.checkpoint_reason == "scheduled"
    p = resolve_training_input_plan(reader_repeat_first_batch=True, latest_checkpoint_step=None, run_steps=10,
                                    target_step=7, checkpoint_interval_steps=50)
    assert p.mode == "repeat_first_batch" and p.source_epochs == 7 and not p.checkpoint_enabled
    with pytest.raises(ValueError):
        resolve_training_input_plan(reader_repeat_first_batch=True, latest_checkpoint_step=3, run_steps=10,
                                    target_step=7, checkpoint_interval_steps=5)


def test_plans_schema_precision():
    plan = TrainingExecutionPlan.sharded(ZeroStage.GRADIENT, micro_steps=4, sync_mode="micro")
    assert plan.accumulation.micro_steps == 4 and plan.zero.stage is ZeroStage.GRADIENT
    with pytest.raises(ValueError):
        PayloadSchema("p", (PayloadField("a", "int32", (None,)), PayloadField("a", "int32", (None,))))
    with pytest.raises(ValueError):
        TrainingStateBlueprint(("g",), (("x", (1,), "float32", "param"), ("x", (1,), "float32", "param")), "d")
    env = EvaluationEnvelope.from_metadata(payload=1, request_id="r", schema_id="s", metadata={"k": 1})
    assert env.metadata["k"] == 1
    assert PrecisionPolicy.BF16.gradient_transport_dtype.is_floating_point
    assert PrecisionPolicy.BF16.sparse_storage_dtype_name == "float16"
    assert PrecisionPolicy.FP32.sparse_gradient_transport_dtype_name == "float32"


def _host_model(pipelined, staleness=1, accum=1):
    from types import SimpleNamespace

    from flare_b200.models.dlrm import DLRM

    m = object.__new__(DLRM)  # no CUDA: only the host-side bookkeeping is exercised
    m.pipelined, m.staleness, m.accum = pipelined, staleness if pipelined else 0, accum
    m._next_slot, m.pending = 0, []
    m.dense, m.emb = SimpleNamespace(step=0), SimpleNamespace(step=0, _slot=0, micro_filled=0, _micro=0)
    return m


def test_pipelined_host_state_machine_without_cuda():
    """Graph keys, capture snapshot / restore and replay advance of the fused DLRM's host state."""
    s = _host_model(False)
    assert s.graph_key() == 0
    s.advance_host_state()
    assert (s.dense.step, s.emb.step) == (1, 1)

    p = _host_model(True)
    assert p.graph_key() is None  # the first step has no pending update: eager, never captured
    p._next_slot, p.pending, p.emb._slot = 1, [0], 0  # after one eager step on slot 0
    keys = []
    for _ in range(4):
        keys.append(p.graph_key())
        snap = p.host_state()
        p._next_slot, p.pending, p.dense.step = 9, [9], 99  # what a capture may leave behind
        p.restore_host_state(snap)
        p.advance_host_state()
    assert keys == [(1, (0,)), (0, (1,)), (1, (0,)), (0, (1,))]  # two graphs, alternating
    assert (p.dense.step, p.emb.step, p.emb._slot, p._next_slot, p.pending_slot) == (4, 4, 0, 1, 0)


def test_pipeline_of_depth_two_host_state_machine_without_cuda():
    """Staleness 2: two updates in flight, three slots in rotation, three graph keys."""
    p = _host_model(True, staleness=2)
    assert p.graph_key() is None
    p._next_slot, p.pending = 2, [0, 1]  # after two eager steps on slots 0 and 1
    keys = []
    for _ in range(6):
        keys.append(p.graph_key())
        p.advance_host_state()
    assert keys == [(2, (0, 1)), (0, (1, 2)), (1, (2, 0))] * 2
    assert (p.dense.step, p.emb.step, p._next_slot, p.pending) == (6, 6, 2, [0, 1])


def test_accumulation_window_host_state_machine_without_cuda():
    """A window of 3 micro-steps: one graph per position, optimizer steps only when the window closes."""
    m = _host_model(False, accum=3)
    keys, steps = [], []
    for _ in range(7):
        keys.append(m.graph_key())
        snap = m.host_state()
        m.emb.micro_filled, m.dense.step = 2, 50  # what a capture may leave behind
        m.restore_host_state(snap)
        m.advance_host_state()
        steps.append((m.dense.step, m.emb.step, m.emb.micro_filled, m.emb._micro))
    assert keys == [("micro", 0), ("micro", 1), ("micro", 2)] * 2 + [("micro", 0)]
    assert steps == [(0, 0, 1, 0), (0, 0, 2, 1), (1, 1, 0, 2), (1, 1, 1, 0), (1, 1, 2, 1), (2, 2, 0, 2),
                     (2, 2, 1, 0)]
