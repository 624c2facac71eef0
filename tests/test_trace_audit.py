"""Semantic trace audit and per-rank profiler helper (CPU); the traced fused step runs on the GPU."""
import pytest
import torch

from flare_b200.runtime.diagnostics import JsonlExecutionTracer
from flare_b200.utils.trace_audit import STAGES, audit_trace


def _write(dirpath, steps=2, nan_at=None, drop=None):
    tr = JsonlExecutionTracer(dirpath, rank=0)
    for st in range(steps):
        for stage in STAGES:
            if drop == (st, stage):
                continue
            f = {}
            if stage == "input_unique":
                f = dict(ids=100, values=torch.arange(100))
            elif stage == "sparse_lookup":
                x = torch.ones(4, 8)
                if nan_at == st:
                    x[1, 2] = float("nan")
                f = dict(pooled=x)
            elif stage == "sparse_update":
                f = dict(unique_rows=40, occurrences=100, heavy_rows=2)
            elif stage == "sparse_commit":
                f = dict(sparse_optimizer_step=st + 1, dense_optimizer_step=st + 1)
            tr.emit(stage, "step", step=st, **f)
    tr.close()


def test_audit_accepts_a_clean_trace_and_flags_problems(tmp_path):
    _write(tmp_path / "ok")
    rep = audit_trace(tmp_path / "ok")
    assert rep["ok"] and rep["steps"] == {0: 2}
    _write(tmp_path / "nan", nan_at=1)
    rep = audit_trace(tmp_path / "nan")
    assert not rep["ok"] and "NaN" in rep["problems"][0][0]
    _write(tmp_path / "gap", drop=(0, "module_update"))
    rep = audit_trace(tmp_path / "gap")
    assert not rep["ok"] and "missing stages ['module_update']" in rep["problems"][0][0]


def test_profile_steps_writes_a_trace_per_rank(tmp_path):
    from flare_b200.utils.profiling import profile_steps

    a = torch.randn(64, 64)
    rep = profile_steps(lambda: a @ a, steps=2, warmup=1, out_dir=tmp_path, rank=3)
    assert (tmp_path / "rank3.json").exists() and rep["steps"] == 2 and "categories" in rep


@pytest.mark.gpu
def test_traced_fused_step_passes_the_audit(cuda, tmp_path):
    from flare_b200.data.synthetic import DLRMSyntheticData
    from flare_b200.models.dlrm import DLRM, DLRMConfig, dlrm_benchmark_tables
    from flare_b200.sparse.config import SparseOptimizerConfig
    from flare_b200.utils.profiling import profile_steps

    opt = SparseOptimizerConfig(kind="rowwise_adagrad", learning_rate=0.05)
    vocabs = [200, 3000, 50]
    cfg = DLRMConfig(tables=dlrm_benchmark_tables(vocabs, 64, opt), bottom=(128, 64), top=(128, 64),
                     sparse_optimizer=opt)
    B = 256
    model = DLRM(cfg, B, max_bag_size=8, device=cuda, seed=1)
    data = DLRMSyntheticData(B, vocabs, max_bag=8, device=cuda, seed=2)
    tr = JsonlExecutionTracer(tmp_path / "trace", rank=0)
    for st in range(3):
        b = data.next()
        model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=False)
        model.traced_step(tr, st)
    tr.close()
    model.check()
    rep = audit_trace(tmp_path / "trace")
    assert rep["ok"], rep
    b = data.next()
    model.set_batch(b.dense, b.labels, b.offsets, b.values, non_blocking=False)
    prof = profile_steps(model.train_step, steps=2, warmup=1, out_dir=tmp_path / "prof", rank=0)
    assert prof["busy_us"] > 0 and "gemm" in prof["categories"]
