import numpy as np
import pytest
import torch
from sklearn.metrics import roc_auc_score

from flare_b200.metrics.ranking import auc, auc_reference, calibration, gauc, gauc_reference


def test_auc_reference_matches_sklearn_with_ties():
    rng = np.random.default_rng(0)
    s = np.round(rng.random(5000), 2)  # many ties
    y = rng.random(5000) < 0.2
    assert abs(auc_reference(s, y) - roc_auc_score(y, s)) < 1e-12


def test_gauc_reference_weights():
    s = np.array([0.9, 0.1, 0.5, 0.5, 0.2, 0.8])
    y = np.array([1, 0, 1, 0, 0, 1])
    g = np.array([0, 0, 1, 1, 2, 2])
    # group 0 AUC 1, group 1 AUC 0.5 (tie), group 2 AUC 1; weights = positives
    assert abs(gauc_reference(s, y, g) - (1 + 0.5 + 1) / 3) < 1e-12
    assert abs(calibration(torch.tensor([0.5, 0.5]), torch.tensor([1.0, 0.0])) - 1.0) < 1e-12


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1000, 300_000])
def test_device_auc_and_gauc(cuda, n):
    g = torch.Generator().manual_seed(n)
    s = torch.round(torch.rand(n, generator=g) * 200) / 200  # ties
    y = (torch.rand(n, generator=g) < 0.1).float()
    grp = torch.randint(0, 500, (n,), generator=g)
    assert abs(auc(s.to(cuda), y.to(cuda)) - auc_reference(s.numpy(), y.numpy())) < 1e-9
    assert abs(gauc(s.to(cuda), y.to(cuda), grp.to(cuda), 0.25) -
               gauc_reference(s.numpy(), y.numpy(), grp.numpy(), 0.25)) < 1e-9


def test_train_metrics_window(tmp_path):
    from flare_b200.metrics.aggregation import JsonlSink, TrainMetricsWindow

    w = TrainMetricsWindow(window_steps=3, sinks=[JsonlSink(tmp_path / "m.jsonl")])
    g = torch.Generator().manual_seed(0)
    out = None
    for _ in range(3):
        y = (torch.rand(64, 1, generator=g) < 0.3).float()
        logits = (y * 2 - 1) + torch.randn(64, 1, generator=g)
        out = w.update(logits, y, loss_sum=torch.tensor(64 * 0.5))
    assert out is not None and out["train/auc_ctr"] > 0.75 and abs(out["train/loss"] - 0.5) < 1e-9
    assert (tmp_path / "m.jsonl").read_text().count("\n") == 1
