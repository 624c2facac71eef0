"""Exact AUC / GAUC / calibration: references vs sklearn, device kernels, distributed merge, metric windows."""
import math

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


def _samples(seed, n=3000, groups=17):
    g = torch.Generator().manual_seed(seed)
    y = (torch.rand(n, generator=g) < 0.35).float()
    # coarse scores so that many samples tie, inside a rank and across ranks
    s = torch.round(torch.sigmoid(y + torch.randn(n, generator=g)) * 64) / 64
    grp = torch.randint(0, groups, (n,), generator=g)
    return s, y, grp


def test_summary_merge_is_exact_for_any_split():
    from flare_b200.metrics.distributed import auc_from_summary, gauc_from_summary, merge_summaries, score_summary

    s, y, grp = _samples(3)
    ref_auc = auc_reference(s.numpy(), y.numpy())
    ref_gauc = gauc_reference(s.numpy(), y.numpy(), grp.numpy(), 0.5)
    for cuts in ([1000, 2000], [1, 2999], [1500]):
        bounds = [0, *cuts, s.numel()]
        parts = [score_summary(s[a:b], y[a:b], grp[a:b]) for a, b in zip(bounds[:-1], bounds[1:])]
        merged = merge_summaries(parts)
        assert merged.shape[0] < s.numel()  # ties collapsed into one key
        assert abs(auc_from_summary(merged) - ref_auc) < 1e-12
        assert abs(gauc_from_summary(merged, 0.5) - ref_gauc) < 1e-12
    one_class = score_summary(s[y > 0.5], y[y > 0.5])
    assert math.isnan(auc_from_summary(one_class))


def _dist_metrics(rank, world):
    from flare_b200.metrics.aggregation import TrainMetricsWindow
    from flare_b200.metrics.distributed import distributed_metrics

    s, y, grp = _samples(7, n=2400)
    n = s.numel() // world
    sl = slice(rank * n, (rank + 1) * n)
    m = distributed_metrics(s[sl], y[sl], grp[sl], negative_factor=0.25)
    # the window: 3 steps of this rank's share, logits whose sigmoid is the score
    w = TrainMetricsWindow(window_steps=3, capacity=n)
    wp = TrainMetricsWindow(window_steps=3, capacity=n, merge="partitioned")
    logits = torch.logit(s[sl].clamp(1e-6, 1 - 1e-6)).reshape(-1, 1)
    k = n // 3
    out = outp = None
    for i in range(3):
        part = slice(i * k, (i + 1) * k)
        out = w.update(logits[part], y[sl][part].reshape(-1, 1), loss_sum=float(rank + 1) * k)
        outp = wp.update(logits[part], y[sl][part].reshape(-1, 1), loss_sum=float(rank + 1) * k)
    assert abs(out["train/auc_ctr"] - outp["train/auc_ctr"]) < 1e-12  # the partitioned merge is exact too
    return m, out


def test_distributed_metrics_over_gloo_ranks():
    from flare_b200.testing.gloo import run_ranks

    s, y, grp = _samples(7, n=2400)
    ref_auc = auc_reference(s.numpy(), y.numpy())
    ref_gauc = gauc_reference(s.numpy(), y.numpy(), grp.numpy(), 0.25)
    ref_cal = float(s.double().sum() / y.double().sum())
    sc = torch.sigmoid(torch.logit(s.clamp(1e-6, 1 - 1e-6)))
    ref_window_auc = auc_reference(sc.numpy(), y.numpy())
    outs = run_ranks(_dist_metrics, 2)
    for m, out in outs:
        assert abs(m["auc"] - ref_auc) < 1e-12 and abs(m["gauc"] - ref_gauc) < 1e-12
        assert abs(m["calibration"] - ref_cal) < 1e-9
        assert abs(out["train/auc_ctr"] - ref_window_auc) < 1e-5  # sigmoid of a slice may differ by an ulp
        assert abs(out["train/loss"] - 1.5) < 1e-12  # (1 * 1200 + 2 * 1200) / 2400
    assert outs[0][1]["train/auc_ctr"] == outs[1][1]["train/auc_ctr"]


class _ListSink:
    def __init__(self):
        self.rows = []

    def write(self, step, metrics):
        self.rows.append((step, metrics))


def test_background_windows_match_synchronous_and_stay_bounded():
    from flare_b200.metrics.aggregation import TrainMetricsWindow

    g = torch.Generator().manual_seed(5)
    steps = [((torch.rand(64, 1, generator=g) < 0.3).float(), torch.randn(64, 1, generator=g)) for _ in range(9)]
    sync_sink, bg_sink = _ListSink(), _ListSink()
    sync = TrainMetricsWindow(window_steps=3, capacity=256, sinks=[sync_sink])
    bg = TrainMetricsWindow(window_steps=3, capacity=256, sinks=[bg_sink], background=True, max_pending=1)
    sync_out = []
    for y, noise in steps:
        logits = (y * 2 - 1) + noise
        r = sync.update(logits, y, loss_sum=64 * 0.25)
        if r is not None:
            sync_out.append(r)
        assert bg.update(logits, y, loss_sum=64 * 0.25) is None
        assert len(bg._pending) <= 1
    got = bg.drain()
    bg.close()
    assert len(got) == len(sync_out) == 3
    for a, b in zip(got, sync_out):
        assert a["train/auc_ctr"] == b["train/auc_ctr"] and a["train/loss"] == b["train/loss"]
    assert [s for s, _ in bg_sink.rows] == [s for s, _ in sync_sink.rows] == [3, 6, 9]


def test_vectorised_host_auc_gauc_equal_the_per_group_oracles():
    import numpy as np

    from flare_b200.metrics.ranking import auc_host, gauc_host

    rng = np.random.default_rng(5)
    for n, groups, levels in ((1, 1, 3), (50, 7, 4), (5000, 300, 20), (20000, 5000, 1000)):
        s = (rng.integers(0, levels, n) / levels).astype(np.float32)  # many ties
        y = (rng.random(n) < 0.3).astype(np.float32)
        g = rng.integers(0, groups, n) * 7 - 3  # negative and sparse group ids
        assert np.isclose(auc_host(s, y), auc_reference(s, y), rtol=0, atol=1e-12, equal_nan=True)
        for nf in (0.0, 0.5):
            assert np.isclose(gauc_host(s, y, g, nf), gauc_reference(s, y, g, nf), rtol=0, atol=1e-12,
                              equal_nan=True)
    assert np.isnan(auc_host(np.zeros(4, np.float32), np.ones(4, np.float32)))
    assert np.isnan(gauc_host(np.zeros(0, np.float32), np.zeros(0, np.float32), np.zeros(0, np.int64)))
    # CPU tensors take the vectorised path
    s, y, g = torch.rand(3000), (torch.rand(3000) < 0.4).float(), torch.randint(0, 50, (3000,))
    assert abs(auc(s, y) - auc_reference(s.numpy(), y.numpy())) < 1e-12
    assert abs(gauc(s, y, g, 0.25) - gauc_reference(s.numpy(), y.numpy(), g.numpy(), 0.25)) < 1e-12
