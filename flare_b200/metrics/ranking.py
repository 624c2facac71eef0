"""Exact ranking metrics: AUC with tie half-credit, grouped AUC, calibration.

Device path: ``auc_device`` sorts (score[, group]) keys with the framework's
own stable radix sort and integrates the Mann-Whitney statistic on the GPU
(csrc/metrics.cu).  Host path (CPU tensors): the same statistic from average
ranks, vectorised over every group at once (``auc_host`` / ``gauc_host``: one
sort by (group, score), tie runs and group segments from boundary masks).
``auc_reference`` / ``gauc_reference`` are the plain per-group oracles the
tests compare both against.  Semantics follow the reference's
exact AUC/GAUC (recipes/recsys/ranking/metrics/ray_data.py:242-554):

* AUC = (sum over positives of [#neg below + 0.5 * #neg tied]) / (P * N);
* GAUC = sum_g AUC_g * w_g / sum_g w_g over groups with both classes,
  w_g = P_g + negative_factor * N_g;
* calibration = mean(prediction) / mean(label).
"""
from __future__ import annotations

import numpy as np
import torch

from .._native import native, on_cuda


def _avg_ranks(x: np.ndarray) -> np.ndarray:
    order = np.argsort(x, kind="mergesort")
    xs = x[order]
    ranks = np.empty(len(x), dtype=np.float64)
    i = 0
    n = len(x)
    while i < n:
        j = i
        while j + 1 < n and xs[j + 1] == xs[i]:
            j += 1
        ranks[order[i:j + 1]] = 0.5 * (i + j) + 1.0
        i = j + 1
    return ranks


def auc_reference(scores, labels) -> float:
    s = np.asarray(scores, dtype=np.float32).astype(np.float64)
    y = np.asarray(labels).astype(np.float64) > 0.5
    P, N = int(y.sum()), int((~y).sum())
    if P == 0 or N == 0:
        return float("nan")
    r = _avg_ranks(s)
    return float((r[y].sum() - P * (P + 1) / 2.0) / (P * N))


def gauc_reference(scores, labels, groups, negative_factor: float = 0.0) -> float:
    s = np.asarray(scores, dtype=np.float32)
    y = np.asarray(labels) > 0.5
    g = np.asarray(groups)
    num = den = 0.0
    for gid in np.unique(g):
        m = g == gid
        P, N = int(y[m].sum()), int((~y[m]).sum())
        if P == 0 or N == 0:
            continue
        w = P + negative_factor * N
        num += auc_reference(s[m], y[m]) * w
        den += w
    return num / den if den else float("nan")


class _AucWorkspace:
    def __init__(self, n: int, device, grouped: bool):
        ntiles = (n + 4095) // 4096
        z = lambda k, dt: torch.empty(k, dtype=dt, device=device)  # noqa: E731
        self.t = dict(keys_a=z(n, torch.int64), keys_b=z(n, torch.int64), vals_a=z(n, torch.int32),
                      vals_b=z(n, torch.int32), negs=z(n, torch.int32), neg_prefix=z(n + 1, torch.int32),
                      hist=z(256 * ntiles, torch.int32), hist_scan=z(256 * ntiles + 1, torch.int32),
                      block_sums=z(512, torch.int32), out=torch.zeros(2, dtype=torch.float64, device=device))
        if grouped:
            self.t.update(credit=z(n, torch.float64), pos_cnt=z(n, torch.int64), neg_cnt=z(n, torch.int64))

    def ptrs(self) -> dict:
        return {k: v.data_ptr() for k, v in self.t.items()}


def _grouped_rank_sums(s: np.ndarray, y: np.ndarray, g: np.ndarray):
    """Per group (in ascending group order): positives, negatives and the sum of the positives'
    average ranks among the group's scores (ties share the mean of their positions)."""
    n = s.shape[0]
    order = np.lexsort((s, g))
    gs, ss, ys = g[order], s[order], y[order]
    gnew = np.empty(n, dtype=bool)
    gnew[0] = True
    gnew[1:] = gs[1:] != gs[:-1]
    gstart = np.flatnonzero(gnew)
    pos = np.arange(n, dtype=np.int64) - gstart[np.cumsum(gnew) - 1]  # 0-based position in the group
    tnew = gnew.copy()
    tnew[1:] |= ss[1:] != ss[:-1]
    tstart = np.flatnonzero(tnew)
    tend = np.append(tstart[1:], n) - 1
    run_rank = 0.5 * (pos[tstart] + pos[tend]).astype(np.float64) + 1.0
    rank = run_rank[np.cumsum(tnew) - 1]
    P = np.add.reduceat(ys.astype(np.int64), gstart)
    N = np.diff(np.append(gstart, n)) - P
    R = np.add.reduceat(np.where(ys, rank, 0.0), gstart)
    return P, N, R


def auc_host(scores, labels) -> float:
    """Exact AUC on the host (numpy), vectorised; equal to ``auc_reference``."""
    s = np.asarray(scores, dtype=np.float32).astype(np.float64).reshape(-1)
    y = (np.asarray(labels).astype(np.float64) > 0.5).reshape(-1)
    if s.size == 0:
        return float("nan")
    P, N, R = _grouped_rank_sums(s, y, np.zeros(s.size, dtype=np.int64))
    if P[0] == 0 or N[0] == 0:
        return float("nan")
    return float((R[0] - P[0] * (P[0] + 1) / 2.0) / (float(P[0]) * float(N[0])))


def gauc_host(scores, labels, groups, negative_factor: float = 0.0) -> float:
    """Exact grouped AUC on the host (numpy), every group in one pass; equal to ``gauc_reference``."""
    s = np.asarray(scores, dtype=np.float32).astype(np.float64).reshape(-1)
    y = (np.asarray(labels).astype(np.float64) > 0.5).reshape(-1)
    g = np.asarray(groups).astype(np.int64).reshape(-1)
    if s.size == 0:
        return float("nan")
    P, N, R = _grouped_rank_sums(s, y, g)
    ok = (P > 0) & (N > 0)
    if not ok.any():
        return float("nan")
    Pf, Nf = P[ok].astype(np.float64), N[ok].astype(np.float64)
    a = (R[ok] - Pf * (Pf + 1) / 2.0) / (Pf * Nf)
    w = Pf + negative_factor * Nf
    den = float(w.sum())
    return float((a * w).sum() / den) if den else float("nan")


def auc(scores: torch.Tensor, labels: torch.Tensor) -> float:
    """Exact AUC; runs on the GPU for CUDA tensors."""
    if not on_cuda(scores, labels):
        return auc_host(scores.detach().float().cpu().numpy(), labels.detach().cpu().numpy())
    s = scores.detach().reshape(-1).float().contiguous()
    y = labels.detach().reshape(-1).float().contiguous()
    n = s.numel()
    P = float((y > 0.5).sum())
    N = n - P
    if P == 0 or N == 0:
        return float("nan")
    ws = _AucWorkspace(n, s.device, grouped=False)
    native().auc_device(s.data_ptr(), y.data_ptr(), 0, n, 0.0, ws.ptrs())
    return float(ws.t["out"][0].item()) / (P * N)


def gauc(scores: torch.Tensor, labels: torch.Tensor, groups: torch.Tensor, negative_factor: float = 0.0) -> float:
    """Grouped AUC weighted by positives (+ negative_factor * negatives)."""
    if not on_cuda(scores, labels, groups):
        return gauc_host(scores.detach().float().cpu().numpy(), labels.detach().cpu().numpy(),
                         groups.detach().cpu().numpy(), negative_factor)
    s = scores.detach().reshape(-1).float().contiguous()
    y = labels.detach().reshape(-1).float().contiguous()
    g = groups.detach().reshape(-1).to(torch.int64).contiguous()
    if int(g.min()) < 0 or int(g.max()) >= 1 << 32:
        raise ValueError("group ids must be in [0, 2^32)")
    ws = _AucWorkspace(s.numel(), s.device, grouped=True)
    native().auc_device(s.data_ptr(), y.data_ptr(), g.data_ptr(), s.numel(), float(negative_factor), ws.ptrs())
    out = ws.t["out"].tolist()
    return out[0] / out[1] if out[1] else float("nan")


def calibration(predictions: torch.Tensor, labels: torch.Tensor) -> float:
    p = float(predictions.float().mean())
    y = float(labels.float().mean())
    return p / y if y else float("nan")


__all__ = ["auc", "auc_host", "auc_reference", "calibration", "gauc", "gauc_host", "gauc_reference"]
