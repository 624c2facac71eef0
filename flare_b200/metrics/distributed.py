"""Exact AUC / GAUC / calibration over the samples of every rank (packed score summaries).

Each rank reduces its window to a score summary: the distinct (group, score)
keys of its samples in ascending order with the number of positives and
negatives at each key, packed as one float64 tensor ``[K, 4]`` (group, score,
positives, negatives; float64 holds group ids below 2^53 and counts exactly).
The ranks all-gather the summaries (padded to the longest one), every rank
merges them into the global summary (a stable sort on the key, equal keys
summed) and integrates the Mann-Whitney statistic with half credit for ties:

    AUC   = sum_k pos_k * (neg below key k + 0.5 * neg_k) / (P * N)
    GAUC  = sum_g AUC_g * w_g / sum_g w_g,  w_g = P_g + negative_factor * N_g,
            over the groups with both classes
    calibration = sum(prediction) / sum(label)

The merge is exact: it gives the same number as the metric over the
concatenated samples, whatever the split across ranks.  The summaries are
built with tensor ops on the samples' device (the GPU during training), so a
window of millions of samples costs one sort per rank and one all-gather of
at most the distinct keys.

Reference behaviour: the score-sorted partial summaries and their exact
merge in recipes/recsys/ranking/metrics/ray_data.py:242-554 (AUC with tie
half-credit, GAUC weighted by positives plus negative_factor * negatives).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _segments(keys: list[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Order that sorts by keys[0] then keys[1]...; segment id of each sorted element; segment count."""
    n = keys[0].numel()
    order = torch.arange(n, device=keys[0].device)
    for k in reversed(keys):  # least significant first: stable sorts compose into a lexicographic sort
        _, o = torch.sort(k[order], stable=True)
        order = order[o]
    new = torch.ones(n, dtype=torch.bool, device=order.device)
    if n > 1:
        diff = torch.zeros(n - 1, dtype=torch.bool, device=order.device)
        for k in keys:
            ks = k[order]
            diff |= ks[1:] != ks[:-1]
        new[1:] = diff
    seg = torch.cumsum(new.to(torch.int64), 0) - 1
    return order, seg, int(seg[-1].item()) + 1 if n else 0


def score_summary(scores: torch.Tensor, labels: torch.Tensor, groups: torch.Tensor | None = None) -> torch.Tensor:
    """Packed summary ``[K, 4]`` float64 (group, score, positives, negatives) of one rank's samples."""
    s = scores.detach().reshape(-1).to(torch.float64) + 0.0  # + 0.0 folds -0.0 into +0.0 (they tie)
    y = (labels.detach().reshape(-1) > 0.5).to(torch.float64)
    g = (torch.zeros_like(s) if groups is None else groups.detach().reshape(-1).to(torch.float64))
    if s.numel() == 0:
        return torch.zeros(0, 4, dtype=torch.float64, device=s.device)
    return _combine(g, s, y, 1.0 - y)


def _combine(g, s, pos, neg) -> torch.Tensor:
    order, seg, K = _segments([g, s])
    out = torch.zeros(K, 4, dtype=torch.float64, device=s.device)
    out[:, 0].scatter_(0, seg, g[order])
    out[:, 1].scatter_(0, seg, s[order])
    out[:, 2].index_add_(0, seg, pos[order])
    out[:, 3].index_add_(0, seg, neg[order])
    return out


def merge_summaries(parts: list[torch.Tensor]) -> torch.Tensor:
    """Exact merge of packed summaries: sorted by (group, score), equal keys summed."""
    parts = [p for p in parts if p.numel()]
    if not parts:
        return torch.zeros(0, 4, dtype=torch.float64)
    cat = torch.cat(parts)
    return _combine(cat[:, 0], cat[:, 1], cat[:, 2], cat[:, 3])


def auc_from_summary(summary: torch.Tensor) -> float:
    """AUC of a merged summary, ignoring the group column."""
    if summary.numel() == 0:
        return float("nan")
    if summary[:, 0].unique().numel() > 1:  # fold the groups: the same score in two groups is one key
        summary = _combine(torch.zeros_like(summary[:, 0]), summary[:, 1], summary[:, 2], summary[:, 3])
    pos, neg = summary[:, 2], summary[:, 3]
    P, N = float(pos.sum()), float(neg.sum())
    if P == 0 or N == 0:
        return float("nan")
    below = torch.cumsum(neg, 0) - neg
    return float((pos * (below + 0.5 * neg)).sum()) / (P * N)


def gauc_from_summary(summary: torch.Tensor, negative_factor: float = 0.0) -> float:
    """Grouped AUC of a merged summary (rows sorted by group, then score)."""
    if summary.numel() == 0:
        return float("nan")
    g, pos, neg = summary[:, 0], summary[:, 2], summary[:, 3]
    start = torch.ones(g.numel(), dtype=torch.bool, device=g.device)
    start[1:] = g[1:] != g[:-1]
    gid = torch.cumsum(start.to(torch.int64), 0) - 1
    G = int(gid[-1].item()) + 1
    Pg = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, pos)
    Ng = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, neg)
    cneg = torch.cumsum(neg, 0)
    first = torch.nonzero(start).reshape(-1)
    base = (cneg - neg)[first]                     # negatives before each group's first key
    below = cneg - neg - base[gid]                 # negatives of the same group below each key
    credit = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, pos * (below + 0.5 * neg))
    ok = (Pg > 0) & (Ng > 0)
    if not bool(ok.any()):
        return float("nan")
    w = Pg + negative_factor * Ng
    auc_g = credit[ok] / (Pg[ok] * Ng[ok])
    den = float(w[ok].sum())
    return float((auc_g * w[ok]).sum()) / den if den else float("nan")


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def _comm_device(group, like: torch.Tensor) -> torch.device:
    return like.device if dist.get_backend(group) != "nccl" else torch.device("cuda", torch.cuda.current_device())


def all_gather_summaries(summary: torch.Tensor, group=None) -> list[torch.Tensor]:
    """Every rank's packed summary (variable lengths, padded to the longest for the all-gather)."""
    W = _world(group)
    if W == 1:
        return [summary]
    dev = _comm_device(group, summary)
    n = torch.tensor([summary.shape[0]], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(n) for _ in range(W)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(x.item()) for x in sizes]
    M = max(max(sizes), 1)
    buf = torch.zeros(M, 4, dtype=torch.float64, device=dev)
    buf[:summary.shape[0]] = summary.to(dev)
    outs = [torch.empty_like(buf) for _ in range(W)]
    dist.all_gather(outs, buf, group=group)
    return [o[:k] for o, k in zip(outs, sizes)]


def _sum_scalars(vals: list[float], group, device) -> list[float]:
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    if _world(group) > 1:
        t = t.to(_comm_device(group, t))
        dist.all_reduce(t, group=group)
    return t.tolist()


def _max_scalar(val: float, group, device) -> float:
    t = torch.tensor([val], dtype=torch.float64, device=device)
    if _world(group) > 1:
        t = t.to(_comm_device(group, t))
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def _exchange_rows(rows: torch.Tensor, owner: torch.Tensor, group) -> torch.Tensor:
    """Send each row of ``rows`` ([n, 4] float64) to rank ``owner[i]``; returns the rows this rank owns."""
    W = _world(group)
    home, dev = rows.device, _comm_device(group, rows)
    order = torch.argsort(owner, stable=True)
    rows, owner = rows[order].to(dev), owner[order]
    send = torch.bincount(owner, minlength=W).to(torch.int64)
    recv = torch.empty_like(send, device=dev)
    dist.all_to_all_single(recv, send.to(dev), group=group)
    send_l, recv_l = send.tolist(), recv.tolist()
    out = torch.empty(sum(recv_l), 4, dtype=torch.float64, device=dev)
    dist.all_to_all_single(out.view(-1), rows.reshape(-1), [4 * k for k in recv_l], [4 * k for k in send_l],
                           group=group)
    return out.to(home)


def _rank_of(group) -> int:
    return dist.get_rank(group) if _world(group) > 1 else 0


def partitioned_gauc(summary: torch.Tensor, negative_factor: float = 0.0, group=None) -> float:
    """Exact GAUC with the groups split over the ranks: group g is merged by rank g mod W only."""
    W = _world(group)
    if W == 1:
        return gauc_from_summary(summary, negative_factor)
    owner = torch.remainder(summary[:, 0].to(torch.int64), W)
    mine = merge_summaries([_exchange_rows(summary, owner, group)])
    num = den = 0.0
    if mine.numel():
        g, pos, neg = mine[:, 0], mine[:, 2], mine[:, 3]
        start = torch.ones(g.numel(), dtype=torch.bool, device=g.device)
        start[1:] = g[1:] != g[:-1]
        gid = torch.cumsum(start.to(torch.int64), 0) - 1
        G = int(gid[-1].item()) + 1
        Pg = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, pos)
        Ng = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, neg)
        cneg = torch.cumsum(neg, 0)
        base = (cneg - neg)[torch.nonzero(start).reshape(-1)]
        below = cneg - neg - base[gid]
        credit = torch.zeros(G, dtype=torch.float64, device=g.device).index_add_(0, gid, pos * (below + 0.5 * neg))
        ok = (Pg > 0) & (Ng > 0)
        w = Pg + negative_factor * Ng
        num = float((credit[ok] / (Pg[ok] * Ng[ok]) * w[ok]).sum())
        den = float(w[ok].sum())
    num, den = _sum_scalars([num, den], group, summary.device)
    return num / den if den else float("nan")


def partitioned_auc(summary: torch.Tensor, group=None) -> float:
    """Exact AUC with the score axis split into one range per rank.

    Every rank proposes W - 1 quantiles of its own distinct scores; the sorted union's every W-th
    value becomes a global splitter, so rank r owns the scores in [split[r-1], split[r]) and equal
    scores always meet at one rank.  Each rank merges its range and credits its positives with the
    negatives below them inside the range plus every negative held by the ranks of lower ranges."""
    W = _world(group)
    if W == 1:
        return auc_from_summary(summary)
    dev = summary.device
    s = summary[:, 1].contiguous()
    k = W - 1
    if s.numel():
        ss = torch.sort(s).values
        q = ss[(torch.arange(1, k + 1, device=dev) * ss.numel()) // (k + 1)]
    else:
        q = torch.full((k,), float("inf"), dtype=torch.float64, device=dev)
    cdev = _comm_device(group, q)
    props = [torch.empty(k, dtype=torch.float64, device=cdev) for _ in range(W)]
    dist.all_gather(props, q.to(cdev), group=group)
    allq = torch.sort(torch.cat(props)).values.to(dev)  # W * (W - 1) proposals
    split = allq[(torch.arange(1, W, device=dev) * allq.numel()) // W]
    owner = torch.searchsorted(split, s, right=True)
    folded = torch.cat([torch.zeros_like(s)[:, None], summary[:, 1:]], 1)
    mine = merge_summaries([_exchange_rows(folded, owner, group)])
    pos, neg = (mine[:, 2], mine[:, 3]) if mine.numel() else (torch.zeros(0, dtype=torch.float64, device=dev),) * 2
    P_r, N_r = float(pos.sum()), float(neg.sum())
    credit = float((pos * (torch.cumsum(neg, 0) - neg + 0.5 * neg)).sum()) if mine.numel() else 0.0
    counts = torch.tensor([P_r, N_r], dtype=torch.float64, device=cdev)
    every = [torch.empty(2, dtype=torch.float64, device=cdev) for _ in range(W)]
    dist.all_gather(every, counts, group=group)
    below = sum(float(every[r][1]) for r in range(_rank_of(group)))
    credit += P_r * below
    credit, P, N = _sum_scalars([credit, P_r, N_r], group, dev)
    return credit / (P * N) if P and N else float("nan")


def distributed_auc(scores: torch.Tensor, labels: torch.Tensor, group=None) -> float:
    """Exact AUC over the samples of every rank of ``group``."""
    return auc_from_summary(merge_summaries(all_gather_summaries(score_summary(scores, labels), group)))


def distributed_gauc(scores: torch.Tensor, labels: torch.Tensor, groups: torch.Tensor, negative_factor: float = 0.0,
                     group=None) -> float:
    """Exact GAUC over every rank's samples (a user's samples may sit on several ranks)."""
    parts = all_gather_summaries(score_summary(scores, labels, groups), group)
    return gauc_from_summary(merge_summaries(parts), negative_factor)


def distributed_calibration(predictions: torch.Tensor, labels: torch.Tensor, group=None) -> float:
    p, y = _sum_scalars([float(predictions.double().sum()), float(labels.double().sum())], group, predictions.device)
    return p / y if y else float("nan")


def distributed_metrics(scores: torch.Tensor, labels: torch.Tensor, groups: torch.Tensor | None = None, *,
                        negative_factor: float = 0.0, group=None, merge: str = "allgather") -> dict[str, float]:
    """AUC, calibration (and GAUC with groups) of every rank's samples.

    ``merge="allgather"`` (default): every rank gathers every summary and merges the whole window
    (one collective; every rank holds all W summaries).  ``merge="partitioned"``: the groups and the
    score ranges are split over the ranks (``partitioned_gauc`` / ``partitioned_auc``), so each rank
    holds and merges about 1/W of the window, for windows too large to gather on every rank; it pays
    two all-to-alls per metric, which on CPU gloo ranks cost more than the all-gather at 200K-row
    windows (``benchmarks.metrics --merge``).  Both are exact."""
    if merge not in ("allgather", "partitioned"):
        raise ValueError(f"merge must be 'allgather' or 'partitioned', got {merge!r}")
    if merge == "partitioned" and _world(group) > 1:
        summ = score_summary(scores, labels, groups)
        out = {"auc": partitioned_auc(summ, group)}
        p_sum, y_sum = _sum_scalars([float(scores.double().sum()), float(labels.double().sum())], group,
                                    scores.device)
        out["calibration"] = p_sum / y_sum if y_sum else float("nan")
        if groups is not None:
            out["gauc"] = partitioned_gauc(summ, negative_factor, group)
        return out
    merged = merge_summaries(all_gather_summaries(score_summary(scores, labels, groups), group))
    out = {"auc": auc_from_summary(merged)}
    p_sum, y_sum = _sum_scalars([float(scores.double().sum()), float(labels.double().sum())], group, scores.device)
    out["calibration"] = p_sum / y_sum if y_sum else float("nan")
    if groups is not None:
        out["gauc"] = gauc_from_summary(merged, negative_factor)
    return out


__all__ = ["all_gather_summaries", "auc_from_summary", "distributed_auc", "distributed_calibration",
           "distributed_gauc", "distributed_metrics", "gauc_from_summary", "merge_summaries", "partitioned_auc", "partitioned_gauc", "score_summary"]
