"""Deterministic synthetic data for the benchmark configurations.

Every generator is seeded and produces the keyed-jagged sparse layout used by
the embedding collection (``offsets`` int32 [F*B+1], ``values`` int32 ids,
feature-major) plus dense features and labels.  Distributions follow the
named configurations:

* DLRM-style: 13 dense features ~ log(1 + |N(0, 3)|); 26 tables with
  log-uniform vocabularies between 1e3 and 4e7 totalling ~200M rows; bag
  lengths ~ U{1..64}; ids ~ Zipf(s=1.05); labels ~ Bernoulli(0.03).
* small CPU config: 13 dense ~ N(0,1); 8 single-id features, Zipf(1.1) over
  1,000 ids; label ~ Bernoulli(sigmoid(a.x + 0.5 N(0,1))).

Zipf ids are drawn by inverting the continuous power-law CDF on [1, V+1) and
scrambled by a multiplicative bijection so hot ids are spread over the table.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

SCRAMBLE = 2654435761  # prime > any vocabulary used here, so k -> k*SCRAMBLE mod V is a bijection


def log_uniform_vocab_sizes(n: int = 26, lo: float = 1e3, hi: float = 4e7, total: float = 2e8) -> list[int]:
    """Stratified log-uniform quantiles, skewed by an exponent fitted so the sum is ~``total``."""
    def sizes(p):
        return [int(round(math.exp(math.log(lo) + (i / max(n - 1, 1)) ** p * (math.log(hi) - math.log(lo)))))
                for i in range(n)]
    a, b = 0.05, 4.0
    for _ in range(80):
        mid = 0.5 * (a + b)
        if sum(sizes(mid)) > total:
            a = mid
        else:
            b = mid
    return sizes(0.5 * (a + b))


def zipf_ids(n: int, vocab: int, s: float, generator: torch.Generator, device="cpu") -> torch.Tensor:
    u = torch.rand(n, generator=generator, device=device, dtype=torch.float64)
    if abs(s - 1.0) < 1e-9:
        x = torch.exp(u * math.log(vocab + 1.0))
    else:
        e = 1.0 - s
        top = (vocab + 1.0) ** e
        x = (1.0 + u * (top - 1.0)) ** (1.0 / e)
    k = torch.clamp(x.floor().to(torch.int64) - 1, 0, vocab - 1)
    return ((k * SCRAMBLE) % vocab).to(torch.int32)


@dataclass
class SparseBatch:
    dense: torch.Tensor     # fp32 [B, num_dense]
    labels: torch.Tensor    # fp32 [B, T]
    offsets: torch.Tensor   # int32 [F*B+1]
    values: torch.Tensor    # int32 [nnz]

    def to(self, device, non_blocking: bool = False) -> "SparseBatch":
        return SparseBatch(*(t.to(device, non_blocking=non_blocking) for t in
                             (self.dense, self.labels, self.offsets, self.values)))

    def pin_memory(self) -> "SparseBatch":
        return SparseBatch(*(t.pin_memory() for t in (self.dense, self.labels, self.offsets, self.values)))

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.dense, self.labels, self.offsets, self.values))


def make_jagged(lengths: torch.Tensor, vocab_sizes: list[int], zipf_s: float, gen: torch.Generator,
                device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """lengths int [F, B] -> (offsets [F*B+1], values) with Zipf ids per feature."""
    F, B = lengths.shape
    flat = lengths.reshape(-1).to(torch.int64)
    offsets = torch.zeros(F * B + 1, dtype=torch.int64, device=device)
    offsets[1:] = torch.cumsum(flat, 0)
    vals = []
    for f in range(F):
        n = int(lengths[f].sum())
        vals.append(zipf_ids(n, vocab_sizes[f], zipf_s, gen, device))
    return offsets.to(torch.int32), torch.cat(vals)


class DLRMSyntheticData:
    """DLRM-style 26-table generator (per-rank stream: seed + rank)."""

    def __init__(self, batch_size: int, vocab_sizes: list[int], *, num_dense: int = 13, max_bag: int = 64,
                 min_bag: int = 1, zipf_s: float = 1.05, pos_rate: float = 0.03, seed: int = 0, rank: int = 0,
                 device="cpu"):
        self.B, self.vocab, self.num_dense = batch_size, list(vocab_sizes), num_dense
        self.max_bag, self.min_bag, self.zipf_s, self.pos_rate = max_bag, min_bag, zipf_s, pos_rate
        self.device = torch.device(device)
        self.gen = torch.Generator(device=self.device).manual_seed(seed * 1000 + rank)

    def next(self) -> SparseBatch:
        B, F, g, dev = self.B, len(self.vocab), self.gen, self.device
        dense = torch.log1p(torch.abs(torch.randn(B, self.num_dense, generator=g, device=dev) * 3.0))
        labels = (torch.rand(B, 1, generator=g, device=dev) < self.pos_rate).float()
        lengths = torch.randint(self.min_bag, self.max_bag + 1, (F, B), generator=g, device=dev)
        offsets, values = make_jagged(lengths, self.vocab, self.zipf_s, g, dev)
        return SparseBatch(dense, labels, offsets, values)


class SmallSyntheticData:
    """13 dense N(0,1), 8 single-id features Zipf(1.1) over 1,000 ids, logistic labels."""

    def __init__(self, batch_size: int = 256, *, num_dense: int = 13, num_sparse: int = 8, vocab: int = 1000,
                 zipf_s: float = 1.1, seed: int = 0, rank: int = 0):
        self.B, self.num_dense, self.F, self.vocab, self.zipf_s = batch_size, num_dense, num_sparse, vocab, zipf_s
        self.gen = torch.Generator().manual_seed(seed * 1000 + rank)
        wgen = torch.Generator().manual_seed(seed)
        self.coef = torch.randn(num_dense, generator=wgen)

    def next(self) -> SparseBatch:
        g = self.gen
        dense = torch.randn(self.B, self.num_dense, generator=g)
        logit = dense @ self.coef + 0.5 * torch.randn(self.B, generator=g)
        labels = (torch.rand(self.B, generator=g) < torch.sigmoid(logit)).float().unsqueeze(1)
        lengths = torch.ones(self.F, self.B, dtype=torch.int64)
        offsets, values = make_jagged(lengths, [self.vocab] * self.F, self.zipf_s, g)
        return SparseBatch(dense, labels, offsets, values)


__all__ = ["DLRMSyntheticData", "SCRAMBLE", "SmallSyntheticData", "SparseBatch", "log_uniform_vocab_sizes",
           "make_jagged", "zipf_ids"]
