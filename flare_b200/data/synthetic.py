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


def synthetic_ranking_batch(B: int, vocabs, num_dense: int, max_bag: int, *, seed: int, device=None,
                            n_labels: int = 3):
    """(dense [B, num_dense], label ids [B], offsets, values) for a ranking model with multi-class labels.

    Bags are U[1, max_bag] uniform ids of each vocabulary, feature-major (the keyed-jagged layout).  Label
    id k is given to scores above the k-th of ``n_labels - 1`` thresholds spaced one unit apart (0 and 1
    for three labels), so higher ids are rarer and predictable from the first dense features."""
    g = torch.Generator().manual_seed(seed)
    dense = torch.randn(B, num_dense, generator=g)
    lens = torch.randint(1, max_bag + 1, (len(vocabs), B), generator=g)
    vals = torch.cat([torch.randint(0, v, (int(lens[f].sum()),), generator=g) for f, v in enumerate(vocabs)])
    offs = torch.cat([torch.zeros(1, dtype=torch.long), lens.reshape(-1).cumsum(0)]).int()
    score = dense[:, 0] + 0.5 * dense[:, 1] + 0.3 * torch.randn(B, generator=g)
    labels = torch.zeros(B, dtype=torch.long)
    for k in range(1, n_labels):
        labels += (score > float(k - 1)).long()
    out = (dense, labels, offs, vals.int())
    return tuple(t.to(device) for t in out) if device is not None else out


@dataclass
class SeqBatch:
    """Packed jagged sequences for the sequential model (one rank's share).

    ``seq_offsets`` [nseq+1] token offsets (each sequence padded at its end to a
    multiple of 8); ``target_row`` [T_cap] = row of token t+1 when token t has a
    next item in its sequence, else -1; the embedding KJT (``emb_offsets``
    [F*(T_cap+N)+1] feature-major, ``emb_values``) has one bag per token (item,
    4 side features; empty for padding) followed by N rows holding the shared
    negative item ids; ``num_valid`` = tokens with a target over ALL ranks.
    """

    seq_offsets: torch.Tensor
    target_row: torch.Tensor
    emb_offsets: torch.Tensor
    emb_values: torch.Tensor
    num_valid: torch.Tensor  # int32 [1]
    tokens: int              # packed tokens (<= T_cap) of this rank

    def to(self, device, non_blocking: bool = False) -> "SeqBatch":
        return SeqBatch(*(t.to(device, non_blocking=non_blocking) for t in
                          (self.seq_offsets, self.target_row, self.emb_offsets, self.emb_values, self.num_valid)),
                        self.tokens)

    def pin_memory(self) -> "SeqBatch":
        return SeqBatch(*(t.pin_memory() for t in (self.seq_offsets, self.target_row, self.emb_offsets,
                                                     self.emb_values, self.num_valid)), self.tokens)


class SeqSyntheticData:
    """Jagged user histories: lengths ~ U[min_len, max_len], items Zipf(s) over ``item_rows``,
    4 side features per token Zipf over ``side_rows``; ``negatives`` shared uniform negatives per step."""

    def __init__(self, nseq: int, *, item_rows: int, side_rows: int = 100_000, num_side: int = 4,
                 min_len: int = 32, max_len: int = 512, zipf_s: float = 1.1, negatives: int = 512,
                 T_cap: int | None = None, seed: int = 0, rank: int = 0, world: int = 1, device="cpu"):
        self.nseq, self.item_rows, self.side_rows, self.num_side = nseq, item_rows, side_rows, num_side
        self.min_len, self.max_len, self.zipf_s, self.negatives = min_len, max_len, zipf_s, negatives
        self.rank, self.world = rank, world
        self.T_cap = T_cap or nseq * ((max_len + 7) // 8 * 8)
        self.device = torch.device(device)
        self.seed = seed
        self.step = 0

    def _lengths(self, r: int, step: int) -> torch.Tensor:
        g = torch.Generator().manual_seed((self.seed * 1000 + r) * 100003 + step)
        return torch.randint(self.min_len, self.max_len + 1, (self.nseq,), generator=g)

    def next(self) -> SeqBatch:
        step = self.step
        self.step += 1
        lens = self._lengths(self.rank, step)
        # the loss mean runs over every rank's tokens: all ranks derive the same count
        num_valid = sum(int((self._lengths(r, step) - 1).sum()) for r in range(self.world))
        padded = (lens + 7) // 8 * 8
        offs = torch.zeros(self.nseq + 1, dtype=torch.int64)
        torch.cumsum(padded, 0, out=offs[1:])
        T = int(offs[-1])
        if T > self.T_cap:
            raise ValueError(f"{T} packed tokens exceed the capacity {self.T_cap}")
        g = torch.Generator(device=self.device).manual_seed((self.seed * 1000 + self.rank) * 7919 + step)
        pos = torch.arange(self.T_cap, dtype=torch.int64)
        seq_id = torch.searchsorted(offs[1:], pos, right=True).clamp(max=self.nseq - 1)
        within = pos - offs[seq_id]
        valid = (pos < T) & (within < lens[seq_id])
        has_next = valid & (within + 1 < lens[seq_id])
        target = torch.where(has_next, pos + 1, torch.full_like(pos, -1)).to(torch.int32)
        n_tok = int(valid.sum())
        B = self.T_cap + self.negatives
        F = 1 + self.num_side
        items = zipf_ids(n_tok, self.item_rows, self.zipf_s, g, self.device)
        sides = [zipf_ids(n_tok, self.side_rows, self.zipf_s, g, self.device) for _ in range(self.num_side)]
        negs = torch.randint(0, self.item_rows, (self.negatives,), generator=g, device=self.device, dtype=torch.int32)
        tok_len = valid.to(torch.int32).to(self.device)
        item_len = torch.cat([tok_len, torch.ones(self.negatives, dtype=torch.int32, device=self.device)])
        side_len = torch.cat([tok_len, torch.zeros(self.negatives, dtype=torch.int32, device=self.device)])
        lengths = torch.cat([item_len] + [side_len] * self.num_side)
        emb_off = torch.zeros(F * B + 1, dtype=torch.int32, device=self.device)
        torch.cumsum(lengths, 0, out=emb_off[1:])
        values = torch.cat([items, negs] + sides)
        return SeqBatch(offs.to(torch.int32).to(self.device), target.to(self.device), emb_off, values,
                        torch.tensor([num_valid], dtype=torch.int32, device=self.device), T)
