"""Sparse embedding operator contract and GPU/CPU implementations.

Mirrors the reference's ``SparseEmbeddingOperator`` (src/flare/kernels/
contracts.py:16-96) and factory (src/flare/ops/factory.py:14): ``gather``,
``gather_pooled``, ``scatter`` and ``scatter_pooled`` over a padded inverse
index with a pad sentinel, plus ``unique_first_occurrence``
(src/flare/ops/sparse_unique.py:52).  Two backends exist: ``cuda`` (the
hand-written sm_100a kernels) and ``cpu`` (native C++ kernels, with PyTorch
reference code as the fallback and test oracle).  The
product training path does not use these padded ops: it uses the fused
sharded embedding kernels in ``flare_b200.sparse.collection``.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from contextlib import contextmanager, nullcontext

import torch

from .._native import dtype_code, native, on_cuda
from ..sparse.precision import require_sparse_gradient_dtype, require_sparse_value_dtype

SPARSE_EMBEDDING_OPERATOR_BACKENDS = ("cuda", "cpu")


def pooled_sparse_widths(target_widths) -> tuple[int, int]:
    """(feature_count, max_elements) of a pooled layout (reference ops/contracts.py:7)."""
    widths = tuple(int(w) for w in target_widths)
    if len(widths) != 2 or widths[0] <= 0 or widths[1] <= 0:
        raise ValueError(f"target_widths must be (feature_count, max_elements), got {target_widths!r}")
    return widths


def _check_inverse(inverse: torch.Tensor) -> torch.Tensor:
    if inverse.dtype != torch.int32:
        raise TypeError(f"inverse must be int32, got {inverse.dtype}")
    return inverse.contiguous()


class SparseEmbeddingOperator(ABC):
    inverse_dtype = torch.int32

    def __init__(self, value_dtype: str, gradient_dtype: str = "float32"):
        self.value_dtype = require_sparse_value_dtype(value_dtype)
        self.gradient_dtype = require_sparse_gradient_dtype(gradient_dtype)

    @abstractmethod
    def gather(self, emb_flat, inverse, batch_size, emb_dim, pad_index): ...

    @abstractmethod
    def gather_pooled(self, emb_flat, inverse, batch_size, emb_dim, target_widths, pad_index): ...

    @abstractmethod
    def scatter(self, emb_rows, emb_dim, inverse, pad_index, gradient): ...

    @abstractmethod
    def scatter_pooled(self, emb_rows, emb_dim, inverse, pad_index, gradient, target_widths): ...

    def execution_context(self):
        return nullcontext()

    def prewarm(self) -> None:
        return None


def _cpu_native():
    """The native CPU kernels (``csrc/sparse_cpu.cpp``), or None when the extension is not built."""
    try:
        return native().cpu
    except Exception:  # pragma: no cover - extension not built
        return None


class CpuSparseEmbeddingOperator(SparseEmbeddingOperator):
    """CPU backend: native C++ kernels (fp32 accumulation, deterministic scatters); PyTorch
    reference code when the extension is not built (and as the oracle in the tests)."""

    def __init__(self, value_dtype: str, gradient_dtype: str = "float32", *, use_native: bool = True):
        super().__init__(value_dtype, gradient_dtype)
        self.nat = _cpu_native() if use_native else None

    def gather(self, emb_flat, inverse, batch_size, emb_dim, pad_index):
        if self.nat is not None:
            inv = _check_inverse(inverse)
            emb = emb_flat.contiguous()
            out = torch.empty((inv.numel(), emb_dim), dtype=emb.dtype)
            self.nat.gather(emb.data_ptr(), dtype_code(emb.dtype), inv.data_ptr(), inv.numel(), emb_dim, pad_index,
                            out.data_ptr())
            return out.reshape(batch_size, -1, emb_dim)
        inv = _check_inverse(inverse).long()
        emb = emb_flat.reshape(-1, emb_dim)
        mask = inv != pad_index
        out = torch.zeros((inv.numel(), emb_dim), dtype=emb.dtype)
        out[mask] = emb[inv[mask]]
        return out.reshape(batch_size, -1, emb_dim)

    def gather_pooled(self, emb_flat, inverse, batch_size, emb_dim, target_widths, pad_index):
        F, E = pooled_sparse_widths(target_widths)
        if self.nat is not None:
            inv = _check_inverse(inverse)
            emb = emb_flat.contiguous()
            out = torch.empty((batch_size, F, emb_dim), dtype=emb.dtype)
            self.nat.gather_pooled(emb.data_ptr(), dtype_code(emb.dtype), inv.data_ptr(), batch_size * F, E,
                                   emb_dim, pad_index, out.data_ptr())
            return out
        inv = _check_inverse(inverse).long().reshape(batch_size, F, E)
        emb = emb_flat.reshape(-1, emb_dim).float()
        mask = (inv != pad_index).unsqueeze(-1)
        rows = emb[torch.where(inv == pad_index, torch.zeros_like(inv), inv)]
        return (rows * mask).sum(2).to(emb_flat.dtype)

    def scatter(self, emb_rows, emb_dim, inverse, pad_index, gradient):
        if self.nat is not None:
            inv = _check_inverse(inverse)
            g = gradient.contiguous()
            out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32)
            self.nat.scatter(g.data_ptr(), dtype_code(g.dtype), inv.data_ptr(), inv.numel(), emb_dim, pad_index,
                             out.data_ptr())
            return out
        inv = _check_inverse(inverse).long().reshape(-1)
        g = gradient.reshape(-1, emb_dim).float()
        out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32)
        keep = inv != pad_index
        out.index_add_(0, inv[keep], g[keep])
        return out

    def scatter_pooled(self, emb_rows, emb_dim, inverse, pad_index, gradient, target_widths):
        F, E = pooled_sparse_widths(target_widths)
        if self.nat is not None:
            inv = _check_inverse(inverse)
            g = gradient.contiguous()
            bags = g.numel() // emb_dim
            if bags * E != inv.numel() or bags % F:
                raise ValueError("inverse and gradient shapes disagree")
            out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32)
            self.nat.scatter_pooled(g.data_ptr(), dtype_code(g.dtype), inv.data_ptr(), bags, E, emb_dim, pad_index,
                                    out.data_ptr())
            return out
        inv = _check_inverse(inverse).long().reshape(-1, F, E)
        g = gradient.reshape(-1, F, 1, emb_dim).float().expand(-1, F, E, emb_dim).reshape(-1, emb_dim)
        flat = inv.reshape(-1)
        keep = flat != pad_index
        out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32)
        out.index_add_(0, flat[keep], g[keep])
        return out


class CudaSparseEmbeddingOperator(SparseEmbeddingOperator):
    """sm_100a kernels on a dedicated non-blocking stream (reference C1 semantics)."""

    def __init__(self, value_dtype: str, gradient_dtype: str = "float32", device: int | None = None):
        super().__init__(value_dtype, gradient_dtype)
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.stream = torch.cuda.Stream(device=self.device)

    @contextmanager
    def execution_context(self):
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            yield self.stream
        cur.wait_stream(self.stream)

    def gather(self, emb_flat, inverse, batch_size, emb_dim, pad_index):
        inv = _check_inverse(inverse)
        out = torch.empty((inv.numel(), emb_dim), dtype=emb_flat.dtype, device=emb_flat.device)
        native().sparse_gather(emb_flat.data_ptr(), dtype_code(emb_flat.dtype), inv.data_ptr(), inv.numel(),
                               emb_dim, pad_index, out.data_ptr())
        return out.reshape(batch_size, -1, emb_dim)

    def gather_pooled(self, emb_flat, inverse, batch_size, emb_dim, target_widths, pad_index):
        F, E = pooled_sparse_widths(target_widths)
        inv = _check_inverse(inverse)
        out = torch.empty((batch_size, F, emb_dim), dtype=emb_flat.dtype, device=emb_flat.device)
        native().sparse_gather_pooled(emb_flat.data_ptr(), dtype_code(emb_flat.dtype), inv.data_ptr(),
                                      batch_size * F, E, emb_dim, pad_index, out.data_ptr())
        return out

    def scatter(self, emb_rows, emb_dim, inverse, pad_index, gradient):
        inv = _check_inverse(inverse)
        g = gradient.contiguous()
        out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32, device=g.device)
        native().sparse_scatter(g.data_ptr(), dtype_code(g.dtype), inv.data_ptr(), inv.numel(), emb_dim,
                                pad_index, out.data_ptr())
        return out

    def scatter_pooled(self, emb_rows, emb_dim, inverse, pad_index, gradient, target_widths):
        F, E = pooled_sparse_widths(target_widths)
        inv = _check_inverse(inverse)
        g = gradient.contiguous()
        bags = g.numel() // emb_dim
        if bags * E != inv.numel() or bags % F:
            raise ValueError("inverse and gradient shapes disagree")
        out = torch.zeros((emb_rows, emb_dim), dtype=torch.float32, device=g.device)
        native().sparse_scatter_pooled(g.data_ptr(), dtype_code(g.dtype), inv.data_ptr(), bags, E, emb_dim,
                                       pad_index, out.data_ptr())
        return out


def create_sparse_embedding_operator(name: str, value_dtype: str = "float32",
                                     gradient_dtype: str = "float32") -> SparseEmbeddingOperator:
    if name == "cuda":
        return CudaSparseEmbeddingOperator(value_dtype, gradient_dtype)
    if name == "cpu":
        return CpuSparseEmbeddingOperator(value_dtype, gradient_dtype)
    raise ValueError(f"unknown sparse operator backend {name!r}; expected one of "
                     f"{SPARSE_EMBEDDING_OPERATOR_BACKENDS}")


def unique_first_occurrence_reference(values: torch.Tensor):
    """Serial first-occurrence dedup (CPU oracle)."""
    flat = values.reshape(-1).tolist()
    seen: dict[int, int] = {}
    unique, inverse, first = [], [], []
    for i, v in enumerate(flat):
        u = seen.get(v)
        if u is None:
            u = len(unique)
            seen[v] = u
            unique.append(v)
            first.append(i)
        inverse.append(u)
    return (torch.tensor(unique, dtype=values.dtype), torch.tensor(inverse, dtype=torch.int32),
            torch.tensor(first, dtype=torch.int64))


def unique_first_occurrence(values: torch.Tensor):
    """Unique keys in first-occurrence order, int32 inverse, int64 first indices."""
    if values.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"sparse unique requires integer keys, got {values.dtype}")
    if not on_cuda(values):
        if values.numel() == 0:
            return values.reshape(-1).clone(), torch.empty(0, dtype=torch.int32), torch.empty(0, dtype=torch.int64)
        nat = _cpu_native()
        if nat is not None:  # open-addressing hash, one pass in occurrence order
            return nat.unique_first(values)
        # Vectorised CPU path: torch.unique + first index per group.
        flat = values.reshape(-1)
        uniq, inv = torch.unique(flat, sorted=True, return_inverse=True)
        first = torch.full((uniq.numel(),), flat.numel(), dtype=torch.int64)
        first.scatter_reduce_(0, inv, torch.arange(flat.numel()), reduce="amin")
        order = torch.argsort(first)
        rank = torch.empty_like(order)
        rank[order] = torch.arange(order.numel())
        return uniq[order], rank[inv].to(torch.int32), first[order]
    keys = values.reshape(-1).to(torch.int64).contiguous()
    n = keys.numel()
    dev = keys.device
    if n == 0:
        return values.reshape(-1).clone(), torch.empty(0, dtype=torch.int32, device=dev), torch.empty(
            0, dtype=torch.int64, device=dev)
    cap = 1
    while cap < 2 * n:
        cap <<= 1
    w = dict(
        tab_keys=torch.empty(cap, dtype=torch.int64, device=dev),
        tab_first=torch.empty(cap, dtype=torch.int32, device=dev),
        slot_of=torch.empty(n, dtype=torch.int64, device=dev),
        is_first=torch.empty(n, dtype=torch.int32, device=dev),
        pos=torch.empty(n + 1, dtype=torch.int32, device=dev),
        block_sums=torch.empty(512, dtype=torch.int32, device=dev),
    )
    unique = torch.empty(n, dtype=torch.int64, device=dev)
    inverse = torch.empty(n, dtype=torch.int32, device=dev)
    first = torch.empty(n, dtype=torch.int64, device=dev)
    native().unique_first_occurrence(
        keys.data_ptr(), n, {k: (v.data_ptr() if isinstance(v, torch.Tensor) else v) for k, v in
                             dict(w, cap=cap).items()}, unique.data_ptr(), inverse.data_ptr(), first.data_ptr())
    count = int(w["pos"][n].item())
    return unique[:count].to(values.dtype), inverse, first[:count]


__all__ = [
    "CpuSparseEmbeddingOperator",
    "CudaSparseEmbeddingOperator",
    "SPARSE_EMBEDDING_OPERATOR_BACKENDS",
    "SparseEmbeddingOperator",
    "create_sparse_embedding_operator",
    "pooled_sparse_widths",
    "unique_first_occurrence",
    "unique_first_occurrence_reference",
]
