"""CPU reference embedding-bag collection (PyTorch, fp32).

Same keyed-jagged input contract and optimizer semantics as the fused GPU
collection; used as the numerics oracle for the CUDA kernels and as the sparse
backend of the CPU (gloo, world size 1) configuration.  Gather/pool semantics
follow the reference's Numba ops (src/flare/ops/sparse_gather.py:40-99) and
its pooled scatter (src/flare/ops/sparse_scatter.py:36-95).
"""
from __future__ import annotations

import math

import torch

from .config import SparseOptimizerConfig, SparseTableSpec
from .precision import TORCH_DTYPES


def pool_reference(weights: list[torch.Tensor], tables: list[SparseTableSpec], offsets: torch.Tensor,
                   values: torch.Tensor, B: int) -> torch.Tensor:
    F = len(tables)
    dims = [t.embedding_dim for t in tables]
    out = torch.zeros(B, sum(dims), dtype=torch.float32)
    offs = offsets.long()
    vals = values.long()
    col = 0
    for f, t in enumerate(tables):
        beg = offs[f * B:(f + 1) * B]
        end = offs[f * B + 1:(f + 1) * B + 1]
        lens = end - beg
        ids = vals[beg[0]:end[-1]] if B else vals[:0]
        bag = torch.repeat_interleave(torch.arange(B), lens)
        keep = ids >= 0
        rows = weights[f].float()[ids.clamp_min(0)] * keep.unsqueeze(1)
        pooled = torch.zeros(B, dims[f])
        pooled.index_add_(0, bag, rows)
        if t.pooling == "mean":
            pooled = pooled / lens.clamp_min(1).unsqueeze(1).float()
        out[:, col:col + dims[f]] = pooled
        col += dims[f]
    return out


def row_gradients(tables, offsets, values, grad_pooled, B):
    """Per table: (unique rows, summed fp32 gradient rows, occurrence counts)."""
    res = []
    offs = offsets.long()
    vals = values.long()
    g = grad_pooled.float()
    col = 0
    for f, t in enumerate(tables):
        d = t.embedding_dim
        beg = offs[f * B:(f + 1) * B]
        end = offs[f * B + 1:(f + 1) * B + 1]
        lens = end - beg
        ids = vals[beg[0]:end[-1]] if B else vals[:0]
        bag = torch.repeat_interleave(torch.arange(B), lens)
        gb = g[:, col:col + d]
        if t.pooling == "mean":
            gb = gb / lens.clamp_min(1).unsqueeze(1).float()
        keep = ids >= 0
        ids, bag = ids[keep], bag[keep]
        uniq, inv = torch.unique(ids, return_inverse=True)
        acc = torch.zeros(uniq.numel(), d)
        acc.index_add_(0, inv, gb[bag])
        cnt = torch.bincount(inv, minlength=uniq.numel()).float()
        res.append((uniq, acc, cnt))
        col += d
    return res


def lr_scale_reference(opt: SparseOptimizerConfig, score: torch.Tensor) -> torch.Tensor:
    p = opt.dynamic_lr_policy
    if p == "constant":
        return torch.ones_like(score)
    if p == "sqrt_decay":
        return torch.rsqrt(score.clamp_min(1.0))
    if p == "log_decay":
        return 1.0 / (1.0 + torch.log1p(score.clamp_min(0.0)))
    if p == "inverse_decay":
        return 1.0 / score.clamp_min(1.0)
    if p == "cosine_frequency":
        S = max(opt.cosine_max_score, 1e-12)
        x = score.clamp(0.0, opt.cosine_max_score) / S
        r = opt.cosine_min_lr_ratio
        return r + (1 - r) * 0.5 * (1 + torch.cos(math.pi * x))
    lut = torch.tensor(opt.custom_lut, dtype=torch.float32)
    idx = score.clamp_min(0).floor().long().clamp_max(len(opt.custom_lut) - 1)
    return lut[idx]


def apply_rows_reference(opt: SparseOptimizerConfig, step: int, w: torch.Tensor, rows: torch.Tensor,
                         g: torch.Tensor, cnt: torch.Tensor, state: dict) -> None:
    """In-place row update of table ``w`` (fp32 math) for the given unique rows."""
    if rows.numel() == 0:
        return
    wr = w[rows].float()
    g = g + opt.weight_decay * wr
    lr = torch.full((rows.numel(), 1), opt.learning_rate)
    if "score" in state:
        sc = state["score"][rows] + cnt
        state["score"][rows] = sc
        lr = lr * lr_scale_reference(opt, sc).unsqueeze(1)
    t = max(step, 1)
    bc1, bc2 = 1 - opt.beta1 ** t, 1 - opt.beta2 ** t
    k = opt.kind
    if k == "sgd":
        wr = wr - lr * g
    elif k == "rowwise_adagrad":
        s = state["row"][rows] + (g * g).mean(1)
        state["row"][rows] = s
        wr = wr - lr * g / (torch.sqrt(s).unsqueeze(1) + opt.eps)
    elif k == "adagrad":
        m = state["m"][rows] + g * g
        state["m"][rows] = m
        wr = wr - lr * g / (torch.sqrt(m) + opt.eps)
    elif k == "adam":
        m = opt.beta1 * state["m"][rows] + (1 - opt.beta1) * g
        v = opt.beta2 * state["v"][rows] + (1 - opt.beta2) * g * g
        state["m"][rows], state["v"][rows] = m, v
        wr = wr - lr * (m / bc1) / (torch.sqrt(v / bc2) + opt.eps)
    elif k == "rowwise_adam":
        m = opt.beta1 * state["m"][rows] + (1 - opt.beta1) * g
        v = opt.beta2 * state["row"][rows] + (1 - opt.beta2) * (g * g).mean(1)
        state["m"][rows], state["row"][rows] = m, v
        wr = wr - lr * (m / bc1) / (torch.sqrt(v / bc2).unsqueeze(1) + opt.eps)
    w[rows] = wr.to(w.dtype)


def _table_stream_seed(seed: int, name: str) -> int:
    """Seed of a table's row-init stream: a function of the run seed and the table's name only."""
    import zlib

    return (int(seed) * 1_000_003 + 17 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF


class CpuEmbeddingBagCollection:
    """Whole tables on the host; same forward/backward contract as the GPU collection.

    With ``storage`` (``SparseStorageOptions``) every table lives in a native paged store instead
    of a tensor: one record per row holds the weights and the optimizer state, pages beyond the
    memory limit spill to disk, and a step reads and writes only the rows of its batch (the
    reference's external store with an AutoStorage memory limit and spill directory).
    """

    def __init__(self, tables: list[SparseTableSpec], batch_size: int, *, optimizer: SparseOptimizerConfig | None = None,
                 seed: int = 0, weights: list[torch.Tensor] | None = None, storage=None, native: bool = False):
        self.tables = list(tables)
        self.B = int(batch_size)
        self.optimizer = optimizer or tables[0].optimizer
        self.total_dim = sum(t.embedding_dim for t in tables)
        self.step = 0
        self._offsets = None
        self._values = None
        self.stores = None
        # native: pooling, per-row gradient sums and the row-wise optimizer in the host C++ ops
        # (parallel over bags / tables / rows, fp32, each row adds its occurrences in order) instead of
        # tensor ops; the tensor-op path stays the plain-PyTorch oracle of the GPU kernels
        self.native = bool(native)
        # hash-keyed tables: any int64 key; a native key -> slot map inserts on first sight (LFU eviction
        # when full) and the table's rows are indexed by slot
        self.maps = {}
        # one row-init generator per table, seeded from (seed, table name): rows of keys inserted later
        # draw from their own table's stream, whichever rank owns the table and whatever else it owns
        self._init_gens = [torch.Generator().manual_seed(_table_stream_seed(seed, t.name)) for t in self.tables]
        if any(t.dynamic for t in self.tables):
            from .._native import native as _nat

            self.maps = {f: _nat().DynamicKeyMap(t.num_embeddings) for f, t in enumerate(self.tables) if t.dynamic}
        if storage is not None:
            self._init_paged(storage, seed, weights)
            return
        g = torch.Generator().manual_seed(seed)
        if weights is None:
            weights = [((torch.rand(t.num_embeddings, t.embedding_dim, generator=g) * 2 - 1) * t.init_scale)
                       .to(TORCH_DTYPES[t.value_dtype]) for t in tables]
        self.weights = weights
        opt = self.optimizer
        self.state = []
        for t in tables:
            st = {}
            if opt.needs_row_state:
                st["row"] = torch.zeros(t.num_embeddings)
            if opt.needs_m:
                st["m"] = torch.zeros(t.num_embeddings, t.embedding_dim)
            if opt.needs_v:
                st["v"] = torch.zeros(t.num_embeddings, t.embedding_dim)
            if opt.needs_score:
                st["score"] = torch.zeros(t.num_embeddings)
            self.state.append(st)

    def set_input(self, offsets: torch.Tensor, values: torch.Tensor, non_blocking: bool = False) -> None:
        self._offsets, self._values = offsets.cpu(), values.cpu()
        self._keys = self._values  # the batch's ids as given (dynamic tables: keys, translated in forward)

    def _translate(self, training: bool) -> None:
        """Dynamic tables: keys -> slots (training lookups insert and re-initialise the new slots' rows)."""
        if not self.maps:
            return
        vals = self._keys.to(torch.int64).clone()
        offs, B = self._offsets.long(), self.B
        for f, m in self.maps.items():
            lo, hi = int(offs[f * B]), int(offs[(f + 1) * B])
            slots, new, _evicted = m.lookup(vals[lo:hi].contiguous(), training)
            vals[lo:hi] = slots
            if new.numel():
                self._init_rows(f, new)
        self._values = vals.to(torch.int32)

    def _init_rows(self, f: int, rows: torch.Tensor) -> None:
        t = self.tables[f]
        w = (torch.rand(rows.numel(), t.embedding_dim, generator=self._init_gens[f]) * 2 - 1) * t.init_scale
        if self.stores is not None:
            rec = torch.zeros(rows.numel(), sum(wd for _, wd in self.layouts[f]))
            rec[:, :t.embedding_dim] = w
            self.stores[f].scatter(rows, rec)
            return
        self.weights[f][rows] = w.to(self.weights[f].dtype)
        for v in self.state[f].values():
            v[rows] = 0

    def dynamic_items(self, f: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(keys, slots, use counts) of dynamic table f's occupied slots."""
        return self.maps[f].items()[:3]

    def _mean_flags(self) -> list[int]:
        return [1 if t.pooling == "mean" else 0 for t in self.tables]

    def forward(self, training: bool = True) -> torch.Tensor:
        self._translate(training)
        if self.stores is not None:
            return self._forward_paged()
        if self.native:
            from .._native import native

            return native().cpu.bag_pool([w.contiguous() for w in self.weights], self._offsets.int().contiguous(),
                                         self._values.int().contiguous(), self.B, self._mean_flags())
        return pool_reference(self.weights, self.tables, self._offsets, self._values, self.B)

    def _row_gradients(self, grad_pooled: torch.Tensor):
        if self.native:
            from .._native import native

            return native().cpu.bag_row_grads(grad_pooled.detach().float().contiguous(),
                                              self._offsets.int().contiguous(), self._values.int().contiguous(),
                                              self.B, [t.embedding_dim for t in self.tables], self._mean_flags())
        return row_gradients(self.tables, self._offsets, self._values, grad_pooled, self.B)

    def backward(self, grad_pooled: torch.Tensor, step: int | None = None) -> None:
        self.step = self.step + 1 if step is None else int(step)
        for f, (rows, g, cnt) in enumerate(self._row_gradients(grad_pooled)):
            if self.stores is not None:
                self._apply_paged(f, rows, g, cnt)
            elif self.native:
                self._apply_native(f, rows, g, cnt)
            else:
                apply_rows_reference(self.optimizer, self.step, self.weights[f], rows, g, cnt, self.state[f])

    def _apply_native(self, f: int, rows: torch.Tensor, g: torch.Tensor, cnt: torch.Tensor) -> None:
        from .._native import native
        from .config import LR_POLICIES, OPTIMIZER_KINDS

        opt, st, none = self.optimizer, self.state[f], torch.empty(0)
        native().cpu.apply_rows(OPTIMIZER_KINDS[opt.kind], LR_POLICIES[opt.dynamic_lr_policy],
                                [opt.learning_rate, opt.beta1, opt.beta2, opt.eps, opt.weight_decay,
                                 opt.cosine_min_lr_ratio, opt.cosine_max_score], list(opt.custom_lut), self.step,
                                self.weights[f], rows.long().contiguous(), g.float().contiguous(),
                                cnt.float().contiguous(), st.get("row", none), st.get("m", none), st.get("v", none),
                                st.get("score", none))

    # ------------------------------------------------------------ paged storage
    def _layout(self, t: SparseTableSpec) -> list[tuple[str, int]]:
        """Record fields (name, width): weights, then the optimizer state the optimizer keeps."""
        opt, d = self.optimizer, t.embedding_dim
        fields = [("weight", d)]
        if opt.needs_m:
            fields.append(("m", d))
        if opt.needs_v:
            fields.append(("v", d))
        if opt.needs_row_state:
            fields.append(("row", 1))
        if opt.needs_score:
            fields.append(("score", 1))
        return fields

    def _init_paged(self, storage, seed: int, weights) -> None:
        self.layouts = [self._layout(t) for t in self.tables]
        specs = [(t.name, t.num_embeddings, sum(w for _, w in lay), t.embedding_dim, t.init_scale)
                 for t, lay in zip(self.tables, self.layouts)]
        self.stores = storage.build_stores(specs, seed)
        if weights is not None:  # start from given tables (every row is written once)
            for f, w in enumerate(weights):
                ids = torch.arange(w.shape[0])
                rec = self.stores[f].gather(ids)
                rec[:, :w.shape[1]] = w.float()
                self.stores[f].scatter(ids, rec)

    def _split(self, f: int, rec: torch.Tensor) -> dict[str, torch.Tensor]:
        out, c = {}, 0
        for name, w in self.layouts[f]:
            out[name] = rec[:, c:c + w] if w > 1 else rec[:, c]
            c += w
        return out

    def _ids_of(self, f: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        B = self.B
        offs, vals = self._offsets.long(), self._values.long()
        beg, end = offs[f * B:(f + 1) * B], offs[f * B + 1:(f + 1) * B + 1]
        lens = end - beg
        ids = vals[beg[0]:end[-1]] if B else vals[:0]
        return ids, torch.repeat_interleave(torch.arange(B), lens), lens

    def _forward_paged(self) -> torch.Tensor:
        out = torch.zeros(self.B, self.total_dim, dtype=torch.float32)
        col = 0
        for f, t in enumerate(self.tables):
            d = t.embedding_dim
            ids, bag, lens = self._ids_of(f)
            keep = ids >= 0
            uniq, inv = torch.unique(ids.clamp_min(0), return_inverse=True)
            w = self._split(f, self.stores[f].gather(uniq))["weight"].to(TORCH_DTYPES[t.value_dtype]).float()
            pooled = torch.zeros(self.B, d)
            pooled.index_add_(0, bag, w[inv] * keep.unsqueeze(1))
            if t.pooling == "mean":
                pooled = pooled / lens.clamp_min(1).unsqueeze(1).float()
            out[:, col:col + d] = pooled
            col += d
        return out

    def _apply_paged(self, f: int, rows: torch.Tensor, g: torch.Tensor, cnt: torch.Tensor) -> None:
        if rows.numel() == 0:
            return
        rec = self.stores[f].gather(rows)
        parts = self._split(f, rec)
        w = parts["weight"].to(TORCH_DTYPES[self.tables[f].value_dtype])
        state = {k: v.clone() for k, v in parts.items() if k != "weight"}
        apply_rows_reference(self.optimizer, self.step, w, torch.arange(rows.numel()), g, cnt, state)
        c = 0
        for name, width in self.layouts[f]:
            v = w.float() if name == "weight" else state[name]
            rec[:, c:c + width] = v if width > 1 else v.unsqueeze(1)
            c += width
        self.stores[f].scatter(rows, rec)

    def table_weights(self, f: int) -> torch.Tensor:
        """Table f's weights (every row; reads the whole paged table when stored)."""
        if self.stores is None:
            return self.weights[f]
        t = self.tables[f]
        return self._split(f, self.stores[f].gather(torch.arange(t.num_embeddings)))["weight"].clone()

    # ------------------------------------------------------------ checkpoint state
    def state_dict(self) -> dict:
        """Step, every table's weights and optimizer state (by table name), dynamic tables' key maps."""
        tables = {}
        for f, t in enumerate(self.tables):
            if self.stores is not None:
                parts = self._split(f, self.stores[f].gather(torch.arange(t.num_embeddings)))
                tables[t.name] = {k: v.clone() for k, v in parts.items()}
            else:
                tables[t.name] = {"weight": self.weights[f].clone(), **{k: v.clone() for k, v in self.state[f].items()}}
            # the table's row-init stream travels with the table (rows of keys inserted later draw from it)
            tables[t.name]["init_rng"] = self._init_gens[f].get_state()
        dynamic = {self.tables[f].name: tuple(x.clone() for x in m.items()) for f, m in self.maps.items()}
        return {"step": self.step, "optimizer": self.optimizer.kind, "tables": tables, "dynamic": dynamic}

    def load_state_dict(self, state: dict) -> None:
        if state.get("optimizer", self.optimizer.kind) != self.optimizer.kind:
            raise ValueError(f"checkpoint optimizer {state['optimizer']!r} is not {self.optimizer.kind!r}")
        for f, t in enumerate(self.tables):
            if t.name not in state["tables"]:
                raise ValueError(f"table {t.name} is not in the checkpoint")
            st = state["tables"][t.name]
            if "init_rng" in st:
                self._init_gens[f].set_state(st["init_rng"])
            if self.stores is not None:
                rec = torch.cat([st[n].float().reshape(t.num_embeddings, -1) for n, _ in self.layouts[f]], 1)
                self.stores[f].scatter(torch.arange(t.num_embeddings), rec)
            else:
                self.weights[f].copy_(st["weight"].to(self.weights[f].dtype))
                for k, v in self.state[f].items():
                    v.copy_(st[k])
        for f, m in self.maps.items():
            m.load(*state["dynamic"][self.tables[f].name])
        self.step = int(state["step"])

    def storage_stats(self) -> list[dict]:
        return [s.stats() for s in self.stores] if self.stores is not None else []


__all__ = ["CpuEmbeddingBagCollection", "apply_rows_reference", "lr_scale_reference", "pool_reference",
           "row_gradients"]
