"""Routed ragged batch ops keep splits and routing metadata consistent (CPU, NumPy and torch)."""
import numpy as np
import pytest
import torch

from flare_b200.data.transport import RoutedRagged, concatenate, pad, take


def _mk(lengths, start, mod=np):
    s = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    vals = np.arange(start * 100, start * 100 + s[-1], dtype=np.int64)
    origin = np.arange(start, start + len(lengths), dtype=np.int64)
    if mod is torch:
        return RoutedRagged(torch.from_numpy(vals), (torch.from_numpy(s),), torch.from_numpy(origin), 10, 3)
    return RoutedRagged(vals, (s,), origin, 10, 3)


@pytest.mark.parametrize("mod", [np, torch])
def test_concat_take_pad(mod):
    a, b = _mk([2, 0, 3], 0, mod), _mk([1, 4], 3, mod)
    c = concatenate([a, b])
    assert c.rows == 5 and list(np.asarray(c.splits[0])) == [0, 2, 2, 5, 6, 10]
    assert list(np.asarray(c.origin)) == [0, 1, 2, 3, 4]
    t = take(c, 2, 2)
    assert list(np.asarray(t.splits[0])) == [0, 3, 4] and list(np.asarray(t.flat_values)) == [2, 3, 4, 300]
    p = pad(t, 2)
    assert p.rows == 4 and p.valid_rows() == 2 and list(np.asarray(p.origin)) == [2, 3, -1, -1]
    assert list(np.asarray(p.flat_values))[-2:] == [300, 300]
    with pytest.raises(ValueError):
        concatenate([a, RoutedRagged(b.flat_values, b.splits, b.origin, 11, 3)])
    with pytest.raises(ValueError):
        take(c, 4, 3)
