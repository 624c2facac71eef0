"""Recipe schema helpers and the synthetic ranking example (CPU)."""
import numpy as np
import pytest

from flare_b200.recipes.examples import run_synthetic_ranking
from flare_b200.recipes.schema import (build_ranking_batch_schema, build_sparse_group_feature_widths,
                                       extract_sparse_base_names, extract_sparse_groups_and_dimensions,
                                       materialize_padded_inverse, parse_sparse_group_name,
                                       parse_sparse_thread_budgets, parse_sparse_workers, validate_inverse_range)

GROUPS = ("users_dim_32", "items_dim_64", "items_dim_16")


def test_batch_schema():
    s = build_ranking_batch_schema(GROUPS[:2])
    assert s["users_dim_32"].is_sparse and s["labels"].is_label and "group_id" in s
    assert s["samples_valid_count"].spec.shape == () and s["side_info"].spec.dtype == "float32"
    assert "group_id" not in build_ranking_batch_schema(GROUPS, include_group_id=False)


def test_group_names_and_counts():
    assert parse_sparse_group_name("a_dim_b_dim_8") == ("a_dim_b", 8)
    for bad in ("", "users", "_dim_8", "users_dim_x", "users_dim_0"):
        with pytest.raises(ValueError):
            parse_sparse_group_name(bad)
    names, dims = extract_sparse_groups_and_dimensions(list(GROUPS))
    assert names == GROUPS and dims == {"users": [32], "items": [16, 64]}
    assert extract_sparse_base_names(GROUPS) == ("items", "users")
    assert parse_sparse_workers("", GROUPS) == {"items": 1, "users": 1}
    assert parse_sparse_workers("4", GROUPS) == {"items": 4, "users": 4}
    assert parse_sparse_workers("users:2", GROUPS) == {"items": 1, "users": 2}
    assert parse_sparse_thread_budgets("items:8", GROUPS) == {"items": 8}
    assert parse_sparse_thread_budgets("", GROUPS) == {}
    for bad in ("users:0", "nobody:2", "users:1,users:2", "users", "users:1:2"):
        with pytest.raises(ValueError):
            parse_sparse_workers(bad, GROUPS)
    w = build_sparse_group_feature_widths({"g": ["a", "b"]}, {"a": 3, "b": 7}, ["g"])
    assert w == {"g": (2, 7)}
    with pytest.raises(KeyError):
        build_sparse_group_feature_widths({"g": ["a"]}, {}, ["g"])


def test_padded_inverse_from_ragged_and_dense():
    # 3 samples, 2 features each, ragged ids per feature; target widths (2 features, 3 ids)
    feature_splits = np.array([0, 2, 4, 6])                 # samples -> features
    id_splits = np.array([0, 1, 3, 3, 7, 8, 9])            # features -> ids (the 4th has 4 ids: one dropped)
    flat = np.array([5, 6, 7, 1, 2, 3, 4, 9, 8])
    out = materialize_padded_inverse(flat, (feature_splits, id_splits), (3, 2, 4), pad_index=10, batch_size=3,
                                     target_widths=(2, 3), group="g", audit=True)
    want = np.full((3, 2, 3), 10)
    want[0, 0, :1] = [5]
    want[0, 1, :2] = [6, 7]
    want[1, 1, :3] = [1, 2, 3]
    want[2, 0, :1] = [9]
    want[2, 1, :1] = [8]
    assert out.tolist() == want.tolist() and out.dtype == np.int32
    dense = materialize_padded_inverse(np.array([[1, 2], [3, 4]]), None, None, pad_index=9, batch_size=2,
                                       target_widths=(3,), group="g", audit=True)
    assert dense.tolist() == [[1, 2, 9], [3, 4, 9]]
    with pytest.raises(ValueError, match="offsets"):
        materialize_padded_inverse(flat, (feature_splits, np.array([0, 1, 3, 2, 7, 8, 9])), (3, 2, 4), pad_index=10,
                                   batch_size=3, target_widths=(2, 3), group="g")
    with pytest.raises(IndexError):
        validate_inverse_range(np.array([0, 11]), 10, "g")
    with pytest.raises(ValueError, match="no slots"):
        validate_inverse_range(np.array([], dtype=np.int64), 10, "g")


def test_synthetic_ranking_example_learns():
    out = run_synthetic_ranking()
    assert out["target_names"] == ["engagement", "reply"]
    assert out["final_loss"] < 0.6 * out["initial_loss"]
    s = np.array(out["scores"])
    assert (s[:2] < 0.5).all() and (s[2:] > 0.5).all()
