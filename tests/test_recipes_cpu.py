"""CPU configuration: training vs the plain PyTorch oracle, paged tables, checkpoint / resume (CPU)."""
import numpy as np
import torch

from flare_b200.recipes.cpu_small import train_small_cpu, train_small_oracle
from flare_b200.recipes.ranking import MultiTargetCrossEntropyLoss, RankingLossAdapter, RankingTask


def test_cpu_small_config_matches_pytorch_oracle_and_learns():
    res = train_small_cpu(steps=200)
    oracle = train_small_oracle(steps=200)
    assert max(abs(a - b) for a, b in zip(res.losses, oracle)) < 1e-4
    assert np.mean(res.losses[-20:]) < np.mean(res.losses[:10]) - 0.1


def test_multitarget_loss_and_adapter():
    loss = MultiTargetCrossEntropyLoss.create(
        {"click": {"sample_weight": {"neg": -1.0, "click": 1.0, "buy": 2.0}},
         "buy": {"sample_weight": {"neg": -1.0, "click": -1.0, "buy": 3.0}, "class_weight": 0.5}},
        {"neg": 0, "click": 1, "buy": 2}, target_names=("click", "buy"))
    assert loss.target_labels.tolist() == [[0, 1, 1], [0, 0, 1]]
    logits = torch.zeros(4, 2)
    labels = torch.tensor([0, 1, 2, 2])
    full = loss(logits, labels, torch.ones(4))
    # BCE(0, y) = ln 2 for every entry; weights: click row |w|, buy row 0.5*|w|
    w = torch.tensor([[1, 0.5], [1, 0.5], [2, 1.5], [2, 1.5]])
    assert torch.allclose(full, w.sum() * np.log(2))
    adapter = RankingLossAdapter(loss)
    out = adapter({"logits": logits}, {"labels": labels, "samples_valid_count": [3], "global_row_start": 0,
                                       "world_size": 1})
    assert torch.allclose(out, w[:3].sum() * np.log(2) / 3)
    RankingTask("label", "group", loss)


def test_cpu_recipe_with_paged_tables_trains_identically(tmp_path):
    from flare_b200.sparse.storage import SparseStorageOptions

    opts = SparseStorageOptions(memory_limit_bytes=64 * 1024, spill_directory=str(tmp_path), entries_per_page=4096)
    a = train_small_cpu(steps=20, batch_size=64, native=False)  # the paged tables use the tensor-op optimizer
    b = train_small_cpu(steps=20, batch_size=64, storage=opts)
    assert a.losses == b.losses


def test_cpu_recipe_checkpoint_resume_matches_an_uninterrupted_run(tmp_path):
    from flare_b200.checkpoint.store import list_steps

    full = train_small_cpu(steps=12, batch_size=32)
    first = train_small_cpu(steps=6, batch_size=32, checkpoint_dir=str(tmp_path), save_every=3)
    assert list_steps(tmp_path) == [3, 6] and first.losses == full.losses[:6]
    second = train_small_cpu(steps=6, batch_size=32, checkpoint_dir=str(tmp_path), resume=True)
    assert second.losses == full.losses[6:]


def test_ranking_phase_schedule_contract():
    """The step's phases in dependency order; the cross-step edge (update -> next train_core) has
    distance 1; a same-step cycle is rejected."""
    import pytest

    from flare_b200.recipes.graph import (RANKING_PHASE_DEPENDENCIES, RANKING_PHASE_ORDER, RANKING_PHASES,
                                          schedule_order)

    order = schedule_order()
    assert set(order) == set(RANKING_PHASE_ORDER)
    pos = {n: i for i, n in enumerate(order)}
    for a, b, d in RANKING_PHASE_DEPENDENCIES:
        if d == 0:
            assert pos[a] < pos[b]
    assert ("update", "train_core", 1) in RANKING_PHASE_DEPENDENCIES
    with pytest.raises(ValueError):
        schedule_order(RANKING_PHASES, RANKING_PHASE_DEPENDENCIES + (("update", "train_core", 0),))


def test_cli_loads_recipes_and_builds_their_batches():
    import pytest
    import torch

    from flare_b200 import cli
    from flare_b200.recipes.multitask import make_recipe
    from flare_b200.recipes.ranking import BaseRankingRecipe

    r = cli.load_recipe("flare_b200.recipes.multitask:make_recipe", 128)
    assert isinstance(r, BaseRankingRecipe) and r.batch_size == 128
    import sys
    import types

    fake = types.ModuleType("_fake_recipe_module")
    fake.RECIPE = make_recipe(32)
    sys.modules[fake.__name__] = fake
    try:
        inst = cli.load_recipe("_fake_recipe_module:RECIPE", 96)  # an instance: batch size replaced
        assert inst.batch_size == 96 and fake.RECIPE.batch_size == 32
    finally:
        del sys.modules[fake.__name__]
    args = cli._parser().parse_args(["recipe", "--recipe", "m:f", "--accumulation-steps", "2", "--resume"])
    assert args.cmd == "recipe" and args.accumulation_steps == 2 and args.resume
    with pytest.raises(SystemExit):
        cli.load_recipe("flare_b200.recipes.multitask", 8)
    with pytest.raises(SystemExit):
        cli.load_recipe("flare_b200.recipes.multitask:multitask_objective", 8)  # not a recipe factory
    b = make_recipe(64).model_builder()
    dense, labels, offs, vals = cli.recipe_batch(b, 3, 64, 7, torch.device("cpu"))
    F = len(b.vocabs)
    assert dense.shape == (64, b.num_dense) and offs.shape == (F * 64 + 1,) and int(offs[-1]) == vals.numel()
    assert int(labels.min()) >= 0 and int(labels.max()) <= 2
    for f, v in enumerate(b.vocabs):
        seg = vals[int(offs[f * 64]):int(offs[(f + 1) * 64])]
        assert int(seg.max()) < v
