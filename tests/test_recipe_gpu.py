"""A user model (multitask PLE recipe) on the fused path: trainer, graph assembly, 2-GPU equivalence."""
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.nn as nn

from flare_b200.models.dlrm import RowwiseAdagradTorch
from flare_b200.recipes.multitask import MultitaskModelBuilder, MultitaskRankingRecipe, synthetic_multitask_batch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _torch_replica(builder, tr, seed):
    """The same model in plain PyTorch fp32: nn.EmbeddingBag tables copied from the fused collection."""
    torch.manual_seed(seed)
    module = builder.create_module().to(tr.device)
    embs = nn.ModuleList()
    for i, s in enumerate(tr.coll.shards):
        e = nn.EmbeddingBag(s.spec.num_embeddings, s.spec.embedding_dim, mode="sum", sparse=True).to(tr.device)
        with torch.no_grad():
            e.weight.copy_(tr.coll.shard_view(i).float())
        embs.append(e)
    return module, embs


def _pooled_ref(embs, offsets, values, B):
    offs = offsets.long()
    outs = []
    for f, e in enumerate(embs):
        seg = offs[f * B:(f + 1) * B + 1]
        outs.append(e(values[seg[0]:seg[-1]].long(), seg[:-1] - seg[0]))
    return torch.cat(outs, 1)


def test_multitask_recipe_trains_on_fused_path_and_tracks_pytorch(cuda):
    builder = MultitaskModelBuilder()
    recipe = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=512, builder=builder)
    tr = recipe.trainer(device=cuda, use_graph=True, seed=4)
    ref_mod, ref_embs = _torch_replica(builder, tr, 4)
    objective = recipe.ranking_task().objective
    opt_d = torch.optim.Adam(ref_mod.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8)
    opt_s = RowwiseAdagradTorch([e.weight for e in ref_embs], lr=0.05)
    B = recipe.batch_size
    fused, plain = [], []
    for step in range(30):
        dense, labels, offs, vals = synthetic_multitask_batch(B, builder.vocabs, builder.num_dense,
                                                             builder.max_bag_size, seed=100 + step, device=cuda)
        fused.append(tr.train_step(dense, labels, offs, vals).loss)
        if step < 8:
            pooled = _pooled_ref(ref_embs, offs, vals, B)
            logits = ref_mod(dense, pooled, {})
            loss = objective(logits, labels, torch.full((B,), 1.0 / B, device=cuda))
            opt_d.zero_grad(set_to_none=True)
            opt_s.zero_grad()
            loss.backward()
            opt_d.step()
            opt_s.step()
            plain.append(float(loss))
    tr.check()
    assert tr.graph is not None  # steps after the warm-up replay one CUDA graph
    for i, (a, p) in enumerate(zip(fused, plain)):
        assert abs(a - p) <= 0.03 * abs(p) + 3e-3, (i, fused[:8], plain)
    assert sum(fused[-5:]) < sum(fused[:5])


def test_assembled_training_and_evaluation_graphs(cuda, tmp_path):
    from flare_b200.recipes.graph import (RANKING_PHASE_ORDER, assemble_ranking_evaluation_graph,
                                          assemble_ranking_training_graph, build_pipeline_nodes)

    builder = MultitaskModelBuilder()
    recipe = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=512, builder=builder)

    def source(seed0):
        s = seed0
        while True:
            yield synthetic_multitask_batch(512, builder.vocabs, builder.num_dense, builder.max_bag_size, seed=s,
                                            device=cuda)
            s += 1

    inputs = build_pipeline_nodes(recipe, source=source(0), device=cuda, seed=1)
    g = assemble_ranking_training_graph(inputs, metrics_static_args=dict(targets=("click", "like"), window_steps=10))
    losses = g["task_graph"].run(40)
    assert set(g["task_graph"].phase_seconds) == set(RANKING_PHASE_ORDER)
    assert losses[-1] < losses[0]
    assert g["metrics"].window.completed or g["metrics"].window.total_steps == 40
    # a timeline without per-step loss reads, at a batch where the GPU step outlasts the host's work per
    # step (pre-built device batches, no metric forward): the host materialises the next step's batch
    # while the GPU trains this one
    import itertools

    from flare_b200.validation.overlap import effective_overlap, phase_overlap
    from flare_b200.validation.perfetto import PerfettoWriter, parse_trace

    big_B = 8192
    big = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=big_B, builder=builder)
    pool = [synthetic_multitask_batch(big_B, builder.vocabs, builder.num_dense, builder.max_bag_size, seed=50 + i,
                                      device=cuda) for i in range(4)]
    tl = assemble_ranking_training_graph(build_pipeline_nodes(big, source=itertools.cycle(pool), device=cuda,
                                                              seed=1))["task_graph"]
    tl.run(4)  # eager steps and the graph capture
    w = PerfettoWriter()
    tl.run(12, read_loss_every=0, trace=w)
    path = w.save(tmp_path / "ranking.pftrace")
    rep = phase_overlap(parse_trace(path), set(range(5, 15)))
    assert len(rep["rows"]) == 10 and all(r["overlaps"]["materialize_next"]["present"] for r in rep["rows"])
    eff = effective_overlap(rep, relations=("materialize_next",))
    assert eff["relations"]["materialize_next"]["positive_hidden_count"] > 0, eff
    ev_inputs = build_pipeline_nodes(recipe, source=source(10_000), device=cuda, seed=1)
    ev_inputs.trainer = inputs.trainer  # evaluate the trained model
    out = assemble_ranking_evaluation_graph(ev_inputs)["task_graph"].run(4)
    assert out["auc/click"] > 0.6 and out["auc/like"] > 0.6, out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multitask_recipe_two_gpus_match_one_gpu_on_global_batch():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           "-m", "flare_b200.recipes.multitask_dist_check"]
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=450)
    assert res.returncode == 0 and "RECIPE_DIST_OK" in res.stdout, (res.stdout + res.stderr)[-5000:]


def test_user_model_accumulation_window_equals_the_union_step(cuda):
    """A user model (multitask PLE) with 2-micro-step windows against the same model stepping once on
    the union of the two micro-batches: equal losses window by window (SGD tables, Adam dense)."""
    from flare_b200.sparse.config import SparseOptimizerConfig

    builder = MultitaskModelBuilder(sparse_optimizer=SparseOptimizerConfig(kind="sgd", learning_rate=0.05))
    B = 256
    win = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=B, builder=builder).trainer(
        device=cuda, use_graph=True, seed=6, accumulation_steps=2)
    one = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=2 * B, builder=builder).trainer(
        device=cuda, use_graph=True, seed=6)
    F = len(builder.vocabs)

    def union(a, b):
        offs, vals, base = [0], [], 0
        for f in range(F):
            for x in (a, b):
                seg = x[2][f * B:(f + 1) * B + 1].long()
                vals.append(x[3][seg[0]:seg[-1]])
                offs.extend((seg[1:] - seg[0] + base).tolist())
                base += int(seg[-1] - seg[0])
        return (torch.cat([a[0], b[0]]), torch.cat([a[1], b[1]]),
                torch.tensor(offs, dtype=torch.int32, device=cuda), torch.cat(vals))

    for w in range(6):
        a, b = [synthetic_multitask_batch(B, builder.vocabs, builder.num_dense, builder.max_bag_size,
                                          seed=500 + 2 * w + k, device=cuda) for k in range(2)]
        la = win.train_step(*a).loss
        lb = win.train_step(*b).loss
        lu = one.train_step(*union(a, b)).loss
        assert abs((la + lb) / 2 - lu) <= 0.02 * abs(lu) + 2e-3, (w, la, lb, lu)
    assert win.coll.step == one.coll.step == 6 and win.coll.micro_filled == 0
    assert len(win.graphs) == 2  # one graph per micro-step position
    win.check()
    one.check()


def test_user_model_checkpoint_resume_matches_an_uninterrupted_run(cuda, tmp_path):
    """Train 4 steps with a checkpoint after step 2; a trainer built from another seed restores step 2 and
    trains steps 3-4 on the same batches: dense master weights and tables equal the uninterrupted run's."""
    from flare_b200.checkpoint.store import CheckpointManager

    builder = MultitaskModelBuilder()
    recipe = MultitaskRankingRecipe(name="mt", task_name="ranking", batch_size=256, builder=builder)
    batches = [synthetic_multitask_batch(256, builder.vocabs, builder.num_dense, builder.max_bag_size,
                                         seed=900 + k, device=cuda) for k in range(4)]
    mgr = CheckpointManager(str(tmp_path / "ck"))
    a = recipe.trainer(device=cuda, use_graph=True, seed=1)
    for k, b in enumerate(batches):
        a.train_step(*b)
        if k == 1:
            a.save_checkpoint(mgr, 2)
    b_tr = recipe.trainer(device=cuda, use_graph=True, seed=2)
    assert b_tr.restore_checkpoint(mgr) == 2 and b_tr.dense.state.step == 2 and b_tr.coll.step == 2
    for b in batches[2:]:
        b_tr.train_step(*b)
    torch.cuda.synchronize()
    a.check()
    b_tr.check()
    dm = (a.dense.state.master - b_tr.dense.state.master).abs().max().item()
    dw = (a.coll.weights - b_tr.coll.weights).abs().max().item()
    assert dm < 1e-5 and dw < 1e-5, (dm, dw)


def test_cli_recipe_trains_checkpoints_resumes_and_evaluates(tmp_path, capsys):
    import json

    from flare_b200 import cli

    ck = str(tmp_path / "ck")
    base = ["recipe", "--recipe", "flare_b200.recipes.multitask:make_recipe", "--batch-per-gpu", "512",
            "--checkpoint-dir", ck, "--log-every", "3", "--eval-batches", "2"]
    assert cli.main(base + ["--steps", "6", "--save-every", "3", "--incremental"]) == 0
    assert cli.main(base + ["--steps", "3", "--save-every", "3", "--resume", "--accumulation-steps", "2"]) == 0
    out = capsys.readouterr().out.strip().splitlines()
    res = json.loads(out[-1])
    assert res["last_step"] == 9 and res["eval_samples"] == 1024
    assert 0.5 < res["auc_click"] <= 1.0 and 0.5 < res["auc_like"] <= 1.0
    assert any(line.startswith("[recipe multitask] step 9 loss") for line in out)
