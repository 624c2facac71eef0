"""Architecture rules checked on the source (AST), no GPU needed.

* The public packages never import the recipes (applications built on the
  framework), as the reference's public / recipe boundary test does
  (tests/architecture/test_public_recipe_boundary.py:13-39).
* The methods that a CUDA graph captures (the fused training step and its
  parts) make no host round trip: no ``.item()``, ``.tolist()``, ``.cpu()``,
  ``.numpy()``, device synchronisation or printing.  The reference checks that
  tracing and validation stay off its hot path by AST inspection
  (tests/architecture/test_training_hot_path.py:25-69).
* No compiler-based kernel layer is imported anywhere: the kernels are the
  hand-written sm_100a sources in ``flare_b200/csrc``.
"""
import ast
from pathlib import Path

import pytest

PKG = Path(__file__).resolve().parents[1] / "flare_b200"

HOT_PATH = {
    "models/dlrm.py": {"DLRM": ["forward_backward", "train_step", "_pipelined_step", "advance_host_state"]},
    "models/mlp.py": {"MLPTower": ["forward", "backward"]},
    "sparse/collection.py": {"ShardedEmbeddingBagCollection": ["forward", "backward", "set_input"]},
    "training/flat.py": {"DenseState": ["apply"]},
}
HOST_SYNC_ATTRS = {"item", "tolist", "cpu", "numpy", "synchronize"}
HOST_SYNC_NAMES = {"print"}


def _modules():
    for path in sorted(PKG.rglob("*.py")):
        yield path, ast.parse(path.read_text(), filename=str(path))


def _imported_names(tree: ast.AST, path: Path) -> list[str]:
    names = []
    pkg_parts = path.relative_to(PKG.parent).with_suffix("").parts[:-1]
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            names += [a.name for a in node.names]
        elif isinstance(node, ast.ImportFrom):
            if node.level:
                base = list(pkg_parts[:len(pkg_parts) - node.level + 1])
                mod = ".".join(base + ([node.module] if node.module else []))
            else:
                mod = node.module or ""
            names.append(mod)
            names += [f"{mod}.{a.name}" for a in node.names]
    return names


def test_public_packages_do_not_import_recipes():
    offenders = []
    for path, tree in _modules():
        rel = path.relative_to(PKG)
        if rel.parts[0] == "recipes":
            continue
        if any(n == "flare_b200.recipes" or n.startswith("flare_b200.recipes.") for n in _imported_names(tree, path)):
            offenders.append(str(rel))
    assert not offenders, f"public modules import recipes: {offenders}"


def test_no_compiler_kernel_layers():
    banned = ("triton", "tilelang")
    offenders = []
    for path, tree in _modules():
        for n in _imported_names(tree, path):
            if n.split(".")[0] in banned:
                offenders.append(f"{path.relative_to(PKG)}: {n}")
        for node in ast.walk(tree):
            if isinstance(node, ast.Attribute) and node.attr == "compile" and isinstance(node.value, ast.Name) \
                    and node.value.id == "torch":
                offenders.append(f"{path.relative_to(PKG)}: torch.compile")
    assert not offenders, offenders


def _method(tree: ast.AST, cls: str, name: str) -> ast.FunctionDef:
    for node in ast.walk(tree):
        if isinstance(node, ast.ClassDef) and node.name == cls:
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == name:
                    return item
    raise AssertionError(f"{cls}.{name} not found")


@pytest.mark.parametrize("rel,cls,meth", [(r, c, m) for r, cs in HOT_PATH.items() for c, ms in cs.items() for m in ms])
def test_graph_captured_methods_make_no_host_round_trip(rel, cls, meth):
    tree = ast.parse((PKG / rel).read_text())
    fn = _method(tree, cls, meth)
    bad = []
    for node in ast.walk(fn):
        if isinstance(node, ast.Call):
            f = node.func
            if isinstance(f, ast.Attribute) and f.attr in HOST_SYNC_ATTRS:
                bad.append(f"line {node.lineno}: .{f.attr}()")
            if isinstance(f, ast.Name) and f.id in HOST_SYNC_NAMES:
                bad.append(f"line {node.lineno}: {f.id}()")
    assert not bad, f"{rel} {cls}.{meth}: {bad}"


def test_nothing_imports_scratch_folders():
    for path, tree in _modules():
        for n in _imported_names(tree, path):
            assert not n.startswith("_work"), f"{path}: imports {n}"
