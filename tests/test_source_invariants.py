"""Structural rules over the Python sources (parsed, never run), as the reference suite enforces
(``tests/unit/test_source_invariants.py:74-218``):

* every raw ``torch.distributed`` collective names its process group (``group=``), so no call
  silently runs on the default world group;
* no ``raise`` sits under a rank-0-only branch (``if ...is_primary`` / ``if rank == 0``): one rank
  raising while its peers enter the next collective hangs them instead of failing them;
* no rank-guarded ``return`` precedes a collective in the same function: the guarded ranks would
  skip a collective that the others wait in.
"""

from __future__ import annotations

import ast
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "build-your-own-hybrid-distributed-training_b200"
FILES = sorted([*PKG.rglob("*.py"), *(ROOT / "examples").glob("*.py"), ROOT / "bench.py"])

RAW_COLLECTIVES = {"all_reduce", "broadcast", "all_gather", "all_gather_into_tensor", "reduce_scatter_tensor", "reduce_scatter",
                   "all_to_all", "all_to_all_single", "send", "recv", "isend", "irecv", "barrier", "all_gather_object",
                   "broadcast_object_list", "reduce", "gather", "scatter"}
WRAPPED_COLLECTIVES = {"all_reduce", "broadcast", "all_gather_tensor", "reduce_scatter_tensor", "all_to_all_tensor",
                       "all_gather_object_in_group", "assert_metadata_consistent", "assert_tensor_consistent", "sum_scalar",
                       "barrier", "send_tensor", "recv_tensor"}


def _trees() -> list[tuple[Path, ast.AST]]:
    return [(p, ast.parse(p.read_text(encoding="utf-8"), filename=str(p))) for p in FILES]


def _is_rank_guard(test: ast.expr) -> bool:
    text = ast.unparse(test)
    return "is_primary" in text or "rank == 0" in text or "rank != 0" in text


def _calls_collective(node: ast.AST) -> bool:
    for sub in ast.walk(node):
        if isinstance(sub, ast.Call):
            f = sub.func
            if isinstance(f, ast.Attribute) and isinstance(f.value, ast.Name) and f.value.id == "dist" and f.attr in RAW_COLLECTIVES:
                return True
            if isinstance(f, ast.Name) and f.id in WRAPPED_COLLECTIVES:
                return True
    return False


def test_sources_parse() -> None:
    assert len(_trees()) > 40


def test_raw_collectives_name_their_group() -> None:
    offenders = []
    for path, tree in _trees():
        for node in ast.walk(tree):
            if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and isinstance(node.func.value, ast.Name)
                    and node.func.value.id == "dist" and node.func.attr in RAW_COLLECTIVES
                    and not any(k.arg == "group" for k in node.keywords)):
                offenders.append(f"{path.relative_to(ROOT)}:{node.lineno} dist.{node.func.attr}")
    assert not offenders, offenders


def test_no_raise_under_a_rank_zero_branch() -> None:
    offenders = []
    for path, tree in _trees():
        for node in ast.walk(tree):
            if isinstance(node, ast.If) and _is_rank_guard(node.test):
                for stmt in node.body:
                    for sub in ast.walk(stmt):
                        if isinstance(sub, ast.Raise):
                            offenders.append(f"{path.relative_to(ROOT)}:{sub.lineno}")
    assert not offenders, offenders


def test_no_rank_guarded_return_before_a_collective() -> None:
    offenders = []
    for path, tree in _trees():
        for fn in ast.walk(tree):
            if not isinstance(fn, (ast.FunctionDef, ast.AsyncFunctionDef)):
                continue
            body = fn.body
            for i, stmt in enumerate(body):
                if isinstance(stmt, ast.If) and _is_rank_guard(stmt.test) and any(isinstance(s, ast.Return) for s in stmt.body):
                    if any(_calls_collective(later) for later in body[i + 1:]):
                        offenders.append(f"{path.relative_to(ROOT)}:{stmt.lineno} in {fn.name}")
    assert not offenders, offenders


@pytest.mark.parametrize("snippet,rule", [
    ("import torch.distributed as dist\ndist.all_reduce(t)\n", "group"),
    ("def f(ctx):\n    if ctx.is_primary:\n        raise ValueError('x')\n", "raise"),
    ("def f(ctx, g, t):\n    if ctx.rank == 0:\n        return 1\n    all_reduce(t, g)\n", "return"),
])
def test_rules_catch_known_violations(snippet: str, rule: str) -> None:
    """The checkers above flag each kind of violation (guards against a rule silently matching nothing)."""
    tree = ast.parse(snippet)
    if rule == "group":
        calls = [n for n in ast.walk(tree) if isinstance(n, ast.Call)]
        assert any(not any(k.arg == "group" for k in c.keywords) for c in calls)
    elif rule == "raise":
        ifs = [n for n in ast.walk(tree) if isinstance(n, ast.If) and _is_rank_guard(n.test)]
        assert ifs and any(isinstance(s, ast.Raise) for n in ifs for s in ast.walk(n))
    else:
        fn = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef))
        guard = next(i for i, s in enumerate(fn.body) if isinstance(s, ast.If) and _is_rank_guard(s.test))
        assert any(_calls_collective(s) for s in fn.body[guard + 1:])
