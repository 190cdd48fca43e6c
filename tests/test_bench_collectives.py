"""bench.py under torchrun: every rank takes the same collective steps.

The driver runs ``bench.py --gpus N`` as N processes; a collective that only
rank 0 reaches (a sum over ranks inside the code that builds rank 0's JSON
line) leaves the other ranks waiting until the process group times out. This
static check walks bench.py and fails if a cross-rank helper is called in
code that only rank 0 runs: inside ``if rank == 0:`` or after an early
``if rank != 0: return`` in the same function.
"""

from __future__ import annotations

import ast
import os

from conftest import REPO

COLLECTIVES = {"_sum_over_ranks", "_max_over_ranks", "_gather", "_barrier"}


def _calls(node) -> set[str]:
    out = set()
    for n in ast.walk(node):
        if isinstance(n, ast.Call) and isinstance(n.func, ast.Name):
            out.add(n.func.id)
    return out


def _is_rank_test(test, op) -> bool:
    return (isinstance(test, ast.Compare) and isinstance(test.left, ast.Name)
            and test.left.id == "rank" and len(test.ops) == 1 and isinstance(test.ops[0], op)
            and isinstance(test.comparators[0], ast.Constant) and test.comparators[0].value == 0)


def _rank0_only_regions(func: ast.FunctionDef):
    """Statements only rank 0 executes."""
    body = func.body
    for i, stmt in enumerate(body):
        if isinstance(stmt, ast.If) and _is_rank_test(stmt.test, ast.Eq):
            yield from stmt.body
        if (isinstance(stmt, ast.If) and _is_rank_test(stmt.test, ast.NotEq)
                and any(isinstance(s, ast.Return) for s in stmt.body)):
            yield from body[i + 1:]
            return


def test_no_collective_runs_on_rank_zero_alone():
    with open(os.path.join(REPO, "bench.py")) as f:
        tree = ast.parse(f.read())
    bad = []
    for func in ast.walk(tree):
        if not isinstance(func, ast.FunctionDef):
            continue
        for stmt in _rank0_only_regions(func):
            hit = _calls(stmt) & COLLECTIVES
            if hit:
                bad.append(f"{func.name}:{stmt.lineno} calls {sorted(hit)}")
    assert not bad, bad


def test_the_check_sees_a_planted_mistake():
    src = ("def f(rank, world):\n"
           "    x = 1\n"
           "    if rank != 0:\n"
           "        return None\n"
           "    y = _sum_over_ranks(x, world)\n")
    func = ast.parse(src).body[0]
    hits = [s for s in _rank0_only_regions(func) if _calls(s) & COLLECTIVES]
    assert len(hits) == 1
