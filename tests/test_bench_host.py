"""Host checks of the driver-facing scripts that need no GPU.

Every name that ``bench.py``, ``__graft_entry__.py`` and the package modules
load must be bound somewhere in the same module (assignment, import, def,
argument) or be a builtin: a module constant lost in an edit otherwise only
shows up as a NameError on the GPU box, in the one bench leg that uses it.
``bench.py --help`` must parse without torch touching a device.
"""

from __future__ import annotations

import ast
import builtins
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SOURCES = [ROOT / "bench.py", ROOT / "__graft_entry__.py",
           *sorted((ROOT / "drama3-studio_b200" / "drama_b200").glob("*.py"))]


def _unbound_names(path: Path) -> list[tuple[str, int]]:
    tree = ast.parse(path.read_text(), filename=str(path))
    bound = set(dir(builtins)) | {"__file__", "__name__", "__doc__", "__spec__", "__package__"}
    for node in ast.walk(tree):
        if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
            bound.add(node.name)
        elif isinstance(node, ast.Name) and isinstance(node.ctx, (ast.Store, ast.Del)):
            bound.add(node.id)
        elif isinstance(node, (ast.Import, ast.ImportFrom)):
            for alias in node.names:
                bound.add((alias.asname or alias.name).split(".")[0])
        elif isinstance(node, ast.arg):
            bound.add(node.arg)
        elif isinstance(node, ast.ExceptHandler) and node.name:
            bound.add(node.name)
        elif isinstance(node, (ast.Global, ast.Nonlocal)):
            bound.update(node.names)
        elif isinstance(node, ast.MatchAs) and node.name:
            bound.add(node.name)
    loads = {(n.id, n.lineno) for n in ast.walk(tree) if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Load)}
    return sorted(((name, line) for name, line in loads if name not in bound), key=lambda t: t[1])


@pytest.mark.parametrize("path", SOURCES, ids=lambda p: p.name)
def test_every_loaded_name_is_bound(path):
    assert _unbound_names(path) == [], f"{path.name}: names loaded but never bound"


def test_bench_help_parses():
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], cwd=ROOT, capture_output=True,
                          text=True, timeout=120)
    assert done.returncode == 0, done.stderr
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--workload"):
        assert flag in done.stdout
