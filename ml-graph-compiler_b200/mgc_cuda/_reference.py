"""Locate the ml-graph-compiler package that this backend plugs into.

The CUDA target consumes the reference compiler's own IR (``ml_graph_compiler.ir``), pass
pipeline (``ml_graph_compiler.passes``), scheduler (``ml_graph_compiler.schedule``) and memory
planner (``ml_graph_compiler.memory``) unchanged; they stay the source of truth for node order,
fused-op semantics and arena offsets. This module makes that package importable.

Search order:

1. an ``ml_graph_compiler`` already importable (installed, or on ``PYTHONPATH``);
2. the directory named by ``$MGC_REFERENCE_PATH``;
3. ``<repo>/baseline/_ref``, where the unmodified reference is pip-installed (see
   ``__graft_entry__.build``).
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path
from types import ModuleType

REPO_ROOT = Path(__file__).resolve().parents[2]
_CANDIDATES = (
    os.environ.get("MGC_REFERENCE_PATH"),
    str(REPO_ROOT / "baseline" / "_ref"),
)


def import_reference() -> ModuleType:
    """Import and return the ``ml_graph_compiler`` package (raising ImportError if absent)."""
    try:
        return importlib.import_module("ml_graph_compiler")
    except ImportError:
        pass
    for cand in _CANDIDATES:
        if cand and (Path(cand) / "ml_graph_compiler" / "__init__.py").exists():
            if cand not in sys.path:
                sys.path.append(cand)
            return importlib.import_module("ml_graph_compiler")
    raise ImportError(
        "ml_graph_compiler (the reference compiler this backend plugs into) is not importable; "
        "install it into baseline/_ref (python -c 'import __graft_entry__ as g; g.build()') or "
        "set MGC_REFERENCE_PATH"
    )


import_reference()
