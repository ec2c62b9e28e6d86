"""Locating the unmodified reference implementation (``packbalance``) on this machine.

Used by the reference arm of ``bench.py`` and by the tests that compare against the
reference.  Nothing here imports the reference or this framework's native extension.
"""

from __future__ import annotations

import contextlib
import importlib.util
import json
import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def locate_reference(root: Path = ROOT) -> tuple[str | None, list[str]]:
    """Directory to put on ``sys.path`` so that ``import packbalance`` loads the
    reference, and a note for every place that was tried.

    Tried in order: the offline install ``baseline/_ref`` (``pip install --target``);
    ``$PB_REFERENCE_PATH``; the ``reference_path`` of ``BASELINE.json`` (a source tree
    whose ``packbalance/`` package is pure Python and imports as it is); a
    ``packbalance`` distribution that the interpreter already finds on its path."""
    tried: list[str] = []
    cands: list[tuple[str, Path]] = [("baseline/_ref", root / "baseline" / "_ref")]
    if os.environ.get("PB_REFERENCE_PATH"):
        cands.append(("$PB_REFERENCE_PATH", Path(os.environ["PB_REFERENCE_PATH"])))
    with contextlib.suppress(OSError, ValueError, KeyError):
        ref = json.loads((root / "BASELINE.json").read_text())["reference_path"]
        cands.append(("BASELINE.json reference_path", Path(ref)))
    for label, path in cands:
        if not path.exists():
            tried.append(f"{label} ({path}): missing")
        elif not (path / "packbalance" / "train" / "train.py").exists():
            tried.append(f"{label} ({path}): no packbalance/train/train.py")
        else:
            return str(path), tried
    spec = importlib.util.find_spec("packbalance")
    if spec is not None and spec.origin and "packbalance_b200" not in spec.origin:
        return str(Path(spec.origin).parent.parent), tried
    tried.append("importable packbalance distribution: none")
    return None, tried
