"""TEST INFRASTRUCTURE ONLY — where the reference tree is: the directory named by the environment variable
LTQ_REF_ROOT, else the reference's install in baseline/_ref of this repository (made by `make -C oracle refpy`).
Used by the golden-fixture scripts, the parity tests that run the reference's own Python, bench.py's reference CPU
arm and build(); none of them ships."""
from __future__ import annotations

import os
import sys
from pathlib import Path
from typing import Optional

REPO = Path(__file__).resolve().parent.parent
INSTALL = REPO / "baseline" / "_ref"


def reference_root() -> Optional[Path]:
    """The reference tree (a directory holding src/liqk_v2.py), or None when there is none."""
    env = os.environ.get("LTQ_REF_ROOT")
    for p in ([Path(env)] if env else []) + [INSTALL]:
        if (p / "src" / "liqk_v2.py").exists():
            return p
    return None


def require_reference_root() -> Path:
    p = reference_root()
    if p is None:
        raise SystemExit("the reference tree is needed: set LTQ_REF_ROOT, or install it with "
                         "`make -C oracle refpy LTQ_REF_ROOT=<reference root>`")
    return p


def import_reference(root: Optional[Path] = None):
    """Put the reference tree on sys.path (its modules import as `src.<name>`), without writing bytecode into it and
    with its torch.compile switched off (TCQ_NO_COMPILE); returns the root."""
    root = root or require_reference_root()
    os.environ.setdefault("TCQ_NO_COMPILE", "1")
    sys.dont_write_bytecode = True
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    return root
