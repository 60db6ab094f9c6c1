"""Make the reference's own PyTorch path importable -- TEST INFRASTRUCTURE ONLY.

The reference package (``src/genie_tk`` of northws/Genie-TK) does not import as
shipped: every triple-quoted class/function docstring was turned into a block that
opens and closes with a line holding only ``#``, leaving bare prose lines in between
(``import genie_tk`` raises ``SyntaxError`` at ``src/genie_tk/triangle_mul.py:193``).
The repair is mechanical and touches no code: each line that is exactly ``#`` after
stripping becomes ``\"\"\"``. The repaired copy is written under ``baseline/_ref/src``
(git-ignored) and is used only to generate golden vectors in this container.
"""

from __future__ import annotations

import os
import shutil
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ROOT_DEFAULT = os.environ.get("GTK_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))
COPY_ROOT = os.path.join(REPO, "baseline", "_ref", "src")


def repaired_copy(ref_root: str = REF_ROOT_DEFAULT) -> str:
    """Copy ``<ref_root>/src/genie_tk`` to ``baseline/_ref/src/genie_tk`` with the docstring repair.

    Returns the directory to put on ``sys.path``. Raises FileNotFoundError when the
    reference is not mounted (e.g. on a GPU box).
    """
    src = os.path.join(ref_root, "src", "genie_tk")
    if not os.path.isdir(src):
        raise FileNotFoundError(f"reference sources not found at {src}")
    dst = os.path.join(COPY_ROOT, "genie_tk")
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    os.makedirs(dst)
    blocks = 0
    for name in sorted(os.listdir(src)):
        if not name.endswith(".py"):
            continue
        with open(os.path.join(src, name), encoding="utf-8") as f:
            lines = f.read().split("\n")
        out = []
        for line in lines:
            if line.strip() == "#":
                indent = line[: len(line) - len(line.lstrip())]
                out.append(indent + '"""')
                blocks += 1
            else:
                out.append(line)
        with open(os.path.join(dst, name), "w", encoding="utf-8") as f:
            f.write("\n".join(out))
    assert blocks % 2 == 0, "unbalanced docstring blocks"
    return COPY_ROOT


def import_reference(ref_root: str = REF_ROOT_DEFAULT):
    """Import the repaired reference package as ``genie_tk`` in a process that has no other ``genie_tk``."""
    path = repaired_copy(ref_root)
    if "genie_tk" in sys.modules:
        mod = sys.modules["genie_tk"]
        if not os.path.abspath(getattr(mod, "__file__", "")).startswith(path):
            raise RuntimeError("another genie_tk is already imported in this process")
    sys.path.insert(0, path)
    import genie_tk  # noqa: E402
    return genie_tk
