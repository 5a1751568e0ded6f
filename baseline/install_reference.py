"""Install the unmodified reference optimizer (``muonium``) under ``baseline/_ref``.

    python baseline/install_reference.py [--source DIR] [--force]

The reference arm of ``bench.py`` and the config-1 parity tests import ``muonium``
from ``baseline/_ref``. That directory is git-ignored (it is not this project's
source) but it travels with the working tree to a GPU box, so it must exist in
the tree before a run. This script creates it and is idempotent:

1. ``pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
   --target baseline/_ref <source>`` — the stock offline install.
2. If that fails (the reference's build backend ``uv_build`` is not in the
   offline wheelhouse), the source tree is copied to a temporary directory, the
   copy's ``[build-system]`` is pointed at setuptools (a build-metadata change
   only), and the same ``pip install`` runs on the copy with ``--no-deps``.

Either way the installed ``muonium`` package is then compared file by file with
``<source>/src/muonium``; any difference is an error, so the arm always runs the
reference's own code. ``ensure_reference()`` is the library entry used by
``bench.py`` and the tests: it installs on demand when a source tree is
available and returns the install root, or raises with the reason.
"""

from __future__ import annotations

import argparse
import filecmp
import os
import re
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
DEFAULT_SOURCES = (os.environ.get("DMB_REFERENCE_SRC", ""), "/root/reference")
WHEELHOUSE = "/opt/wheelhouse"


def _find_source(source: str | None) -> str | None:
    for cand in ([source] if source else []) + [s for s in DEFAULT_SOURCES if s]:
        if os.path.isfile(os.path.join(cand, "src", "muonium", "__init__.py")):
            return cand
    return None


def _tree_diff(a: str, b: str) -> list[str]:
    """Relative paths of ``.py`` files that differ or are missing between two trees."""
    bad = []
    for root, _, files in os.walk(a):
        for f in files:
            if not f.endswith(".py"):
                continue
            pa = os.path.join(root, f)
            pb = os.path.join(b, os.path.relpath(pa, a))
            if not os.path.isfile(pb) or not filecmp.cmp(pa, pb, shallow=False):
                bad.append(os.path.relpath(pa, a))
    return bad


def installed(source: str | None = None) -> bool:
    """True when ``baseline/_ref/muonium`` exists (and equals ``source`` if one is found)."""
    pkg = os.path.join(TARGET, "muonium")
    if not os.path.isfile(os.path.join(pkg, "__init__.py")):
        return False
    src = _find_source(source)
    return src is None or not _tree_diff(os.path.join(src, "src", "muonium"), pkg)


def _pip(src: str, extra: list[str]) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           WHEELHOUSE, "--target", TARGET, "--upgrade", *extra, src]
    return subprocess.run(cmd, capture_output=True, text=True)


def install(source: str | None = None, force: bool = False, log=print) -> str:
    src = _find_source(source)
    if src is None:
        raise RuntimeError("reference source not found (set DMB_REFERENCE_SRC)")
    if installed(src) and not force:
        return TARGET
    os.makedirs(TARGET, exist_ok=True)
    r = _pip(src, [])
    how = "pip install (stock build backend)"
    if r.returncode != 0:
        log(f"stock install failed ({r.stderr.strip().splitlines()[-1] if r.stderr.strip() else r.returncode}); "
            "retrying from a copy with a setuptools build backend")
        with tempfile.TemporaryDirectory() as tmp:
            copy = os.path.join(tmp, "muonium_src")
            shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "__pycache__", ".venv"))
            pp = os.path.join(copy, "pyproject.toml")
            text = open(pp).read()
            text = re.sub(r"\[build-system\][^\[]*",
                          '[build-system]\nrequires = ["setuptools"]\nbuild-backend = "setuptools.build_meta"\n\n'
                          '[tool.setuptools.packages.find]\nwhere = ["src"]\n\n', text, count=1)
            open(pp, "w").write(text)
            r = _pip(copy, ["--no-deps"])
            how = "pip install --no-deps from a copy (build backend switched to setuptools)"
        if r.returncode != 0:
            raise RuntimeError("reference install failed: " + (r.stderr.strip().splitlines() or ["?"])[-1])
    diff = _tree_diff(os.path.join(src, "src", "muonium"), os.path.join(TARGET, "muonium"))
    if diff:
        raise RuntimeError(f"installed muonium differs from the reference source: {diff[:5]}")
    log(f"reference installed under {TARGET} via {how}; src/muonium identical to {src}")
    return TARGET


def ensure_reference() -> str:
    """Return the directory to put on ``sys.path`` for ``import muonium``.

    Installs on demand when a reference source tree is reachable; raises
    ``RuntimeError`` naming the reason when neither an install nor a source exists.
    """
    if installed():
        return TARGET
    return install(log=lambda *_: None)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--source")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    install(a.source, a.force)


if __name__ == "__main__":
    main()
