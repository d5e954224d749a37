"""Install the unmodified reference framework (Koas-W/Femtotron) into ``baseline/_ref``.

    python baseline/install_reference.py [--source DIR] [--force]

The reference arm of ``bench.py`` and the reference-parity tests import the reference from
``baseline/_ref``.  The reference's ``pyproject.toml`` names the build backend
``setuptools.backends._legacy:_Backend``, which the installed setuptools does not provide, so
the plain ``pip install --target baseline/_ref <reference>`` fails while resolving the
backend.  This script therefore

  1. tries that plain offline install first;
  2. on failure copies the reference tree to a temporary directory, rewrites only the
     ``build-backend`` line of the copy's ``pyproject.toml`` to ``setuptools.build_meta``,
     and installs the copy with ``--no-deps`` (its dependencies, torch and transformers,
     come from this image).

No Python source of the reference is changed.  Every step is offline
(``--no-index --find-links /opt/wheelhouse``).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
DEFAULT_SOURCE = os.environ.get("FT_REFERENCE_SRC", "/root/reference")
WHEELHOUSE = os.environ.get("FT_WHEELHOUSE", "/opt/wheelhouse")


def installed(target: str = TARGET) -> bool:
    return os.path.isfile(os.path.join(target, "femtotron", "__init__.py")) or \
        os.path.isdir(os.path.join(target, "femtotron", "training"))


def _pip(src: str, target: str, no_deps: bool) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--find-links", WHEELHOUSE, "--target", target, "--upgrade"]
    if no_deps:
        cmd.append("--no-deps")
    cmd.append(src)
    return subprocess.run(cmd, capture_output=True, text=True)


def install(source: str = DEFAULT_SOURCE, target: str = TARGET, force: bool = False) -> str:
    """Install the reference; returns a one-line description of what happened."""
    if installed(target) and not force:
        return f"already installed in {target}"
    if not os.path.isdir(os.path.join(source, "femtotron")):
        raise FileNotFoundError(f"reference source not found at {source}")
    os.makedirs(target, exist_ok=True)
    r = _pip(source, target, no_deps=False)
    if r.returncode == 0 and installed(target):
        return "installed with the plain offline pip command"
    with tempfile.TemporaryDirectory(prefix="ft_ref_") as tmp:
        copy = os.path.join(tmp, "reference")
        shutil.copytree(source, copy, ignore=shutil.ignore_patterns("__pycache__", "*.pyc", ".git"))
        pp = os.path.join(copy, "pyproject.toml")
        with open(pp) as f:
            lines = f.read().splitlines()
        lines = ['build-backend = "setuptools.build_meta"' if ln.strip().startswith("build-backend")
                 else ln for ln in lines]
        with open(pp, "w") as f:
            f.write("\n".join(lines) + "\n")
        r2 = _pip(copy, target, no_deps=True)
        if r2.returncode != 0 or not installed(target):
            tail = (r2.stderr or r2.stdout or "").strip().splitlines()[-3:]
            raise RuntimeError("reference install failed: " + " | ".join(tail))
    return ("installed from a copy whose pyproject.toml names setuptools.build_meta "
            "(--no-deps); the plain command failed: " +
            ((r.stderr or r.stdout or "").strip().splitlines() or ["?"])[-1][:160])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--source", default=DEFAULT_SOURCE)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(install(a.source, TARGET, a.force))


if __name__ == "__main__":
    main()
