"""The reference installer (``baseline/install_reference.py``) puts the reference's own Python
sources, byte for byte, into the target directory: the benchmark's reference arm and the
reference-parity tests run unmodified reference code."""
from __future__ import annotations

import filecmp
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))
import install_reference  # noqa: E402


def _py_files(top):
    out = set()
    for d, _, fs in os.walk(top):
        for f in fs:
            if f.endswith(".py"):
                out.add(os.path.relpath(os.path.join(d, f), top))
    return out


@pytest.mark.skipif(not os.path.isdir(os.path.join(install_reference.DEFAULT_SOURCE, "femtotron")),
                    reason="reference source tree not present on this machine")
def test_installed_reference_sources_are_identical(tmp_path):
    target = str(tmp_path / "ref")
    msg = install_reference.install(target=target)
    assert install_reference.installed(target), msg
    src = os.path.join(install_reference.DEFAULT_SOURCE, "femtotron")
    dst = os.path.join(target, "femtotron")
    src_files = _py_files(src)
    assert src_files, "no Python sources in the reference tree"
    assert _py_files(dst) == src_files
    _, mismatch, errors = filecmp.cmpfiles(src, dst, sorted(src_files), shallow=False)
    assert not mismatch and not errors, (mismatch, errors)
    # a second call leaves the installation alone
    assert install_reference.install(target=target).startswith("already installed")


def test_missing_source_is_reported(tmp_path):
    with pytest.raises(FileNotFoundError):
        install_reference.install(source=str(tmp_path / "nowhere"), target=str(tmp_path / "t"))
