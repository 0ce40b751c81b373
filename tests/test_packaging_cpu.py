"""The installable package (pyproject.toml), on the CPU: pip builds the
repository into a target directory, the install carries the sm_100a library
and the C++ host path as package data, declares the vLLM general-plugin entry
point the reference declares (its pyproject.toml:56-57) and imports under
both names (flashdec_b200 and the flashdec alias)."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_pip_install_ships_libraries_and_the_vllm_entry_point(tmp_path):
    pkg = ROOT / "flashdec_b200"
    if not (pkg / "libflashdec_b200.so").exists() or not list(pkg.glob("_hostpath*.so")):
        pytest.skip("libraries not built in this checkout (python -m flashdec_b200.build)")
    src = tmp_path / "src"
    src.mkdir()
    shutil.copy(ROOT / "pyproject.toml", src / "pyproject.toml")
    shutil.copytree(pkg, src / "flashdec_b200",
                    ignore=shutil.ignore_patterns("__pycache__", "_build", "csrc"))
    shutil.copytree(ROOT / "flashdec", src / "flashdec", ignore=shutil.ignore_patterns("__pycache__"))
    site = tmp_path / "site"
    subprocess.run([sys.executable, "-m", "pip", "install", "--quiet", "--no-index", "--no-deps",
                    "--no-build-isolation", "--target", str(site), str(src)],
                   check=True, timeout=600)
    assert (site / "flashdec_b200" / "libflashdec_b200.so").exists()
    assert list((site / "flashdec_b200").glob("_hostpath*.so"))
    eps = list(site.glob("flashdec_b200-*.dist-info/entry_points.txt"))
    assert eps, "no entry_points.txt in the install"
    text = eps[0].read_text()
    assert "[vllm.general_plugins]" in text
    assert "flashdec_b200 = flashdec_b200.vllm_plugin:register" in text
    # the installed copy (not the checkout) imports under both names
    code = ("import flashdec_b200, flashdec, flashdec.kernels.paged_decode as pd; "
            "import flashdec_b200.kernels.paged_decode as pd2; "
            "assert flashdec_b200.__file__.startswith(%r), flashdec_b200.__file__; "
            "assert pd is pd2" % str(site))
    subprocess.run([sys.executable, "-c", code], cwd=tmp_path, check=True, timeout=300,
                   env=dict(os.environ, PYTHONPATH=str(site)))
