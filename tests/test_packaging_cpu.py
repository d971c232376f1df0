"""The package installs with the reference's SGLang plugin entry point
(tri-sds pyproject.toml:16-17: group ``sglang.srt.plugins``, name
``tri_sds``), and SGLang's discovery path - importlib.metadata entry points
of that group, loaded and called - registers TriSDSWorker in place of
StandaloneWorker (tri_sds/__init__.py:1-10)."""
import os
import shutil
import subprocess
import sys
import tomllib

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pyproject_declares_the_plugin_entry_point():
    with open(os.path.join(ROOT, "pyproject.toml"), "rb") as f:
        meta = tomllib.load(f)
    eps = meta["project"]["entry-points"]["sglang.srt.plugins"]
    assert eps == {"tri_sds": "tri_sds_b200:create_plugin"}
    assert "libtsds.so" in meta["tool"]["setuptools"]["package-data"]["tri_sds_b200"]


def test_installed_entry_point_registers_the_worker(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    shutil.copy(os.path.join(ROOT, "pyproject.toml"), src)
    shutil.copytree(os.path.join(ROOT, "tri_sds_b200"), src / "tri_sds_b200",
                    ignore=shutil.ignore_patterns("_build", "__pycache__", "*.o"))
    site = tmp_path / "site"
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "--no-build-isolation",
                        "--quiet", "--target", str(site), str(src)], capture_output=True, text=True, timeout=600)
    if r.returncode != 0 and "No module named" in r.stderr and "setuptools" in r.stderr:
        pytest.skip("setuptools is not installed")
    assert r.returncode == 0, r.stderr
    probe = (
        "import importlib.metadata as md\n"
        "eps = [e for e in md.entry_points(group='sglang.srt.plugins') if e.name == 'tri_sds']\n"
        "assert len(eps) == 1, eps\n"
        "fn = eps[0].load()\n"
        "import tri_sds_b200\n"
        "assert tri_sds_b200.__file__.startswith(%r), tri_sds_b200.__file__\n"
        "fn()\n"
        "from tri_sds_b200.sglang_compat import HAVE_SGLANG, HookRegistry, HookType\n"
        "from tri_sds_b200.worker import TriSDSWorker\n"
        "if not HAVE_SGLANG:\n"
        "    assert HookRegistry.lookup(tri_sds_b200.STANDALONE_WORKER) == (TriSDSWorker, HookType.REPLACE)\n"
        "print('ok', eps[0].value)\n" % str(site))
    env = {**os.environ, "PYTHONPATH": str(site)}
    r = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True, cwd=str(tmp_path), env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert "ok tri_sds_b200:create_plugin" in r.stdout
