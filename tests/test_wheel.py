"""Packaging: the wheel builder produces a platform wheel whose installed package finds its
library and header, and whose library answers through the C ABI (no GPU needed)."""

import importlib.util
import os
import pathlib
import subprocess
import sys
import zipfile

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _builder():
    spec = importlib.util.spec_from_file_location(
        "build_wheel_under_test", ROOT / "onnxruntime-musa_b200" / "build_wheel.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_wheel_builds_installs_and_loads(pkg, tmp_path):
    bw = _builder()
    whl = bw.build(tmp_path / "dist", name="onnxruntime-b200-moe", version="0.1.0")
    assert whl.name.startswith("onnxruntime_b200_moe-0.1.0-py3-none-")
    names = set(zipfile.ZipFile(whl).namelist())
    for n in ("__init__.py", "ep.py", "py.typed", "lib/libmoe_b200.so", "include/moe_b200.h"):
        assert f"onnxruntime_musa_b200/{n}" in names
    target = tmp_path / "site"
    subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "-q",
                    "--target", str(target), str(whl)], check=True)
    code = ("import onnxruntime_musa_b200 as m, pathlib;"
            "p = pathlib.Path(m.get_library_path());"
            "assert p.is_file() and p.parent.parent == pathlib.Path(m.__file__).parent;"
            "assert (p.parent.parent / 'include' / 'moe_b200.h').is_file();"
            "print(m.lib().moe_b200_abi_version(), m.get_ep_name())")
    env = dict(os.environ, PYTHONPATH=str(target))
    env.pop("MOE_B200_LIBRARY", None)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       cwd=tmp_path)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["1", "B200MoEExecutionProvider"]


def test_wheel_builder_rejects_bad_metadata(tmp_path):
    import pytest
    bw = _builder()
    with pytest.raises(ValueError):
        bw.build(tmp_path, name="bad name")
    with pytest.raises(ValueError):
        bw.build(tmp_path, version="one")
