"""CPU-side checks of the C-ABI library: it loads and exports every symbol that
include/nfx.h declares (no GPU calls)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "nfx.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nfx_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_declared_symbols():
    from neuroflow_b200 import _nfx
    names = _declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(_nfx.lib, n)]
    assert not missing, missing


def test_library_is_sm100a_only():
    # the build targets sm_100a exclusively
    from neuroflow_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_nflow_infer_cli_usage():
    """The command-line front-end is built next to the library and keeps the
    reference's flags and exit codes (cpp/src/main.cpp:27-50)."""
    import subprocess
    cli = os.path.join(ROOT, "neuroflow_b200", "nflow_infer")
    assert os.path.exists(cli)
    r = subprocess.run([cli, "--help"], capture_output=True, text=True)
    assert r.returncode == 0 and "--model" in r.stdout and "--input" in r.stdout
    r = subprocess.run([cli, "--model", "m.nneuroir"], capture_output=True, text=True)
    assert r.returncode == 1
