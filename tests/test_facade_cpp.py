"""Runs the C++ facade tests (tests/cpp/test_facade.cpp): the cuOP-style
operator and plugin classes compiled against include/cuop and linked with
libcuopx.so (and the oracle, as the checker)."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "cpp" / "test_facade.cpp"
OUT = ROOT / "tests" / "cpp" / "_build" / "test_facade"


def build_facade_test() -> Path:
    from cuop_b200 import build as b

    lib = b.build()
    oracle_lib = ROOT / "oracle" / "liboracle.so"
    if not oracle_lib.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)
    deps = [SRC, lib, oracle_lib] + list((ROOT / "include").rglob("*.h*"))
    if OUT.exists() and all(OUT.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = [b._nvcc(), "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{ROOT / 'include' / 'cuop'}", str(SRC),
           "-o", str(OUT), f"-L{lib.parent}", "-lcuopx", f"-L{oracle_lib.parent}", "-l:liboracle.so",
           f"-Xlinker=-rpath={lib.parent}", f"-Xlinker=-rpath={oracle_lib.parent}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return OUT


def _run(args):
    exe = build_facade_test()
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    return r.stdout


def test_facade_host_only():
    out = _run(["--host-only"])
    assert "0 failures" in out


@pytest.mark.gpu
def test_facade_on_gpu():
    out = _run([])
    assert "0 failures" in out
