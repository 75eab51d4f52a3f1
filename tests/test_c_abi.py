"""The reference's C ABI used from C: tests/c_abi/abi_check.c is compiled
with gcc against include/ndtensors_capi.h and linked to the built
libndtensors_capi.so, as a C / Julia / Rust caller would bind it."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIBDIR = ROOT / "ndtensors-rs_b200" / "lib"


@pytest.fixture(scope="module")
def abi_check(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    if not (LIBDIR / "libndtensors_capi.so").exists():
        pytest.fail("libndtensors_capi.so is not built (make -C ndtensors-rs_b200)")
    exe = tmp_path_factory.mktemp("abi") / "abi_check"
    subprocess.run(["gcc", "-std=c11", "-O1", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi" / "abi_check.c"), "-L", str(LIBDIR), "-lndtensors_capi",
                    f"-Wl,-rpath,{LIBDIR}", "-lm", "-o", str(exe)], check=True)
    return exe


def _run(exe, mode):
    r = subprocess.run([str(exe), mode], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout


def test_c_caller_host(abi_check, ndt):
    if ndt.device_available():
        pytest.skip("host mode checks the no-device behaviour")
    _run(abi_check, "host")


@pytest.mark.gpu
def test_c_caller_device(abi_check, gpu):
    _run(abi_check, "device")
