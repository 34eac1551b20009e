"""Runs the C++ host-API tests (tests/cpp, include/bjf.hpp).

test_host_api needs no GPU; test_device_api ports the reference's device-path tests and
needs an sm_100a GPU.  Each binary prints one PASS/FAIL line per case."""
from __future__ import annotations

import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CPP = os.path.join(HERE, "cpp")


def _build():
    subprocess.run(["make", "-s", "-C", CPP], check=True)


def _run(binary: str) -> str:
    _build()
    proc = subprocess.run([os.path.join(CPP, "_build", binary)], capture_output=True, text=True, timeout=600)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out
    assert "0 failed" in out, out
    return out


def test_cpp_host_api():
    out = _run("test_host_api")
    assert out.count("PASS ") >= 18


@pytest.mark.gpu
def test_cpp_device_api(cuda_device):
    out = _run("test_device_api")
    assert out.count("PASS ") >= 17
