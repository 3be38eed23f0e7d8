"""The C++ host layer (include/oxide_host.hpp): build its test program and run
it.  Without a device only the host-side tests run (argument checks, error
mapping, broadcast rules, the host RoPE table); on a GPU every op is checked
against the CPU oracle through the Rust-shaped interface."""
import os
import subprocess

import pytest

from conftest import ROOT

CPP = os.path.join(ROOT, "tests", "cpp")
EXE = os.path.join(CPP, "_build", "test_host_ops")


def _build():
    subprocess.run(["make", "-s", "-C", CPP], check=True, timeout=600)
    assert os.path.exists(EXE)


def _run(*args):
    r = subprocess.run([EXE, *args], capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout + r.stderr


def test_host_layer_builds_and_host_tests_pass():
    _build()
    rc, out = _run("--host")
    assert rc == 0, out
    assert " 0 failed" in out and "PASS broadcast_shape_follows_reference_rules" in out, out


@pytest.mark.gpu
def test_host_layer_ops_on_device(cuda):
    _build()
    rc, out = _run()
    assert rc == 0, out
    assert "SKIP" not in out and " 0 failed" in out, out
