"""The C ABI driven from C++ (tests/c/matmul_abi_test.cpp): the reference's
matmul regression test (cpp_ggml/src/matmul_backend_test.cpp:17-98,166-188)
restated as a caller of include/b2q.h, with the reference's shapes, inputs,
two iterations and pass criteria, F16 / Q8_0 / Q4_0 / Q4_K weights."""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "sam-3d-objects-ggml_b200")
BIN = os.path.join(PKG, "lib", "matmul_abi_test")


@pytest.fixture(scope="module")
def abi_test_binary(b2q_mod):
    subprocess.run(["make", "-s", "-C", PKG, "abi-test"], check=True)
    assert os.access(BIN, os.X_OK)
    return BIN


def test_abi_test_program_builds_and_links_the_library(abi_test_binary):
    out = subprocess.run(["ldd", abi_test_binary], capture_output=True, text=True, check=True).stdout
    assert "libb2q.so" in out and "not found" not in out


@pytest.mark.gpu
@pytest.mark.parametrize("args", [[], ["--large"]])
def test_reference_regression_shapes_through_the_c_abi(abi_test_binary, args):
    r = subprocess.run([abi_test_binary] + args, capture_output=True, text=True, timeout=600)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("b2q weights=")]
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert lines and all(ln.endswith("PASS") for ln in lines)
    assert "ALL PASS" in r.stdout
    # both iterations of every shape and type ran: 4 types x 4 shapes (+ 4 large) x 2
    assert len(lines) == (40 if args else 32)
