"""The C++ drop-in (include/Kernels.hpp, include/Weight.hpp) driven by a
compiled C++ caller, as the reference's own tests drive its API
(src/tests/MatmulTests.cpp:12-132, src/tests/AttentionTests.cpp:9-74, and the
exception types of the launch functions). The program is tests/cxx/dropin_test.cpp;
it checks every product and attention output against the CPU oracle."""
import os
import subprocess

import pytest

from conftest import ROOT

CXX = os.path.join(ROOT, "tests", "cxx")
BINARY = os.path.join(CXX, "_build", "dropin_test")


def _build():
    subprocess.run(["make", "-s", "-C", CXX], check=True, capture_output=True, text=True)
    assert os.path.exists(BINARY)


def test_cpp_dropin_compiles_against_the_headers():
    """Kernels.hpp / Weight.hpp and the template Weight(model, name)
    constructor compile and link against the library (no GPU needed)."""
    _build()


@pytest.mark.gpu
def test_cpp_dropin_replays_reference_tests(cuda):
    _build()
    r = subprocess.run([BINARY], capture_output=True, text=True, timeout=600)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "0 failures" in r.stdout
