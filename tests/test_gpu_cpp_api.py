"""The C++ drop-in API (reference class and function names over the C ABI),
exercised by tests/cpp/api_test.cpp: reference known-answer cases, error
behaviour, Layer/Loss/Optimizer classes and the arena ZeroLLM model."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_api_program():
    from zerollm_b200.build import API_TEST_BIN
    assert os.path.exists(API_TEST_BIN), "build() compiles tests/cpp/api_test.cpp"
    r = subprocess.run([API_TEST_BIN], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
