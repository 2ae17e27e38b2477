"""ft::CudaBackend's KV cache and attention (kv_alloc, attention) from C++,
as the engine's layer loop would call them in place of its CPU attention
(ft/src/engine.cpp:553-566): tests/cpp/test_cuda_backend.cpp --attention,
checked against the oracle's restatement of Engine::Impl::attn.  Runs late
in the suite."""
import os
import subprocess

import pytest

from tests.test_cpp_backend import compile_test

pytestmark = pytest.mark.gpu


def test_adapter_attention_on_gpu(tmp_path):
    exe = compile_test(os.path.join(tmp_path, "test_cuda_backend"))
    r = subprocess.run([exe, "--attention"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all tests passed" in r.stdout
