"""The C++ ft::IBackend adapter (xwfes_b200/host/cuda_backend.cpp): it must
compile against the interface header (CPU, no GPU needed) and pass the C++
test binary tests/cpp/test_cuda_backend.cpp on a B200."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "xwfes_b200", "host")


def compile_test(out):
    from oracle import oracle as O
    from xwfes_b200 import build, ftc
    if not os.path.exists(ftc.LIB_PATH):
        build.build()
    O.lib()  # builds oracle/liboracle.so if needed
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(HOST, "compat"), "-I", HOST,
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "oracle"),
           os.path.join(ROOT, "tests", "cpp", "test_cuda_backend.cpp"),
           os.path.join(HOST, "cuda_backend.cpp"), os.path.join(HOST, "gguf.cpp"),
           "-L", os.path.dirname(ftc.LIB_PATH), "-lftcuda",
           "-L", os.path.join(ROOT, "oracle"), "-loracle",
           "-Wl,-rpath," + os.path.dirname(ftc.LIB_PATH) + ":" + os.path.join(ROOT, "oracle"),
           "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def _ref_include():
    from oracle import oracle as O
    tree = O.reference_tree()
    return os.path.join(tree, "include") if tree else ""


# the reference tree's headers, where the reference is checked out (CPU-only check)
REF_INCLUDE = _ref_include()


@pytest.mark.skipif(not REF_INCLUDE or not os.path.isdir(REF_INCLUDE),
                    reason="reference tree not present")
def test_adapter_compiles_against_reference_headers():
    """cuda_backend.cpp drops into the reference tree as is: it compiles
    against the reference's own, unmodified ft/ headers (C++20, as its
    CMake build)."""
    r = subprocess.run(["g++", "-std=c++20", "-Wall", "-fsyntax-only", "-I", REF_INCLUDE,
                        "-I", HOST, "-I", os.path.join(ROOT, "include"),
                        os.path.join(HOST, "cuda_backend.cpp")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_adapter_compiles(tmp_path):
    assert os.path.exists(compile_test(str(tmp_path / "test_cuda_backend")))


def test_adapter_host_checks(tmp_path):
    """The parts of the adapter that need no device (the down-weight layout)."""
    exe = compile_test(str(tmp_path / "test_cuda_backend"))
    r = subprocess.run([exe, "--host-only"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "all tests passed" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_adapter_passes_on_gpu(tmp_path):
    exe = compile_test(str(tmp_path / "test_cuda_backend"))
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "all tests passed" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_gguf_file_upload_and_matmul_on_gpu(tmp_path):
    """A small model file (Q4_K, Q6_K and Q8_0 weights and a 4-expert Q4_K
    tensor, written by tests/gguf_write.py) loaded by the engine-side reader,
    uploaded whole with CudaBackend::upload_all, then matmuls (M = 1, 3, 16)
    and expert-chunk windows on the device copies against the oracle."""
    import gguf_write as G
    from xwfes_b200 import formats as F, synth as S
    ggml = {F.Q4_K: 12, F.Q6_K: 14, F.Q8_0: 8}
    specs = [("blk.0.attn_q.weight", F.Q4_K, 512, 1024, 1),
             ("blk.0.ffn_down.weight", F.Q6_K, 256, 512, 1),
             ("blk.0.attn_k.weight", F.Q8_0, 128, 1024, 1),
             ("blk.0.ffn_gate_exps.weight", F.Q4_K, 256, 1024, 4)]
    tensors = []
    for name, t, n, k, e in specs:
        raw = b"".join(S.weight(t, n, k, seed=10 + p, name=name).tobytes() for p in range(e))
        dims = (k, n) if e == 1 else (k, n, e)
        tensors.append((name, dims, ggml[t], raw))
    path = G.write_gguf(str(tmp_path / "tiny.gguf"), [("general.name", G.STR, "tiny")], tensors)
    exe = compile_test(str(tmp_path / "test_cuda_backend"))
    r = subprocess.run([exe, "--gguf", path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "all tests passed" in r.stdout, r.stdout + r.stderr
