"""The C ABI library without a GPU: it loads, exports every entry point
include/ftc.h declares, and rejects bad arguments before touching CUDA."""
import ctypes as C
import os
import re
import subprocess
import sys

import pytest

from xwfes_b200 import formats as F, ftc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "ftc.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ftc_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(ftc.LIB_PATH):
        from xwfes_b200 import build
        build.build()
    return ftc.lib()


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/ftc.h but not exported"
    assert set(syms) == set(ftc.SIGNATURES), "ctypes signatures out of sync with include/ftc.h"


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++17")])
def test_header_compiles_as_c_and_cpp(lang, std):
    """include/ftc.h is a plain C header (an FFI binding or a C engine can
    include it), warning-free in C and C++."""
    cc = "gcc" if lang == "c" else "g++"
    r = subprocess.run([cc, "-x", lang, std, "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        os.path.join(ROOT, "include", "ftc.h")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_row_bytes_matches_formats(lib):
    for t in (F.F32, F.F16, F.BF16, F.Q4_0, F.Q4_1, F.Q8_0, F.Q4_K, F.Q6_K):
        for k in (256, 4096, 14336):
            assert lib.ftc_row_bytes(t, k) == F.row_bytes(t, k)
    assert lib.ftc_row_bytes(99, 256) == -1
    assert lib.ftc_abi_version() == 1


def test_kernel_entry_points_validate_before_launch(lib):
    # null pointers / bad shapes are refused before any CUDA call
    rc = lib.ftc_mul_mat_vec(F.Q4_K, None, 16, 256, 144, None, 1, None, None)
    assert rc == -1 and "null" in ftc.last_error()
    rc = lib.ftc_mul_mat_vec(F.Q4_K, 16, 16, 255, 144, 16, 1, 16, None)
    assert rc == -1 and "whole number of blocks" in ftc.last_error()
    rc = lib.ftc_mul_mat_vec(F.Q4_K, 16, 16, 256, 144, 16, 9, 16, None)
    assert rc == -1 and "M must be" in ftc.last_error()
    rc = lib.ftc_mul_mat_vec(F.Q4_K, 16, 16, 256, 100, 16, 1, 16, None)
    assert rc == -1 and "row_stride" in ftc.last_error()
    rc = lib.ftc_mul_mat_vec(7, 16, 16, 256, 144, 16, 1, 16, None)
    assert rc == -2
    rc = lib.ftc_dequant(F.Q6_K, 16, 4, 100, 210, 16, None)
    assert rc == -1


def test_down_axpy_validates_before_launch(lib):
    rb = F.row_bytes(F.Q4_K, 4096)
    ws = lib.ftc_matmul_down_axpy_workspace_bytes
    # a Llama-sized down projection at one token splits the rows into slabs
    assert ws(F.Q4_K, 14336, 4096, 1) > 0
    assert ws(F.Q4_K, 14336, 4096, 0) == 0 and ws(7, 14336, 4096, 1) == 0
    assert ws(F.Q4_K, 4, 4096, 1) == 0  # one slab: sums go straight into y
    call = lib.ftc_matmul_down_axpy
    assert call(F.Q4_K, 16, 14336, 4096, rb, 16, 1, 16, None, 0, None) == -1
    assert "workspace" in ftc.last_error()
    assert call(F.Q4_K, 16, 64, 4000, rb, 16, 1, 16, None, 0, None) == -1
    assert "whole number of blocks" in ftc.last_error()
    assert call(F.Q4_K, 16, 64, 4096, rb - 1, 16, 1, 16, None, 0, None) == -1
    assert "row_stride" in ftc.last_error()
    assert call(F.Q4_K, None, 64, 4096, rb, 16, 1, 16, None, 0, None) == -1
    assert "null" in ftc.last_error()
    assert call(7, 16, 64, 4096, rb, 16, 1, 16, None, 0, None) == -2
    # nothing to add: no pointer is touched, no launch
    assert call(F.Q4_K, None, 64, 4096, rb, None, 0, None, None, 0, None) == 0
    assert call(F.Q4_K, None, 0, 4096, rb, None, 3, None, None, 0, None) == 0


def test_fused_silu_gemv_validates_before_launch(lib):
    call = lib.ftc_mul_mat_vec_silu
    rb = F.row_bytes(F.Q4_K, 3584)
    assert call(None, F.Q4_K, None, 8192, 3584, rb, 16, 3584, 16, None) == -1
    assert "null" in ftc.last_error()
    assert call(None, F.Q8_0, 16, 8192, 3584, rb, 16, 3584, 16, None) == -2
    assert call(None, F.Q4_K, 16, 8192, 3500, rb, 16, 3584, 16, None) == -1
    assert "bad shape" in ftc.last_error()
    assert call(None, F.Q4_K, 16, 8192, 3584, rb, 16, 3000, 16, None) == -1
    assert "up_offset" in ftc.last_error()
    assert call(None, F.Q4_K, 16, 8192, 3584, rb, 16, 3586, 16, None) == -1
    assert "up_offset" in ftc.last_error()


def _moe_desc(**kw):
    rs, rd = F.row_bytes(F.Q4_K, 1024), F.row_bytes(F.Q4_K, 2048)
    v = dict(dtype=F.Q4_K, n_experts=8, top_k=2, n_embd=1024, n_ff=2048, gate_exps=256,
             up_exps=256, down_exps=256, gu_row_stride=rs, gu_plane_stride=rs * 2048,
             dn_row_stride=rd, dn_plane_stride=rd * 1024)
    v.update(kw)
    return ftc.MoeDesc(**v)


def test_moe_entry_validates_before_launch(lib):
    import ctypes as C
    d = _moe_desc()
    need = lib.ftc_moe_workspace_bytes(C.byref(d), 64)
    # routing arrays, row scales, gathered x, fp32 gate|up, fp16 h, fp32 expert outputs
    assert need >= 128 * (1024 * 2 + 2 * 2048 * 4 + 2048 * 2 + 1024 * 4)
    for bad in (dict(top_k=0), dict(top_k=9), dict(n_experts=2, top_k=3),
                dict(n_experts=300), dict(n_ff=1000), dict(n_embd=100), dict(dtype=F.Q8_0),
                dict(n_ff=65536)):
        assert lib.ftc_moe_workspace_bytes(C.byref(_moe_desc(**bad)), 64) == 0, bad
        rc = lib.ftc_moe_ffn(C.byref(_moe_desc(**bad)), 256, 256, F.BF16, 64, 256, 256, need, None)
        assert rc in (-1, -2), bad
    # T == 0 is a no-op that touches nothing
    assert lib.ftc_moe_ffn(C.byref(d), None, None, F.BF16, 0, None, None, 0, None) == 0
    assert lib.ftc_moe_ffn(C.byref(d), 256, None, F.BF16, 4, 256, 256, need, None) == -1
    assert "null" in ftc.last_error()
    rc = lib.ftc_moe_ffn(C.byref(d), 256, 256, F.BF16, 64, 256, 256, need - 256, None)
    assert rc == -1 and "workspace too small" in ftc.last_error()
    rc = lib.ftc_moe_ffn(C.byref(d), 256, 256, F.BF16, 64, 256, 128, need, None)
    assert rc == -1 and "alignment" in ftc.last_error()
    rc = lib.ftc_moe_ffn(C.byref(d), 256, 256, F.Q8_0, 64, 256, 256, need, None)
    assert rc == -2
    # the expert FFN entry on pre-grouped rows ignores top_k: an
    # expert-parallel rank may hold one expert of a top-2 layer
    one = _moe_desc(n_experts=1, top_k=2)
    assert lib.ftc_moe_experts_workspace_bytes(C.byref(one), 64) > 0
    assert lib.ftc_moe_workspace_bytes(C.byref(one), 64) == 0


def _run_child(code, env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=120)


def test_fault_injection_fires_before_cuda():
    code = ("import ctypes as C; from xwfes_b200 import ftc; L = ftc.lib(); h = C.c_void_p();"
            "rc = L.ftc_backend_create(0, C.byref(h)); print(rc, h.value, ftc.last_error())")
    r = _run_child(code, {"FTC_INJECT_FAIL": "ftc_backend_create"})
    assert r.returncode == 0, r.stderr
    rc, hv, *msg = r.stdout.split()
    assert int(rc) == -5 and hv == "None" and "injected" in " ".join(msg)


def test_backend_create_without_device_fails_cleanly():
    """No GPU here: creating a backend returns an error status, never a
    half-built handle (the engine then keeps its CPU backend)."""
    code = ("import ctypes as C; from xwfes_b200 import ftc; L = ftc.lib(); h = C.c_void_p();"
            "rc = L.ftc_backend_create(0, C.byref(h)); print(rc, h.value)")
    r = _run_child(code, {"CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr
    rc, hv = r.stdout.split()
    assert int(rc) in (-1, -3) and hv == "None"


def test_library_refuses_to_fall_back(monkeypatch, tmp_path):
    monkeypatch.setattr(ftc, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(ftc, "_lib", None)
    with pytest.raises(FileNotFoundError):
        ftc.lib()


def test_exchange_entry_points_validate_before_launch(lib):
    """The expert-parallel bookkeeping, the row helpers and the peer
    allreduce refuse bad arguments before any CUDA call."""
    import ctypes as C
    # ftc_ep_pack: per-token arrays may be empty only for T == 0
    rc = lib.ftc_ep_pack(None, F.BF16, 4, 256, None, 256, None, None, 8, 2, 2, 8, 256, None, None)
    assert rc == -1 and "null pointer" in ftc.last_error()
    rc = lib.ftc_ep_pack(256, F.BF16, 4, 256, 256, 256, 256, 256, 8, 2, 3, 8, 256, 256, None)
    assert rc == -1 and "split evenly" in ftc.last_error()
    rc = lib.ftc_ep_pack(256, F.BF16, 4, 256, 256, 256, 256, 256, 8, 2, 2, 7, 256, 256, None)
    assert rc == -1 and "capacity" in ftc.last_error()
    rc = lib.ftc_ep_pack(256, F.Q4_K, 4, 256, 256, 256, 256, 256, 8, 2, 2, 8, 256, 256, None)
    assert rc == -2
    rc = lib.ftc_ep_pack(264, F.BF16, 4, 256, 256, 256, 256, 256, 8, 2, 2, 8, 256, 256, None)
    assert rc == -1 and "aligned" in ftc.last_error()
    # ftc_ep_regroup
    rc = lib.ftc_ep_regroup(None, 2, 4, 8, 256, 256, 256, 256, None)
    assert rc == -1 and "null" in ftc.last_error()
    rc = lib.ftc_ep_regroup(256, 16, 32, 8, 256, 256, 256, 256, None)
    assert rc == -1 and "1..256" in ftc.last_error()
    # ftc_silu_mul_rows: [gate | up] rows need ld >= 2n; fp16 rows an even n
    rc = lib.ftc_silu_mul_rows(256, 4, 100, 150, 256, None, None, None)
    assert rc == -1 and "ld >= 2n" in ftc.last_error()
    rc = lib.ftc_silu_mul_rows(256, 4, 101, 202, None, 256, 256, None)
    assert rc == -1 and "even n" in ftc.last_error()
    rc = lib.ftc_silu_mul_rows(256, 4, 100, 200, None, None, None, None)
    assert rc == -1 and "null" in ftc.last_error()
    # peer allreduce: bad group / size, missing buffer
    h = (C.c_uint8 * 64)()
    out = C.c_void_p()
    rc = lib.ftc_peer_ar_create(2, 2, 1024, C.byref(out), h)
    assert rc == -1 and "rank < world" in ftc.last_error()
    rc = lib.ftc_peer_ar_create(0, 9, 1024, C.byref(out), h)
    assert rc == -1 and "1..8 ranks" in ftc.last_error()
    rc = lib.ftc_peer_ar_create(0, 2, 0, C.byref(out), h)
    assert rc == -1 and "max_elems" in ftc.last_error()
    assert lib.ftc_peer_ar_sum_f32(None, 256, 256, 16, None) == -1
    assert lib.ftc_mul_mat_vec_allreduce(None, F.Q4_K, 256, 16, 256, 144, 256, 256, None) == -1
    assert lib.ftc_peer_ar_max_elems(None) == 0
    assert lib.ftc_peer_ar_destroy(None) == 0
