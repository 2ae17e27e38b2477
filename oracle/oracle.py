"""ctypes front-end of the CPU checkers.  TEST INFRASTRUCTURE ONLY.

* ``liboracle.so`` -- ftoracle.c, the C restatement of the reference path.
* ``_ref/libftref.so`` -- the reference's own ``ft/src/cpu_backend.cpp``
  compiled from its sources (oracle/Makefile), reached through ref_shim.cpp.
* ``_ref/libftref_engine.so`` -- the reference engine's attention and RoPE
  (``ft/src/engine.cpp``), reached through ref_engine_shim.cpp.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module; the product path never does.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libftref.so")
_REF_ENGINE = os.path.join(HERE, "_ref", "libftref_engine.so")

_f = C.c_float
_i64 = C.c_int64
_p = C.c_void_p


def reference_tree():
    """The reference's source tree (the directory holding its ``src/`` and
    ``include/``): ``$FT_REF_SRC`` when set, else ``reference/ft-igpu-src``
    checked out beside this repository, else None."""
    env = os.environ.get("FT_REF_SRC")
    if env:
        return env if os.path.isdir(env) else None
    side = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "ft-igpu-src")
    return side if os.path.isdir(os.path.join(side, "src")) else None


def build():
    """Compile liboracle.so (and _ref/libftref.so where the reference tree
    exists) with oracle/Makefile."""
    ref = reference_tree()
    subprocess.run(["make", "-s", "-C", HERE] + ([f"REF_SRC={ref}"] if ref else []), check=True)


def _load(path):
    lib = C.CDLL(path)
    return lib


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        _lib = _load(_LIB)
        _lib.ftor_half_to_float.restype = _f
        _lib.ftor_half_to_float.argtypes = [C.c_uint16]
        _lib.ftor_float_to_half.restype = C.c_uint16
        _lib.ftor_float_to_half.argtypes = [_f]
        _lib.ftor_dot_row_f32.restype = _f
        _lib.ftor_dot_row_f32.argtypes = [_p, _p, C.c_int, _i64]
        _lib.ftor_dequant_row.argtypes = [_p, _p, C.c_int, _i64]
        _lib.ftor_matmul.argtypes = [_p, _i64, _i64, _p, C.c_int, _i64, _i64, _p, C.c_int]
        _lib.ftor_expert_chunk.argtypes = [_p, _p, _p, _p, _p, C.c_int, _i64, _i64, _i64,
                                           _i64, _i64, C.c_int]
        _lib.ftor_expert_ffn.argtypes = [_p, _p, _p, _p, _p, C.c_int, _i64, _i64, _i64,
                                         _i64, _i64, C.c_int]
        _lib.ftor_matmul_down_axpy.argtypes = [_p, _i64, _i64, _p, C.c_int, _i64, _i64, _p,
                                               C.c_int]
        _lib.ftor_route_topk.argtypes = [_p, _p, _i64, _i64, _i64, _p, _p]
        _lib.ftor_moe_ffn.argtypes = [_p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                                      C.c_int, _p, C.c_int]
        _lib.ftor_attention.argtypes = [_p, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _p,
                                        C.c_int]
        _lib.ftor_rope.argtypes = [_p, _i64, _i64, _i64, _i64, C.c_double, C.c_int]
        for fn in ("ftor_block_elems", "ftor_block_bytes", "ftor_row_bytes"):
            getattr(_lib, fn).restype = _i64
        _lib.ftor_row_bytes.argtypes = [C.c_int, _i64]
    return _lib


def have_ref():
    return os.path.exists(_REF)


def ref():
    """The reference's own CPU code (None when _ref was never built)."""
    global _ref
    if _ref is None and have_ref():
        r = _load(_REF)
        r.ftref_half_to_float.restype = _f
        r.ftref_half_to_float.argtypes = [C.c_uint16]
        r.ftref_float_to_half.restype = C.c_uint16
        r.ftref_float_to_half.argtypes = [_f]
        r.ftref_dequant_row.argtypes = [_p, _p, C.c_uint32, _i64]
        r.ftref_dot_row_f32.argtypes = [_p, _p, C.c_uint32, _i64, _p]
        r.ftref_matmul.argtypes = [_p, _i64, _i64, _p, C.c_uint32, _i64, _p, C.c_int]
        r.ftref_run_expert_chunk.argtypes = [_p, _p, _p, _p, _p, C.c_uint32, _i64, _i64, _i64,
                                             C.c_size_t, C.c_size_t, C.c_int]
        r.ftref_matmul_down_axpy.argtypes = [_p, _i64, _i64, _p, C.c_uint32, _i64, _p]
        _ref = r
    return _ref


_ref_engine = None


def ref_engine():
    """The reference engine's own attention and RoPE (None when
    _ref/libftref_engine.so was never built)."""
    global _ref_engine
    if _ref_engine is None and os.path.exists(_REF_ENGINE):
        r = _load(_REF_ENGINE)
        r.ftref_attn.argtypes = [_p, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _p, C.c_int]
        r.ftref_rope_vec.restype = None
        r.ftref_rope_vec.argtypes = [_p, _i64, _i64, C.c_double, C.c_int]
        r.ftref_softmax.restype = None
        r.ftref_softmax.argtypes = [_p, _i64]
        _ref_engine = r
    return _ref_engine


def _ptr(a):
    return a.ctypes.data_as(_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed (rc={rc})")


# ----------------------------------------------------------------- oracle

def dequant_rows(w, dtype, k):
    """Dequantize every row of ``w`` ``[n, row_bytes]`` -> fp32 ``[n, k]``."""
    w = _c(w, np.uint8)
    n = w.shape[0]
    out = np.empty((n, k), dtype=np.float32)
    for r in range(n):
        _check(lib().ftor_dequant_row(_ptr(out[r]), _ptr(w[r]), dtype, k), "ftor_dequant_row")
    return out


def dot_row(x, wrow, dtype, k):
    x = _c(x, np.float32)
    wrow = _c(wrow, np.uint8)
    return float(lib().ftor_dot_row_f32(_ptr(x), _ptr(wrow), dtype, k))


def matmul(x, w, dtype, k, threads=1):
    """Per-row semantics ``y[m][n] = dot(x_m, W_n)``; x fp32 ``[m, k]``."""
    x = _c(x, np.float32).reshape(-1, k)
    w = _c(w, np.uint8)
    m, n = x.shape[0], w.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    _check(lib().ftor_matmul(_ptr(x), m, k, _ptr(w), dtype, n, w.shape[1], _ptr(y), threads),
           "ftor_matmul")
    return y


def expert_chunk(x, out, gate, up, down, dtype, k, ic, threads=1):
    """Reference-layout expert chunk (down rows = neurons); ``out`` += ..."""
    x = _c(x, np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    m = x.shape[0]
    _check(lib().ftor_expert_chunk(_ptr(x), _ptr(out), _ptr(gate), _ptr(up), _ptr(down), dtype,
                                   m, k, ic, gate.shape[1], down.shape[1], threads),
           "ftor_expert_chunk")
    return out


def matmul_down_axpy(x, w, dtype, n, y, threads=1):
    """``y[m] += x_m . W`` with W = ``w`` ``[n_in, row_bytes(n)]`` (n_in rows of
    ``n`` weights, the reference's transposed down convention); x fp32
    ``[m, n_in]``, ``y`` fp32 ``[m, n]`` accumulated in place."""
    w = _c(w, np.uint8)
    x = _c(x, np.float32).reshape(-1, w.shape[0])
    assert y.dtype == np.float32 and y.flags.c_contiguous and y.shape == (x.shape[0], n)
    _check(lib().ftor_matmul_down_axpy(_ptr(x), x.shape[0], w.shape[0], _ptr(w), dtype, n,
                                       w.shape[1], _ptr(y), threads), "ftor_matmul_down_axpy")
    return y


def expert_ffn(x, out, gate, up, down, dtype, k, n_ff, threads=1):
    """Standard-layout expert FFN (down ``[k][n_ff]``); ``out`` += ..."""
    x = _c(x, np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    m = x.shape[0]
    _check(lib().ftor_expert_ffn(_ptr(x), _ptr(out), _ptr(gate), _ptr(up), _ptr(down), dtype,
                                 m, k, n_ff, gate.shape[1], down.shape[1], threads),
           "ftor_expert_ffn")
    return out


def route_topk(logits, u):
    logits = _c(logits, np.float32)
    t, e = logits.shape
    idx = np.empty((t, u), dtype=np.int32)
    w = np.empty((t, u), dtype=np.float32)
    _check(lib().ftor_route_topk(_ptr(logits), None, t, e, u, _ptr(idx), _ptr(w)),
           "ftor_route_topk")
    return idx, w


def moe_ffn(x, logits, gate_exps, up_exps, down_exps, dtype, k, n_ff, u, threads=1):
    """Routed-expert MoE FFN; returns ``out[t][k]`` (starting from zero)."""
    x = _c(x, np.float32)
    logits = _c(logits, np.float32)
    gate_exps, up_exps, down_exps = (_c(a, np.uint8) for a in (gate_exps, up_exps, down_exps))
    t, e = logits.shape
    out = np.zeros((t, k), dtype=np.float32)
    _check(lib().ftor_moe_ffn(_ptr(x), _ptr(logits), t, k, n_ff, e, u, _ptr(gate_exps),
                              _ptr(up_exps), _ptr(down_exps), dtype, _ptr(out), threads),
           "ftor_moe_ffn")
    return out


# -------------------------------------------------------------- reference

def ref_dequant_rows(w, dtype, k):
    w = _c(w, np.uint8)
    out = np.empty((w.shape[0], k), dtype=np.float32)
    for r in range(w.shape[0]):
        _check(ref().ftref_dequant_row(_ptr(out[r]), _ptr(w[r]), dtype, k), "ftref_dequant_row")
    return out


def ref_dot_row(x, wrow, dtype, k):
    x = _c(x, np.float32)
    wrow = _c(wrow, np.uint8)
    out = np.zeros(1, dtype=np.float32)
    _check(ref().ftref_dot_row_f32(_ptr(x), _ptr(wrow), dtype, k, _ptr(out)), "ftref_dot_row_f32")
    return float(out[0])


def ref_matmul(x, w, dtype, k, threads=1):
    """The reference's CpuBackend::matmul, unmodified (sums rows for M>1)."""
    x = _c(x, np.float32).reshape(-1, k)
    w = _c(w, np.uint8)
    y = np.zeros(w.shape[0] * x.shape[0], dtype=np.float32)
    _check(ref().ftref_matmul(_ptr(x), x.shape[0], k, _ptr(w), dtype, w.shape[0], _ptr(y),
                              threads), "ftref_matmul")
    return y


def ref_expert_chunk(x, out, gate, up, down, dtype, k, ic, threads=1):
    x = _c(x, np.float32)
    gate, up, down = (_c(a, np.uint8) for a in (gate, up, down))
    _check(ref().ftref_run_expert_chunk(_ptr(x), _ptr(out), _ptr(gate), _ptr(up), _ptr(down),
                                        dtype, x.shape[0], k, ic, gate.shape[1], down.shape[1],
                                        threads), "ftref_run_expert_chunk")
    return out


def ref_matmul_down_axpy(x, w, dtype, n, y):
    """The reference's own ft::matmul_down_axpy; ``y`` accumulated in place."""
    w = _c(w, np.uint8)
    x = _c(x, np.float32).reshape(-1, w.shape[0])
    assert y.dtype == np.float32 and y.flags.c_contiguous and y.shape == (x.shape[0], n)
    _check(ref().ftref_matmul_down_axpy(_ptr(x), x.shape[0], w.shape[0], _ptr(w), dtype, n,
                                        _ptr(y)), "ftref_matmul_down_axpy")
    return y


# -------------------------------------------------------------- attention

def attention(q, n_head, n_head_kv, head_dim, k_cache, v_cache, base, k_blk, v_blk, threads=1):
    """Engine::Impl::attn (ft/src/engine.cpp:137-177) restated: q fp32
    ``[M, n_head*head_dim]`` after RoPE, cache rows ``[base, dk]`` (rows
    below ``base`` are read), the block's rows ``[M, dk]``; returns the
    attention output ``[M, n_head*head_dim]``."""
    q = _c(q, np.float32)
    M = q.shape[0]
    dk = n_head_kv * head_dim
    kc = _c(k_cache, np.float32) if base else np.zeros((1, dk), np.float32)
    vc = _c(v_cache, np.float32) if base else np.zeros((1, dk), np.float32)
    kb, vb = _c(k_blk, np.float32), _c(v_blk, np.float32)
    out = np.empty((M, n_head * head_dim), dtype=np.float32)
    _check(lib().ftor_attention(_ptr(q), M, n_head, n_head_kv, head_dim, _ptr(kc), _ptr(vc), base,
                                _ptr(kb), _ptr(vb), _ptr(out), threads), "ftor_attention")
    return out


def rope(x, heads, head_dim, base, theta, neox):
    """RoPE of rows m at positions base + m (ft/src/engine.cpp:43-60, 545-551),
    on a copy of x ``[M, heads*head_dim]``."""
    x = np.array(x, dtype=np.float32, order="C", copy=True)
    _check(lib().ftor_rope(_ptr(x), x.shape[0], heads, head_dim, base, theta, 1 if neox else 0),
           "ftor_rope")
    return x
