"""ctypes binding of libftcuda.so (include/ftc.h).

Device-pointer entry points take torch CUDA tensors (their ``data_ptr()``)
and launch on torch's current stream unless a stream is given.  The library
must exist: there is no CPU fallback, a missing or unbuildable library raises.
"""
import ctypes as C
import os

import numpy as np

from . import formats as F

PKG = os.path.dirname(os.path.abspath(__file__))
# FTC_LIB overrides the library path (e.g. a build of the sources elsewhere)
LIB_PATH = os.environ.get("FTC_LIB") or os.path.join(PKG, "libftcuda.so")

_p = C.c_void_p
_i64 = C.c_int64

# name -> (restype, argtypes); one line per declaration in include/ftc.h
SIGNATURES = {
    "ftc_last_error": (C.c_char_p, []),
    "ftc_abi_version": (C.c_int, []),
    "ftc_row_bytes": (_i64, [C.c_int, _i64]),
    "ftc_backend_create": (C.c_int, [C.c_int, C.POINTER(_p)]),
    "ftc_backend_destroy": (None, [_p]),
    "ftc_backend_info": (C.c_int, [_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_uint64)]),
    "ftc_backend_upload": (C.c_int, [_p, _p, C.c_size_t]),
    "ftc_backend_evict": (C.c_int, [_p, _p]),
    "ftc_backend_cached_bytes": (C.c_int, [_p, C.POINTER(C.c_uint64)]),
    "ftc_backend_matmul": (C.c_int, [_p, _p, _i64, _i64, _p, C.c_int, _i64, _p]),
    "ftc_backend_run_expert_chunk": (C.c_int, [_p, _p]),
    "ftc_backend_matmul_down_axpy": (C.c_int, [_p, _p, _i64, _i64, _p, C.c_int, _i64, _p]),
    "ftc_matmul_down_axpy_workspace_bytes": (C.c_size_t, [C.c_int, _i64, _i64, _i64]),
    "ftc_matmul_down_axpy": (C.c_int, [C.c_int, _p, _i64, _i64, _i64, _p, _i64, _p, _p,
                                       C.c_size_t, _p]),
    "ftc_backend_moe_ffn": (C.c_int, [_p, _p, _p, _p, _p, _i64, _p]),
    "ftc_backend_sync": (C.c_int, [_p]),
    "ftc_backend_stream": (_p, [_p]),
    "ftc_backend_device_ptr": (_p, [_p, _p]),
    "ftc_device_status": (C.c_int, [_p, C.POINTER(C.c_int)]),
    "ftc_dequant": (C.c_int, [C.c_int, _p, _i64, _i64, _i64, _p, _p]),
    "ftc_mul_mat_vec": (C.c_int, [C.c_int, _p, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "ftc_mul_mat_vec_multi": (C.c_int, [C.c_int, C.c_int, C.POINTER(_p), C.POINTER(_i64), _i64,
                                        _i64, _p, _i64, C.POINTER(_p), _p]),
    "ftc_mul_mat_vec_multi_hint": (C.c_int, [C.c_int, C.c_int, C.POINTER(_p), C.POINTER(_i64),
                                             _i64, _i64, _p, _i64, C.POINTER(_p), C.c_int,
                                             C.POINTER(_p), C.POINTER(_i64), _p]),
    "ftc_gemm": (C.c_int, [C.c_int, _p, _i64, _i64, _i64, _p, C.c_int, _i64, _p, C.c_int, _p]),
    "ftc_expert_chunk_static": (C.c_int, [C.c_int, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                          _i64, _p]),
    "ftc_gemm_rowscaled": (C.c_int, [C.c_int, _p, _i64, _i64, _i64, _p, _i64, _p, C.c_int, _p,
                                     _p]),
    "ftc_rows_to_f16": (C.c_int, [_p, C.c_int, _i64, _i64, _i64, _p, _p, _p]),
    "ftc_silu_mul": (C.c_int, [_p, _p, _i64, _p, _p]),
    "ftc_moe_route": (C.c_int, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p]),
    "ftc_moe_combine": (C.c_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p]),
    "ftc_moe_experts_workspace_bytes": (C.c_size_t, [_p, _i64]),
    "ftc_moe_experts": (C.c_int, [_p, _p, C.c_int, _i64, _p, _p, _i64, _p, _p, C.c_size_t, _p]),
    "ftc_moe_workspace_bytes": (C.c_size_t, [_p, _i64]),
    "ftc_moe_ffn": (C.c_int, [_p, _p, _p, C.c_int, _i64, _p, _p, C.c_size_t, _p]),
    "ftc_silu_mul_rows": (C.c_int, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "ftc_ep_pack": (C.c_int, [_p, C.c_int, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                              _p, _p, _p]),
    "ftc_ep_regroup": (C.c_int, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "ftc_peer_ar_create": (C.c_int, [C.c_int, C.c_int, _i64, C.POINTER(_p), _p]),
    "ftc_peer_ar_open": (C.c_int, [_p, _p]),
    "ftc_peer_ar_max_elems": (_i64, [_p]),
    "ftc_peer_ar_sum_f32": (C.c_int, [_p, _p, _p, _i64, _p]),
    "ftc_peer_ar_destroy": (C.c_int, [_p]),
    "ftc_mul_mat_vec_allreduce": (C.c_int, [_p, C.c_int, _p, _i64, _i64, _i64, _p, _p, _p]),
    "ftc_mul_mat_vec_silu": (C.c_int, [_p, C.c_int, _p, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "ftc_attention_workspace_bytes": (C.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "ftc_attention": (C.c_int, [_p, _i64, _i64, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _p, _p,
                                C.c_size_t, _p]),
    "ftc_rope": (C.c_int, [_p, _i64, _i64, _i64, _i64, C.c_double, C.c_int, _p]),
    "ftc_backend_kv_alloc": (C.c_int, [_p, _i64, _i64, _i64]),
    "ftc_backend_attention": (C.c_int, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                                        C.c_int, _p]),
    "ftc_backend_kv_read": (C.c_int, [_p, _i64, _i64, _i64, _p, _p]),
    "ftc_backend_kv_write": (C.c_int, [_p, _i64, _i64, _i64, _p, _p]),
}


class FtcError(RuntimeError):
    def __init__(self, fn, rc, msg):
        super().__init__(f"{fn} failed (status {rc}): {msg}")
        self.rc = rc


class ExpertChunkJob(C.Structure):
    """``ftc_expert_chunk_job`` == ft::ExpertChunkJob (ft/include/ft/backend.h:7-19)."""
    _fields_ = [("x", _p), ("out", _p), ("gate", _p), ("up", _p), ("down", _p),
                ("dtype", C.c_int), ("M", _i64), ("K", _i64), ("IC", _i64),
                ("gate_up_row_stride", C.c_size_t), ("down_row_stride", C.c_size_t)]


class MoeDesc(C.Structure):
    """``ftc_moe_desc``: expert weights and shapes of one MoE layer."""
    _fields_ = [("dtype", C.c_int), ("n_experts", _i64),
                ("top_k", _i64), ("n_embd", _i64), ("n_ff", _i64), ("gate_exps", _p),
                ("up_exps", _p), ("down_exps", _p), ("gu_row_stride", _i64),
                ("gu_plane_stride", _i64), ("dn_row_stride", _i64), ("dn_plane_stride", _i64)]


_lib = None


def lib():
    """Load libftcuda.so (raises if it was never built: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -m xwfes_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    return lib().ftc_last_error().decode(errors="replace")


def check(rc, fn):
    if rc != 0:
        raise FtcError(fn, rc, last_error())


def _stream(stream):
    if stream is not None:
        return C.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def device_status(stream=None):
    """Synchronize the stream and return (and clear) the kernels' status word
    (0: every bounded wait completed)."""
    v = C.c_int()
    check(lib().ftc_device_status(_stream(stream), C.byref(v)), "ftc_device_status")
    return v.value


def row_bytes(dtype, k):
    return int(lib().ftc_row_bytes(F.dtype_id(dtype), k))


# ------------------------------------------------------------ kernels

def mul_mat_vec(w, dtype, n, k, x, y=None, row_stride=None, stream=None):
    """y[m][n] = sum_k x[m][k] W[n][k] on the GPU (fp32, M = x.shape[0] <= 8).

    ``w``: uint8 CUDA tensor of GGUF blocks; ``x``: fp32 CUDA tensor [M, k].
    """
    import torch
    t = F.dtype_id(dtype)
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if y is None:
        y = torch.empty((m, n), dtype=torch.float32, device=x.device)
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    check(lib().ftc_mul_mat_vec(t, w.data_ptr(), n, k, rs, x2.data_ptr(), m, y.data_ptr(),
                                _stream(stream)), "ftc_mul_mat_vec")
    return y


def matmul_down_axpy(w, dtype, n_in, n, x, y, row_stride=None, ws=None, stream=None):
    """y[m][j] += sum_i x[m][i] W_i[j] on the GPU (ftc_matmul_down_axpy): ``w``
    uint8 CUDA tensor of ``n_in`` rows of ``n`` weights (the reference's
    transposed down layout), ``x`` fp32 [M, n_in], ``y`` fp32 [M, n]
    accumulated in place.  ``ws``: scratch (allocated when None)."""
    import torch
    t = F.dtype_id(dtype)
    x2 = x.reshape(-1, n_in)
    m = x2.shape[0]
    need = lib().ftc_matmul_down_axpy_workspace_bytes(t, n_in, n, m)
    if ws is None and need:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    rs = row_stride if row_stride is not None else row_bytes(t, n)
    check(lib().ftc_matmul_down_axpy(t, w.data_ptr(), n_in, n, rs, x2.data_ptr(), m, y.data_ptr(),
                                     ws.data_ptr() if ws is not None else None,
                                     ws.numel() if ws is not None else 0, _stream(stream)),
          "ftc_matmul_down_axpy")
    return y


def mul_mat_vec_silu(w, dtype, n, k, gu, up_offset=None, y=None, row_stride=None, ar=None,
                     stream=None):
    """y = (silu(gate) * up) . W^T for one token, the SiLU product computed as
    the GEMV loads its activation (ftc_mul_mat_vec_silu): ``gu`` fp32 CUDA
    tensor holding [gate (k) | up (k)] (up at ``up_offset``, default k).
    With ``ar`` (a PeerAllreduce) y is summed over its ranks as well."""
    import torch
    t = F.dtype_id(dtype)
    if y is None:
        y = torch.empty((1, n), dtype=torch.float32, device=gu.device)
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    off = k if up_offset is None else up_offset
    check(lib().ftc_mul_mat_vec_silu(ar._ar if ar is not None else None, t, w.data_ptr(), n, k, rs,
                                     gu.data_ptr(), off, y.data_ptr(), _stream(stream)),
          "ftc_mul_mat_vec_silu")
    return y


def mul_mat_vec_multi(ws, dtype, ns, k, x, ys=None, row_stride=None, stream=None):
    """Several GEMVs sharing x in one launch: ys[i] = x @ W_i^T."""
    import torch
    t = F.dtype_id(dtype)
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if ys is None:
        ys = [torch.empty((m, n), dtype=torch.float32, device=x.device) for n in ns]
    P = len(ws)
    wa = (_p * P)(*[w.data_ptr() for w in ws])
    na = (_i64 * P)(*ns)
    ya = (_p * P)(*[y.data_ptr() for y in ys])
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    check(lib().ftc_mul_mat_vec_multi(t, P, wa, na, k, rs, x2.data_ptr(), m, ya, _stream(stream)),
          "ftc_mul_mat_vec_multi")
    return ys


def attention(q, n_head, n_head_kv, head_dim, k_blk, v_blk, base=0, k_cache=None, v_cache=None,
              kv_stride=None, out=None, ws=None, stream=None):
    """Causal grouped-query attention on the GPU (ftc_attention): q fp32 CUDA
    [M, n_head*head_dim] at positions base .. base+M-1; K/V rows [pos,
    kv_stride] -- rows below ``base`` from k_cache / v_cache, the block's
    from k_blk / v_blk.  Returns out [M, n_head*head_dim]."""
    import torch
    q2 = q.reshape(q.shape[0], -1)
    M = q2.shape[0]
    ks = kv_stride if kv_stride is not None else n_head_kv * head_dim
    if out is None:
        out = torch.empty((M, n_head * head_dim), dtype=torch.float32, device=q.device)
    need = int(lib().ftc_attention_workspace_bytes(M, n_head, n_head_kv, head_dim, base))
    if need and (ws is None or ws.numel() < need):
        ws = torch.empty(need, dtype=torch.uint8, device=q.device)
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    check(lib().ftc_attention(q2.data_ptr(), M, n_head, n_head_kv, head_dim, ptr(k_cache),
                              ptr(v_cache), ks, base, k_blk.data_ptr(), v_blk.data_ptr(),
                              out.data_ptr(), ptr(ws) if need else None, need, _stream(stream)),
          "ftc_attention")
    return out


def rope(x, heads, head_dim, base, theta, neox, stream=None):
    """RoPE in place on fp32 CUDA x [M, heads*head_dim], row m at position
    base + m (ftc_rope); returns x."""
    check(lib().ftc_rope(x.data_ptr(), x.shape[0], heads, head_dim, base, float(theta),
                         1 if neox else 0, _stream(stream)), "ftc_rope")
    return x


_TORCH_OUT = {F.F32: "float32", F.BF16: "bfloat16", F.F16: "float16"}


def gemm(w, dtype, n, k, x, y=None, y_dtype=F.BF16, row_stride=None, stream=None):
    """Tensor-core dequant-GEMM: y[m][n] = sum_k x[m][k] W[n][k].

    ``x``: bf16 or fp16 CUDA tensor [M, k]; ``y`` in ``y_dtype``."""
    import torch
    t = F.dtype_id(dtype)
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    xt = {torch.bfloat16: F.BF16, torch.float16: F.F16}[x2.dtype]
    yt = F.dtype_id(y_dtype)
    if y is None:
        y = torch.empty((m, n), dtype=getattr(torch, _TORCH_OUT[yt]), device=x.device)
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    check(lib().ftc_gemm(t, w.data_ptr(), n, k, rs, x2.data_ptr(), xt, m, y.data_ptr(), yt,
                         _stream(stream)), "ftc_gemm")
    return y


def rows_to_f16(x, out=None, row_exp=None, stream=None):
    """fp16 copy of the rows of ``x`` (fp32 / bf16 / fp16 CUDA tensor [M, K]),
    each scaled by 2**-row_exp[m] into fp16's range; returns (out, row_exp)."""
    import torch
    x2 = x.reshape(x.shape[0], -1)
    m, k = x2.shape
    xt = {torch.float32: F.F32, torch.bfloat16: F.BF16, torch.float16: F.F16}[x2.dtype]
    if out is None:
        out = torch.empty((m, k), dtype=torch.float16, device=x.device)
    if row_exp is None:
        row_exp = torch.empty((m,), dtype=torch.int32, device=x.device)
    check(lib().ftc_rows_to_f16(x2.data_ptr(), xt, m, k, x2.stride(0), out.data_ptr(),
                                row_exp.data_ptr(), _stream(stream)), "ftc_rows_to_f16")
    return out, row_exp


def gemm_rowscaled(w, dtype, n, k, x16, row_exp, y=None, y_dtype=F.F32, row_stride=None,
                   stream=None):
    """y = (x16 @ W^T) with row m multiplied by 2**row_exp[m]: the GEMM on the
    output of :func:`rows_to_f16`, giving the unscaled product."""
    import torch
    t = F.dtype_id(dtype)
    m = x16.shape[0]
    yt = F.dtype_id(y_dtype)
    if y is None:
        y = torch.empty((m, n), dtype=getattr(torch, _TORCH_OUT[yt]), device=x16.device)
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    check(lib().ftc_gemm_rowscaled(t, w.data_ptr(), n, k, rs, x16.data_ptr(), m, y.data_ptr(), yt,
                                   row_exp.data_ptr(), _stream(stream)), "ftc_gemm_rowscaled")
    return y


def silu_mul(g, u, out=None, stream=None):
    """silu(g) * u elementwise (fp32 CUDA tensors)."""
    import torch
    if out is None:
        out = torch.empty_like(g)
    check(lib().ftc_silu_mul(g.data_ptr(), u.data_ptr(), g.numel(), out.data_ptr(),
                             _stream(stream)), "ftc_silu_mul")
    return out


def silu_mul_rows(gu, n, to_f16=False, stream=None):
    """Rows of ``gu`` (fp32 CUDA [M, >= 2n], row pitch gu.stride(0)) hold
    [gate | up]; returns silu(gate) * up as fp32 [M, n], or with ``to_f16``
    the fp16 rows and row exponents of :func:`rows_to_f16` of that result."""
    import torch
    m = gu.shape[0]
    if gu.dtype != torch.float32 or gu.stride(1) != 1:
        raise ValueError("silu_mul_rows: fp32 rows with unit column stride")
    if to_f16:
        out = torch.empty((m, n), dtype=torch.float16, device=gu.device)
        e = torch.empty((m,), dtype=torch.int32, device=gu.device)
        check(lib().ftc_silu_mul_rows(gu.data_ptr(), m, n, gu.stride(0), None, out.data_ptr(),
                                      e.data_ptr(), _stream(stream)), "ftc_silu_mul_rows")
        return out, e
    h = torch.empty((m, n), dtype=torch.float32, device=gu.device)
    check(lib().ftc_silu_mul_rows(gu.data_ptr(), m, n, gu.stride(0), h.data_ptr(), None, None,
                                  _stream(stream)), "ftc_silu_mul_rows")
    return h


def _align(n, a=256):
    return (n + a - 1) // a * a


def moe_route(logits, top_k, stream=None):
    """Device routing (ftc_moe_route) of fp32 logits [T, E]: returns a dict of
    int32 / fp32 CUDA tensors idx, w, counts, offsets, rank, pos, row_token."""
    import torch
    T, E = logits.shape
    dev = logits.device
    i32 = dict(dtype=torch.int32, device=dev)
    r = {"idx": torch.empty((T, top_k), **i32), "w": torch.empty((T, top_k), dtype=torch.float32,
                                                                  device=dev),
         "counts": torch.empty((E,), **i32), "offsets": torch.empty((E + 1,), **i32),
         "rank": torch.empty((E,), **i32), "pos": torch.empty((T, top_k), **i32),
         "row_token": torch.empty((max(1, T * top_k),), **i32)}
    check(lib().ftc_moe_route(logits.data_ptr(), T, E, top_k, r["idx"].data_ptr(),
                              r["w"].data_ptr(), r["counts"].data_ptr(), r["offsets"].data_ptr(),
                              r["rank"].data_ptr(), r["pos"].data_ptr(), r["row_token"].data_ptr(),
                              _stream(stream)), "ftc_moe_route")
    return r


def moe_combine(y, route, out=None, stream=None, pos=None):
    """out[t] = sum_u w[t][u] * y[pos[t][u]] in expert first-use order
    (``pos`` defaults to the routing's row positions)."""
    import torch
    T, U = route["idx"].shape
    K = y.shape[-1]
    if out is None:
        out = torch.empty((T, K), dtype=torch.float32, device=y.device)
    pos = route["pos"] if pos is None else pos
    check(lib().ftc_moe_combine(y.data_ptr(), pos.data_ptr(), route["idx"].data_ptr(),
                                route["w"].data_ptr(), route["rank"].data_ptr(), T, U, K,
                                out.data_ptr(), _stream(stream)), "ftc_moe_combine")
    return out


def ep_pack(x, route, world, cap, send=None, stream=None):
    """Rows of this rank's tokens into the equal-split send buffer
    [world, cap, n_embd] (ftc_ep_pack); returns (send, pos_padded)."""
    import torch
    T, K = x.shape
    U = route["idx"].shape[1]
    E = route["counts"].shape[0]
    xt = {torch.float32: F.F32, torch.bfloat16: F.BF16, torch.float16: F.F16}[x.dtype]
    if send is None:
        send = torch.empty((world, cap, K), dtype=x.dtype, device=x.device)
    pp = torch.empty((T, U), dtype=torch.int32, device=x.device)
    check(lib().ftc_ep_pack(x.data_ptr(), xt, T, K, route["idx"].data_ptr(),
                            route["counts"].data_ptr(), route["pos"].data_ptr(),
                            route["row_token"].data_ptr(), E, U, world, cap, send.data_ptr(),
                            pp.data_ptr(), _stream(stream)), "ftc_ep_pack")
    return send, pp


def ep_regroup(recv_counts, world, n_local, cap, stream=None):
    """(perm, inv, counts, offsets) int32 CUDA tensors of ftc_ep_regroup."""
    import torch
    dev = recv_counts.device
    i32 = dict(dtype=torch.int32, device=dev)
    perm, inv = torch.empty(world * cap, **i32), torch.empty(world * cap, **i32)
    counts, offsets = torch.empty(n_local, **i32), torch.empty(n_local, **i32)
    check(lib().ftc_ep_regroup(recv_counts.data_ptr(), world, n_local, cap, perm.data_ptr(),
                               inv.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                               _stream(stream)), "ftc_ep_regroup")
    return perm, inv, counts, offsets


class MoeLayer:
    """One MoE FFN layer on the device (``ftc_moe_ffn``).

    ``gate_exps``/``up_exps``: uint8 CUDA tensors of E planes of n_ff Q4_K rows
    of n_embd; ``down_exps``: E planes of n_embd rows of n_ff (standard GGUF
    layout)."""

    def __init__(self, gate_exps, up_exps, down_exps, n_experts, top_k, n_embd, n_ff,
                 dtype=F.Q4_K):
        t = F.dtype_id(dtype)
        gu_rs, dn_rs = row_bytes(t, n_embd), row_bytes(t, n_ff)
        self._keep = (gate_exps, up_exps, down_exps)
        self.desc = MoeDesc(t, n_experts, top_k, n_embd, n_ff,
                            gate_exps.data_ptr(), up_exps.data_ptr(), down_exps.data_ptr(),
                            gu_rs, gu_rs * n_ff, dn_rs, dn_rs * n_embd)
        self.n_experts, self.top_k, self.n_embd = n_experts, top_k, n_embd
        self._ws = None
        self._ews = None

    def workspace_bytes(self, T):
        n = int(lib().ftc_moe_workspace_bytes(C.byref(self.desc), T))
        if n == 0 and T > 0:
            raise FtcError("ftc_moe_workspace_bytes", -1, last_error())
        return n

    def workspace(self, T, device="cuda"):
        import torch
        n = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(max(n, 256), dtype=torch.uint8, device=device)
        return self._ws

    def __call__(self, logits, x, out=None, stream=None):
        """out[t] = routed-expert FFN of x[t]; logits fp32 [T, E], x [T, n_embd]
        (fp32, bf16 or fp16 CUDA tensor); returns fp32 [T, n_embd]."""
        import torch
        T = x.shape[0]
        xt = {torch.float32: F.F32, torch.bfloat16: F.BF16, torch.float16: F.F16}[x.dtype]
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=x.device)
        ws = self.workspace(T, x.device)
        check(lib().ftc_moe_ffn(C.byref(self.desc), logits.data_ptr(), x.data_ptr(), xt, T,
                                out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(stream)),
              "ftc_moe_ffn")
        return out

    def experts(self, x, counts, offsets, max_rows, out=None, stream=None):
        """Expert FFNs on rows of x already grouped by expert (ftc_moe_experts):
        counts / offsets int32 CUDA tensors [E]; returns fp32 [rows, n_embd]."""
        import torch
        R = x.shape[0]
        xt = {torch.float32: F.F32, torch.bfloat16: F.BF16, torch.float16: F.F16}[x.dtype]
        if out is None:
            out = torch.empty((R, self.n_embd), dtype=torch.float32, device=x.device)
        n = int(lib().ftc_moe_experts_workspace_bytes(C.byref(self.desc), R))
        if self._ews is None or self._ews.numel() < n:
            self._ews = torch.empty(max(n, 256), dtype=torch.uint8, device=x.device)
        check(lib().ftc_moe_experts(C.byref(self.desc), x.data_ptr(), xt, R, counts.data_ptr(),
                                    offsets.data_ptr(), max_rows, out.data_ptr(),
                                    self._ews.data_ptr(), self._ews.numel(), _stream(stream)),
              "ftc_moe_experts")
        return out

    def routing(self, T):
        """(idx [T, U] int32, weights [T, U] fp32, counts [E] int32) of the last
        call, read from the start of the workspace."""
        import torch
        R = T * self.top_k
        ws = self._ws
        o_w = _align(R * 4)
        o_c = o_w + _align(R * 4)
        idx = ws[:R * 4].view(torch.int32).reshape(T, self.top_k)
        w = ws[o_w:o_w + R * 4].view(torch.float32).reshape(T, self.top_k)
        cnt = ws[o_c:o_c + self.n_experts * 4].view(torch.int32)
        return idx, w, cnt


def dequant(w, dtype, n_rows, k, out=None, row_stride=None, stream=None):
    import torch
    t = F.dtype_id(dtype)
    if out is None:
        out = torch.empty((n_rows, k), dtype=torch.float32, device=w.device)
    rs = row_stride if row_stride is not None else row_bytes(t, k)
    check(lib().ftc_dequant(t, w.data_ptr(), n_rows, k, rs, out.data_ptr(), _stream(stream)),
          "ftc_dequant")
    return out


# ------------------------------------------------------------ host tensor

class HostTensor:
    """ft::HostTensor (ft/include/ft/types.h:119-140): a view of GGUF blocks in
    host memory.  ne[0] = cols (K, the block axis), ne[1] = rows (N),
    ne[2] = expert planes."""

    def __init__(self, data, dtype, ne, name="t"):
        self.data = np.ascontiguousarray(data, dtype=np.uint8)
        self.dtype = F.dtype_id(dtype)
        self.ne = tuple(int(v) for v in ne) + (1,) * (4 - len(ne))
        self.name = name
        if self.data.nbytes < self.row_stride_bytes() * self.ne[1] * self.ne[2] * self.ne[3]:
            raise ValueError("HostTensor: data smaller than its shape")
        self._base = self.data.ctypes.data  # the array owns its buffer: fixed address

    def cols(self):
        return self.ne[0]

    def rows(self):
        return self.ne[1]

    def row_stride_bytes(self):
        return F.row_bytes(self.dtype, self.ne[0])

    def slice_bytes(self):
        return self.row_stride_bytes() * self.ne[1]

    def ptr(self, offset=0):
        return self._base + offset

    def slice(self, e):
        """Host address of expert plane e (HostTensor::slice)."""
        return self.ptr(self.slice_bytes() * e)

    @property
    def nbytes(self):
        return self.data.nbytes


# ------------------------------------------------------------ backend

LOOP_PATH = os.path.join(PKG, "libftcloop.so")
_loop = None


def loop_lib():
    """Load libftcloop.so (host/call_loop.c): the native caller loop."""
    global _loop
    if _loop is None:
        if not os.path.exists(LOOP_PATH):
            raise FileNotFoundError(
                f"{LOOP_PATH} is missing: build it with `python -m xwfes_b200.build`")
        L = C.CDLL(LOOP_PATH)
        L.ftc_call_loop.restype = C.c_int
        L.ftc_call_loop.argtypes = [_p, _p, C.c_int, C.POINTER(_p), C.POINTER(_i64),
                                    C.POINTER(_i64), C.POINTER(_p), C.POINTER(C.c_int),
                                    C.POINTER(_i64), C.POINTER(_p), C.c_int]
        _loop = L
    return _loop


class MatmulSequence:
    """A fixed list of IBackend::matmul calls on one backend, replayed by
    ``run(reps)`` from native code: each call is ftc_backend_matmul with
    host buffers, synchronous, in list order -- what an engine's decode loop
    does per step -- with no interpreter between the calls.  The arrays are
    checked and their addresses taken once, here; they must stay alive and
    in place while the sequence is used (it keeps references)."""

    def __init__(self, backend, calls):
        n = len(calls)
        self._be = backend
        self._keep = [c for c in calls]
        xs, ws, ys = (_p * n)(), (_p * n)(), (_p * n)()
        ms, ks, ns = (_i64 * n)(), (_i64 * n)(), (_i64 * n)()
        dts = (C.c_int * n)()
        for i, (x, M, K, W, y) in enumerate(calls):
            N = W.ne[1]
            assert x.dtype == np.float32 and x.flags.c_contiguous and x.size >= M * K
            assert y.dtype == np.float32 and y.flags.c_contiguous and y.size >= M * N
            xs[i], ws[i], ys[i] = x.ctypes.data, W._base, y.ctypes.data
            ms[i], ks[i], ns[i], dts[i] = M, K, N, W.dtype
        self._args = (n, xs, ms, ks, ws, dts, ns, ys)
        self._fn = C.cast(lib().ftc_backend_matmul, _p)

    def run(self, reps=1):
        n, xs, ms, ks, ws, dts, ns, ys = self._args
        rc = loop_lib().ftc_call_loop(self._fn, self._be._h, n, xs, ms, ks, ws, dts, ns, ys, reps)
        if rc:
            raise FtcError("ftc_backend_matmul", rc, last_error())


class CudaBackend:
    """Python mirror of the ft::IBackend a CUDA build plugs in
    (ft/include/ft/backend.h:21-40), over the ftc_backend_* C ABI.  Host
    buffers in, host buffers out.  Weights passed to ``upload`` stay in HBM
    (keyed by host address; the HostTensor is kept alive until ``evict``);
    any other weight is copied to the device for the one call."""

    def __init__(self, device=0):
        h = C.c_void_p()
        check(lib().ftc_backend_create(device, C.byref(h)), "ftc_backend_create")
        self._h = h
        self._keep = {}  # uploaded host tensors (their addresses key the cache)

    def close(self):
        if self._h:
            lib().ftc_backend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def name(self):
        buf = C.create_string_buffer(256)
        mem = C.c_uint64()
        check(lib().ftc_backend_info(self._h, buf, 256, C.byref(mem)), "ftc_backend_info")
        return buf.value.decode()

    def info(self):
        buf = C.create_string_buffer(256)
        mem = C.c_uint64()
        check(lib().ftc_backend_info(self._h, buf, 256, C.byref(mem)), "ftc_backend_info")
        return {"name": buf.value.decode(), "integrated": False, "uma": False,
                "mem_bytes": mem.value}

    def ready(self):
        return bool(self._h)

    def stream(self):
        return lib().ftc_backend_stream(self._h)

    def upload(self, t):
        """Pre-load a HostTensor's blocks into HBM (Engine::load time)."""
        self._keep[t.ptr()] = t
        check(lib().ftc_backend_upload(self._h, t.ptr(), t.nbytes), "ftc_backend_upload")

    def evict(self, t):
        check(lib().ftc_backend_evict(self._h, t.ptr()), "ftc_backend_evict")
        self._keep.pop(t.ptr(), None)

    def cached_bytes(self):
        v = C.c_uint64()
        check(lib().ftc_backend_cached_bytes(self._h, C.byref(v)), "ftc_backend_cached_bytes")
        return v.value

    def device_ptr(self, t, offset=0):
        return lib().ftc_backend_device_ptr(self._h, t.ptr(offset))

    def matmul(self, x, M, K, W, y):
        """IBackend::matmul: x fp32 [M][K] host, y fp32 [M][N] host (written)."""
        n = W.ne[1]
        assert x.dtype == np.float32 and x.flags.c_contiguous and x.size >= M * K
        assert y.dtype == np.float32 and y.flags.c_contiguous and y.size >= M * n
        rc = _lib.ftc_backend_matmul(self._h, x.ctypes.data, M, K, W._base, W.dtype, n,
                                     y.ctypes.data)
        if rc:
            raise FtcError("ftc_backend_matmul", rc, last_error())

    def kv_alloc(self, n_layers, capacity, dim):
        """The engine's KV cache in this backend's HBM (ftc_backend_kv_alloc)."""
        check(lib().ftc_backend_kv_alloc(self._h, n_layers, capacity, dim), "ftc_backend_kv_alloc")

    def attention(self, layer, base, q, k_new, v_new, n_head, n_head_kv, head_dim, write_kv=True,
                  out=None):
        """One layer's attention with host arrays (ftc_backend_attention): q
        fp32 [M, n_head*head_dim], k_new / v_new [M, n_head_kv*head_dim];
        returns out [M, n_head*head_dim]."""
        q = np.ascontiguousarray(q, dtype=np.float32)
        k_new = np.ascontiguousarray(k_new, dtype=np.float32)
        v_new = np.ascontiguousarray(v_new, dtype=np.float32)
        M = q.shape[0]
        assert q.size == M * n_head * head_dim
        assert k_new.size == v_new.size == M * n_head_kv * head_dim
        if out is None:
            out = np.empty((M, n_head * head_dim), dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.size >= q.size
        check(lib().ftc_backend_attention(self._h, layer, base, M, n_head, n_head_kv, head_dim,
                                          q.ctypes.data, k_new.ctypes.data, v_new.ctypes.data,
                                          1 if write_kv else 0, out.ctypes.data),
              "ftc_backend_attention")
        return out

    def kv_read(self, layer, pos0, n, dim):
        """Rows [pos0, pos0+n) of a layer of the device KV cache -> (k, v)
        host arrays [n, dim] (the engine's prefix-cache snapshot copy)."""
        k = np.empty((n, dim), dtype=np.float32)
        v = np.empty((n, dim), dtype=np.float32)
        check(lib().ftc_backend_kv_read(self._h, layer, pos0, n, k.ctypes.data, v.ctypes.data),
              "ftc_backend_kv_read")
        return k, v

    def kv_write(self, layer, pos0, k, v):
        """Host rows k, v [n, dim] into rows [pos0, pos0+n) of a layer of the
        device KV cache (the engine's prefix-cache restore copy)."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        assert k.shape == v.shape and k.ndim == 2
        check(lib().ftc_backend_kv_write(self._h, layer, pos0, k.shape[0], k.ctypes.data,
                                         v.ctypes.data), "ftc_backend_kv_write")

    def matmul_sequence(self, calls):
        """A fixed list of ``matmul`` calls, ``calls`` = [(x, M, K, W, y), ...]
        with the same argument rules, replayed from native code (see
        MatmulSequence)."""
        return MatmulSequence(self, calls)

    def matmul_down_axpy(self, x, M, n_in, W, y):
        """ft::matmul_down_axpy: y[m] += x_m . W over the first ``n_in`` rows of
        W (``W.cols()`` weights each); x fp32 [M][n_in], y fp32 [M][W.cols()]
        host arrays, y accumulated."""
        if n_in > W.rows():
            raise ValueError("matmul_down_axpy: n_in exceeds W.rows()")
        assert x.dtype == np.float32 and x.flags.c_contiguous and x.size >= M * n_in
        assert y.dtype == np.float32 and y.flags.c_contiguous and y.size >= M * W.cols()
        check(lib().ftc_backend_matmul_down_axpy(self._h, x.ctypes.data, M, n_in, W.ptr(),
                                                 W.dtype, W.cols(), y.ctypes.data),
              "ftc_backend_matmul_down_axpy")

    def moe_ffn(self, x, logits, gate_exps, up_exps, down_exps, top_k, out, bias=None):
        """ftc_backend_moe_ffn: the routed experts of the engine's moe_ffn with
        host arrays; gate/up/down_exps are HostTensors with ne = (n_embd, n_ff,
        E) / (n_ff, n_embd, E) (standard down layout); ``out`` fp32 [T][n_embd]
        is accumulated."""
        T, K = x.shape
        E = gate_exps.ne[2]
        assert x.dtype == np.float32 and x.flags.c_contiguous
        assert logits.dtype == np.float32 and logits.flags.c_contiguous and logits.shape == (T, E)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.shape == (T, K)
        d = MoeDesc(dtype=gate_exps.dtype, n_experts=E, top_k=top_k, n_embd=K,
                    n_ff=gate_exps.rows(), gate_exps=gate_exps.ptr(), up_exps=up_exps.ptr(),
                    down_exps=down_exps.ptr(), gu_row_stride=gate_exps.row_stride_bytes(),
                    gu_plane_stride=gate_exps.slice_bytes(),
                    dn_row_stride=down_exps.row_stride_bytes(),
                    dn_plane_stride=down_exps.slice_bytes())
        b = None
        if bias is not None:
            bias = np.ascontiguousarray(bias, dtype=np.float32)
            assert bias.shape == (E,)
            b = bias.ctypes.data
        check(lib().ftc_backend_moe_ffn(self._h, C.byref(d), logits.ctypes.data, b,
                                        x.ctypes.data, T, out.ctypes.data), "ftc_backend_moe_ffn")

    def run_expert_chunk(self, x, out, gate, up, down, dtype, M, K, IC, gu_stride, dn_stride):
        """IBackend::run_expert_chunk with host addresses (ints) for the
        gate/up/down windows; ``out`` is accumulated into."""
        assert out.dtype == np.float32 and out.flags.c_contiguous
        job = ExpertChunkJob(x.ctypes.data, out.ctypes.data, gate, up, down, F.dtype_id(dtype),
                             M, K, IC, gu_stride, dn_stride)
        check(lib().ftc_backend_run_expert_chunk(self._h, C.byref(job)),
              "ftc_backend_run_expert_chunk")

    def sync(self):
        check(lib().ftc_backend_sync(self._h), "ftc_backend_sync")


IPC_HANDLE_BYTES = 64  # FTC_IPC_HANDLE_BYTES in include/ftc.h


class PeerAllreduce:
    """Sum of fp32 vectors over the ranks of a process group through NVLink
    peer memory (ftc_peer_ar_*): one process per GPU, small vectors.  The
    CUDA IPC handles are exchanged with an all-gather over ``group``."""

    def __init__(self, max_elems, group=None):
        import torch
        import torch.distributed as dist
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_elems = int(max_elems)
        self.torch = torch
        self._ar = None
        # Each step's outcome is shared before the next one, so that a rank
        # whose allocation or mapping failed makes every rank raise the same
        # error instead of leaving the others waiting in a later collective.
        h = (C.c_uint8 * IPC_HANDLE_BYTES)()
        ptr = _p()
        err = None
        try:
            check(lib().ftc_peer_ar_create(self.rank, self.world, self.max_elems, C.byref(ptr), h),
                  "ftc_peer_ar_create")
            self._ar = ptr
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            err = f"{type(e).__name__}: {e}"
        handles = [None] * self.world
        dist.all_gather_object(handles, (err, bytes(h)), group=group)
        self._agree([e for e, _ in handles], "ftc_peer_ar_create")
        allh = (C.c_uint8 * (IPC_HANDLE_BYTES * self.world)).from_buffer_copy(
            b"".join(b for _, b in handles))
        err = None
        try:
            check(lib().ftc_peer_ar_open(self._ar, allh), "ftc_peer_ar_open")
        except Exception as e:  # noqa: BLE001
            err = f"{type(e).__name__}: {e}"
        errs = [None] * self.world
        # also the barrier after which every rank has mapped every other
        # rank's buffer, before the first call
        dist.all_gather_object(errs, err, group=group)
        self._agree(errs, "ftc_peer_ar_open")

    def _agree(self, errs, step):
        bad = [(r, e) for r, e in enumerate(errs) if e is not None]
        if bad:
            try:
                self.close()
            except FtcError:
                self._ar = None  # the set-up failure is the error to report
            raise RuntimeError(f"PeerAllreduce: {step} failed on rank(s) "
                               + "; ".join(f"{r}: {e}" for r, e in bad))

    def fits(self, t):
        return t.dtype == self.torch.float32 and t.is_contiguous() and t.numel() <= self.max_elems

    def sum_(self, t, stream=None):
        """In-place sum of the fp32 CUDA tensor ``t`` over the ranks."""
        if not self.fits(t):
            raise ValueError("PeerAllreduce: contiguous fp32 tensor of at most max_elems")
        check(lib().ftc_peer_ar_sum_f32(self._ar, t.data_ptr(), t.data_ptr(), t.numel(),
                                        _stream(stream)), "ftc_peer_ar_sum_f32")
        return t

    def mul_mat_vec_sum(self, w, dtype, n, k, x, y=None, row_stride=None, stream=None):
        """y = sum over the ranks of x . W^T for this rank's shard W (one token,
        fp32), GEMV and allreduce in one kernel (ftc_mul_mat_vec_allreduce)."""
        import torch
        t = F.dtype_id(dtype)
        if y is None:
            y = torch.empty((1, n), dtype=torch.float32, device=x.device)
        rs = row_stride if row_stride is not None else row_bytes(t, k)
        check(lib().ftc_mul_mat_vec_allreduce(self._ar, t, w.data_ptr(), n, k, rs, x.data_ptr(),
                                              y.data_ptr(), _stream(stream)),
              "ftc_mul_mat_vec_allreduce")
        return y

    def silu_mul_mat_vec_sum(self, w, dtype, n, k, gu, up_offset=None, y=None, row_stride=None,
                             stream=None):
        """y = sum over the ranks of (silu(gate) * up) . W^T for this rank's
        shard W, gu = [gate (k) | up (k)] fp32 (ftc_mul_mat_vec_silu): the
        SiLU product, the GEMV and the allreduce in one kernel."""
        return mul_mat_vec_silu(w, dtype, n, k, gu, up_offset=up_offset, y=y,
                                row_stride=row_stride, ar=self, stream=stream)

    def close(self):
        if self._ar:
            check(lib().ftc_peer_ar_destroy(self._ar), "ftc_peer_ar_destroy")
            self._ar = None
