"""tp.CudaOps's routing between the decode GEMV and the GEMM, on the CPU
with a stand-in for the library: which entry each row count reaches, and
that GEMV passes of 8 rows cover every row exactly once (gemv_max_m)."""
import pytest

from xwfes_b200 import tp

torch = pytest.importorskip("torch")


class FakeLib:
    """Records calls; computes x . W^T with W given as a float tensor."""

    def __init__(self):
        self.calls = []

    def mul_mat_vec(self, w, dtype, n, k, x, y=None):
        assert x.shape[0] <= 8 and x.is_contiguous()
        self.calls.append(("gemv", x.shape[0]))
        r = x @ w.T
        if y is None:
            return r
        assert y.shape == r.shape and y.is_contiguous()
        y.copy_(r)
        return y

    def mul_mat_vec_multi(self, ws, dtype, ns, k, x):
        self.calls.append(("gemv_multi", x.shape[0]))
        return [x @ w.T for w in ws]

    def rows_to_f16(self, x):
        self.calls.append(("rows_to_f16", x.shape[0]))
        return x.clone(), None

    def gemm_rowscaled(self, w, dtype, n, k, x16, e):
        self.calls.append(("gemm", x16.shape[0]))
        return x16 @ w.T

    def silu_mul_rows(self, gu, n, to_f16=False):
        h = gu[:, :n] / (1 + torch.exp(-gu[:, :n])) * gu[:, n:2 * n]
        return (h, None) if to_f16 else h


def ops(gemv_max_m):
    o = tp.CudaOps(torch.device("cpu"), gemv_max_m=gemv_max_m)
    o.ftc = FakeLib()
    return o


@pytest.mark.parametrize("M,limit,kind", [(1, 8, "gemv"), (8, 8, "gemv"), (9, 8, "gemm"),
                                          (16, 8, "gemm"), (9, 32, "gemv"), (32, 32, "gemv"),
                                          (33, 32, "gemm")])
def test_row_count_picks_the_entry(M, limit, kind):
    o = ops(limit)
    w = torch.randn(24, 16)
    x = torch.randn(M, 16)
    y = o.matmuls(x, [(w, 24, 16)])[0]
    assert torch.allclose(y, x @ w.T, atol=1e-5)
    kinds = {c[0] for c in o.ftc.calls}
    assert kinds == ({"gemv"} if kind == "gemv" else {"rows_to_f16", "gemm"})
    if kind == "gemv":
        assert sum(m for _, m in o.ftc.calls) == M  # every row once, <= 8 per pass
        assert all(m <= 8 for _, m in o.ftc.calls)


def test_strided_rows_and_silu_path():
    o = ops(32)
    w = torch.randn(20, 12)
    big = torch.randn(21, 40)
    x = big[:, 3:15]  # a column slice: not contiguous
    y = o.matmuls(x, [(w, 20, 12)])[0]
    assert torch.allclose(y, x @ w.T, atol=1e-5)
    gu = torch.randn(21, 24)
    wd = torch.randn(10, 12)
    out = o.silu_matmul(gu, 12, (wd, 10, 12))
    h = gu[:, :12] / (1 + torch.exp(-gu[:, :12])) * gu[:, 12:]
    assert torch.allclose(out, h @ wd.T, atol=1e-5)
