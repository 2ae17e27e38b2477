"""The Python binding's argument marshalling for the engine-glue entries, on
the CPU with a stand-in for libftcuda.so: the MoE descriptor built from the
expert HostTensors, the router bias, the down projection's shapes and its
workspace request."""

import numpy as np
import pytest

from xwfes_b200 import formats as F, ftc, synth as S

torch = pytest.importorskip("torch")


class Fake:
    def __init__(self, ws_bytes=0):
        self.calls = {}
        self.ws_bytes = ws_bytes

    def ftc_backend_create(self, device, out):
        out._obj.value = 0x51
        return 0

    def ftc_backend_destroy(self, h):
        self.calls["destroy"] = h

    def ftc_backend_moe_ffn(self, h, desc, logits, bias, x, T, out):
        d = desc._obj
        self.calls["moe"] = dict(h=h, T=T, bias=bias, logits=logits, x=x, out=out,
                                 desc={f: getattr(d, f) for f, _ in ftc.MoeDesc._fields_})
        return 0

    def ftc_backend_matmul_down_axpy(self, h, x, M, n_in, w, dtype, N, y):
        self.calls["axpy_be"] = (M, n_in, w, dtype, N)
        return 0

    def ftc_matmul_down_axpy_workspace_bytes(self, t, n_in, n, m):
        return self.ws_bytes

    def ftc_matmul_down_axpy(self, t, w, n_in, n, rs, x, m, y, ws, wsb, st):
        self.calls["axpy"] = (t, n_in, n, rs, m, ws, wsb)
        return 0

    def ftc_row_bytes(self, t, k):
        return F.row_bytes(t, k)

    def ftc_last_error(self):
        return b""


def test_moe_desc_from_expert_tensors(monkeypatch):
    fake = Fake()
    monkeypatch.setattr(ftc, "_lib", fake)
    E, K, FF, T = 4, 512, 768, 3
    g = ftc.HostTensor(S.expert_weights(F.Q4_K, E, FF, K, seed=1), F.Q4_K, (K, FF, E))
    u = ftc.HostTensor(S.expert_weights(F.Q4_K, E, FF, K, seed=2), F.Q4_K, (K, FF, E))
    d = ftc.HostTensor(S.expert_weights(F.Q4_K, E, K, FF, seed=3), F.Q4_K, (FF, K, E))
    x = np.zeros((T, K), np.float32)
    logits = np.zeros((T, E), np.float32)
    out = np.zeros((T, K), np.float32)
    be = ftc.CudaBackend(0)
    be.moe_ffn(x, logits, g, u, d, 2, out, bias=np.arange(E, dtype=np.float32))
    c = fake.calls["moe"]
    assert c["h"].value == 0x51 and c["T"] == T and c["bias"] is not None
    assert (c["x"], c["out"], c["logits"]) == (x.ctypes.data, out.ctypes.data,
                                               logits.ctypes.data)
    rb, rd = F.row_bytes(F.Q4_K, K), F.row_bytes(F.Q4_K, FF)
    assert c["desc"] == dict(dtype=F.Q4_K, n_experts=E, top_k=2, n_embd=K, n_ff=FF,
                             gate_exps=g.ptr(), up_exps=u.ptr(), down_exps=d.ptr(),
                             gu_row_stride=rb, gu_plane_stride=rb * FF,
                             dn_row_stride=rd, dn_plane_stride=rd * K)
    be.moe_ffn(x, logits, g, u, d, 2, out)
    assert fake.calls["moe"]["bias"] is None
    with pytest.raises(AssertionError):
        be.moe_ffn(x, logits[:, :2].copy(), g, u, d, 2, out)  # logits not [T][E]
    be.close()
    assert fake.calls["destroy"] is not None


def test_down_axpy_shapes_and_workspace(monkeypatch):
    fake = Fake(ws_bytes=4096)
    monkeypatch.setattr(ftc, "_lib", fake)
    n_in, n = 300, 512
    w = ftc.HostTensor(S.weight(F.Q4_K, n_in, n, seed=4), F.Q4_K, (n, n_in))
    be = ftc.CudaBackend(0)
    x = np.zeros((2, n_in), np.float32)
    y = np.zeros((2, n), np.float32)
    be.matmul_down_axpy(x, 2, n_in, w, y)
    assert fake.calls["axpy_be"] == (2, n_in, w.ptr(), F.Q4_K, n)
    with pytest.raises(ValueError):
        be.matmul_down_axpy(np.zeros((2, n_in + 1), np.float32), 2, n_in + 1, w, y)  # > W.rows()
    be.close()
    # device entry: the workspace the library asks for is allocated and passed
    wt = torch.from_numpy(w.data)
    xt = torch.zeros((2, n_in))
    yt = torch.zeros((2, n))
    ftc.matmul_down_axpy(wt, F.Q4_K, n_in, n, xt, yt, stream=0)
    t, ni, nn, rs, m, ws, wsb = fake.calls["axpy"]
    assert (t, ni, nn, rs, m, wsb) == (F.Q4_K, n_in, n, F.row_bytes(F.Q4_K, n), 2, 4096)
    assert ws is not None
    fake.ws_bytes = 0
    ftc.matmul_down_axpy(wt, F.Q4_K, n_in, n, xt, yt, stream=0)
    assert fake.calls["axpy"][5] is None and fake.calls["axpy"][6] == 0
