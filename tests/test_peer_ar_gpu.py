"""The NVLink peer allreduce (ftc_peer_ar) between two processes on two GPUs.

Exactness: with two ranks every element is in[rank 0] + in[rank 1] in fp32,
one rounding, so the result must equal numpy's a0 + a1 bit for bit on both
ranks -- for vector lengths that take the float4 path and the scalar path,
for repeated calls (the two buffer parities alternate) and for calls
replayed from a CUDA graph (the call counters live on the device).

Fused GEMV + allreduce (ftc_mul_mat_vec_allreduce): every rank's GEMV
partial pushed by the GEMV kernel itself and summed there must equal the
separate GEMV followed by ftc_peer_ar_sum_f32, bit for bit, on every rank --
also interleaved with plain sums (the two share the call counters) and
replayed from a CUDA graph.

Failure path: when one rank does not join a call, the other's kernel gives
up after the library's wait bound, records status 1 (ftc_device_status) and
the process stays usable.  Nothing faults: the waiting rank only polls its
own flags; the absent rank keeps its buffer mapped until both have left."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MAX = 1 << 17
SIZES = (1, 3, 4, 8192, 8194, 131072)


def inputs(rank, n, call):
    return np.random.default_rng(1000 * call + 10 * rank + n).standard_normal(n).astype(np.float32)


_CHILD = r"""
import os, sys, time, datetime, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from xwfes_b200 import ftc
import test_peer_ar_gpu as T
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
ar = ftc.PeerAllreduce(T.MAX)
out = {{}}
mode = {mode!r}
if mode == "sum":
    for call in range(3):
        for n in T.SIZES:
            t = torch.from_numpy(T.inputs(rank, n, call)).cuda()
            ar.sum_(t)
            out[f"{{call}}_{{n}}"] = t.cpu().numpy()
    # graph replay: the captured call, replayed on new inputs
    n = 8192
    t = torch.empty(n, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ar.sum_(t, stream=s)
    for call in (10, 11):
        t.copy_(torch.from_numpy(T.inputs(rank, n, call)))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        out[f"{{call}}_{{n}}"] = t.cpu().numpy()
    del g
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
elif mode == "fused":
    from xwfes_b200 import formats as F, synth as S
    shapes = [(8192, 1024), (1000, 3584), (4096, 4096)]
    for i, (n, k) in enumerate(shapes):
        w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=rank, name=f"par.{{i}}")).cuda()
        for call in range(2):
            x = torch.from_numpy(T.inputs(rank, k, 100 + call)).cuda().reshape(1, k)
            yf = ar.mul_mat_vec_sum(w, F.Q4_K, n, k, x)
            yr = ftc.mul_mat_vec(w, F.Q4_K, n, k, x)
            ar.sum_(yr)
            out[f"f{{i}}_{{call}}"] = yf.cpu().numpy()
            out[f"r{{i}}_{{call}}"] = yr.cpu().numpy()
    n, k = shapes[0]
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=rank, name="par.0")).cuda()
    x = torch.from_numpy(T.inputs(rank, k, 200)).cuda().reshape(1, k)
    y = torch.empty(1, n, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ar.mul_mat_vec_sum(w, F.Q4_K, n, k, x, y=y, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ar.mul_mat_vec_sum(w, F.Q4_K, n, k, x, y=y, stream=s)
    for call in range(3):
        y.zero_()
        g.replay()
        torch.cuda.synchronize()
        out[f"g_{{call}}"] = y.cpu().numpy()
    del g
    yr = ftc.mul_mat_vec(w, F.Q4_K, n, k, x)
    ar.sum_(yr)
    out["g_ref"] = yr.cpu().numpy()
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
elif mode == "fused_silu":
    from xwfes_b200 import formats as F, synth as S
    for i, (n, k) in enumerate([(8192, 3584), (4096, 1024)]):
        w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=rank, name=f"ps.{{i}}")).cuda()
        gu = (4 * torch.from_numpy(T.inputs(rank, 2 * k, 300 + i))).cuda().reshape(1, 2 * k)
        yf = ar.silu_mul_mat_vec_sum(w, F.Q4_K, n, k, gu)
        yr = ftc.mul_mat_vec(w, F.Q4_K, n, k, ftc.silu_mul_rows(gu, k))
        ar.sum_(yr)
        out[f"sf{{i}}"] = yf.cpu().numpy()
        out[f"sr{{i}}"] = yr.cpu().numpy()
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
else:  # rank 1 stays out of the call; rank 0 must time out cleanly
    if rank == 0:
        t = torch.ones(8192, device="cuda")
        t0 = time.time()
        ar.sum_(t)
        st = ftc.device_status()
        out["status"] = np.array([st, time.time() - t0])
        # the context still works
        out["after"] = (torch.arange(4, device="cuda") * 2).cpu().numpy()
dist.barrier()
ar.close()
np.savez(os.path.join({out_dir!r}, f"r{{rank}}.npz"), **out)
dist.destroy_process_group()
"""


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(tmp_path, mode):
    code = _CHILD.format(root=ROOT, out_dir=str(tmp_path), mode=mode)
    port = _free_port()
    procs = []
    for r in range(2):
        # vectors of 65536+ elements take the two-shot exchange (by default only
        # used on 4+ ranks), so both exchanges are covered on two GPUs
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                   FTC_PEER_AR_TWO_SHOT="65536")
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, cwd=ROOT))
    for p in procs:
        assert p.wait(timeout=300) == 0
    return [np.load(tmp_path / f"r{r}.npz") for r in range(2)]


def test_two_ranks_sum_exactly(tmp_path):
    r0, r1 = _run(tmp_path, "sum")
    keys = [f"{c}_{n}" for c in range(3) for n in SIZES] + ["10_8192", "11_8192"]
    for key in keys:
        call, n = (int(v) for v in key.split("_"))
        want = inputs(0, n, call) + inputs(1, n, call)
        assert np.array_equal(r0[key], want), key
        assert np.array_equal(r1[key], want), key


def test_absent_rank_times_out(tmp_path):
    r0, _ = _run(tmp_path, "absent")
    status, secs = r0["status"]
    assert status == 1 and secs >= 1.0
    assert r0["after"].tolist() == [0, 2, 4, 6]


def test_fused_gemv_allreduce_matches_separate(tmp_path):
    r0, r1 = _run(tmp_path, "fused")
    for i in range(3):
        for call in range(2):
            f, r = f"f{i}_{call}", f"r{i}_{call}"
            assert np.array_equal(r0[f], r0[r]) and np.array_equal(r1[f], r1[r]), (i, call)
            assert np.array_equal(r0[f], r1[f]), (i, call)
    for call in range(3):
        assert np.array_equal(r0[f"g_{call}"], r0["g_ref"])
        assert np.array_equal(r1[f"g_{call}"], r0["g_ref"])
