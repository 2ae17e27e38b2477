"""The native caller loop (xwfes_b200/host/call_loop.c) behind
MatmulSequence: it must pass each call's arguments through unchanged, in
list order, repeat the list `reps` times, and stop at the first non-zero
status.  Checked on the CPU with a recording stand-in for
ftc_backend_matmul (no GPU, no CUDA library call)."""
import ctypes as C

import numpy as np
import pytest

from xwfes_b200 import build, ftc

MM = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int,
                 C.c_int64, C.c_void_p)


@pytest.fixture(scope="module")
def loop():
    build.build()
    return ftc.loop_lib()


def marshal(calls):
    n = len(calls)
    P, I64 = C.c_void_p * n, C.c_int64 * n
    xs, ws, ys = P(*[c[0] for c in calls]), P(*[c[3] for c in calls]), P(*[c[6] for c in calls])
    ms, ks, ns = I64(*[c[1] for c in calls]), I64(*[c[2] for c in calls]), I64(*[c[5] for c in calls])
    dts = (C.c_int * n)(*[c[4] for c in calls])
    return n, xs, ms, ks, ws, dts, ns, ys


def test_calls_in_order_and_repeated(loop):
    seen = []

    def fake(be, x, M, K, w, dtype, N, y):
        seen.append((be, x, M, K, w, dtype, N, y))
        return 0

    cb = MM(fake)
    calls = [(0x1000 + i, i + 1, 256 * (i + 1), 0x9000 + i, 12 + i, 64 * i + 8, 0x5000 + i)
             for i in range(5)]
    rc = loop.ftc_call_loop(C.cast(cb, C.c_void_p), C.c_void_p(0xBEEF), *marshal(calls), 3)
    assert rc == 0
    want = [(0xBEEF, x, M, K, w, dt, N, y) for _ in range(3) for (x, M, K, w, dt, N, y) in calls]
    assert seen == want


def test_stops_at_first_error(loop):
    seen = []

    def fake(be, x, M, K, w, dtype, N, y):
        seen.append(x)
        return -7 if len(seen) == 4 else 0

    cb = MM(fake)
    calls = [(0x100 + i, 1, 256, 0x200, 12, 8, 0x300) for i in range(3)]
    rc = loop.ftc_call_loop(C.cast(cb, C.c_void_p), C.c_void_p(1), *marshal(calls), 5)
    assert rc == -7
    assert seen == [0x100, 0x101, 0x102, 0x100]  # the fourth call failed; nothing after it


def test_rejects_missing_function_or_backend(loop):
    calls = [(0x100, 1, 256, 0x200, 12, 8, 0x300)]
    assert loop.ftc_call_loop(None, C.c_void_p(1), *marshal(calls), 1) == -1
    cb = MM(lambda *a: 0)
    assert loop.ftc_call_loop(C.cast(cb, C.c_void_p), None, *marshal(calls), 1) == -1


def test_sequence_checks_arrays_once():
    """MatmulSequence validates dtype, layout and sizes at construction,
    like CudaBackend.matmul does per call."""
    class FakeBe:
        _h = C.c_void_p(1)

    w = ftc.HostTensor(np.zeros((4, 144), np.uint8), 12, (256, 4))
    x = np.zeros((1, 256), np.float32)
    y = np.zeros((1, 4), np.float32)
    with pytest.raises(AssertionError):
        ftc.MatmulSequence(FakeBe(), [(x.astype(np.float64), 1, 256, w, y)])
    with pytest.raises(AssertionError):
        ftc.MatmulSequence(FakeBe(), [(x, 1, 256, w, np.zeros((1, 3), np.float32))])
