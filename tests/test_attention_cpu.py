"""ftc_attention / ftc_rope / ftc_backend_attention without a GPU: bad
arguments are refused before any CUDA call, with a message naming the
problem (the checks a caller can rely on)."""
import ctypes as C

import pytest

from xwfes_b200 import ftc


@pytest.fixture(scope="module")
def lib():
    from xwfes_b200 import build
    build.build()
    return ftc.lib()


def test_attention_argument_checks(lib):
    p = 4096  # any non-null, 16-byte aligned value: nothing is dereferenced
    cases = [
        ((p, 0, 32, 8, 128, p, p, 1024, 0, p, p, p, None, 0, None), "empty"),
        ((p, 1, 32, 8, 128, p, p, 1024, -1, p, p, p, None, 0, None), "negative base"),
        ((p, 1, 30, 8, 128, p, p, 1024, 0, p, p, p, None, 0, None), "multiple of n_head_kv"),
        ((p, 1, 32, 8, 96, p, p, 768, 0, p, p, p, None, 0, None), "head_dim"),
        ((p, 1, 32, 8, 128, None, None, 1024, 5, p, p, p, None, 0, None), "null"),
        ((p, 1, 32, 8, 128, p, p, 1020, 0, p, p, p, None, 0, None), "kv_stride"),
        ((p, 1, 32, 8, 128, p, p, 1026, 0, p, p, p, None, 0, None), "kv_stride"),
        ((p + 8, 1, 32, 8, 128, p, p, 1024, 0, p, p, p, None, 0, None), "aligned"),
        ((p, 70000, 32, 8, 128, p, p, 1024, 0, p, p, p, None, 0, None), "too many"),
    ]
    for args, word in cases:
        assert lib.ftc_attention(*args) != 0, word
        assert word in ftc.last_error(), (word, ftc.last_error())


def test_rope_argument_checks(lib):
    assert lib.ftc_rope(None, 1, 8, 128, 0, 1e4, 0, None) != 0
    assert lib.ftc_rope(4096, 1, 8, 127, 0, 1e4, 0, None) != 0
    assert "bad argument" in ftc.last_error()
    assert lib.ftc_rope(4096, 0, 8, 128, 0, 1e4, 1, None) == 0  # no rows: nothing to do


def test_backend_entries_need_a_backend(lib):
    assert lib.ftc_backend_kv_alloc(None, 2, 16, 1024) != 0
    z = (C.c_float * 4)()
    assert lib.ftc_backend_attention(None, 0, 0, 1, 32, 8, 128, z, z, z, 1, z) != 0


def test_kv_copies_need_a_backend(lib):
    z = (C.c_float * 4)()
    assert lib.ftc_backend_kv_read(None, 0, 0, 1, z, z) != 0
    assert lib.ftc_backend_kv_write(None, 0, 0, 1, z, z) != 0
