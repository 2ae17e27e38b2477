"""GGUF block formats handled by the dequant-matmul path.

Type ids are the reference's ``ft::DType`` values (ft/include/ft/types.h:20-27)
extended with the GGUF ids of the two K-quants the reference does not load
(ft/src/gguf.cpp:129-137 rejects them).  Row geometry follows
``ft::dtype_row_bytes`` (ft/include/ft/types.h:51-55): a row of ``K`` weights
is ``ceil(K / block_elems)`` whole blocks.
"""

F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 3, 8, 12, 14, 30

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q8_0: "Q8_0",
         Q4_K: "Q4_K", Q6_K: "Q6_K", BF16: "BF16"}
BY_NAME = {v: k for k, v in NAMES.items()}

# (weights per block, bytes per block)
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20),
         Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

QK_K = 256


def dtype_id(t):
    """Accept a type id or a name such as ``"Q4_K"``."""
    if isinstance(t, str):
        return BY_NAME[t.upper()]
    if t not in BLOCK:
        raise ValueError(f"unknown GGUF dtype id {t}")
    return int(t)


def row_bytes(t, k):
    """Bytes of one row of ``k`` weights (whole blocks)."""
    eb, bb = BLOCK[dtype_id(t)]
    return -(-int(k) // eb) * bb


def bytes_per_weight(t):
    eb, bb = BLOCK[dtype_id(t)]
    return bb / eb
