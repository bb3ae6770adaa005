"""Seeded random GGUF tensor blocks of each ggml type the loader dequantises
(test data). Every byte is random except the fp16 scale fields, which are set
to finite values so the blocks decode to ordinary weights."""
import numpy as np

# type id -> (elements per block, bytes per block, byte offsets of fp16 fields)
GGML_TYPES = {
    0: (1, 4, ()),            # F32
    1: (1, 2, ()),            # F16
    30: (1, 2, ()),           # BF16
    2: (32, 18, (0,)),        # Q4_0
    3: (32, 20, (0, 2)),      # Q4_1
    6: (32, 22, (0,)),        # Q5_0
    7: (32, 24, (0, 2)),      # Q5_1
    8: (32, 34, (0,)),        # Q8_0
    12: (256, 144, (0, 2)),   # Q4_K
    14: (256, 210, (208,)),   # Q6_K
}
NAMES = {0: "F32", 1: "F16", 30: "BF16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 12: "Q4_K",
         14: "Q6_K"}


def random_blocks(ggml_type, n, seed, scale=0.01):
    """Raw bytes of n elements of `ggml_type` (n a multiple of its block)."""
    be, bb, f16 = GGML_TYPES[ggml_type]
    assert n % be == 0
    rng = np.random.default_rng(seed)
    nb = n // be
    if ggml_type == 0:
        return rng.normal(0, 0.02, n).astype(np.float32).tobytes()
    if ggml_type == 1:
        return rng.normal(0, 0.02, n).astype(np.float16).tobytes()
    if ggml_type == 30:
        return (rng.normal(0, 0.02, n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    raw = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
    for off in f16:
        v = np.abs(rng.normal(0, scale, nb)).astype(np.float16) + np.float16(1e-4)
        raw[:, off:off + 2] = v.view(np.uint8).reshape(nb, 2)
    return raw.tobytes()
