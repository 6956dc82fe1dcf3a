"""The u8 scorer's half-precision split test, checked exhaustively on the CPU.

k_predict_u8_tiled (predict_kernels.cu) stages each bin b as the half value 1024 + b, the
threshold t as -(1024 + t), takes c = sat(bin + threshold) (a saturating half add: 1.0
exactly when b > t, else 0.0) and updates the leaf as leaf = leaf * 2 + c (a fused
multiply-add) from a start of 2^(10 - D), so after D levels the half holds 1024 + index and
its low byte is the index. numpy's float16 rounds every operation to nearest even like the
GPU's half arithmetic, so these identities can be checked for every input here.
"""
import numpy as np
import pytest

H = np.float16


def test_saturated_difference_is_the_split_bit():
    b = np.arange(256, dtype=np.float32)[:, None]
    t = np.arange(256, dtype=np.float32)[None, :]
    hb = (H(1024.0) + b.astype(H)).astype(H)       # staged bins: exact
    ht = (-(H(1024.0) + t.astype(H))).astype(H)    # staged thresholds: exact
    assert np.all(hb.astype(np.float32) == 1024 + b)
    assert np.all(ht.astype(np.float32) == -(1024 + t))
    c = np.clip((hb + ht).astype(H), H(0.0), H(1.0))
    assert np.array_equal(c.astype(np.float32), (b > t).astype(np.float32))
    # the staged bins' bit pattern is 0x64 in the high byte, the bin in the low byte
    assert np.array_equal(hb[:, 0].view(np.uint16), 0x6400 + np.arange(256, dtype=np.uint16))


@pytest.mark.parametrize("depth", range(1, 9))
def test_leaf_accumulates_exactly_and_its_low_byte_is_the_index(depth):
    n = 1 << depth
    bits = ((np.arange(n)[:, None] >> np.arange(depth - 1, -1, -1)[None, :]) & 1).astype(H)
    leaf = np.full(n, H(2.0 ** (10 - depth)), H)
    for d in range(depth):  # leaf = leaf * 2 + c, every intermediate exact in half
        leaf = (leaf * H(2.0) + bits[:, d]).astype(H)
    assert np.array_equal(leaf.astype(np.float32), 1024 + np.arange(n, dtype=np.float32))
    assert np.array_equal(leaf.view(np.uint16) & 0xFF, np.arange(n, dtype=np.uint16))
