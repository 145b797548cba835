"""CPU checks of the block top-k oracle's stated rules."""
import math

import numpy as np

from oracle import blocktopk as bt
from oracle import sage
from oracle.numerics import round_bf16


def test_select_ties_and_order():
    s = np.array([[1.0, 3.0, 3.0, 0.5, 3.0]], dtype=np.float32)
    assert bt.select(s, 2).tolist() == [[1, 2]]        # equal scores: lower index first
    assert bt.select(s, 4).tolist() == [[0, 1, 2, 4]]  # reported ascending
    assert bt.select(s, 9).shape == (1, 5)


def test_pool_ragged_block_and_exactness():
    x = round_bf16(np.random.default_rng(0).standard_normal((300, 128)).astype(np.float32))
    p = bt.pool_blocks(x)
    assert p.shape == (3, 128)
    np.testing.assert_array_equal(p[2], (x[256:].astype(np.float64).sum(0) / 44).astype(np.float32))


def test_keep_all_blocks_equals_dense_attention():
    rng = np.random.default_rng(1)
    q, k, v = (round_bf16(rng.standard_normal((1, 2, 300, 128)).astype(np.float32)) for _ in range(3))
    o, idx = bt.blocksparse_attention(q, k, v, keep=3)
    assert (idx == np.arange(3)).all()
    np.testing.assert_allclose(o, sage.sdpa_reference(q, k, v), rtol=1e-5, atol=1e-6)


def test_hot_blocks_are_found():
    q, k, v = bt.make_hot_inputs(1, 1, 1024, 128, hot=2, boost=4.0, seed=3)
    idx = bt.select_head(q[0, 0], k[0, 0], keep=2)
    assert idx.shape == (8, 2)
