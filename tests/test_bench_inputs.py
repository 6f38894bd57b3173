"""The benchmark's shared inputs (bench.py): both arms and every rank must
draw the same values.  x is one stream, so a prefix of rows equals the same
rows of a longer draw; W^T comes in 256-column blocks from their own
streams, so a rank's column shard equals the same columns of the whole
matrix.  CPU only."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_x_prefix_rows_are_the_same():
    b = _bench()
    full = b.synthetic_x(40, 96)
    assert full.dtype == np.float32 and full.shape == (40, 96)
    assert np.array_equal(b.synthetic_x(7, 96), full[:7])


def test_w_shards_equal_the_whole_matrix():
    b = _bench()
    K, N = 64, 1100  # not a multiple of the 256-column block
    whole = b.synthetic_wT(K, N, 0, N)
    assert whole.shape == (N, K) and whole.dtype == np.float32
    for c0, n in [(0, 550), (550, 550), (256, 300), (1000, 100), (255, 2)]:
        assert np.array_equal(b.synthetic_wT(K, N, c0, n), whole[c0:c0 + n]), (c0, n)
    assert abs(float(whole.std()) - 0.02) < 0.002


def test_output_digest_is_of_the_fp32_bytes():
    b = _bench()
    y = np.arange(12, dtype=np.float32).reshape(3, 4)
    assert b.output_digest(y) == b.output_digest(y.astype(np.float64))
    assert b.output_digest(y) != b.output_digest(y + 1)
