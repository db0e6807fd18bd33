"""The oracle's kv_cache_rotate restatement (kv_cache.metal:200-236) on the
CPU: positions below the new length take the rows `shift` further on, the
rest stay, and a shift beyond the length is refused."""
import numpy as np
import pytest

from oracle import oracle as O


def test_kv_rotate_rows_semantics():
    rng = np.random.default_rng(5)
    rows = rng.integers(0, 1 << 16, size=(50, 2, 8), dtype=np.uint16)
    for shift in (0, 1, 16, 33, 40):
        out, new_len = O.kv_rotate_rows(rows, 40, shift)
        assert new_len == 40 - shift
        assert np.array_equal(out[:new_len], rows[shift:40])
        assert np.array_equal(out[new_len:], rows[new_len:])  # untouched past the new length
    with pytest.raises(ValueError):
        O.kv_rotate_rows(rows, 40, 41)
