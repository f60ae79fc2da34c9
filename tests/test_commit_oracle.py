"""CPU: the commit-step oracle against the reference's own cache compaction (golden fixture made by running
inference/hf/ddtree.py _compact_appended_window / compact_dynamic_cache)."""
import numpy as np

from oracle import oracle
from tests._golden import load


def test_compact_tail_oracle_matches_reference():
    f = load("compact_cache.npz")
    i = 0
    while f"c{i}_in" in f:
        out = oracle.compact_tail(f[f"c{i}_in"], int(f[f"c{i}_past"]), f[f"c{i}_keep"])
        assert np.array_equal(out, f[f"c{i}_out"]), i
        i += 1
    assert i == 5
    past, keep, n = int(f["dyn_past"]), f["dyn_keep"], int(f["dyn_len"])
    for layer in range(2):
        for kv in "kv":
            out = oracle.compact_tail(f[f"dyn_{kv}{layer}_in"], past, keep)[..., :n, :]
            assert np.array_equal(out, f[f"dyn_{kv}{layer}_out"])


def test_commit_kv_moves_oracle_reads_sources_first():
    pool = np.arange(2 * 10 * 3).reshape(2, 10, 3)
    src = np.array([[4, 5, 6, 0]])  # slot 5 is both a target (of 4) and a source (for 6 -> ... )
    tgt = np.array([[5, 6, 7, 0]])
    out = oracle.commit_kv_moves(pool, src, tgt)
    assert np.array_equal(out[:, 5], pool[:, 4]) and np.array_equal(out[:, 6], pool[:, 5])
    assert np.array_equal(out[:, 7], pool[:, 6]) and np.array_equal(out[:, 0], pool[:, 0])
