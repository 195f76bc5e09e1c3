"""CPU: the gap vector behind AKVLayer's hot-tier order vectors behaves like
a plain list under removals anywhere and appends."""
import numpy as np


def test_gapvec_matches_list():
    from akv.drop_in import _GapVec
    rng = np.random.default_rng(0)
    ref = list(range(100))
    g = _GapVec(np.array(ref), np.int64)
    nxt = 100
    for step in range(3000):
        if ref and rng.random() < 0.5:
            i = int(rng.integers(0, len(ref))) if rng.random() < 0.5 else int(rng.integers(0, min(6, len(ref))))
            ref.pop(i)
            g.remove(i)
        else:
            ref.append(nxt)
            g.append(nxt)
            nxt += 1
        assert len(g) == len(ref)
        if step % 97 == 0:
            np.testing.assert_array_equal(g.view(), np.array(ref, dtype=np.int64))
    np.testing.assert_array_equal(g.view(), np.array(ref, dtype=np.int64))
