"""bench.py's exactness check (count_mismatches), the rule behind every
`check.mismatches` in the bench line, on crafted cases (CPU)."""
import numpy as np
import torch

import bench


def _exact(n=40, k=10, extra=8, seed=0):
    rng = np.random.default_rng(seed)
    scores = np.sort(rng.random(n))[::-1].astype(np.float64)
    ids = rng.permutation(n).astype(np.int64)
    return scores, ids, torch.tensor(scores[:k + extra])[None], torch.tensor(ids[:k + extra])[None]


def _count(got_s, got_i, ex_s, ex_i, k=10):
    return bench.count_mismatches(torch.tensor(got_s, dtype=torch.float32)[None],
                                  torch.tensor(got_i, dtype=torch.int32)[None], ex_s, ex_i, k)


def test_exact_answer_passes():
    s, i, ex_s, ex_i = _exact()
    assert _count(s[:10], i[:10], ex_s, ex_i) == 0


def test_tie_at_the_kth_may_swap():
    s, i, ex_s, ex_i = _exact()
    s = s.copy()
    s[10] = s[9]  # rows 9 and 10 tied at the k-th score
    ex_s = torch.tensor(s[:18])[None]
    got_i = i[:10].copy()
    got_i[9] = i[10]
    assert _count(s[:10], got_i, ex_s, ex_i) == 0


def test_wrong_id_with_a_plausible_score_is_caught():
    s, i, ex_s, ex_i = _exact(n=60)
    got_i = i[:10].copy()
    got_i[9] = i[50]  # far below the k-th, outside the exact top-18, reported with the k-th's score
    assert _count(s[:10], got_i, ex_s, ex_i) == 1


def test_wrong_score_unsorted_and_duplicates_are_caught():
    s, i, ex_s, ex_i = _exact()
    bad_s = s[:10].copy()
    bad_s[3] *= 1.0 + 1e-4  # 1e-4 relative error
    assert _count(bad_s, i[:10], ex_s, ex_i) == 1
    assert _count(s[:10][::-1].copy(), i[:10][::-1].copy(), ex_s, ex_i) == 1
    dup = i[:10].copy()
    dup[9] = dup[8]
    assert _count(s[:10], dup, ex_s, ex_i) == 1


def test_missing_clear_winner_is_caught():
    s, i, ex_s, ex_i = _exact()
    got_i = i[1:11].copy()  # the best row left out
    assert _count(s[1:11], got_i, ex_s, ex_i) == 1
