"""Known-answer cases of the promotion-table policy (the oracle restatement)."""

import numpy as np

import oracle


def _table(slots):
    return np.full((1, slots), -1, np.int32), np.zeros((1, slots), np.int32)


def test_insert_hit_and_expire():
    pages, last = _table(4)
    oracle.promotion_update(pages, last, np.array([[7, 3]]), step=0, ttl=3)
    assert pages.tolist() == [[7, 3, -1, -1]] and last.tolist()[0][:2] == [0, 0]
    oracle.promotion_update(pages, last, np.array([[3, 9]]), step=1, ttl=3)
    assert pages.tolist() == [[7, 3, 9, -1]] and last.tolist()[0][:3] == [0, 1, 1]
    # step 3: page 7 idle for 3 steps -> freed before insertion, its slot reused
    oracle.promotion_update(pages, last, np.array([[5, 3]]), step=3, ttl=3)
    assert pages.tolist() == [[5, 3, 9, -1]] and last.tolist()[0][:3] == [3, 3, 1]


def test_eviction_smallest_last_hit_then_smallest_page():
    pages = np.array([[40, 10, 30, 20]], np.int32)
    last = np.array([[5, 2, 2, 7]], np.int32)
    oracle.promotion_update(pages, last, np.array([[99]]), step=8, ttl=100)
    # slots 1 and 2 tie on last_hit 2: the smaller page id (10, slot 1) goes
    assert pages.tolist() == [[40, 99, 30, 20]] and last.tolist() == [[5, 8, 2, 7]]


def test_negative_ids_and_duplicates_ignored():
    pages, last = _table(3)
    oracle.promotion_update(pages, last, np.array([[-1, 4, 4]]), step=2, ttl=5)
    assert pages.tolist() == [[4, -1, -1]] and last.tolist()[0][0] == 2
