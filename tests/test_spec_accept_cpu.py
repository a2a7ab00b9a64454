"""The greedy speculative acceptance rule of the runner (solort_b200/runner.py, accept_drafts),
the rule of the reference's SpecCudaGraphQwen3Executor._spec_round
(src/solort/model/cuda_graph_executor.py:476-481): drafts are kept while they equal the target's
argmax, and the target's token after the last kept draft closes the round."""

from __future__ import annotations

import pytest

from solort_b200.runner import accept_drafts


def test_every_draft_accepted_adds_the_bonus_token():
    assert accept_drafts([5, 6, 7, 8], [5, 6, 7, 8, 9]) == [5, 6, 7, 8, 9]


def test_first_draft_rejected_gives_the_target_token_only():
    assert accept_drafts([5, 6, 7, 8], [1, 6, 7, 8, 9]) == [1]


def test_partial_prefix_stops_at_the_first_mismatch():
    # a later agreement (index 3) does not count once index 2 disagrees
    assert accept_drafts([5, 6, 7, 8], [5, 6, 2, 8, 9]) == [5, 6, 2]


def test_single_draft():
    assert accept_drafts([4], [4, 3]) == [4, 3]
    assert accept_drafts([4], [2, 3]) == [2]


def test_target_row_count_must_be_drafts_plus_one():
    with pytest.raises(ValueError):
        accept_drafts([1, 2], [1, 2])
