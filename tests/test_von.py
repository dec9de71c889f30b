"""Independent-options layout rules (`independent_options_tensors`,
src/engine.rs:531-590) restated in oracle/von.py, on hand-worked rows."""

import numpy as np
import pytest

from oracle.von import von_allowed, von_layout


def test_positions_restart_inside_each_option_and_the_last_token_stays_shared():
    # [CLS] a b [SEP] [M] x [M] y z [SEP]   real_len 10, markers at 4 and 6
    pos, opt = von_layout(10, [4, 6], 12)
    assert opt.tolist() == [-1, -1, -1, -1, 0, 0, 1, 1, 1, -1, -1, -1]
    assert pos.tolist() == [0, 1, 2, 3, 4, 5, 4, 5, 6, 9, 10, 11]


def test_full_mask_isolates_options_and_keeps_shared_tokens():
    pos, opt = von_layout(10, [4, 6], 12)
    allowed = von_allowed(10, pos, opt, None)
    # shared tokens see shared tokens (incl. the final [SEP]) only
    assert allowed[0].tolist() == [True] * 4 + [False] * 5 + [True] + [False] * 2
    # an option token sees the shared tokens and its own option
    assert allowed[5].tolist() == [True] * 4 + [True, True] + [False] * 3 + [True] + [False] * 2
    assert allowed[7].tolist() == [True] * 4 + [False, False] + [True] * 3 + [True] + [False] * 2
    # padded queries attend only to themselves
    assert allowed[11].tolist() == [True] * 4 + [False] * 5 + [True] + [False, True]


def test_sliding_mask_uses_option_invariant_distance():
    pos, opt = von_layout(10, [4, 6], 12)
    allowed = von_allowed(10, pos, opt, 1)
    # token 6 (position 4, option 1) reaches positions 3..5: token 3 (shared) and token 7
    assert np.flatnonzero(allowed[6]).tolist() == [3, 6, 7]
    # token 4 (position 4, option 0) reaches token 3 and token 5
    assert np.flatnonzero(allowed[4]).tolist() == [3, 4, 5]


def test_rows_without_markers_inside_the_row_are_refused():
    with pytest.raises(ValueError, match="no marker"):
        von_layout(5, [], 5)
    with pytest.raises(ValueError, match="no marker"):
        von_layout(5, [5], 6)
