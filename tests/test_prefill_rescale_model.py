"""CPU check of the replay that the sharp-score prefill test relies on: given scores that raise
the running max of some rows of a 32-row warp by more than 2^8 at a later key tile and leave
their neighbours' max alone, the replay reports that warp (and only that one) as mixed."""
import numpy as np

from tests.test_gpu_prefill import _mixed_rescale_warps


def _case(q_rows_hot):
    # One sequence, one head, head_dim 2, 64 cached keys then 64 new tokens: key tile 0 (keys
    # 0-63) is visible to every row with score 0, key 64 (tile 1) is visible to every row.
    T, past, D = 64, 64, 2
    q = np.zeros((1, T, 1, D), np.float32)
    q[0, :q_rows_hot, 0, 0] = 10.0
    k = np.zeros((past + T, 1, D), np.float32)
    k[64, 0, 0] = 10.0  # score 100 / sqrt(2) for the hot rows: far more than 2^8 above 0
    return _mixed_rescale_warps(q, [k], [past], 1, 1, D)


def test_replay_flags_only_the_split_warp():
    assert _case(16) == 1   # rows 0-15 rescale at tile 1, rows 16-31 do not: warp 0 is mixed
    assert _case(32) == 0   # the whole warp rescales together
    assert _case(0) == 0    # nobody rescales
