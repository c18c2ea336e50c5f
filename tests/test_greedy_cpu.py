"""Greedy next-token selection: the oracle's restatement of the reference's
where(all(isfinite(logits)), argmax(logits), -1) and the C ABI's argument
checks (no GPU needed)."""
import ctypes as C

import numpy as np

import oracle


def test_oracle_greedy_semantics():
    lg = np.zeros((5, 7), np.float32)
    lg[0, 3] = 2.0
    lg[1, [2, 5]] = 4.0                 # tie: the lower index wins
    lg[2, 1] = np.nan                   # any non-finite logit -> -1
    lg[3, 6] = np.inf
    lg[4, :] = -3.0
    lg[4, 0] = -np.inf
    assert oracle.greedy_token(lg).tolist() == [3, 2, -1, -1, -1]
    assert oracle.greedy_token(lg[0]).item() == 3


def test_greedy_abi_argument_checks():
    from trifuse_b200._lib import lib
    L = lib()
    assert L.tf_greedy_tokens(None, 0, 10, None, None) == 0        # nothing to do
    assert L.tf_greedy_tokens(None, 2, 10, None, None) == 1        # TF_ERR_INVALID_ARGUMENT
    assert L.tf_greedy_tokens(None, 2, 0, None, None) == 2         # TF_ERR_SHAPE
    out = (C.c_int64 * 1)()
    assert L.tf_session_decode_greedy(None, None, None, 1, out, None, 0, None) == 1
    assert L.tf_session_decode_greedy(None, None, None, 1, None, None, 0, None) == 1
