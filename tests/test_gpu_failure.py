"""Dispatched failures through the session ABI, on a real bounded wait.

The test hook tf_set_wait_limit shortens the tensor-core pipeline waits to a
few hundred cycles, so the first wait of a prefill's projection expires: the
kernel records the expiry, waits for its own copies and MMAs, releases its
tensor memory and returns (no trap, no fault).  The session call then
returns TF_ERR_TIMEOUT and invalidates the session; the next call is refused
with TF_ERR_STATE until tf_session_reset, after which the same prefill gives
the same logits as before the failure (TFETResidentSession.mm:388-392, 667)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_invalidates_session_until_reset():
    from trifuse_b200 import ops
    from trifuse_b200._lib import TriFuseError, check, lib
    from trifuse_b200.model import Config, Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = Config(layers=1, vocab=512, capacity=128)
    w = synthetic_olmoe(cfg, seed=11, device="cuda")
    model = Model(cfg, w)
    del w
    sess = Session(model, max_batch=1, capacity=128, max_prefill_tokens=64)
    ids = torch.from_numpy(np.random.default_rng(4).integers(0, cfg.vocab, size=64))
    try:
        want = sess.prefill([0], [ids]).clone()
        sess.reset()
        check(lib().tf_set_wait_limit(300))
        try:
            with pytest.raises(TriFuseError, match="TIMEOUT"):
                sess.prefill([0], [ids])
        finally:
            check(lib().tf_set_wait_limit(0))
        with pytest.raises(TriFuseError, match="STATE.*invalid"):
            sess.prefill([0], [ids])
        with pytest.raises(TriFuseError, match="STATE.*invalid"):
            sess.decode(torch.tensor([1]))
        sess.reset()
        got = sess.prefill([0], [ids])
        assert torch.equal(got, want)
        assert ops.device_error() == 0
    finally:
        sess.close()
        model.close()


def test_session_check_reports_no_failure_on_a_clean_step():
    from trifuse_b200._lib import check, lib
    from trifuse_b200.model import Config, Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    import ctypes as C
    cfg = Config(layers=1, vocab=512, capacity=64)
    w = synthetic_olmoe(cfg, seed=12, device="cuda")
    model = Model(cfg, w)
    del w
    sess = Session(model, max_batch=16, capacity=64)
    try:
        sess.set_lengths([3] * 16)
        logits = torch.empty((16, cfg.vocab), dtype=torch.float32, device="cuda")
        sess.decode(torch.arange(16, device="cuda"), logits=logits)
        check(lib().tf_session_check(sess.handle, C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        assert torch.isfinite(logits).all()
    finally:
        sess.close()
        model.close()
