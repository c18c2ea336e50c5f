"""Tolerances shared by the CPU and GPU parity tests.

The bar for floating-point outputs is max-abs 2e-2 and mean relative 5e-3,
with fp32 accumulation; the relative error is averaged over elements whose
reference magnitude is at least 1e-2 (smaller ones are covered by max-abs).

Layer outputs that include the residual stream (out = act(residual + moe))
use ``ulp_act``: there max-abs may also reach one unit in the last place of
the activation dtype at the reference value's magnitude.  Both sides round
the same fp32 sum to bf16/f16, and at |out| >= 4 one bf16 ulp is 3.1e-2, so
any accumulation-order difference flips a final rounding by exactly one ulp.
The MoE contribution itself (residual = 0) always meets the plain bar."""
import numpy as np

MAX_ABS = 2e-2
MEAN_REL = 5e-3


def errors(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    diff = np.abs(got - ref)
    big = np.abs(ref) >= 1e-2
    rel = float((diff[big] / np.abs(ref[big])).mean()) if big.any() else 0.0
    return float(diff.max()) if diff.size else 0.0, rel


def act_ulp(ref, act):
    """One unit in the last place of `act` (f16 / bf16) at |ref|."""
    mant = {"f16": 10, "bf16": 7}[act]
    mag = np.maximum(np.abs(np.asarray(ref, np.float64)), 2.0 ** -14)
    return np.exp2(np.floor(np.log2(mag)) - mant)


def assert_close(got, ref, act=None, max_abs=MAX_ABS, mean_rel=MEAN_REL, ulp_act=None):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), "NaN pattern differs"
    m = ~np.isnan(ref)
    mx, rel = errors(got[m], ref[m])
    if ulp_act is not None:
        bound = np.maximum(max_abs, act_ulp(ref[m], ulp_act))
        over = np.abs(got[m] - ref[m]) > bound
        assert not over.any() and rel <= mean_rel, (
            f"max_abs={mx:.3e} ({int(over.sum())} above max(2e-2, 1 ulp)) mean_rel={rel:.3e}")
        return mx, rel
    assert mx <= max_abs and rel <= mean_rel, f"max_abs={mx:.3e} mean_rel={rel:.3e}"
    return mx, rel


def assert_logits_close(got, ref, act, max_abs=MAX_ABS, mean_rel=MEAN_REL, ulps=1):
    """End-to-end logits: max-abs within max(2e-2, 1 act ulp), normalized L1
    error mean|d| / mean|ref| within 5e-3, and identical top-1 token per row.

    Logits pass through a whole forward of act-dtype roundings on both
    sides, so small-magnitude logits carry percent-level relative noise that
    the per-element mean-relative bar (meant for one layer's output) would
    over-weight; the normalized L1 error measures the same 5e-3 bar on the
    vector as a whole.

    ``ulps`` widens the per-element bound to that many act ulps for deep
    models: after 16 layers each side's final fp32 logit carries the
    accumulated act-dtype roundings of the whole stack, so the single
    rounding to the act dtype can land one more ulp apart."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape
    d = np.abs(got - ref)
    bound = np.maximum(max_abs, ulps * act_ulp(ref, act))
    l1 = float(d.mean() / max(np.abs(ref).mean(), 1e-30))
    assert not (d > bound).any(), f"max_abs={d.max():.3e} normalized_l1={l1:.3e}"
    assert l1 <= mean_rel, f"normalized L1 {l1:.3e}"
    g2 = got.reshape(-1, got.shape[-1])
    r2 = ref.reshape(-1, ref.shape[-1])
    assert np.array_equal(g2.argmax(-1), r2.argmax(-1)), "top-1 token differs"
    return float(d.max()), l1
