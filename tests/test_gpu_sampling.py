"""Nucleus (top-p) sampling on the device (gaje_cuda_sample_top_p) against
the oracle's restatement of sample_top_p_core (src/compute/sampling.rs:14-55)
with the same uniform draw r.

The device sums probabilities exactly (fixed point); the reference runs f32
running sums, whose normalising sum over 10^5 terms drifts from the exact sum
by about 2e-4 relative (measured per case by _f32_drift).
The two choices agree unless the draw (or top_p) lies within that drift of a
boundary between tokens; every disagreement must be such a near tie, checked
in float64 on the reference's own ordering (EPS below).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _f64_walk(logits, T, top_p, r):
    """float64 sorted-order view of sample_top_p_core: (probs sorted, ids, cum,
    cutoff, target)."""
    lg = logits.astype(np.float32)
    p = np.exp(((lg - lg.max()) / np.float32(T)).astype(np.float32)).astype(np.float64)
    p /= p.sum()
    order = np.argsort(-p, kind="stable")
    ps = p[order]
    cum = np.cumsum(ps)
    over = np.nonzero(cum > top_p)[0]
    cutoff = int(over[0]) + 1 if over.size else p.size
    target = r * cum[cutoff - 1]
    return ps, order, cum, cutoff, target


EPS = 1e-4  # the floor of the tolerance below


def _f32_drift(logits, T, top_p):
    """How far the reference's f32 arithmetic moves the cumulative masses from
    their exact values on this case: the normalising sum is an f32 running sum
    over the whole vocabulary (about 2e-4 relative over 151936 terms), and the
    sorted running sum adds its own rounding.  Returned with a 25 % margin and
    never below EPS."""
    lg = logits.astype(np.float32)
    p32 = np.exp(((lg - lg.max()) / np.float32(T)).astype(np.float32))
    s32 = np.cumsum(p32, dtype=np.float32)[-1]
    p64 = p32.astype(np.float64)
    q64 = p64 / p64.sum()
    order = np.argsort(-q64, kind="stable")
    c64 = np.cumsum(q64[order])
    c32 = np.cumsum((p32 / s32)[order], dtype=np.float32)
    return max(EPS, 1.25 * float(np.abs(c32.astype(np.float64) - c64).max()))


def _near_tie(logits, T, top_p, r, a, b, eps=EPS):
    """True when tokens a and b sit on either side of a decision boundary that
    the draw or top_p is within eps of (float64 of the reference's ordering)."""
    ps, order, cum, cutoff, target = _f64_walk(logits, T, top_p, r)
    pos = {int(t): i for i, t in enumerate(order)}
    ia, ib = pos[a], pos[b]
    lo, hi = min(ia, ib), max(ia, ib)
    # every cumulative boundary between the two positions is within eps of the target,
    # or top_p is within eps of the cumulative mass around the cut
    near_draw = all(abs(cum[k] - target) <= eps for k in range(lo, hi))
    near_cut = abs(cum[cutoff - 1] - top_p) <= eps or (cutoff >= 2 and abs(cum[cutoff - 2] - top_p) <= eps)
    return near_draw or near_cut


def _cases():
    rng = np.random.default_rng(11)
    V = 151936
    yield "normal", (rng.standard_normal(V) * 3).astype(np.float32)
    peaked = (rng.standard_normal(V) * 0.5).astype(np.float32)
    peaked[rng.integers(0, V, 5)] += 12.0
    yield "peaked", peaked
    yield "ties", np.round(rng.standard_normal(V) * 2).astype(np.float32)
    yield "small", np.array([1.0, 3.0, 3.0, 0.5, 3.0, -1.0, 2.0, 2.0, 3.0, 0.0], np.float32)
    yield "flat", np.zeros(4096, np.float32)


@pytest.mark.parametrize("T,top_p", [(1.0, 0.9), (0.7, 0.5), (1.3, 1.0), (0.8, 0.0)])
def test_top_p_matches_oracle(g, O, T, top_p):
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    mism = total = 0
    for name, lg in _cases():
        d = torch.from_numpy(lg).cuda()
        rs = [0.0] + list(np.random.default_rng(len(lg)).random(23)) + [0.999999]
        eps = _f32_drift(lg, T, top_p)
        for r in rs:
            r = float(np.float32(r))
            if r >= 1.0:
                continue
            g.sample_top_p(d.data_ptr(), lg.size, T, top_p, r, out.data_ptr(), out.data_ptr() + 4)
            torch.cuda.synchronize()
            tok, kept = (int(v) for v in out.cpu().numpy().view(np.uint32))
            otok, okept = O.sample_top_p(lg, T, top_p, r)
            total += 1
            if tok != otok:
                mism += 1
                assert _near_tie(lg, T, top_p, r, tok, otok, eps), (name, T, top_p, r, tok, otok, eps)
            if kept != okept:
                ps, order, cum, cutoff, target = _f64_walk(lg, T, top_p, r)
                # every kept count between the two sits at a cumulative mass within the drift of top_p
                assert all(abs(cum[k - 1] - top_p) <= eps for k in range(min(kept, okept), max(kept, okept))), (
                    name, kept, okept, eps)
    assert mism <= total // 2, (mism, total)  # near ties are the exception, not the rule


def test_top_p_deterministic_and_errors(g):
    lg = (np.random.default_rng(2).standard_normal(50000) * 2).astype(np.float32)
    d = torch.from_numpy(lg).cuda()
    out = torch.zeros(4, dtype=torch.int32, device="cuda")
    g.sample_top_p(d.data_ptr(), lg.size, 0.9, 0.8, 0.37, out.data_ptr())
    g.sample_top_p(d.data_ptr(), lg.size, 0.9, 0.8, 0.37, out.data_ptr() + 4)
    torch.cuda.synchronize()
    a, b = out.cpu().numpy()[:2]
    assert a == b
    with pytest.raises(ValueError):
        g.sample_top_p(d.data_ptr(), lg.size, 0.0, 0.8, 0.3, out.data_ptr())
    with pytest.raises(ValueError):
        g.sample_top_p(d.data_ptr(), lg.size, 1.0, 0.8, 1.0, out.data_ptr())
