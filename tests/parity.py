"""Code-parity helpers shared by the GPU tests: fp32 distance ties proven in float64.

The reference picks codes by the first minimum of the fp32 distance
||x||^2 - 2 x.c + ||c||^2 (quantization.py:92-96, 124-144, 206-252).  The
CUDA encoder evaluates the same formula with the dot products in a different
summation order, so two candidates whose distances agree to fp32 rounding may
swap.  A code mismatch counts as a tie only if the float64 distances of the
two candidates differ by no more than the rounding bound of the fp32 formula
(tie_bound); anything else is a failure.
"""
import numpy as np

from oracle import restate as R

F32_EPS = 2.0 ** -23


def tie_bound(x, c_a, c_b):
    """Largest fp32 rounding error of the reference's ||x||^2 - 2 x.c + ||c||^2 (quantization.py:92-96)
    for either candidate: (dim + 4) ulps of the largest term, per row."""
    dim = x.shape[-1]
    nx = np.linalg.norm(x, axis=-1)
    nc = np.maximum(np.linalg.norm(c_a, axis=-1), np.linalg.norm(c_b, axis=-1))
    return (dim + 4) * F32_EPS * (nx + nc) ** 2


def prove_ties(x, cb_got, cb_want):
    """x [n, d] float64 vectors, cb_got / cb_want [n, d] the two chosen centroids: True where the
    float64 distances of the two choices differ by no more than the fp32 rounding bound."""
    d_got = ((x - cb_got) ** 2).sum(-1)
    d_want = ((x - cb_want) ** 2).sum(-1)
    return np.abs(d_got - d_want) <= tie_bound(x, cb_got, cb_want)


def check_codes(x16, pq_cb, rvq_cb, thr, got, want, what):
    """got / want: dicts of pq [N, M], mask [N], rvq [N] (dense, L = 1), optional sp_idx / sp_val.
    Returns (pq mismatches, rvq mismatches); every mismatch must be a proven tie."""
    N, D = x16.shape
    M, _, ds = pq_cb.shape
    x = x16.astype(np.float64)
    bad_n, bad_m = np.nonzero(got["pq"] != want["pq"])
    if bad_n.size:
        sub = x.reshape(N, M, ds)[bad_n, bad_m]
        cg = pq_cb[bad_m, got["pq"][bad_n, bad_m]].astype(np.float64)
        cw = pq_cb[bad_m, want["pq"][bad_n, bad_m]].astype(np.float64)
        ok = prove_ties(sub, cg, cw)
        assert ok.all(), f"{what}: {int((~ok).sum())} PQ code mismatches are not fp32 ties"
    agree = (got["pq"] == want["pq"]).all(axis=1)
    n_rvq = 0
    if rvq_cb is not None and rvq_cb.shape[0]:
        np.testing.assert_array_equal(got["mask"][agree], want["mask"][agree], err_msg=f"{what}: RVQ gate")
        sel = agree & want["mask"]
        diff = sel & (got["rvq"] != want["rvq"])
        n_rvq = int(diff.sum())
        if n_rvq:
            _, res = R.pq_quantize(x16[diff], pq_cb)
            r = res.astype(np.float32).astype(np.float64)
            cg = rvq_cb[0, got["rvq"][diff].astype(np.int64)].astype(np.float64)
            cw = rvq_cb[0, want["rvq"][diff].astype(np.int64)].astype(np.float64)
            ok = prove_ties(r, cg, cw)
            assert ok.all(), f"{what}: {int((~ok).sum())} RVQ code mismatches are not fp32 ties"
        agree = agree & (~want["mask"] | (got["rvq"] == want["rvq"]))
    if "sp_idx" in want:
        np.testing.assert_array_equal(got["sp_idx"][agree], want["sp_idx"][agree], err_msg=f"{what}: sparse idx")
        np.testing.assert_array_equal(got["sp_val"][agree].view(np.uint16), want["sp_val"][agree].view(np.uint16),
                                      err_msg=f"{what}: sparse val")
    return bad_n.size, n_rvq


def rvq_ties_ok(residual16, rvq_cb, got, want):
    """Multi-layer RVQ: for every vector whose codes differ, the first differing layer must be a
    proven tie of the running residual (fp32, quantization.py:236-250) against the two rows."""
    bad = np.flatnonzero((got != want).any(axis=1))
    if bad.size == 0:
        return 0
    L = rvq_cb.shape[0]
    running = residual16[bad].astype(np.float32)
    pending = np.ones(bad.size, bool)
    for layer in range(L):
        g, w = got[bad, layer].astype(np.int64), want[bad, layer].astype(np.int64)
        diff = pending & (g != w)
        if diff.any():
            x = running[diff].astype(np.float64)
            ok = prove_ties(x, rvq_cb[layer, g[diff]].astype(np.float64), rvq_cb[layer, w[diff]].astype(np.float64))
            assert ok.all(), f"{int((~ok).sum())} RVQ code mismatches at layer {layer} are not fp32 ties"
            pending &= ~diff
        running = running - rvq_cb[layer].astype(np.float32)[w]
    return int(bad.size)
