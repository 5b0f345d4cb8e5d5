"""The algebra of the Sinkhorn-Knopp backward kernel, checked on the CPU.

The kernel (mhc-proj_b200/csrc/sinkhorn_n4.cuh, "the backward in potential
form") does not differentiate the row/column steps one by one: it writes the
forward after k iterations as diag(u_k) M diag(v_k), with u_k = 1/(M v_{k-1})
and v_k = 1/(M^T u_k), takes the eps masks of the first iteration for every
iteration, and forms the vector-Jacobian product from M and the potentials.
Here that algorithm is restated in float32 numpy and compared with the
oracle's step-by-step exact VJP (oracle/birkhoff_oracle.c, the reference's
row/column form of sinkhorn_knopp.cuh:851-906 differentiated exactly) on
ordinary inputs and on inputs whose rows or columns fall to eps or below.
"""
import numpy as np
import pytest

import oracle

EPS = np.float32(1e-8)


def potential_vjp(M, G, iters):
    """dL/dM of L = sum(G * SK_iters(M)) by the kernel's potential form."""
    f32 = np.float32
    n = M.shape[0]
    one = np.ones((n, 4), f32)
    with np.errstate(divide="ignore"):
        s = np.einsum("nij,nj->ni", M, one).astype(f32)
        mr = s > EPS
        u = np.where(mr, f32(1) / np.where(mr, s, f32(1)), f32(0)).astype(f32)
        t = np.einsum("nij,ni->nj", M, u).astype(f32)
        mc = t > EPS
        v = np.where(mc, f32(1) / np.where(mc, t, f32(1)), f32(0)).astype(f32)
        us, vs = [u], [one, v]
        for _ in range(1, iters):
            s = np.einsum("nij,nj->ni", M, v).astype(f32)
            u = np.where(mr, f32(1) / np.where(mr, s, f32(1)), f32(0)).astype(f32)
            t = np.einsum("nij,ni->nj", M, u).astype(f32)
            v = np.where(mc, f32(1) / np.where(mc, t, f32(1)), f32(0)).astype(f32)
            us.append(u)
            vs.append(v)
    H = (G * M).astype(f32)
    du = np.einsum("nij,nj->ni", H, v).astype(f32)
    dv = np.einsum("nij,ni->nj", H, u).astype(f32)
    dM = (G * u[:, :, None] * v[:, None, :]).astype(f32)
    for k in reversed(range(iters)):
        u, v, vp = us[k], vs[k + 1], vs[k]
        dt = (-dv * v * v).astype(f32)
        du = (du + np.einsum("nij,nj->ni", M, dt)).astype(f32)
        dM = (dM + u[:, :, None] * dt[:, None, :]).astype(f32)
        ds = (-du * u * u).astype(f32)
        dv = np.einsum("nij,ni->nj", M, ds).astype(f32)
        dM = (dM + ds[:, :, None] * vp[:, None, :]).astype(f32)
        du = np.zeros_like(du)
    return dM


def masked_inputs(n, seed):
    """N(0,1) logits with, by matrix index mod 8: a row of -40 (its sum below
    eps), a column of -40 (below eps after the row step), both, a row of -19.5
    (just above eps), a column of -21, two rows of -40, or nothing."""
    rng = np.random.default_rng(seed)
    R = rng.standard_normal((n, 4, 4)).astype(np.float32)
    for m in range(n):
        i, j, c = m % 4, (m // 4) % 4, m % 8
        if c in (1, 3):
            R[m, i, :] = -40.0
        if c in (2, 3):
            R[m, :, j] = -40.0
        if c == 4:
            R[m, i, :] = -19.5
        if c == 5:
            R[m, :, j] = -21.0
        if c == 6:
            R[m, i, :] = -40.0
            R[m, (i + 1) % 4, :] = -40.0
    G = rng.standard_normal((n, 4, 4)).astype(np.float32)
    return np.exp(R).astype(np.float32), G


@pytest.mark.parametrize("iters", [1, 2, 5, 20])
@pytest.mark.parametrize("kind", ["normal", "masked"])
def test_potential_form_is_the_exact_vjp(kind, iters):
    n = 2048
    if kind == "normal":
        rng = np.random.default_rng(iters)
        M = np.exp(rng.standard_normal((n, 4, 4))).astype(np.float32)
        G = rng.standard_normal((n, 4, 4)).astype(np.float32)
    else:
        M, G = masked_inputs(n, 30 + iters)
    D = potential_vjp(M, G, iters)
    Do = oracle.sinkhorn_knopp_n4_backward(G, M, iters, 1e-8, exact=True)
    # the same zeros (rows with a zero factor get no gradient in either form)
    assert np.array_equal(D == 0, Do == 0)
    # dR = dM * M within 2e-6; dM itself where M is not tiny
    assert (np.abs(D * M - Do * M) <= 2e-6).all()
    big = M > 1e-6
    assert (np.abs(D - Do)[big] <= 2e-6 * np.maximum(1.0, np.abs(Do[big]))).all()
