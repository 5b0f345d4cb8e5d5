"""The fused H_res producer + projection on the host side: the oracle's
float64 chain rule against autograd, and the argument checks of the binding
and the module (which raise before any device work)."""
import numpy as np
import pytest
import torch

import mhc_proj
import oracle


def _inputs(n, seed):
    g = np.random.default_rng(seed)
    h = g.standard_normal((n, 16)).astype(np.float32)
    rms = g.uniform(0.5, 2.0, n).astype(np.float32)
    b = g.standard_normal(16).astype(np.float32)
    D = g.standard_normal((n, 4, 4)).astype(np.float32)
    return h, rms, b, D


def test_logits_formula():
    h, rms, b, _ = _inputs(64, 1)
    R = oracle.hres_logits(h, rms, 0.7, b)
    want = (0.7 * h.astype(np.float64) / rms.astype(np.float64)[:, None] + b.astype(np.float64)).reshape(-1, 4, 4)
    np.testing.assert_allclose(R, want, rtol=0, atol=1e-15)


def test_backward_chain_matches_autograd():
    h, rms, b, D = _inputs(257, 2)
    ht = torch.tensor(h, dtype=torch.float64, requires_grad=True)
    rt = torch.tensor(rms, dtype=torch.float64, requires_grad=True)
    at = torch.tensor(1.3, dtype=torch.float64, requires_grad=True)
    bt = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    R = at * ht / rt[:, None] + bt
    (R * torch.tensor(D, dtype=torch.float64).reshape(-1, 16)).sum().backward()
    dh, drms, dalpha, db = oracle.hres_backward_chain(D, h, rms, 1.3)
    np.testing.assert_allclose(dh, ht.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(drms, rt.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dalpha, at.grad.item(), rtol=1e-12)
    np.testing.assert_allclose(db, bt.grad.numpy().reshape(4, 4), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("h,rms,b,msg", [
    (torch.zeros(3, 15), torch.zeros(3), torch.zeros(16), "h_res must be"),
    (torch.zeros(3, 4, 5), torch.zeros(3), torch.zeros(16), "h_res must be"),
    (torch.zeros(3, 16), torch.zeros(4), torch.zeros(16), "rms must have"),
    (torch.zeros(3, 16), torch.zeros(3), torch.zeros(15), "b_res must have"),
])
def test_binding_rejects_bad_shapes(h, rms, b, msg):
    with pytest.raises(RuntimeError, match=msg):
        mhc_proj.torch.birkhoff_proj_n4_hres(h, rms, 1.0, b)


def test_binding_rejects_multi_element_alpha():
    with pytest.raises(RuntimeError, match="alpha_res"):
        mhc_proj.torch.birkhoff_proj_n4_hres(torch.zeros(2, 16), torch.ones(2), torch.ones(2), torch.zeros(16))


def test_backward_binding_rejects_bad_shapes():
    with pytest.raises(RuntimeError, match="G must be"):
        mhc_proj.torch.birkhoff_proj_n4_hres_backward(torch.zeros(2, 16), torch.zeros(2, 4, 4), torch.zeros(2, 16),
                                                      torch.ones(2), 1.0)
    with pytest.raises(RuntimeError, match="batch size"):
        mhc_proj.torch.birkhoff_proj_n4_hres_backward(torch.zeros(2, 4, 4), torch.zeros(2, 4, 4),
                                                      torch.zeros(3, 16), torch.ones(3), 1.0)


def test_module_rejects_bad_shapes():
    m = mhc_proj.MHCProjectionN4HRes()
    with pytest.raises(ValueError, match="h_res"):
        m(torch.zeros(3, 15), torch.zeros(3), 1.0, torch.zeros(16))
    with pytest.raises(ValueError, match="rms"):
        m(torch.zeros(2, 3, 16), torch.zeros(6), 1.0, torch.zeros(16))
