"""The Python surface mirrors the reference package (mhc_proj/__init__.py,
mhc_proj/module.py, src/bindings.cpp): names, defaults, error types."""
import inspect

import pytest
import torch

import mhc_proj
from mhc_proj import sharding


def test_public_names():
    assert hasattr(mhc_proj, "MHCProjectionN4") and hasattr(mhc_proj, "MHCSinkhornN4")
    for f in ("birkhoff_proj_n4", "birkhoff_proj_n4_backward", "sinkhorn_knopp_n4", "sinkhorn_knopp_n4_backward",
              "sinkhorn_knopp_n4_logits", "sinkhorn_knopp_n4_logits_backward"):
        assert callable(getattr(mhc_proj.torch, f))


def test_binding_signatures_and_defaults():
    doc = mhc_proj.torch.birkhoff_proj_n4.__doc__
    assert "R: torch.Tensor" in doc and "tol" in doc and "1e-06" in doc and "**kwargs" in doc
    doc = mhc_proj.torch.birkhoff_proj_n4_backward.__doc__
    assert "G: torch.Tensor" in doc and "T: torch.Tensor" in doc
    doc = mhc_proj.torch.sinkhorn_knopp_n4.__doc__
    assert "M: torch.Tensor" in doc and "max_iter" in doc and "= 20" in doc
    doc = mhc_proj.torch.sinkhorn_knopp_n4_backward.__doc__
    assert "G: torch.Tensor" in doc and "M: torch.Tensor" in doc and "= 20" in doc


def test_module_defaults():
    assert mhc_proj.MHCProjectionN4().tol == 1e-6
    assert mhc_proj.MHCSinkhornN4().max_iter == 20
    assert inspect.signature(mhc_proj.MHCProjectionN4).parameters["tol"].default == 1e-6


@pytest.mark.parametrize("shape", [(3,), (2, 4, 3), (2, 3, 4), (4, 5)])
def test_module_rejects_non_4x4(shape):
    with pytest.raises(ValueError):
        mhc_proj.MHCProjectionN4()(torch.zeros(shape))
    with pytest.raises(ValueError):
        mhc_proj.MHCSinkhornN4()(torch.zeros(shape))


@pytest.mark.parametrize("shape", [(4, 4), (2, 2, 4, 4), (2, 4, 3), (2, 3, 4)])
def test_low_level_rejects_non_batch(shape):
    x = torch.zeros(shape)
    with pytest.raises(RuntimeError):
        mhc_proj.torch.birkhoff_proj_n4(x, 1e-6)
    with pytest.raises(RuntimeError):
        mhc_proj.torch.sinkhorn_knopp_n4(x)
    ok = torch.zeros(2, 4, 4)
    with pytest.raises(RuntimeError):
        mhc_proj.torch.birkhoff_proj_n4_backward(ok, x)
    with pytest.raises(RuntimeError):
        mhc_proj.torch.sinkhorn_knopp_n4_backward(x, ok)


def test_fused_logits_signatures():
    doc = mhc_proj.torch.sinkhorn_knopp_n4_logits.__doc__
    assert "R: torch.Tensor" in doc and "= 20" in doc
    doc = mhc_proj.torch.sinkhorn_knopp_n4_logits_backward.__doc__
    assert "G: torch.Tensor" in doc and "R: torch.Tensor" in doc
    with pytest.raises(RuntimeError):
        mhc_proj.torch.sinkhorn_knopp_n4_logits(torch.zeros(2, 4, 3))


def test_backward_batch_mismatch():
    with pytest.raises(RuntimeError):
        mhc_proj.torch.birkhoff_proj_n4_backward(torch.zeros(2, 4, 4), torch.zeros(3, 4, 4))


def test_shard_ranges_cover_the_batch():
    for n in (0, 1, 7, 1000, 2 ** 26):
        for world in (1, 2, 3, 4, 8):
            rs = [sharding.shard_range(n, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sz = sharding.shard_sizes(n, world)
            assert max(sz) - min(sz) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(10, 2, 2)
