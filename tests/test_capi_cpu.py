"""The C-ABI library loads, exports every entry point include/mhc_proj.h
declares, and rejects bad arguments before touching a device (so these run
without a GPU)."""
import os
import re

import pytest

from conftest import ROOT
from mhc_proj import capi

HEADER = os.path.join(ROOT, "include", "mhc_proj.h")


def declared_functions():
    txt = open(HEADER).read()
    return re.findall(r"^MHC_API\s+[\w\s\*]+?\b(mhc_\w+)\s*\(", txt, flags=re.M)


def test_header_declares_the_abi():
    names = declared_functions()
    assert sorted(names) == sorted(capi.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings():
    assert capi.abi_version() == 1
    assert capi.status_string(0) == "success"
    assert "invalid" in capi.status_string(capi.MHC_ERR_INVALID_VALUE)
    assert "iteration" in capi.status_string(capi.MHC_ERR_ITERS)
    assert capi.status_string(-77) == "unknown status"


FAKE = 256  # a non-null address that is never dereferenced by these calls


@pytest.mark.parametrize("fn,args", [
    (capi.birkhoff_proj_n4, (FAKE, FAKE, 1e-6, -1)),
    (capi.birkhoff_proj_n4, (0, FAKE, 1e-6, 5)),
    (capi.birkhoff_proj_n4_backward, (FAKE, 0, FAKE, 5)),
    (capi.birkhoff_proj_n4_backward, (FAKE, FAKE, FAKE, -3)),
    (capi.sinkhorn_knopp_n4, (FAKE, 0, 5, 20)),
    (capi.sinkhorn_knopp_n4_backward, (0, FAKE, FAKE, 5, 20)),
])
def test_invalid_arguments_rejected(fn, args):
    with pytest.raises(capi.MhcError) as e:
        fn(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE


def test_backward_iteration_limit():
    with pytest.raises(capi.MhcError) as e:
        capi.sinkhorn_knopp_n4_backward(FAKE, FAKE, FAKE, 5, capi.MHC_SK_BACKWARD_MAX_ITERS + 1)
    assert e.value.code == capi.MHC_ERR_ITERS


@pytest.mark.parametrize("fn,args", [
    (capi.birkhoff_proj_n4, (0, 0, 1e-6, 0)),
    (capi.birkhoff_proj_n4_backward, (0, 0, 0, 0)),
    (capi.sinkhorn_knopp_n4, (0, 0, 0, 20)),
    (capi.sinkhorn_knopp_n4_backward, (0, 0, 0, 0, 20)),
])
def test_empty_batch_is_a_no_op(fn, args):
    fn(*args)  # no launch, no error


@pytest.mark.parametrize("fn,args", [
    (capi.birkhoff_proj_n4_ex, (FAKE, -16, FAKE, capi.MHC_DTYPE_F32, 1e-6, 5)),
    (capi.birkhoff_proj_n4_ex, (FAKE, 16, FAKE, 7, 1e-6, 5)),
    (capi.birkhoff_proj_n4_ex, (0, 16, FAKE, capi.MHC_DTYPE_BF16, 1e-6, 5)),
    (capi.birkhoff_proj_n4_backward_ex, (FAKE, 16, 3, FAKE, 16, 0, FAKE, 5)),
    (capi.birkhoff_proj_n4_backward_ex, (FAKE, 16, 0, FAKE, -1, 0, FAKE, 5)),
    (capi.birkhoff_proj_n4_backward_ex, (FAKE, 16, 0, FAKE, 16, -2, FAKE, 5)),
])
def test_ex_invalid_arguments_rejected(fn, args):
    with pytest.raises(capi.MhcError) as e:
        fn(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE


@pytest.mark.parametrize("fn,args", [
    (capi.sinkhorn_knopp_n4_strided, (FAKE, 16, FAKE, capi.MHC_DTYPE_F32, -1, 20, 0)),
    (capi.sinkhorn_knopp_n4_strided, (FAKE, -16, FAKE, capi.MHC_DTYPE_F32, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_strided, (FAKE, 16, FAKE, 9, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_strided, (FAKE, 16, 0, capi.MHC_DTYPE_BF16, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_strided, (FAKE, 16, FAKE, capi.MHC_DTYPE_F16, 5, 20, 4)),
    (capi.sinkhorn_knopp_n4_backward_strided, (FAKE, 16, 5, FAKE, 16, 0, FAKE, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_backward_strided, (FAKE, 16, 0, FAKE, 16, -1, FAKE, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_backward_strided, (FAKE, -1, 0, FAKE, 16, 0, FAKE, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_backward_strided, (FAKE, 16, 0, 0, 16, 0, FAKE, 5, 20, 0)),
    (capi.sinkhorn_knopp_n4_backward_strided, (FAKE, 16, 0, FAKE, 16, 0, FAKE, 5, 20, capi.MHC_SK_HW_RECIPROCAL)),
])
def test_strided_sinkhorn_invalid_arguments_rejected(fn, args):
    with pytest.raises(capi.MhcError) as e:
        fn(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE


def test_strided_sinkhorn_backward_iteration_limit():
    with pytest.raises(capi.MhcError) as e:
        capi.sinkhorn_knopp_n4_backward_strided(FAKE, 16, 1, FAKE, 16, 1, FAKE, 5,
                                                capi.MHC_SK_BACKWARD_MAX_ITERS + 1, capi.MHC_SK_LOGITS)
    assert e.value.code == capi.MHC_ERR_ITERS


def test_strided_sinkhorn_empty_batch_is_a_no_op():
    capi.sinkhorn_knopp_n4_strided(0, 16, 0, capi.MHC_DTYPE_BF16, 0, 20, capi.MHC_SK_LOGITS)
    capi.sinkhorn_knopp_n4_backward_strided(0, 16, 1, 0, 16, 2, 0, 0, 20, capi.MHC_SK_LOGITS)


@pytest.mark.parametrize("fn,args", [
    (capi.birkhoff_proj_n4_hres, (FAKE, 24, FAKE, FAKE, FAKE, FAKE, 1e-6, -1)),
    (capi.birkhoff_proj_n4_hres, (FAKE, -24, FAKE, FAKE, FAKE, FAKE, 1e-6, 5)),
    (capi.birkhoff_proj_n4_hres, (FAKE, 24, 0, FAKE, FAKE, FAKE, 1e-6, 5)),
    (capi.birkhoff_proj_n4_hres, (FAKE, 24, FAKE, 0, FAKE, FAKE, 1e-6, 5)),
    (capi.birkhoff_proj_n4_hres, (FAKE, 24, FAKE, FAKE, 0, FAKE, 1e-6, 5)),
    (capi.birkhoff_proj_n4_hres_backward, (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, -1,
                                           FAKE, 68)),
    (capi.birkhoff_proj_n4_hres_backward, (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, -16, FAKE, FAKE, FAKE, 5,
                                           FAKE, 68)),
    (capi.birkhoff_proj_n4_hres_backward, (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, 0, FAKE, 5,
                                           FAKE, 68)),
    (capi.birkhoff_proj_n4_hres_backward, (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, 5,
                                           0, 68)),
    (capi.birkhoff_proj_n4_hres_backward, (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, 5,
                                           FAKE, -4)),
    (capi.birkhoff_proj_n4_hres_backward_workspace, (-1,)),
])
def test_hres_invalid_arguments_rejected(fn, args):
    with pytest.raises(capi.MhcError) as e:
        fn(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE


def test_hres_forward_empty_batch_is_a_no_op():
    capi.birkhoff_proj_n4_hres(0, 24, 0, 0, 0, 0, 1e-6, 0)


@pytest.mark.parametrize("args", [
    (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, -1),
    (FAKE, FAKE, FAKE, -24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, 5),
    (FAKE, FAKE, FAKE, 24, FAKE, FAKE, FAKE, 16, FAKE, 0, FAKE, 5),
    (FAKE, FAKE, 0, 24, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, 5),
])
def test_hres_noalloc_invalid_arguments_rejected(args):
    with pytest.raises(capi.MhcError) as e:
        capi.birkhoff_proj_n4_hres_backward_noalloc(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE


@pytest.mark.parametrize("fn,args", [
    (capi.birkhoff_proj_n4_duals, (FAKE, FAKE, FAKE, 1e-6, -1)),
    (capi.birkhoff_proj_n4_duals, (FAKE, FAKE, 0, 1e-6, 5)),
    (capi.birkhoff_proj_n4_backward_duals, (FAKE, FAKE, 0, FAKE, 5)),
    (capi.birkhoff_proj_n4_backward_duals, (FAKE, FAKE, FAKE, FAKE, -2)),
])
def test_duals_invalid_arguments_rejected(fn, args):
    with pytest.raises(capi.MhcError) as e:
        fn(*args)
    assert e.value.code == capi.MHC_ERR_INVALID_VALUE
