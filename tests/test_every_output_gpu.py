"""Every matrix of a batch is projected and written exactly once.

The persistent forward hands each SM's slice of the batch to its warps 32
matrices at a time (the first chunk of warp w fixed, later ones claimed
through a shared counter), and the small-batch kernel takes two lanes per
matrix; a slip in either would leave some T unwritten.  Outputs here are
filled with NaN before the call (a buffer from the caching allocator may
already hold the right values from an earlier call), inputs are finite, and
the results must equal the reference kernel's at sizes on both sides of the
chunk, block and small-batch boundaries -- for the plain, counting,
dual-saving and H_res forwards."""
import pytest
import torch

import oracle
from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu

# 2^13 and 2^13 + 1: the small-batch threshold; 148 * 32 +- 1: one chunk per
# SM; 148 * 640 +- 1: one chunk per warp of every SM; 148 * 1280 + 7: a second
# round of claims; larger ragged sizes.
SIZES = [8192, 8193, 4735, 4737, 94719, 94721, 189447, (1 << 20) + 12345, (1 << 22) + 3]


def nan_like(x):
    return torch.full_like(x, float("nan"))


def same_bits(a, b):
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.fixture(scope="module")
def ref():
    if not oracle.RefCuda.available():
        pytest.skip("reference kernels not built")
    return oracle.RefCuda()


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("kind", ["normal", "mixture"])
def test_every_forward_output_written(ref, kind, n):
    s = torch.cuda.current_stream().cuda_stream
    R = make_logits(kind, n, seed=n % 977)
    Tr = nan_like(R)
    ref.birkhoff_proj_n4(R.data_ptr(), Tr.data_ptr(), 1e-6, n, s)

    T = nan_like(R)
    capi.birkhoff_proj_n4(R.data_ptr(), T.data_ptr(), 1e-6, n, s)

    Ts = nan_like(R)
    it = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    gn = torch.full((n,), float("nan"), device="cuda")
    capi.birkhoff_proj_n4_stats(R.data_ptr(), Ts.data_ptr(), 1e-6, n, it.data_ptr(), gn.data_ptr(), s)

    Td = nan_like(R)
    beta = torch.full((n, 4), float("nan"), device="cuda")
    capi.birkhoff_proj_n4_duals(R.data_ptr(), Td.data_ptr(), beta.data_ptr(), 1e-6, n, s)
    torch.cuda.synchronize()

    assert not torch.isnan(Tr).any()
    for out in (T, Ts, Td):
        assert same_bits(out, Tr)
    assert int((it < 0).sum()) == 0 and not torch.isnan(gn).any() and not torch.isnan(beta).any()


@pytest.mark.parametrize("n", [94721, (1 << 20) + 12345])
def test_every_hres_forward_output_written(n):
    """The H_res forward against the plain forward on the producer's logits."""
    g = torch.Generator(device="cuda").manual_seed(n)
    H = torch.randn(n, 24, device="cuda", generator=g)
    rms = torch.rand(n, device="cuda", generator=g) + 0.5
    a = torch.tensor([0.9], device="cuda")
    b = torch.randn(16, device="cuda", generator=g)
    h = H[:, 8:24]
    s = torch.cuda.current_stream().cuda_stream
    T = torch.full((n, 4, 4), float("nan"), device="cuda")
    capi.birkhoff_proj_n4_hres(h.data_ptr(), 24, rms.data_ptr(), a.data_ptr(), b.data_ptr(), T.data_ptr(), 1e-6, n, s)
    torch.cuda.synchronize()
    assert not torch.isnan(T).any()
