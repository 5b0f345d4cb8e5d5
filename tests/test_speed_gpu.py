"""The kernels against the reference's own kernels (built from its sources)
on the same device and the same inputs: N = 2^22, x ~ N(0,1) and the
training-shaped sigma mix, CUDA-event timing after warm-up.  The Newton
forward must be at least 1.5x faster and the IFT backward at least 1.5x
faster; the measured times are printed."""
import pytest
import torch

import oracle
from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu


def _ms(fn, reps=5):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


@pytest.mark.parametrize("kind", ["normal", "sigma_mix"])
def test_faster_than_reference_kernels(kind):
    if not oracle.RefCuda.available():
        pytest.skip("reference kernels not built")
    ref = oracle.RefCuda()
    n = 1 << 22
    R = make_logits(kind, n, seed=0)
    G = make_logits("normal", n, seed=1)
    T = torch.empty_like(R)
    D = torch.empty_like(R)
    s = torch.cuda.current_stream().cuda_stream
    ref_f = _ms(lambda: ref.birkhoff_proj_n4(R.data_ptr(), T.data_ptr(), 1e-6, n, s))
    ref_b = _ms(lambda: ref.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), n, s))
    our_f = _ms(lambda: capi.birkhoff_proj_n4(R.data_ptr(), T.data_ptr(), 1e-6, n, s))
    our_b = _ms(lambda: capi.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), n, s))
    print(f"\n[{kind} N=2^22] reference fwd {ref_f:.3f} ms bwd {ref_b:.3f} ms | this fwd {our_f:.3f} ms "
          f"bwd {our_b:.3f} ms | speed-up fwd {ref_f / our_f:.2f}x bwd {ref_b / our_b:.2f}x")
    assert ref_f / our_f > 1.5
    assert ref_b / our_b > 1.5
