"""The counting forward (mhc_birkhoff_proj_n4_pass_counts): same T and
per-matrix iterations as the plain and stats forwards, and pass counts that
add up the way the reference's control flow (src/birkhoff_proj_n4.cu:400-495)
requires: every Newton iteration starts with candidate k = 0 and ends with
an accepted candidate or a Sinkhorn sweep, a candidate k+1 follows every
rejected candidate k < 4, and each busy lane slot of the state machine is
exactly one pass."""
import pytest
import torch

from mhc_proj import capi
from mhc_proj.workloads import make_logits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["normal", "sigma_mix", "mixture"])
@pytest.mark.parametrize("tol", [1e-6, 1e-3])
def test_counts_add_up(kind, tol):
    n = (1 << 18) + 13
    R = make_logits(kind, n, seed=31)
    T, it, gn, c = capi.birkhoff_proj_n4_pass_counts_tensor(R, tol)
    T0 = capi.birkhoff_proj_n4_tensor(R, tol)
    it1 = torch.empty(n, dtype=torch.int32, device="cuda")
    gn1 = torch.empty(n, device="cuda")
    T1 = torch.empty_like(R)
    capi.birkhoff_proj_n4_stats(R.data_ptr(), T1.data_ptr(), tol, n, it1.data_ptr(), gn1.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(T.view(torch.int32), T0.view(torch.int32))
    assert torch.equal(T1.view(torch.int32), T0.view(torch.int32))
    assert torch.equal(it, it1) and torch.equal(gn.view(torch.int32), gn1.view(torch.int32))

    iterations = int(it.sum())
    cand = [c[f"candidate_{k}"] for k in range(5)]
    acc = [c[f"accepted_{k}"] for k in range(5)]
    assert c["matrices"] == n and c["fill"] == 2 * n and c["start"] == n
    assert cand[0] == iterations
    for k in range(4):
        assert cand[k + 1] == cand[k] - acc[k]
    assert c["sweep_column"] == c["sweep_eval"] == cand[4] - acc[4]
    assert sum(acc) + c["sweep_eval"] == iterations
    assert c["at_cap"] == int(((it == 20) & ~(gn < tol)).sum())
    passes = c["start"] + sum(cand) + c["sweep_column"] + c["sweep_eval"]
    assert c["busy_lane_slots"] == passes
    assert c["lane_slots"] >= passes and c["lane_slots"] % 32 == 0


def test_counts_accumulate():
    R = make_logits("normal", 5000, seed=32)
    c = torch.zeros(18, dtype=torch.int64, device="cuda")
    T = torch.empty_like(R)
    it = torch.empty(5000, dtype=torch.int32, device="cuda")
    gn = torch.empty(5000, device="cuda")
    for _ in range(2):
        capi.birkhoff_proj_n4_pass_counts(R.data_ptr(), T.data_ptr(), 1e-6, 5000, it.data_ptr(), gn.data_ptr(),
                                          c.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(c[0]) == 10000 and int(c[1]) == 20000
