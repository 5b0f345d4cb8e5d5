"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's CUDA kernels, compiled unmodified from its sources into
oracle/_ref/libmhcref.so (`make -C oracle ref`), on a GPU, plus the
reference's vanilla PyTorch Sinkhorn-Knopp (README.md:37-46), and stores
inputs and outputs as .npz files:

  golden_<case>.npz   R, T_ref (birkhoff_proj_n4, tol 1e-6), G,
                      D_ref (birkhoff_proj_n4_backward on T_ref),
                      M = exp(R), T_sk_ref (sinkhorn_knopp_n4, 20 iters),
                      D_sk_ref (the reference's SK backward, 20 iters),
                      P_vanilla / dR_vanilla (vanilla SK20 fwd and autograd)
  readme_example.npz  the README's N=2 example inputs (torch.manual_seed(123),
                      CUDA RNG) with the reference's outputs

Usage (needs a GPU):  python tests/golden/make_golden.py --out tests/golden
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

N_CASE = 2048


def cases(dev):
    """(name, R, G) with seeded generators.  cfg1 uses the CPU generator
    exactly as its recipe states; the others use CPU generators too so the
    inputs are reproducible anywhere, then move to the device."""
    out = []
    torch.manual_seed(123)
    x = torch.randn(4096, 4, 4)
    G = torch.randn(4096, 4, 4)
    out.append(("cfg1_n4096_seed123", x, G))

    g = torch.Generator().manual_seed(0)
    out.append(("cfg2_normal", torch.randn(N_CASE, 4, 4, generator=g), torch.randn(N_CASE, 4, 4, generator=g)))

    g = torch.Generator().manual_seed(3)
    s = torch.rand(N_CASE, 1, 1, generator=g) * 3.5 + 0.5
    out.append(("cfg3_sigma_mix", s * torch.randn(N_CASE, 4, 4, generator=g), torch.randn(N_CASE, 4, 4, generator=g)))

    g = torch.Generator().manual_seed(5)
    x = torch.randn(N_CASE, 4, 4, generator=g)
    u = torch.rand(N_CASE, generator=g)
    x = torch.where(((u >= 0.5) & (u < 0.75))[:, None, None], 3 * x, x)
    col = torch.randint(0, 4, (N_CASE, 4), generator=g)
    x = torch.where((u >= 0.75)[:, None, None], x + 6 * torch.nn.functional.one_hot(col, 4).float(), x)
    out.append(("cfg5_mixture", x, torch.randn(N_CASE, 4, 4, generator=g)))

    g = torch.Generator().manual_seed(10)
    out.append(("wide_normal_sigma10", 10 * torch.randn(N_CASE, 4, 4, generator=g), torch.randn(N_CASE, 4, 4, generator=g)))
    return out


def run_ref(ref, R, G):
    N = R.shape[0]
    T = torch.empty_like(R)
    D = torch.empty_like(R)
    ref.birkhoff_proj_n4(R.data_ptr(), T.data_ptr(), 1e-6, N, 0)
    ref.birkhoff_proj_n4_backward(G.data_ptr(), T.data_ptr(), D.data_ptr(), N, 0)
    M = torch.exp(R)
    Tsk = torch.empty_like(R)
    Dsk = torch.empty_like(R)
    ref.sinkhorn_knopp_n4(M.data_ptr(), Tsk.data_ptr(), N, 20, 0)
    ref.sinkhorn_knopp_n4_backward(G.data_ptr(), M.data_ptr(), Dsk.data_ptr(), N, 20, 0)
    torch.cuda.synchronize()
    return T, D, M, Tsk, Dsk


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    dev = torch.device("cuda:0")
    ref = oracle.RefCuda()
    for name, x, G in cases(dev):
        R = x.to(dev).contiguous()
        Gd = G.to(dev).contiguous()
        T, D, M, Tsk, Dsk = run_ref(ref, R, Gd)
        P, dR = oracle.vanilla_sinkhorn(R, Gd)
        np.savez_compressed(
            os.path.join(a.out, f"golden_{name}.npz"),
            R=R.cpu().numpy(), G=Gd.cpu().numpy(), T_ref=T.cpu().numpy(), D_ref=D.cpu().numpy(),
            M=M.cpu().numpy(), T_sk_ref=Tsk.cpu().numpy(), D_sk_ref=Dsk.cpu().numpy(),
            P_vanilla_gpu=P.cpu().numpy(), dR_vanilla_gpu=dR.cpu().numpy())
        print("wrote", name, flush=True)

    # README.md:27-133: torch.manual_seed(123); x, G = randn(2,4,4) on CUDA
    torch.manual_seed(123)
    x = torch.randn(2, 4, 4, device=dev)
    G = torch.randn(2, 4, 4, device=dev)
    T, D, M, Tsk, Dsk = run_ref(ref, x.contiguous(), G.contiguous())
    P, dR = oracle.vanilla_sinkhorn(x, G)
    np.savez_compressed(os.path.join(a.out, "readme_example.npz"), R=x.cpu().numpy(), G=G.cpu().numpy(),
                        T_ref=T.cpu().numpy(), D_ref=D.cpu().numpy(), P_vanilla_gpu=P.cpu().numpy(),
                        dR_vanilla_gpu=dR.cpu().numpy())
    print("wrote readme_example", flush=True)


if __name__ == "__main__":
    main()
