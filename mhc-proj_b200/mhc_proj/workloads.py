"""Seeded synthetic logits with the distributions of the benchmark workloads,
generated on the device with torch generators:

  normal     x ~ N(0,1)                                   (Newton workload)
  sigma_mix  x ~ sigma_k N(0,1), sigma_k ~ U[0.5, 4]      (training-shaped,
             per matrix; ill-conditioned, near-permutation projections)
  mixture    50% N(0,1), 25% N(0,9), 25% N(0,1) with +6 on one entry per row
             (multi-GPU sweep)
  wide       N(0, 100)
  uniform    U(-1, 1)
"""
import torch


def make_logits(kind: str, n: int, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if kind == "normal":          # x ~ N(0,1)
        return torch.randn(n, 4, 4, device=device, generator=g)
    if kind == "sigma_mix":       # x ~ sigma_k N(0,1), sigma_k ~ U[0.5, 4] per matrix
        s = torch.rand(n, 1, 1, device=device, generator=g) * 3.5 + 0.5
        return s * torch.randn(n, 4, 4, device=device, generator=g)
    if kind == "mixture":         # 50% N(0,1), 25% N(0,9), 25% N(0,1) + 6 on one entry per row
        x = torch.randn(n, 4, 4, device=device, generator=g)
        u = torch.rand(n, device=device, generator=g)
        x = torch.where(((u >= 0.5) & (u < 0.75))[:, None, None], 3 * x, x)
        col = torch.randint(0, 4, (n, 4), device=device, generator=g)
        bump = 6 * torch.nn.functional.one_hot(col, 4).to(x.dtype)
        return torch.where((u >= 0.75)[:, None, None], x + bump, x)
    if kind == "wide":            # N(0, 100): near-permutation projections
        return 10 * torch.randn(n, 4, 4, device=device, generator=g)
    if kind == "uniform":         # U(-1, 1)
        return 2 * torch.rand(n, 4, 4, device=device, generator=g) - 1
    raise ValueError(kind)
