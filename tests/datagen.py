"""Seeded synthetic point clouds with the shapes and distributions of the five
benchmark configurations (no public dataset is involved)."""
import math

import torch


def uniform(B, N, seed, lo=0.0, hi=1.0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(B, N, 3, generator=g, dtype=torch.float64) * (hi - lo) + lo).to(dtype)


def sphere_noise(B, N, seed, sigma=0.01, dtype=torch.float32):
    """Config 2: unit-sphere surface + isotropic Gaussian noise."""
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(B, N, 3, generator=g, dtype=torch.float64)
    v = v / v.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    return (v + sigma * torch.randn(B, N, 3, generator=g, dtype=torch.float64)).to(dtype)


def gmm(B, N, seed, k=8, dtype=torch.float32):
    """Config 3: 8-component anisotropic Gaussian mixture per cloud (means U[-1,1]^3,
    per-axis std U[0.02,0.2], weights Dirichlet(1))."""
    g = torch.Generator().manual_seed(seed)
    out = torch.empty(B, N, 3, dtype=torch.float64)
    for b in range(B):
        means = torch.rand(k, 3, generator=g, dtype=torch.float64) * 2 - 1
        std = torch.rand(k, 3, generator=g, dtype=torch.float64) * 0.18 + 0.02
        e = -torch.log(torch.rand(k, generator=g, dtype=torch.float64))   # Dirichlet(1) via Exp(1)
        w = e / e.sum()
        comp = torch.multinomial(w, N, replacement=True, generator=g)
        out[b] = means[comp] + std[comp] * torch.randn(N, 3, generator=g, dtype=torch.float64)
    return out.to(dtype)


def lidar(N, seed, boxes=200, dtype=torch.float32):
    """Config 5: 40% ground plane (x,y U[-50,50], z N(0,0.02^2)), 60% in 200
    axis-aligned boxes (centres on the plane, sizes U[0.5,4] m)."""
    g = torch.Generator().manual_seed(seed)
    n_ground = int(round(0.4 * N))
    n_box = N - n_ground
    ground = torch.empty(n_ground, 3, dtype=torch.float64)
    ground[:, :2] = torch.rand(n_ground, 2, generator=g, dtype=torch.float64) * 100 - 50
    ground[:, 2] = torch.randn(n_ground, generator=g, dtype=torch.float64) * 0.02
    centres = torch.rand(boxes, 2, generator=g, dtype=torch.float64) * 100 - 50
    sizes = torch.rand(boxes, 3, generator=g, dtype=torch.float64) * 3.5 + 0.5
    which = torch.randint(0, boxes, (n_box,), generator=g)
    u = torch.rand(n_box, 3, generator=g, dtype=torch.float64)
    pts = torch.empty(n_box, 3, dtype=torch.float64)
    pts[:, :2] = centres[which] + (u[:, :2] - 0.5) * sizes[which, :2]
    pts[:, 2] = u[:, 2] * sizes[which, 2]
    allp = torch.cat([ground, pts])
    perm = torch.randperm(N, generator=g)
    return allp[perm].unsqueeze(0).to(dtype)


def knn_config4(seed=4, dtype=torch.float32, B=8, P=8192):
    """Config 4: U[-1,1]^3, ragged lengths uniform in [4096, 8192]."""
    g = torch.Generator().manual_seed(seed)
    p1 = (torch.rand(B, P, 3, generator=g, dtype=torch.float64) * 2 - 1).to(dtype)
    p2 = (torch.rand(B, P, 3, generator=g, dtype=torch.float64) * 2 - 1).to(dtype)
    l1 = torch.randint(P // 2, P + 1, (B,), generator=g)
    l2 = torch.randint(P // 2, P + 1, (B,), generator=g)
    return p1, p2, l1, l2
