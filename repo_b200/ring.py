"""Closed control polygon -> ring of piecewise-Hermite cubics, with autograd
(mirrors closed_cubic_fill_segments_tilelang, manbo/ops/cubic_splatting.py:81-543)."""
from __future__ import annotations

import math

import torch

from . import _native as nat

_BASIS: dict = {}


def ring_basis(control_points_per_bezier: int, subdiv: int, device: torch.device):
    """basis [S+1, Kb], deriv_basis [S+1, Kb-1], dt [S] at linspace(0, 1, S+1)
    (cubic_splatting.py:81-134), computed with torch on the host."""
    kb, sub = int(control_points_per_bezier), int(subdiv)
    if kb < 2:
        raise ValueError(f"control_points_per_bezier must be >=2, got {kb}")
    if sub <= 0:
        raise ValueError(f"subdiv must be >0, got {sub}")
    key = (kb, sub, str(device))
    hit = _BASIS.get(key)
    if hit is not None:
        return hit
    n = kb - 1
    t = torch.linspace(0.0, 1.0, sub + 1, dtype=torch.float32)
    tc, omt = t.view(-1, 1), (1.0 - t).view(-1, 1)
    idx = torch.arange(kb, dtype=torch.float32)
    comb = torch.tensor([math.comb(n, i) for i in range(kb)], dtype=torch.float32)
    basis = comb.view(1, kb) * torch.pow(omt, (n - idx).view(1, kb)) * torch.pow(tc, idx.view(1, kb))
    didx = torch.arange(kb - 1, dtype=torch.float32)
    dcomb = torch.tensor([math.comb(n - 1, i) for i in range(kb - 1)], dtype=torch.float32)
    dbasis = (dcomb.view(1, kb - 1) * torch.pow(omt, ((n - 1) - didx).view(1, kb - 1))
              * torch.pow(tc, didx.view(1, kb - 1)))
    dt = t[1:] - t[:-1]
    out = (basis.contiguous().to(device), dbasis.contiguous().to(device), dt.contiguous().to(device))
    _BASIS[key] = out
    return out


class ClosedRingSegmentsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, control_points, subdiv):
        cp = control_points.contiguous().to(torch.float32)
        n, k = int(cp.shape[0]), int(cp.shape[1])
        basis, dbasis, dt = ring_basis((k + 2) // 2, int(subdiv), cp.device)
        out = torch.empty((n * 2 * int(subdiv), 4, 2), dtype=torch.float32, device=cp.device)
        if n > 0:
            nat.check(nat.call("cs_ring_segments_forward", nat.ptr(cp), nat.ptr(basis),
                               nat.ptr(dbasis), nat.ptr(dt), nat.ptr(out), n, k, int(subdiv),
                               nat.stream(cp.device)), "cs_ring_segments_forward")
        ctx.shape = (n, k, int(subdiv))
        return out

    @staticmethod
    def backward(ctx, grad_out):
        n, k, sub = ctx.shape
        dev = grad_out.device
        basis, dbasis, dt = ring_basis((k + 2) // 2, sub, dev)
        gcp = torch.zeros((n, k, 2), dtype=torch.float32, device=dev)
        if n > 0:
            g = grad_out.contiguous().to(torch.float32)
            nat.check(nat.call("cs_ring_segments_backward", nat.ptr(g), nat.ptr(basis),
                               nat.ptr(dbasis), nat.ptr(dt), nat.ptr(gcp), n, k, sub,
                               nat.stream(dev)), "cs_ring_segments_backward")
        return gcp, None


def closed_cubic_fill_segments(control_points: torch.Tensor, *, subdiv: int = 4,
                               threads: int = 256):
    """[N, K, 2] closed control polygons -> ([N*2*subdiv, 4, 2] cubics, [N+1] int32
    offsets with stride 2*subdiv).  Requires K >= 4 and (K-2) % 2 == 0."""
    if control_points.ndim != 3 or int(control_points.shape[-1]) != 2:
        raise ValueError(f"control_points must be [N,K,2], got {tuple(control_points.shape)}")
    if not control_points.is_cuda:
        raise ValueError("closed_cubic_fill_segments_tilelang requires CUDA tensor")
    if int(subdiv) <= 0:
        raise ValueError(f"subdiv must be >0, got {int(subdiv)}")
    n, k = int(control_points.shape[0]), int(control_points.shape[1])
    if k < 4 or ((k - 2) % 2) != 0:
        raise ValueError(
            "closed cubic fill expects control point count K that satisfies K>=4 and (K-2)%2==0, "
            f"got K={k}")
    spc = 2 * int(subdiv)
    offs = torch.arange(0, (n + 1) * spc, spc, dtype=torch.int32, device=control_points.device)
    if n <= 0:
        return torch.empty((0, 4, 2), dtype=torch.float32, device=control_points.device), offs
    segs = ClosedRingSegmentsFunction.apply(control_points, int(subdiv))
    return segs.contiguous(), offs.contiguous()
