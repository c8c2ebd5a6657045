"""Seeded synthetic scenes for the benchmark configurations.

The reference's paper datasets (DIV2K, Kodak) are not used; these generators
stand in for them with the shapes, sizes and value distributions of the five
benchmark configurations.  Every tensor is drawn from a CPU ``torch.Generator``
so that the CUDA path, the CPU oracle and the TileLang reference all see the
same bits.

Closed fill paths are stored as rings of ``3*G`` pixel-space points: segment
``k`` of a path is the cubic ``(r[3k], r[3k+1], r[3k+2], r[3k+3 mod 3G])``, so
consecutive segments share endpoints.  The renderer consumes normalised
cubics ``n = p / (W/2) - 1`` (the inverse of the projection in
``manbo/ops/cubic_splatting.py:588-595``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F


@dataclass
class FillScene:
    """A closed-fill optimisation problem (configs 1, 2, 3 and 5)."""

    height: int
    width: int
    samples: int                 # S, polyline samples per cubic segment
    ring: torch.Tensor           # [P, 3G, 2] float32 pixel-space ring points
    colors: torch.Tensor         # [P, 3]
    opacities: torch.Tensor      # [P]
    depths: torch.Tensor         # [P]
    aa_widths: torch.Tensor      # [P]
    fill_rules: torch.Tensor     # [P] int32 (0 even-odd, else nonzero)
    background: torch.Tensor     # [3]
    target: torch.Tensor         # [1, 3, H, W]
    segs_per_path: int
    meta: dict = field(default_factory=dict)

    @property
    def num_paths(self) -> int:
        return int(self.ring.shape[0])

    def seg_offsets(self) -> torch.Tensor:
        g = self.segs_per_path
        return torch.arange(0, (self.num_paths + 1) * g, g, dtype=torch.int32)

    def cubics_px(self) -> torch.Tensor:
        return ring_to_cubics(self.ring)

    def cubics_norm(self) -> torch.Tensor:
        return px_to_norm(self.cubics_px(), self.width, self.height)


@dataclass
class StrokeScene:
    """An open-stroke optimisation problem (config 4)."""

    height: int
    width: int
    samples: int
    cubics_px: torch.Tensor      # [P, 4, 2] one cubic per primitive
    colors: torch.Tensor
    opacities: torch.Tensor
    stroke_widths: torch.Tensor
    depths: torch.Tensor
    aa_widths: torch.Tensor
    background: torch.Tensor
    target: torch.Tensor
    meta: dict = field(default_factory=dict)

    @property
    def num_paths(self) -> int:
        return int(self.cubics_px.shape[0])

    def seg_offsets(self) -> torch.Tensor:
        return torch.arange(0, self.num_paths + 1, dtype=torch.int32)

    def cubics_norm(self) -> torch.Tensor:
        return px_to_norm(self.cubics_px, self.width, self.height)


# --------------------------------------------------------------------------
# geometry helpers


def ring_to_cubics(ring: torch.Tensor) -> torch.Tensor:
    """[P, 3G, 2] ring points -> [P*G, 4, 2] cubic control points."""
    p, n, _ = ring.shape
    g = n // 3
    k = torch.arange(g)
    idx = torch.stack([3 * k, 3 * k + 1, 3 * k + 2, (3 * k + 3) % n], dim=1)  # [G,4]
    return ring[:, idx.reshape(-1), :].reshape(p * g, 4, 2).contiguous()


def ring_gather_index(segs_per_path: int) -> torch.Tensor:
    """Index [G*4] into a ring of 3G points, in cubic control-point order."""
    n = 3 * segs_per_path
    k = torch.arange(segs_per_path)
    return torch.stack([3 * k, 3 * k + 1, 3 * k + 2, (3 * k + 3) % n], 1).reshape(-1)


def px_to_norm(p: torch.Tensor, width: int, height: int) -> torch.Tensor:
    half = torch.tensor([0.5 * float(width), 0.5 * float(height)], dtype=p.dtype, device=p.device)
    return (p / half - 1.0).contiguous()


def circle_rings(centres: torch.Tensor, radii: torch.Tensor, phases: torch.Tensor,
                 segs: int) -> torch.Tensor:
    """Closed circles as rings of ``segs`` cubic arcs: [P, 3*segs, 2]."""
    kappa = 4.0 / 3.0 * math.tan(math.pi / (2.0 * segs))
    k = torch.arange(segs, dtype=torch.float32)
    theta = phases[:, None] + k[None, :] * (2.0 * math.pi / segs)          # [P,G]
    theta_n = theta + (2.0 * math.pi / segs)
    r = radii[:, None]
    cx, cy = centres[:, 0:1], centres[:, 1:2]
    p0 = torch.stack([cx + r * torch.cos(theta), cy + r * torch.sin(theta)], -1)
    t0 = torch.stack([-torch.sin(theta), torch.cos(theta)], -1)
    p3 = torch.stack([cx + r * torch.cos(theta_n), cy + r * torch.sin(theta_n)], -1)
    t3 = torch.stack([-torch.sin(theta_n), torch.cos(theta_n)], -1)
    p1 = p0 + kappa * r[..., None] * t0
    p2 = p3 - kappa * r[..., None] * t3
    ring = torch.stack([p0, p1, p2], dim=2).reshape(centres.shape[0], 3 * segs, 2)
    return ring.to(torch.float32).contiguous()


def distinct_depths(gen: torch.Generator, n: int) -> torch.Tensor:
    """U(0,1) depths, redrawn until all float32 values are distinct."""
    for _ in range(64):
        d = torch.rand(n, generator=gen, dtype=torch.float32)
        if torch.unique(d).numel() == n:
            return d
    # fall back to a seeded permutation of an evenly spaced grid
    perm = torch.randperm(n, generator=gen)
    return ((perm.to(torch.float32) + 0.5) / float(n)).contiguous()


# --------------------------------------------------------------------------
# targets


def value_noise(gen: torch.Generator, h: int, w: int, octaves: int = 4,
                base_cell: int = 96) -> torch.Tensor:
    """Sum of ``octaves`` bilinear value-noise layers, [3,H,W] in [0,1]."""
    acc = torch.zeros(1, 3, h, w)
    amp_total = 0.0
    for o in range(octaves):
        cell = max(2, base_cell >> o)
        gh, gw = h // cell + 2, w // cell + 2
        grid = torch.rand(1, 3, gh, gw, generator=gen)
        up = F.interpolate(grid, size=(h, w), mode="bilinear", align_corners=False)
        amp = 0.5 ** o
        acc += amp * up
        amp_total += amp
    return (acc / amp_total)[0]


def paint_ellipses(gen: torch.Generator, img: torch.Tensor, count: int,
                   rmin: float, rmax: float) -> torch.Tensor:
    """Paint ``count`` random rotated filled ellipses (1 px anti-aliased)."""
    _, h, w = img.shape
    ys = torch.arange(h, dtype=torch.float32)[:, None] + 0.5
    xs = torch.arange(w, dtype=torch.float32)[None, :] + 0.5
    for _ in range(count):
        c = torch.rand(2, generator=gen) * torch.tensor([float(w), float(h)])
        rad = rmin + (rmax - rmin) * torch.rand(2, generator=gen)
        ang = float(torch.rand(1, generator=gen)) * math.pi
        col = torch.rand(3, generator=gen)
        ca, sa = math.cos(ang), math.sin(ang)
        dx, dy = xs - c[0], ys - c[1]
        u = (ca * dx + sa * dy) / rad[0]
        v = (-sa * dx + ca * dy) / rad[1]
        rr = torch.sqrt(u * u + v * v)
        # approximate signed distance in pixels for a 1 px smooth edge
        sd = (rr - 1.0) * torch.minimum(rad[0], rad[1])
        cov = torch.clamp(0.5 - sd, 0.0, 1.0)
        img = img * (1.0 - cov) + col[:, None, None] * cov
    return img


def paint_lines(gen: torch.Generator, img: torch.Tensor, count: int) -> torch.Tensor:
    """Paint ``count`` random anti-aliased straight lines of width U[1,4]."""
    _, h, w = img.shape
    ys = torch.arange(h, dtype=torch.float32)[:, None] + 0.5
    xs = torch.arange(w, dtype=torch.float32)[None, :] + 0.5
    for _ in range(count):
        a = torch.rand(2, generator=gen) * torch.tensor([float(w), float(h)])
        b = torch.rand(2, generator=gen) * torch.tensor([float(w), float(h)])
        width = 1.0 + 3.0 * float(torch.rand(1, generator=gen))
        col = torch.rand(3, generator=gen)
        v = b - a
        vv = float(v.dot(v)) + 1e-12
        t = ((xs - a[0]) * v[0] + (ys - a[1]) * v[1]) / vv
        t = torch.clamp(t, 0.0, 1.0)
        d = torch.sqrt((a[0] + t * v[0] - xs) ** 2 + (a[1] + t * v[1] - ys) ** 2)
        cov = torch.clamp(0.5 * width + 0.5 - d, 0.0, 1.0)
        img = img * (1.0 - cov) + col[:, None, None] * cov
    return img


# --------------------------------------------------------------------------
# configurations


def config1(seed: int = 0) -> FillScene:
    """256x256 CPU plumbing run: 64 random-control-point paths x 4 segments, S=8."""
    gen = torch.Generator().manual_seed(seed)
    h = w = 256
    bg_img = torch.full((3, h, w), 0.5)
    target = paint_ellipses(gen, bg_img, 8, 10.0, 80.0)[None].contiguous()
    p, g = 64, 4
    ring = (torch.rand(p, 3 * g, 2, generator=gen) * 256.0).contiguous()
    colors = torch.rand(p, 3, generator=gen)
    opac = torch.rand(p, generator=gen)
    depths = distinct_depths(gen, p)
    return FillScene(h, w, 8, ring, colors, opac, depths, torch.ones(p),
                     torch.ones(p, dtype=torch.int32), torch.ones(3), target, g,
                     {"config": 1, "seed": seed})


def circles_scene(seed: int, h: int, w: int, paths: int, segs: int, samples: int,
                  ellipses: int, rmin: float = 5.0, rmax: float = 40.0) -> FillScene:
    """Config-2 style scene: random small circles over a noise+ellipse target."""
    gen = torch.Generator().manual_seed(seed)
    target = value_noise(gen, h, w)
    target = paint_ellipses(gen, target, ellipses, 8.0, max(16.0, min(h, w) / 6.0))
    target = target.clamp(0.0, 1.0)[None].contiguous()
    centres = torch.rand(paths, 2, generator=gen) * torch.tensor([float(w), float(h)])
    radii = rmin + (rmax - rmin) * torch.rand(paths, generator=gen)
    phases = torch.rand(paths, generator=gen) * (2.0 * math.pi)
    ring = circle_rings(centres, radii, phases, segs)
    colors = torch.rand(paths, 3, generator=gen)
    depths = distinct_depths(gen, paths)
    return FillScene(h, w, samples, ring, colors, torch.ones(paths), depths,
                     torch.ones(paths), torch.ones(paths, dtype=torch.int32),
                     torch.ones(3), target, segs,
                     {"seed": seed, "paths": paths, "segs": segs, "samples": samples})


def config2(seed: int = 1) -> FillScene:
    s = circles_scene(seed, 512, 768, 512, 4, 16, 32)
    s.meta["config"] = 2
    return s


def config3(seed: int = 2) -> FillScene:
    s = circles_scene(seed, 1356, 2040, 4096, 6, 16, 128)
    s.meta["config"] = 3
    return s


def config5(scene_index: int, paths: int, samples: int) -> FillScene:
    s = circles_scene(1000 + scene_index, 512, 768, paths, 4, samples, 32)
    s.meta.update({"config": 5, "scene": scene_index})
    return s


def config4(seed: int = 3) -> StrokeScene:
    """1024x1024 stroke run: 2048 open one-segment cubics, width U[1,4], S=16."""
    gen = torch.Generator().manual_seed(seed)
    h = w = 1024
    target = paint_lines(gen, torch.ones(3, h, w), 256).clamp(0, 1)[None].contiguous()
    p = 2048
    cubics = (torch.rand(p, 4, 2, generator=gen) * torch.tensor([float(w), float(h)])).contiguous()
    widths = 1.0 + 3.0 * torch.rand(p, generator=gen)
    colors = torch.rand(p, 3, generator=gen)
    opac = torch.rand(p, generator=gen)
    depths = distinct_depths(gen, p)
    return StrokeScene(h, w, 16, cubics, colors, opac, widths, depths, torch.ones(p),
                       torch.ones(3), target, {"config": 4, "seed": seed})


def small_fill_scene(seed: int, h: int = 48, w: int = 64, paths: int = 6, segs: int = 4,
                     samples: int = 6, mixed: bool = True) -> FillScene:
    """Tiny scene for exhaustive parity tests (mixed rules, widths, opacities)."""
    gen = torch.Generator().manual_seed(seed)
    centres = torch.rand(paths, 2, generator=gen) * torch.tensor([float(w), float(h)])
    radii = 4.0 + 18.0 * torch.rand(paths, generator=gen)
    phases = torch.rand(paths, generator=gen) * (2.0 * math.pi)
    ring = circle_rings(centres, radii, phases, segs)
    # perturb control points so paths are not perfect circles (and may self-intersect)
    ring = ring + 4.0 * (torch.rand(ring.shape, generator=gen) - 0.5)
    colors = torch.rand(paths, 3, generator=gen)
    if mixed:
        opac = 0.3 + 0.7 * torch.rand(paths, generator=gen)
        aa = 0.6 + 1.2 * torch.rand(paths, generator=gen)
        rules = (torch.rand(paths, generator=gen) < 0.5).to(torch.int32)
    else:
        opac, aa, rules = torch.ones(paths), torch.ones(paths), torch.ones(paths, dtype=torch.int32)
    depths = distinct_depths(gen, paths)
    target = torch.rand(1, 3, h, w, generator=gen)
    bg = torch.rand(3, generator=gen)
    return FillScene(h, w, samples, ring.contiguous(), colors, opac, depths, aa, rules, bg,
                     target, segs, {"seed": seed, "small": True})


def small_stroke_scene(seed: int, h: int = 48, w: int = 64, paths: int = 8,
                       samples: int = 6) -> StrokeScene:
    gen = torch.Generator().manual_seed(seed)
    cubics = (torch.rand(paths, 4, 2, generator=gen) * torch.tensor([float(w), float(h)])).contiguous()
    widths = 1.0 + 3.0 * torch.rand(paths, generator=gen)
    colors = torch.rand(paths, 3, generator=gen)
    opac = 0.3 + 0.7 * torch.rand(paths, generator=gen)
    aa = 0.6 + 1.2 * torch.rand(paths, generator=gen)
    depths = distinct_depths(gen, paths)
    target = torch.rand(1, 3, h, w, generator=gen)
    bg = torch.rand(3, generator=gen)
    return StrokeScene(h, w, samples, cubics, colors, opac, widths, depths, aa, bg, target,
                       {"seed": seed, "small": True})


def seeded_grad(seed: int, h: int, w: int, scale: float = 1e-3) -> torch.Tensor:
    """A seeded upstream image gradient [H, W, 3] for standalone backward tests."""
    gen = torch.Generator().manual_seed(seed)
    return ((torch.rand(h, w, 3, generator=gen) - 0.5) * (2.0 * scale)).contiguous()


__all__ = [
    "FillScene", "StrokeScene", "ring_to_cubics", "ring_gather_index", "px_to_norm",
    "circle_rings", "config1", "config2", "config3", "config4", "config5",
    "circles_scene", "small_fill_scene", "small_stroke_scene", "seeded_grad",
    "value_noise", "paint_ellipses", "paint_lines", "distinct_depths",
]
