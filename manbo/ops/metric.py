"""Metric kernels with the reference's factory names (manbo/ops/metric.py).

The reference composes its metrics from per-block partial-sum kernels; the
B200 build computes MSE in one fused launch and SSIM with a separable window.
The factories below keep the reference's call shapes: the partial-sum
factories fill one partial per ``threads * items_per_thread`` span.
"""
from __future__ import annotations

import torch

from repo_b200 import _native as nat
from repo_b200 import metric as _m

DEFAULT_THREADS = _m.DEFAULT_THREADS
DEFAULT_ITEMS_PER_THREAD = _m.DEFAULT_ITEMS_PER_THREAD
DEFAULT_SSIM_THREADS = _m.DEFAULT_SSIM_THREADS
DEFAULT_SSIM_BLOCK_H = _m.DEFAULT_SSIM_BLOCK_H
DEFAULT_SSIM_BLOCK_W = _m.DEFAULT_SSIM_BLOCK_W


def _ceildiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _span_sums(x, y, span, partial):
    n = int(x.numel())
    for b in range(int(partial.numel())):
        lo, hi = b * span, min(n, (b + 1) * span)
        xs = x.view(-1)[lo:hi].contiguous()
        if y is None:
            ys = torch.zeros_like(xs)
            sq = False
        else:
            ys = y.view(-1)[lo:hi].contiguous()
            sq = True
        if sq:
            _m.sse_mse(xs, ys, out_sse=partial[b:b + 1])
        else:
            partial[b:b + 1].copy_(xs.sum().reshape(1))


def mse_partial_sum_kernel(threads: int = DEFAULT_THREADS,
                           items_per_thread: int = DEFAULT_ITEMS_PER_THREAD, dtype="float32",
                           target="auto"):
    span = int(threads) * int(items_per_thread)

    def kernel(x, y, partial):
        _span_sums(x, y, span, partial)
    return kernel


def reduce_sum_partial_kernel(threads: int = DEFAULT_THREADS,
                              items_per_thread: int = DEFAULT_ITEMS_PER_THREAD, target="auto"):
    span = int(threads) * int(items_per_thread)

    def kernel(x, partial):
        _span_sums(x, None, span, partial)
    return kernel


def mse_backward_diff_kernel(threads: int = DEFAULT_THREADS, dtype="float32"):
    def kernel(lhs, rhs, scale, grad):
        nat.check(nat.call("cs_mse_backward", nat.ptr(lhs), nat.ptr(rhs), None, float(scale),
                           nat.ptr(grad), int(grad.numel()), nat.stream(grad.device)),
                  "cs_mse_backward")
    return kernel


def mse_backward_diff_tilelang(lhs, rhs, *, scale: float, threads: int = DEFAULT_THREADS):
    lf = lhs.float().contiguous().view(-1)
    rf = rhs.float().contiguous().view(-1)
    grad = torch.empty_like(lf, dtype=torch.float32)
    mse_backward_diff_kernel(threads)(lf, rf, scale, grad)
    return grad.view(lhs.shape)


def reduce_sum_1d_tilelang(x, *, threads: int = DEFAULT_THREADS,
                           items_per_thread: int = DEFAULT_ITEMS_PER_THREAD):
    return x.contiguous().sum()


def ssim_map_kernel(win_size: int = 11, block_h: int = DEFAULT_SSIM_BLOCK_H,
                    block_w: int = DEFAULT_SSIM_BLOCK_W, threads: int = DEFAULT_SSIM_THREADS,
                    target="auto"):
    """Returns kernel(x, y, win2d, out, c1, c2) for [C, H, W] inputs.  The window
    must be separable, outer(g, g) as the reference builds it; g is recovered
    as the row sums of win2d."""
    def kernel(x, y, win2d, out, c1, c2):
        c, h, w = (int(v) for v in x.shape)
        g = win2d.sum(dim=1).contiguous().to(torch.float32)
        dev = x.device
        means = torch.empty((c,), dtype=torch.float32, device=dev)
        ws = _m._workspace(dev, "ssim", int(nat.call("cs_ssim_workspace_size", c, h, w, win_size)))
        nat.check(nat.call("cs_ssim", nat.ptr(x), nat.ptr(y), nat.ptr(g), c, h, w, int(win_size),
                           float(c1), float(c2), nat.ptr(means), nat.ptr(out), ws.data_ptr(),
                           nat.stream(dev)), "cs_ssim")
    return kernel
