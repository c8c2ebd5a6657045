"""MSE loss, PSNR and SSIM on the B200 kernels (mirrors manbo/metric.py).

``mse_loss_tilelang`` keeps the reference's autograd contract
(manbo/metric.py:133-212) but reads the gradient scale on the device, so the
backward performs no host synchronisation (the reference calls ``.item()``,
manbo/metric.py:168).  ``ssim`` is forward-only, like the reference.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import _ext
from . import _native as nat

DEFAULT_THREADS = 256
DEFAULT_ITEMS_PER_THREAD = 8
DEFAULT_SSIM_THREADS = 64
DEFAULT_SSIM_BLOCK_H = 8
DEFAULT_SSIM_BLOCK_W = 16

_GAUSS_CACHE: Dict[Tuple[str, int, float], torch.Tensor] = {}
_WS_CACHE: Dict[Tuple[str, str], torch.Tensor] = {}


def _workspace(device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
    """Per-device scratch buffer, grown on demand, used in stream order.  It is
    zeroed when allocated: the kernels' completion tickets start at zero and
    are reset by the kernels themselves."""
    key = (str(device), kind)
    buf = _WS_CACHE.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros((max(nbytes, 256),), dtype=torch.uint8, device=device)
        _WS_CACHE[key] = buf
    return buf


def _as_cuda_f32(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.dtype != torch.float32:
        x = x.float()
    if not x.is_contiguous():
        x = x.contiguous()
    return x


def _validate_pair_4d(x: torch.Tensor, y: torch.Tensor) -> None:
    if x.shape != y.shape:
        raise ValueError(f"x and y must have the same shape, got {x.shape} and {y.shape}")
    if x.dim() != 4:
        raise ValueError(f"expected input shape [N, C, H, W], got {x.shape}")
    if min(x.shape) <= 0:
        raise ValueError(f"all dimensions must be > 0, got {x.shape}")


def gaussian_1d(win_size: int, win_sigma: float, device: torch.device) -> torch.Tensor:
    """Normalised 1-D Gaussian g; the reference's window is outer(g, g)
    (manbo/metric.py:47-61)."""
    key = (device.type, device.index, int(win_size), float(win_sigma))
    g = _GAUSS_CACHE.get(key)
    if g is None:
        coords = torch.arange(win_size, dtype=torch.float32, device=device)
        coords -= win_size // 2
        g = torch.exp(-(coords ** 2) / (2 * (win_sigma ** 2)))
        g /= g.sum()
        g = g.contiguous()
        _GAUSS_CACHE[key] = g
    return g


def sse_mse(x: torch.Tensor, y: torch.Tensor, out_sse=None, out_mse=None):
    """Device-resident SSE and MSE of two flattened float32 CUDA tensors."""
    if out_mse is None:
        return out_sse, _ext.load().mse_forward(x, y, out_sse)
    n = int(x.numel())
    dev = x.device
    ws = _workspace(dev, "mse", int(nat.call("cs_mse_workspace_size", n)))
    nat.check(nat.call("cs_mse_forward", nat.ptr(x), nat.ptr(y), n, nat.ptr(out_sse),
                       nat.ptr(out_mse), ws.data_ptr(), nat.stream(dev)), "cs_mse_forward")
    return out_sse, out_mse


def mse_backward(lhs: torch.Tensor, rhs: torch.Tensor, scale: torch.Tensor,
                 factor: float = 1.0) -> torch.Tensor:
    """grad = scale * factor * (lhs - rhs), scale a device scalar."""
    return _ext.load().mse_backward(lhs, rhs, scale, float(factor))


class MSELossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, threads, items_per_thread, tilelang_backward):
        if x.shape != y.shape:
            raise ValueError(f"x and y must have the same shape, got {x.shape} and {y.shape}")
        x32 = _as_cuda_f32(x, "x")
        y32 = _as_cuda_f32(y, "y")
        _, loss = sse_mse(x32, y32)
        ctx.save_for_backward(x32, y32)
        ctx.numel = int(x.numel())
        ctx.x_dtype, ctx.y_dtype = x.dtype, y.dtype
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        x, y = ctx.saved_tensors
        grad_x = grad_y = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            # d loss / dx = grad_output * (2 / N) * (x - y); the product with
            # the device scalar grad_output is formed in the kernel
            g = _as_cuda_f32(grad_output.reshape(1), "grad_output")
            factor = 2.0 / float(ctx.numel)
            if ctx.needs_input_grad[0]:
                grad_x = mse_backward(x, y, g, factor).to(ctx.x_dtype)
            if ctx.needs_input_grad[1]:
                grad_y = mse_backward(y, x, g, factor).to(ctx.y_dtype)
        return grad_x, grad_y, None, None, None


def mse_loss(x: torch.Tensor, y: torch.Tensor, *, threads: int = DEFAULT_THREADS,
             items_per_thread: int = DEFAULT_ITEMS_PER_THREAD,
             tilelang_backward: bool = True) -> torch.Tensor:
    """mean((x - y)^2) with the reference's autograd contract (manbo/metric.py:198-212)."""
    return MSELossFunction.apply(x, y, int(threads), int(items_per_thread),
                                 int(bool(tilelang_backward)))


def psnr(x: torch.Tensor, y: torch.Tensor, *, data_range: float = 1.0, eps: float = 1e-12,
         threads: int = DEFAULT_THREADS,
         items_per_thread: int = DEFAULT_ITEMS_PER_THREAD) -> torch.Tensor:
    """10 log10(R^2 / (mse + eps)) (manbo/metric.py:64-99)."""
    _validate_pair_4d(x, y)
    if data_range <= 0.0:
        raise ValueError("data_range must be > 0")
    if eps < 0.0:
        raise ValueError("eps must be >= 0")
    x32 = _as_cuda_f32(x, "x")
    y32 = _as_cuda_f32(y, "y")
    _, mse = sse_mse(x32.view(-1), y32.view(-1))
    return 10.0 * torch.log10((data_range * data_range) / (mse + eps))


def ssim_per_plane(x32: torch.Tensor, y32: torch.Tensor, win_size: int, win_sigma: float,
                   c1: float, c2: float, ssim_map=None) -> torch.Tensor:
    """Mean SSIM of each of the N*C planes of [N, C, H, W] float32 CUDA inputs."""
    n, c, h, w = x32.shape
    g = gaussian_1d(win_size, win_sigma, x32.device)
    return _ext.load().ssim_planes(x32, y32, g, n * c, h, w, int(win_size), float(c1), float(c2),
                                   ssim_map)


def ssim(x: torch.Tensor, y: torch.Tensor, *, data_range: float = 1.0, size_average: bool = True,
         win_size: int = 11, win_sigma: float = 1.5, k1: float = 0.01, k2: float = 0.03,
         nonnegative_ssim: bool = False, block_h: int = DEFAULT_SSIM_BLOCK_H,
         block_w: int = DEFAULT_SSIM_BLOCK_W, threads: int = DEFAULT_SSIM_THREADS) -> torch.Tensor:
    """Valid-window Gaussian SSIM, forward only (manbo/metric.py:215-273)."""
    _validate_pair_4d(x, y)
    if data_range <= 0.0:
        raise ValueError("data_range must be > 0")
    if win_size <= 0 or win_size % 2 == 0:
        raise ValueError("win_size must be a positive odd integer")
    if win_sigma <= 0.0:
        raise ValueError("win_sigma must be > 0")
    x32 = _as_cuda_f32(x, "x")
    y32 = _as_cuda_f32(y, "y")
    n, c, h, w = x32.shape
    if h - win_size + 1 <= 0 or w - win_size + 1 <= 0:
        raise ValueError(f"input spatial size {(h, w)} is smaller than win_size {win_size}")
    c1 = (k1 * data_range) ** 2
    c2 = (k2 * data_range) ** 2
    per_channel = ssim_per_plane(x32, y32, win_size, win_sigma, c1, c2).view(n, c)
    if nonnegative_ssim:
        per_channel = torch.relu(per_channel)
    if size_average:
        return per_channel.mean()
    return per_channel.mean(1)


__all__ = ["mse_loss", "psnr", "ssim", "sse_mse", "mse_backward", "gaussian_1d", "ssim_per_plane"]
