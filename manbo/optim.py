"""Adan optimiser on the B200 step kernel (mirrors manbo/optim.py:10-190).

Same constructor, validation, state (``exp_avg``, ``exp_avg_sq``,
``exp_avg_diff``, ``neg_pre_grad`` per parameter), ``restart_opt`` and global
gradient-norm clipping as the reference; every parameter's update is one
``cs_adan_step`` launch.  Like the reference, clipping (max_grad_norm > 0)
reads the norm on the host, once per step.
"""
from __future__ import annotations

import math

import torch
from torch.optim.optimizer import Optimizer

from .ops.optim import adan_step_from_grad_kernel

DEFAULT_TILELANG_THREADS = 256
_STATE_KEYS = ("exp_avg", "exp_avg_sq", "exp_avg_diff", "neg_pre_grad")


class Adan(Optimizer):
    """Adan (adaptive Nesterov momentum) with decoupled or proximal weight decay."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.98, 0.92, 0.99), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 0.0, no_prox: bool = False,
                 tilelang_threads: int = DEFAULT_TILELANG_THREADS):
        if not 0.0 <= max_grad_norm:
            raise ValueError(f"Invalid max_grad_norm: {max_grad_norm}")
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        for i in range(3):
            if not 0.0 <= betas[i] < 1.0:
                raise ValueError(f"Invalid beta parameter at index {i}: {betas[i]}")
        if tilelang_threads <= 0:
            raise ValueError(f"Invalid tilelang_threads: {tilelang_threads}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      max_grad_norm=max_grad_norm, no_prox=no_prox,
                                      tilelang_threads=tilelang_threads))

    def __setstate__(self, state):
        super().__setstate__(state)
        for group in self.param_groups:
            group.setdefault("no_prox", False)
            group.setdefault("tilelang_threads", DEFAULT_TILELANG_THREADS)

    @torch.no_grad()
    def restart_opt(self):
        """Zero the step count and every moment (the reference's restart)."""
        for group in self.param_groups:
            group["step"] = 0
            for p in group["params"]:
                if p.requires_grad:
                    st = self.state[p]
                    for k in _STATE_KEYS:
                        st[k] = torch.zeros_like(p)

    def _clip_factor(self) -> float:
        max_norm = self.defaults["max_grad_norm"]
        if max_norm <= 0:
            return 1.0
        dev = self.param_groups[0]["params"][0].device
        sq = torch.zeros(1, device=dev)
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is not None:
                    sq.add_(p.grad.pow(2).sum())
        eps = self.param_groups[0]["eps"]
        factor = torch.clamp(torch.tensor(max_norm, device=dev) / (torch.sqrt(sq) + eps), max=1.0)
        return float(factor.item())

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        clip = self._clip_factor()
        for group in self.param_groups:
            b1, b2, b3 = group["betas"]
            group["step"] = group.get("step", 0) + 1
            t = int(group["step"])
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            no_prox = bool(group["no_prox"])
            key = (int(group["tilelang_threads"]), no_prox)
            if group.get("_b200_kernel_key") != key:
                group["_b200_kernel"] = adan_step_from_grad_kernel(threads=key[0], no_prox=no_prox)
                group["_b200_kernel_key"] = key
            kernel = group["_b200_kernel"]
            bc1, bc2, bc3_sqrt = 1.0 - b1 ** t, 1.0 - b2 ** t, math.sqrt(1.0 - b3 ** t)
            for p in params:
                if p.dtype != torch.float32:
                    raise ValueError("TileLang Adan currently expects float32 params")
                if not p.is_contiguous():
                    raise ValueError("TileLang Adan expects contiguous params")
                st = self.state[p]
                if not st:
                    for k in _STATE_KEYS:
                        st[k] = torch.zeros_like(p)
                moments = [st[k] for k in _STATE_KEYS]
                if any(m.dtype != torch.float32 or not m.is_contiguous() for m in moments):
                    raise ValueError("TileLang Adan expects contiguous float32 states")
                g = p.grad
                if g.dtype != torch.float32 or g.device != p.device or not g.is_contiguous():
                    buf = st.get("_grad_buf")
                    if buf is None or buf.shape != p.shape:
                        buf = torch.empty_like(p)
                        st["_grad_buf"] = buf
                    buf.copy_(g)
                    g = buf
                n = p.numel()
                kernel(p.view(n), g.view(n), *(m.view(n) for m in moments), t, b1, b2, b3, bc1,
                       bc2, bc3_sqrt, group["lr"], group["weight_decay"], group["eps"], clip)
        return loss


__all__ = ["Adan"]
