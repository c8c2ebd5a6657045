"""Adan step operator on the B200 kernel (mirrors manbo/ops/optim.py).

``adan_step_from_grad_kernel`` returns a callable with the reference kernel's
argument list (flat float32 tensors, then step and the scalar
hyper-parameters; manbo/ops/optim.py:29-47); ``adan_step_from_grad_tilelang``
is the keyword front end (:109-170).  Both run ``cs_adan_step``.
"""
from __future__ import annotations

import torch

from repo_b200 import _native as nat

DEFAULT_THREADS = 256


def _check_flat(name, t, numel):
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise ValueError(f"{name} must be float32")
    if not t.is_contiguous() or t.numel() != numel:
        raise ValueError(f"{name} must be contiguous with {numel} elements")


def adan_step_from_grad_kernel(threads: int = DEFAULT_THREADS, dtype: str = "float32",
                               no_prox: bool = False):
    """Adan step callable: kernel(param, grad, exp_avg, exp_avg_sq, exp_avg_diff,
    neg_pre_grad, step, beta1, beta2, beta3, bias_correction1, bias_correction2,
    bias_correction3_sqrt, lr, weight_decay, eps, clip_global_grad_norm), all
    tensors flat float32 of one length, updated in place."""
    if threads <= 0:
        raise ValueError("threads must be > 0")
    if dtype != "float32":
        raise ValueError("the B200 Adan step computes in float32")
    prox_flag = int(bool(no_prox))

    def kernel(param, grad, exp_avg, exp_avg_sq, exp_avg_diff, neg_pre_grad, step_i32, beta1,
               beta2, beta3, bias_correction1, bias_correction2, bias_correction3_sqrt, lr,
               weight_decay, eps, clip_global_grad_norm):
        numel = int(param.numel())
        for name, t in (("param", param), ("grad", grad), ("exp_avg", exp_avg),
                        ("exp_avg_sq", exp_avg_sq), ("exp_avg_diff", exp_avg_diff),
                        ("neg_pre_grad", neg_pre_grad)):
            _check_flat(name, t, numel)
        nat.check(nat.call("cs_adan_step", nat.ptr(param), nat.ptr(grad), nat.ptr(exp_avg),
                           nat.ptr(exp_avg_sq), nat.ptr(exp_avg_diff), nat.ptr(neg_pre_grad),
                           numel, int(step_i32), float(beta1), float(beta2), float(beta3),
                           float(bias_correction1), float(bias_correction2),
                           float(bias_correction3_sqrt), float(lr), float(weight_decay),
                           float(eps), float(clip_global_grad_norm), prox_flag,
                           nat.stream(param.device)), "cs_adan_step")

    return kernel


def adan_step_from_grad_tilelang(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor,
                                 exp_avg_sq: torch.Tensor, exp_avg_diff: torch.Tensor,
                                 neg_pre_grad: torch.Tensor, *, step: int, lr: float = 1e-3,
                                 betas: tuple = (0.98, 0.92, 0.99), eps: float = 1e-8,
                                 weight_decay: float = 0.0, no_prox: bool = False,
                                 clip_global_grad_norm: float = 1.0,
                                 threads: int = DEFAULT_THREADS) -> None:
    """One Adan step in place from an externally provided gradient; the bias
    corrections are computed on the host from `step` (manbo/ops/optim.py:109-170)."""
    b1, b2, b3 = betas
    n = param.numel()
    g = grad if grad.is_contiguous() else grad.contiguous()
    adan_step_from_grad_kernel(threads=threads, no_prox=no_prox)(
        param.view(n), g.view(n), exp_avg.view(n), exp_avg_sq.view(n), exp_avg_diff.view(n),
        neg_pre_grad.view(n), int(step), b1, b2, b3, 1.0 - b1 ** step, 1.0 - b2 ** step,
        (1.0 - b3 ** step) ** 0.5, lr, weight_decay, eps, clip_global_grad_norm)


__all__ = ["adan_step_from_grad_kernel", "adan_step_from_grad_tilelang", "DEFAULT_THREADS"]
