"""The drop-in Adan optimiser (manbo.Adan on cs_adan_step) against the
reference's own outputs (tests/golden/adan.npz) and the CPU oracle, on the GPU."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu

VARIANTS = {
    "prox": dict(lr=0.05, weight_decay=0.02),
    "noprox": dict(lr=0.05, weight_decay=0.02, no_prox=True),
    "clip": dict(lr=0.05, max_grad_norm=0.5),
}
KEYS = ("exp_avg", "exp_avg_sq", "exp_avg_diff", "neg_pre_grad")


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_adan_matches_reference_golden(variant):
    import manbo
    g = load_golden("adan")
    ps = [torch.from_numpy(g[f"param0_{i}"]).cuda().requires_grad_(True) for i in range(2)]
    opt = manbo.Adan(ps, **VARIANTS[variant])
    for t in range(3):
        for i, p in enumerate(ps):
            p.grad = torch.from_numpy(g[f"grad{t}_{i}"]).cuda()
        opt.step()
    for i, p in enumerate(ps):
        np.testing.assert_allclose(p.detach().cpu().numpy(), g[f"{variant}_param_{i}"],
                                   rtol=1e-5, atol=1e-7)
        for k in KEYS:
            np.testing.assert_allclose(opt.state[p][k].cpu().numpy(), g[f"{variant}_{k}_{i}"],
                                       rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
def test_adan_step_operator_matches_oracle(n):
    """manbo.ops.adan_step_from_grad_tilelang on both the 4-wide and the
    single-element paths (n % 4 != 0), several steps, against the oracle."""
    from manbo.ops import adan_step_from_grad_tilelang
    gen = torch.Generator().manual_seed(n)
    p = torch.randn(n, generator=gen)
    dev = [p.cuda()] + [torch.zeros(n, device="cuda") for _ in KEYS]
    host = [p.numpy().copy()] + [np.zeros(n, np.float32) for _ in KEYS]
    for t in range(1, 5):
        grad = torch.randn(n, generator=gen) * 0.3
        adan_step_from_grad_tilelang(dev[0], grad.cuda(), *dev[1:], step=t, lr=0.01,
                                     weight_decay=0.01, clip_global_grad_norm=0.9)
        oracle.adan_step(host[0], grad.numpy().copy(), *host[1:], step=t, lr=0.01,
                         weight_decay=0.01, clip_global_grad_norm=0.9)
    torch.cuda.synchronize()
    for d, h in zip(dev, host):
        np.testing.assert_allclose(d.cpu().numpy(), h, rtol=1e-5, atol=1e-7)


def test_adan_rejects_what_the_reference_rejects():
    import manbo
    p = torch.zeros(4, device="cuda", requires_grad=True)
    with pytest.raises(ValueError, match="Invalid beta parameter at index 2"):
        manbo.Adan([p], betas=(0.9, 0.9, 1.0))
    with pytest.raises(ValueError, match="Invalid learning rate"):
        manbo.Adan([p], lr=-1.0)
    q = torch.zeros(4, device="cuda", dtype=torch.float64, requires_grad=True)
    opt = manbo.Adan([q])
    q.grad = torch.ones_like(q)
    with pytest.raises(ValueError, match="float32"):
        opt.step()
