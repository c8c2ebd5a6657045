"""Regularisation loss kernels (cs_regularization_forward / _backward) against
the CPU oracle (oracle/regularization.py) and the reference's own loss and
gradients (tests/golden/regularization.npz, made by tests/golden/make_golden.py
from manbo/regularization.py:359 on a GPU)."""
import numpy as np
import pytest
import torch

from conftest import load_golden as golden, rel_l2
from oracle import regularization as reg

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
KW = dict(num_beziers=2, bezier_degree=4, num_samples=3, lambda_proj=0.7, opacity_weight=0.3,
          boundary_bound=1.0, curvature_angle_thresh_deg=60.0)


def _gpu(cp, op, xyz, mode, **kw):
    from repo_b200.regularization import regularization_loss
    tcp = torch.from_numpy(np.ascontiguousarray(cp, np.float32)).to(DEV).requires_grad_(True)
    top = torch.from_numpy(np.ascontiguousarray(op, np.float32)).to(DEV).requires_grad_(True)
    txyz = None
    if xyz is not None:
        txyz = torch.from_numpy(np.ascontiguousarray(xyz, np.float32)).to(DEV).requires_grad_(True)
    loss = regularization_loss(tcp, top, txyz, mode=mode, **kw)
    loss.backward()
    return (float(loss), tcp.grad.cpu().numpy(), top.grad.cpu().numpy(),
            None if txyz is None else txyz.grad.cpu().numpy())


def _scene(mode, seed, n):
    rng = np.random.default_rng(seed)
    k = 10 if mode == "closed" else 4
    cp = rng.uniform(-1.3, 1.3, (n, k, 2)).astype(np.float32)
    op = rng.normal(0, 2, (n, 1)).astype(np.float32)
    xyz = rng.uniform(-1, 1, (n, 2, 24, 2)).astype(np.float32) if mode == "closed" else None
    return cp, op, xyz


@pytest.mark.parametrize("mode", ["closed", "unclosed"])
def test_regularisation_matches_reference_golden(mode):
    g = golden("regularization")
    cp, op = g[f"{mode}_cp"], g[f"{mode}_op"]
    xyz = g[f"{mode}_xyz"] if mode == "closed" else None
    loss, g_cp, g_op, g_xyz = _gpu(cp, op, xyz, mode, **KW)
    want = float(g[f"{mode}_loss"][0])
    assert abs(loss - want) <= 1e-5 * abs(want)
    assert rel_l2(g_cp, g[f"{mode}_g_cp"]) <= 1e-4
    assert rel_l2(g_op, g[f"{mode}_g_op"]) <= 1e-4
    if mode == "closed":
        assert rel_l2(g_xyz, g[f"{mode}_g_xyz"]) <= 1e-4


@pytest.mark.parametrize("mode", ["closed", "unclosed"])
@pytest.mark.parametrize("seed,n", [(0, 1), (1, 7), (2, 300), (3, 5000)])
def test_regularisation_matches_oracle(mode, seed, n):
    cp, op, xyz = _scene(mode, seed, n)
    loss, g_cp, g_op, g_xyz = _gpu(cp, op, xyz, mode, **KW)
    c64 = cp.astype(np.float64)
    o64 = op.astype(np.float64)
    x64 = None if xyz is None else xyz.astype(np.float64)
    want = reg.regularization_loss(c64, o64, x64, mode=mode, **KW)
    w_cp, w_op, w_xyz = reg.regularization_grads(c64, o64, x64, mode=mode, **KW)
    assert abs(loss - want) <= 1e-5 * abs(want)
    assert rel_l2(g_cp, w_cp) <= 1e-4
    assert rel_l2(g_op, w_op) <= 1e-4
    if mode == "closed":
        assert rel_l2(g_xyz, w_xyz) <= 1e-4


def test_regularisation_gradient_scales_with_grad_output():
    from repo_b200.regularization import regularization_loss
    cp, op, xyz = _scene("closed", 5, 9)
    tcp = torch.from_numpy(cp).to(DEV).requires_grad_(True)
    top = torch.from_numpy(op).to(DEV).requires_grad_(True)
    txyz = torch.from_numpy(xyz).to(DEV)
    (3.0 * regularization_loss(tcp, top, txyz, mode="closed", **KW)).backward()
    g3 = tcp.grad.clone()
    tcp.grad = None
    regularization_loss(tcp, top, txyz, mode="closed", **KW).backward()
    torch.testing.assert_close(g3, 3.0 * tcp.grad, rtol=1e-6, atol=0)


def test_manbo_name_runs_the_kernels():
    import manbo
    cp, op, xyz = _scene("closed", 8, 11)
    tcp = torch.from_numpy(cp).to(DEV).requires_grad_(True)
    loss = manbo.regularization_loss_tilelang(tcp, torch.from_numpy(op).to(DEV),
                                              torch.from_numpy(xyz).to(DEV), mode="closed",
                                              threads=128, items_per_thread=4, **KW)
    want = reg.regularization_loss(cp.astype(np.float64), op.astype(np.float64),
                                   xyz.astype(np.float64), mode="closed", **KW)
    assert abs(float(loss.detach()) - want) <= 1e-5 * abs(want)
    loss.backward()
    assert tcp.grad is not None and torch.isfinite(tcp.grad).all()
