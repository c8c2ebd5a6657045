"""The regularisation oracle (oracle/regularization.py, a restatement of
manbo/regularization.py and manbo/ops/regularization.py): closed-form cases
and its gradients against central differences of its own loss (float64)."""
import numpy as np
import pytest

from conftest import rel_l2
from oracle import regularization as reg


def _scene(mode, seed):
    rng = np.random.default_rng(seed)
    n = 5
    if mode == "closed":
        k = 2 * reg.shape_degree("closed", 2, 4) + 2          # 10 control points
        xyz = rng.uniform(-1, 1, (n, 2, 24, 2))
    else:
        k = 4
        xyz = None
    cp = rng.uniform(-1.3, 1.3, (n, k, 2))
    op = rng.normal(0, 2, (n, 1))
    return cp, op, xyz


KW = dict(num_beziers=2, bezier_degree=4, num_samples=3, lambda_proj=0.7, opacity_weight=0.3,
          boundary_bound=1.0, curvature_angle_thresh_deg=60.0)


def _fd(f, x, eps=1e-6):
    g = np.zeros_like(x)
    for i in np.ndindex(x.shape):
        up, dn = x.copy(), x.copy()
        up[i] += eps
        dn[i] -= eps
        g[i] = (f(up) - f(dn)) / (2 * eps)
    return g


@pytest.mark.parametrize("mode", ["closed", "unclosed"])
@pytest.mark.parametrize("seed", [0, 1])
def test_regularisation_gradients_match_finite_differences(mode, seed):
    cp, op, xyz = _scene(mode, seed)
    # keep the boundary hinge away from its kink at +-bound
    cp = np.where(np.abs(np.abs(cp) - 1.0) < 1e-3, cp * 1.01, cp)
    g_cp, g_op, g_xyz = reg.regularization_grads(cp, op, xyz, mode=mode, **KW)
    loss = lambda c=cp, o=op, x=xyz: reg.regularization_loss(c, o, x, mode=mode, **KW)
    assert rel_l2(g_cp, _fd(lambda c: loss(c=c), cp)) <= 1e-6
    assert rel_l2(g_op, _fd(lambda o: loss(o=o), op)) <= 1e-6
    if mode == "closed":
        fd_x = _fd(lambda x: loss(x=x), xyz)
        assert np.abs(fd_x).max() > 0  # some sample passes the angle mask
        assert rel_l2(g_xyz, fd_x) <= 1e-6
    else:
        assert g_xyz is None


def test_shape_penalty_closed_form():
    # open curve p0=(0,0), mid, pend=(2,0): alpha = mid.x / (4 + 1e-8)
    cp = np.array([[[0.0, 0.0], [3.0, 1.0], [-1.0, 5.0], [2.0, 0.0]]])
    a1, a2 = 6.0 / (4 + 1e-8), -2.0 / (4 + 1e-8)
    assert reg.shape_sum(cp) == pytest.approx((a1 - 1) ** 2 + a2 ** 2, rel=1e-12)
    # inside the chord: no penalty
    assert reg.shape_sum(np.array([[[0.0, 0.0], [1.0, 3.0], [2.0, 0.0]]])) == 0.0


def test_closed_shape_skips_the_split_point_and_projects_onto_it():
    cp = np.zeros((1, 6, 2))
    cp[0, 2] = (1.0, 0.0)            # split = 2: the chord end
    cp[0, 1] = (2.0, 0.0)            # alpha 2 -> phi 1
    cp[0, 3] = (-1.0, 0.0)           # alpha -1 -> phi 1
    cp[0, 4] = (0.5, 9.0)            # alpha 0.5 -> 0
    cp[0, 5] = (0.0, 0.0)            # alpha 0 -> 0
    assert reg.shape_sum(cp, split_idx=2) == pytest.approx(2.0, rel=1e-7)


def test_opacity_boundary_and_curvature_closed_form():
    assert reg.opacity_sum(np.zeros(4)) == pytest.approx(2.0)    # |0.5 - 1| * 4
    cp = np.array([[[1.5, 0.0], [9.0, 9.0], [-2.0, 0.5]]])         # joints (degree 2): 0 and 2
    assert reg.boundary_sum(cp, 2, 1.0) == pytest.approx(0.5 + 1.0)
    # a finely sampled circle (the closed path is the first half followed by
    # the reversed second half) turns by far less than 120 degrees over 10
    # samples, so no sample passes the angle mask
    m = 32
    th = np.linspace(0.0, 2.0 * np.pi, 2 * m, endpoint=False)
    circle = np.stack([np.cos(th), np.sin(th)], axis=-1)
    xyz = np.stack([circle[:m], circle[m:][::-1]])[None]
    s, per = reg.curvature_sum(xyz, 4, 60.0)
    assert per == 16 and s == 0.0
    # a hairpin (both halves run the same way) does pass it where it folds
    fold = np.stack([circle[:m], circle[:m]])[None]
    s, _ = reg.curvature_sum(fold, 1, 60.0)
    assert s > 0.0


def test_loss_shape_checks():
    cp, op, xyz = _scene("closed", 3)
    with pytest.raises(ValueError):
        reg.regularization_loss(cp[:, :8], op, xyz, mode="closed", **KW)


def test_host_wrapper_checks_arguments_like_the_reference():
    """repo_b200.regularization validates before any device work
    (manbo/regularization.py:79-105, :359-380) and rejects host tensors."""
    import torch

    from repo_b200.regularization import regularization_loss
    cp = torch.zeros(3, 10, 2)
    op = torch.zeros(3, 1)
    xyz = torch.zeros(3, 2, 8, 2)
    kw = dict(num_beziers=2, bezier_degree=4, num_samples=3)
    with pytest.raises(ValueError, match="Unsupported mode"):
        regularization_loss(cp, op, xyz, mode="spiral", **kw)
    with pytest.raises(ValueError, match="xyz must be provided"):
        regularization_loss(cp, op, None, mode="closed", **kw)
    with pytest.raises(ValueError, match="expected K=10"):
        regularization_loss(cp[:, :8], op, xyz, mode="closed", **kw)
    with pytest.raises(ValueError, match="at least one curve"):
        regularization_loss(cp[:0], op, xyz, mode="unclosed", **kw)
    with pytest.raises(ValueError, match="CUDA"):
        regularization_loss(cp, op, xyz, mode="closed", **kw)


@pytest.mark.parametrize("mode", ["closed", "unclosed"])
def test_oracle_matches_reference_golden(mode):
    """The restatement against the reference's own loss and gradients
    (tests/golden/regularization.npz, from manbo/regularization.py:359 run by
    tests/golden/make_golden.py on a GPU; the reference runs in float32 with
    fast math)."""
    from conftest import load_golden
    g = load_golden("regularization")
    cp = g[f"{mode}_cp"].astype(np.float64)
    op = g[f"{mode}_op"].astype(np.float64)
    xyz = g[f"{mode}_xyz"].astype(np.float64) if mode == "closed" else None
    loss = reg.regularization_loss(cp, op, xyz, mode=mode, **KW)
    want = float(g[f"{mode}_loss"][0])
    assert abs(loss - want) <= 1e-5 * abs(want)
    g_cp, g_op, g_xyz = reg.regularization_grads(cp, op, xyz, mode=mode, **KW)
    assert rel_l2(g_cp, g[f"{mode}_g_cp"]) <= 1e-4
    assert rel_l2(g_op, g[f"{mode}_g_op"]) <= 1e-4
    if mode == "closed":
        assert rel_l2(g_xyz, g[f"{mode}_g_xyz"]) <= 1e-4
