"""The drop-in API under CUDA graph capture and with cached intersect capacities.

The renderer sizes its intersect buffers from the previous frame of the same
shape.  An eager frame that outgrows them is binned again with the exact
sizes (same result as a first frame); a frame enqueued under graph capture
reads nothing back, so an overflow there leaves the status word set and the
image NaN.  A training step of the API (render, MSE, SSIM, backward, Adam)
captured into a CUDA graph by the caller replays to the eager results.
"""
import numpy as np
import pytest
import torch

import oracle
from repo_b200 import scenes

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _scene(radius_lo, radius_hi, seed=5, paths=48, h=256, w=256):
    return scenes.circles_scene(seed, h, w, paths, 4, 8, 6, rmin=radius_lo, rmax=radius_hi)


def _fill_args(sc):
    return (sc.cubics_norm().to(DEV), sc.seg_offsets().to(DEV), sc.colors.to(DEV),
            sc.opacities.to(DEV), sc.depths.to(DEV), sc.height, sc.width, 16, 16,
            sc.background.to(DEV))


def _oracle_image(sc):
    st = oracle.render_fill(sc.cubics_norm().numpy(), sc.seg_offsets().numpy(),
                            sc.colors.numpy(), sc.opacities.numpy(), sc.depths.numpy(),
                            sc.height, sc.width, sc.background.numpy(),
                            fill_rules=sc.fill_rules.numpy(), aa_widths=sc.aa_widths.numpy(),
                            samples=sc.samples)
    return st["image"]


def test_frame_that_outgrows_the_cached_capacity_is_binned_again():
    import manbo
    from repo_b200 import _ext
    _ext.load().forget_capacities()
    small, big = _scene(2.0, 3.0), _scene(90.0, 120.0)
    assert small.num_paths == big.num_paths and small.height == big.height
    kw = dict(fill_rules=small.fill_rules.to(DEV), aa_widths=small.aa_widths.to(DEV),
              distance_samples=small.samples)
    manbo.ops.render_cubic_fill_splat_tilelang(*_fill_args(small), **kw)  # caches a small size
    out = manbo.ops.render_cubic_fill_splat_tilelang(*_fill_args(big), **kw)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - _oracle_image(big)).max() <= 1e-6
    # and back: a smaller frame fits the grown buffers
    out = manbo.ops.render_cubic_fill_splat_tilelang(*_fill_args(small), **kw)
    assert np.abs(out.cpu().numpy() - _oracle_image(small)).max() <= 1e-6


def test_capture_before_an_eager_frame_of_the_shape_is_refused():
    from repo_b200 import _ext, render
    _ext.load().forget_capacities()
    sc = _scene(5.0, 20.0, seed=6)
    a = _fill_args(sc)
    raw = sc.aa_widths.to(DEV)
    rules = sc.fill_rules.to(DEV)
    basis = render.bernstein_basis(sc.samples, DEV)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with pytest.raises(RuntimeError, match="outside CUDA graph capture"):
        with torch.cuda.graph(g, stream=s):
            _ext.load().render_forward(a[0], a[1], a[2], a[3], a[4], rules, None, raw, a[9],
                                       basis, sc.height, sc.width, sc.samples, 1.0, False, 0,
                                       -1, False)
    torch.cuda.synchronize()


def test_captured_overflow_poisons_the_image_and_sets_the_status():
    from repo_b200 import _ext, _native, render
    ext = _ext.load()
    ext.forget_capacities()
    small, big = _scene(2.0, 3.0, seed=7), _scene(90.0, 120.0, seed=7)
    cn = small.cubics_norm().to(DEV).contiguous()
    a = _fill_args(small)
    raw = small.aa_widths.to(DEV)
    rules = small.fill_rules.to(DEV)
    basis = render.bernstein_basis(small.samples, DEV)

    def fwd():
        return ext.render_forward(cn, a[1], a[2], a[3], a[4], rules, None, raw, a[9], basis,
                                  small.height, small.width, small.samples, 1.0, False, 0, -1,
                                  False)

    fwd()  # eager: caches a capacity sized for the small circles
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fwd()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out, fts, fidx, frame, _, _ = fwd()
    g.replay()
    torch.cuda.synchronize()
    assert int(frame.counters[1]) == _native.CS_OK
    assert np.abs(out.cpu().numpy() - _oracle_image(small)).max() <= 1e-6
    cn.copy_(big.cubics_norm().to(DEV))  # the same graph now sees far more intersects
    g.replay()
    torch.cuda.synchronize()
    assert int(frame.counters[1]) == _native.CS_ERR_CAPACITY
    assert torch.isnan(out).all()
    del g


class _TrainState:
    """The user's training step on the drop-in API (render, clamp + CHW, MSE,
    SSIM as a forward metric, backward, Adam)."""

    def __init__(self, sc):
        self.sc = sc
        self.ring = sc.ring.to(DEV).clone().requires_grad_(True)
        self.colors = sc.colors.to(DEV).clone().requires_grad_(True)
        self.opac, self.depths = sc.opacities.to(DEV), sc.depths.to(DEV)
        self.rules, self.aa = sc.fill_rules.to(DEV), sc.aa_widths.to(DEV)
        self.bg = sc.background.to(DEV)
        self.offs = sc.seg_offsets().to(DEV)
        self.gidx = scenes.ring_gather_index(sc.segs_per_path).to(DEV)
        self.half = torch.tensor([0.5 * sc.width, 0.5 * sc.height], device=DEV)
        self.target = sc.target.to(DEV)
        self.opt = torch.optim.Adam([{"params": [self.ring], "lr": 0.5},
                                     {"params": [self.colors], "lr": 0.01}], capturable=True)
        self.loss = None

    def step(self):
        import manbo
        sc = self.sc
        self.opt.zero_grad(set_to_none=False)
        cn = self.ring[:, self.gidx, :].reshape(-1, 4, 2) / self.half - 1.0
        out = manbo.ops.render_cubic_fill_splat_tilelang(
            cn, self.offs, self.colors, self.opac, self.depths, sc.height, sc.width, 16, 16,
            self.bg, fill_rules=self.rules, aa_widths=self.aa, distance_samples=sc.samples)
        img = torch.clamp(out, 0, 1).permute(2, 0, 1).unsqueeze(0).contiguous()
        loss = manbo.mse_loss_tilelang(img, self.target)
        with torch.no_grad():
            self.ssim = manbo.ssim(img.detach(), self.target)
        loss.backward()
        self.opt.step()
        self.loss = loss.detach()

    def reset(self):
        """Back to the starting parameters and an empty optimiser state (in
        place, so that a captured graph keeps its addresses)."""
        with torch.no_grad():
            self.ring.copy_(self.sc.ring.to(DEV))
            self.colors.copy_(self.sc.colors.to(DEV))
            for st in self.opt.state.values():
                for v in st.values():
                    v.zero_()


def test_api_training_step_captured_in_a_graph_replays_to_the_eager_result():
    sc = scenes.circles_scene(9, 128, 160, 24, 4, 8, 6)
    n = 4
    eager = _TrainState(sc)
    losses_e, ssim_e = [], []
    for _ in range(n):
        eager.step()
        losses_e.append(float(eager.loss))
        ssim_e.append(float(eager.ssim))
    graphed = _TrainState(sc)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up: optimiser state, gradients, capacity cache
        graphed.step()
        graphed.step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphed.reset()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        graphed.step()
    losses_g, ssim_g = [], []
    for _ in range(n):
        g.replay()
        losses_g.append(float(graphed.loss))
        ssim_g.append(float(graphed.ssim))
    np.testing.assert_allclose(losses_g, losses_e, rtol=1e-4, atol=0)
    np.testing.assert_allclose(ssim_g, ssim_e, rtol=1e-4, atol=0)
    del g
