"""The device-resident training step (repo_b200.train.FillTrainer) against the
autograd path through the drop-in manbo API, on the GPU."""
import numpy as np
import pytest
import torch

from conftest import rel_l2
from repo_b200 import scenes
from repo_b200.train import FillTrainer

pytestmark = pytest.mark.gpu


def _api_step(sc, dev):
    import manbo
    h, w = sc.height, sc.width
    ring = sc.ring.to(dev).clone().requires_grad_(True)
    colors = sc.colors.to(dev).clone().requires_grad_(True)
    gidx = scenes.ring_gather_index(sc.segs_per_path).to(dev)
    half = torch.tensor([0.5 * w, 0.5 * h], device=dev)
    cn = ring[:, gidx, :].reshape(-1, 4, 2) / half - 1.0
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        cn, sc.seg_offsets().to(dev), colors, sc.opacities.to(dev), sc.depths.to(dev), h, w, 16,
        16, sc.background.to(dev), fill_rules=sc.fill_rules.to(dev),
        aa_widths=sc.aa_widths.to(dev), distance_samples=sc.samples)
    img = torch.clamp(out, 0, 1).permute(2, 0, 1).unsqueeze(0).contiguous()
    target = sc.target.to(dev)
    loss = manbo.mse_loss_tilelang(img, target)
    s = manbo.ssim(img.detach(), target)
    loss.backward()
    return out.detach(), float(loss), float(s), ring.grad, colors.grad


@pytest.mark.parametrize("seed", [31, 32])
def test_fused_step_matches_api_autograd(seed):
    dev = torch.device("cuda")
    sc = scenes.small_fill_scene(seed, h=64, w=80, paths=9)
    tr = FillTrainer(sc, dev)
    tr.forward_backward()
    out, loss, s, g_ring, g_col = _api_step(sc, dev)
    torch.cuda.synchronize()
    assert torch.equal(tr.out, out)
    assert abs(tr.loss_value() - loss) <= 1e-6 * max(loss, 1e-12) + 1e-9
    assert abs(tr.ssim_value() - s) <= 1e-5
    assert rel_l2(tr.v_ring.view_as(g_ring).cpu().numpy(), g_ring.cpu().numpy()) <= 1e-4
    assert rel_l2(tr.v_colors.view_as(g_col).cpu().numpy(), g_col.cpu().numpy()) <= 1e-4
    assert float(tr.v_edges.abs().max()) == 0.0, "edge gradients are cleared once consumed"


def test_adam_kernel_matches_host_adam_and_clears_grads():
    dev = torch.device("cuda")
    sc = scenes.small_fill_scene(40, h=48, w=64, paths=6)
    tr = FillTrainer(sc, dev, lr_points=0.5, lr_colors=0.01)
    p = tr.params.double().cpu().numpy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    lr = np.where(np.arange(p.size) < tr.n_ring, 0.5, 0.01)
    for t in range(1, 4):
        tr.forward_backward()
        g = tr.flat_grad[:tr.n_params].double().cpu().numpy()
        tr.optimizer_step()
        m = 0.9 * m + 0.1 * g
        v = 0.999 * v + 0.001 * g * g
        p = p - lr * (m / (1 - 0.9 ** t)) / (np.sqrt(v / (1 - 0.999 ** t)) + 1e-8)
        got = tr.params.double().cpu().numpy()
        assert np.abs(got - p).max() <= 1e-4, t
        p = got  # follow the device state so rounding does not compound
        assert float(tr.flat_grad[:tr.n_params].abs().max()) == 0.0
    assert int(tr.step_count.item()) == 3


def test_graph_replay_matches_eager_steps():
    dev = torch.device("cuda")
    sc = scenes.small_fill_scene(50, h=64, w=96, paths=12)
    a = FillTrainer(sc, dev)
    b = FillTrainer(sc, dev, capacity=(a.capacity, a.dcapacity))
    b.capture(warmup=0)
    losses_a, losses_b = [], []
    for _ in range(6):
        a.step_eager()
        b.step()
        losses_a.append(a.loss_value())
        losses_b.append(b.loss_value())
    n, status = b.check_status()
    assert status == 0 and n > 0
    np.testing.assert_allclose(losses_a, losses_b, rtol=1e-4)
    assert rel_l2(b.params.cpu().numpy(), a.params.cpu().numpy()) <= 1e-4


def test_capacity_overflow_is_reported_not_out_of_bounds():
    dev = torch.device("cuda")
    sc = scenes.small_fill_scene(60, h=64, w=80, paths=10)
    tr = FillTrainer(sc, dev, capacity=(8, 64))
    tr.forward_backward()
    _, status = tr.check_status()
    assert status == 2  # CS_ERR_CAPACITY
    # everything renders as background; nothing was written out of bounds
    bg = sc.background.to(dev).view(1, 1, 3).expand_as(tr.out)
    assert torch.equal(tr.out, bg)


def test_config2_training_reduces_loss():
    dev = torch.device("cuda")
    tr = FillTrainer(scenes.config2(), dev)
    tr.capture()
    tr.step()
    first = tr.loss_value()
    for _ in range(60):
        tr.step()
    torch.cuda.synchronize()
    _, status = tr.check_status()
    assert status == 0
    assert tr.loss_value() < 0.8 * first


def test_band_gradients_sum_to_the_full_image_gradient():
    """The multi-GPU band layout, emulated on one GPU: each band renders its own
    rows bit-exactly and the sum of the bands' gradient buffers (what the
    all-reduce forms) is the full-image gradient."""
    from repo_b200.bands import balanced_bands, tile_row_work
    dev = torch.device("cuda")
    sc = scenes.small_fill_scene(70, h=96, w=80, paths=14)
    full = FillTrainer(sc, dev, with_ssim=False)
    full.forward_backward()
    bands = balanced_bands(tile_row_work(sc, dev), 3)
    assert len({b for b in bands}) == 3
    parts = [FillTrainer(sc, dev, with_ssim=False, tile_rows=b) for b in bands]
    for t in parts:
        t.forward_backward()
    torch.cuda.synchronize()
    n = full.n_params
    total = sum(t.flat_grad for t in parts)
    assert rel_l2(total[:n].cpu().numpy(), full.flat_grad[:n].cpu().numpy()) <= 1e-5
    assert abs(float(total[n]) - float(full.flat_grad[n])) <= 1e-5 * float(full.flat_grad[n])
    assert abs(float(total[n + 1]) - float(full.flat_grad[n + 1])) <= 1e-5 * float(full.flat_grad[n + 1])
    for t, (r0, r1) in zip(parts, bands):
        rows = slice(r0 * 16, min(sc.height, r1 * 16))
        assert torch.equal(t.out[rows], full.out[rows])


def test_band_ssim_sums_add_up_to_the_whole_image_ssim():
    """Band SSIM of the fused step (FillTrainer with tile_rows and a halo):
    each band's per-plane SSIM output sums, from its own rows plus the next
    band's first rows, add up to the whole image's."""
    from repo_b200.train import FillTrainer
    dev = torch.device("cuda")
    sc = scenes.config1()
    full = FillTrainer(sc, dev, with_ssim=True)
    full.forward_backward()
    torch.cuda.synchronize()
    img = full.img_chw.clone()
    h, w = sc.height, sc.width
    want = full.ssim_planes.double() * float((h - 10) * (w - 10))
    tby = (h + 15) // 16
    total = torch.zeros(3, dtype=torch.float64, device=dev)
    for r0, r1 in ((0, 5), (5, 9), (9, tby)):
        y1 = min(r1 * 16, h)

        def gather(send, y1=y1):
            n = min(send.shape[1], h - y1)
            if n <= 0:
                return None
            out = torch.zeros_like(send)
            out[:, :n] = img[:, y1:y1 + n]
            return out

        tr = FillTrainer(sc, dev, with_ssim=True, tile_rows=(r0, r1), halo_gather=gather)
        tr.forward_backward()
        torch.cuda.synchronize()
        total += tr.ssim_sums.double()
    torch.testing.assert_close(total, want, rtol=1e-5, atol=0)
