"""cs_ssim_noalloc (fixed device scratch, no workspace argument) against cs_ssim
(caller workspace), both called through the C ABI on the GPU.

The file name sorts last so that the suite also exercises the entry point
after every other GPU test has run in the same process; it passes run alone
as well (``pytest tests/test_zz_no_alloc.py -m gpu``).
"""
import pytest
import torch

from repo_b200 import _native as nat
from repo_b200.metric import gaussian_1d

pytestmark = pytest.mark.gpu

CS_ERR_CAPACITY = 2
TOL = 1e-6  # same kernel and reduction order: expected bit-identical


def _inputs(seed, planes, h, w):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand((planes, h, w), generator=g)
    y = (x + 0.1 * torch.randn((planes, h, w), generator=g)).clamp(0, 1)
    return x.cuda().contiguous(), y.cuda().contiguous()


def _ssim_with_workspace(x, y, gauss, win, c1, c2):
    planes, h, w = x.shape
    means = torch.empty(planes, device=x.device)
    smap = torch.empty((planes, h - win + 1, w - win + 1), device=x.device)
    ws = torch.zeros(int(nat.call("cs_ssim_workspace_size", planes, h, w, win)),
                     dtype=torch.uint8, device=x.device)
    nat.check(nat.call("cs_ssim", nat.ptr(x), nat.ptr(y), nat.ptr(gauss), planes, h, w, win,
                       c1, c2, nat.ptr(means), nat.ptr(smap), ws.data_ptr(),
                       nat.stream(x.device)), "cs_ssim")
    return means, smap


def _ssim_noalloc(x, y, gauss, win, c1, c2, with_map=True):
    planes, h, w = x.shape
    means = torch.empty(planes, device=x.device)
    smap = torch.empty((planes, h - win + 1, w - win + 1), device=x.device) if with_map else None
    nat.check(nat.call("cs_ssim_noalloc", nat.ptr(x), nat.ptr(y), nat.ptr(gauss), planes, h, w,
                       win, c1, c2, nat.ptr(means), nat.ptr(smap), nat.stream(x.device)),
              "cs_ssim_noalloc")
    return means, smap


@pytest.mark.parametrize("planes,h,w", [(3, 512, 512), (2, 75, 131)])
def test_noalloc_ssim_matches_workspace_ssim_twice_in_a_row(planes, h, w):
    win, c1, c2 = 11, 0.01 ** 2, 0.03 ** 2
    x, y = _inputs(planes * 1000 + h, planes, h, w)
    gauss = gaussian_1d(win, 1.5, x.device)
    ref_means, ref_map = _ssim_with_workspace(x, y, gauss, win, c1, c2)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        means, smap = _ssim_noalloc(x, y, gauss, win, c1, c2)
        torch.cuda.synchronize()
        assert torch.allclose(means, ref_means, rtol=0, atol=TOL)
        assert torch.allclose(smap, ref_map, rtol=0, atol=TOL)
    # a different input right after: results follow the new input
    x2, y2 = _inputs(7, planes, h, w)
    ref2, _ = _ssim_with_workspace(x2, y2, gauss, win, c1, c2)
    means2, _ = _ssim_noalloc(x2, y2, gauss, win, c1, c2, with_map=False)
    torch.cuda.synchronize()
    assert torch.allclose(means2, ref2, rtol=0, atol=TOL)


def test_noalloc_ssim_rejects_sizes_beyond_its_scratch():
    # 64 planes of 600 x 600: 64 * 19 * 19 = 23104 partials fit; 256 planes do not.
    gauss = gaussian_1d(11, 1.5, torch.device("cuda"))
    means = torch.empty(256, device="cuda")
    x = torch.zeros((256, 600, 600), device="cuda")
    rc = nat.call("cs_ssim_noalloc", nat.ptr(x), nat.ptr(x), nat.ptr(gauss), 256, 600, 600, 11,
                  1e-4, 9e-4, nat.ptr(means), None, nat.stream(x.device))
    assert rc == CS_ERR_CAPACITY
    x64 = x[:64].contiguous()
    m64, _ = _ssim_noalloc(x64, x64, gauss, 11, 1e-4, 9e-4, with_map=False)
    torch.cuda.synchronize()
    assert torch.allclose(m64, torch.ones_like(m64), atol=1e-6)
