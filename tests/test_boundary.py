"""The C-ABI library and the drop-in Python surface (no GPU needed)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "cubicsplat_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^CS_API [^;]*?\b(cs_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 20
    for required in ["cs_project_cubics", "cs_bin_count", "cs_bin_sort", "cs_fill_forward",
                     "cs_fill_backward", "cs_stroke_forward", "cs_stroke_backward",
                     "cs_mse_forward", "cs_ssim", "cs_ring_segments_forward"]:
        assert required in syms


def test_library_loads_and_exports_every_declared_symbol():
    from repo_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        from repo_b200 import build
        build.build()
    lib = ctypes.CDLL(_native.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) == set(_native.SIGNATURES), "ctypes table out of sync"
    lib.cs_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.cs_version()


def test_workspace_size_queries_need_no_gpu():
    from repo_b200 import _native
    assert _native.call("cs_bin_workspace_size", 1536) >= 2 * 4 * 1536
    assert _native.call("cs_mse_workspace_size", 1 << 20) > 0
    assert _native.call("cs_ssim_workspace_size", 3, 512, 768, 11) > 0


def test_manbo_surface_imports():
    import manbo
    import manbo.ops as ops
    for name in ["mse_loss_tilelang", "psnr", "ssim", "Adan", "gs_render",
                 "regularization_loss_tilelang", "set_gs_profile_ctx_factory"]:
        assert hasattr(manbo, name)
    for name in ops.__all__:
        assert hasattr(ops, name), name
    from manbo.ops.cubic_polyline_splatting import render_cubic_polyline_splat_tilelang  # noqa
    from manbo.ops.cubic_splatting import _flatten_cubics_to_edges  # noqa
    from manbo.ops.tile_bins import get_tile_bin_edges_tilelang  # noqa


def test_out_of_scope_names_raise():
    import manbo
    import manbo.ops as ops
    with pytest.raises(NotImplementedError):
        ops.rasterize_forward_tilelang()
    with pytest.raises(NotImplementedError):
        manbo.gs_render()


def test_adan_is_a_real_optimizer_with_reference_validation():
    import torch
    import manbo
    p = torch.zeros(3, requires_grad=True)
    with pytest.raises(ValueError, match="Invalid epsilon value"):
        manbo.Adan([p], eps=-1.0)
    opt = manbo.Adan([p], lr=0.1)
    assert opt.defaults["betas"] == (0.98, 0.92, 0.99)
    p.grad = torch.ones(3)
    with pytest.raises(ValueError):  # CPU tensors: no host fallback
        opt.step()


def test_cpu_tensors_are_rejected_without_fallback():
    import torch
    import manbo
    x = torch.rand(1, 3, 16, 16)
    with pytest.raises(ValueError):
        manbo.psnr(x, x)
    with pytest.raises(ValueError):
        manbo.ops.render_cubic_fill_splat_tilelang(
            torch.zeros(4, 4, 2), torch.tensor([0, 4], dtype=torch.int32), torch.rand(1, 3),
            torch.ones(1), torch.rand(1), 32, 32, 16, 16, torch.ones(3))


def test_flatten_method_validation():
    from repo_b200.render import normalize_cubic_flatten_method
    assert normalize_cubic_flatten_method("De-Casteljau") == "de_casteljau"
    with pytest.raises(ValueError):
        normalize_cubic_flatten_method("spline")


def test_scenes_are_deterministic():
    from repo_b200 import scenes
    a, b = scenes.config2(), scenes.config2()
    assert (a.ring == b.ring).all() and (a.target == b.target).all()
    assert a.num_paths == 512 and a.cubics_norm().shape == (2048, 4, 2)
    assert scenes.config3().cubics_norm().shape == (4096 * 6, 4, 2)
    assert len(set(a.depths.tolist())) == 512


def test_workspace_and_list_sizes():
    """Sizes the host allocates from: raster workspace (dispatch counter,
    ticket, one loss partial per strip) and unit lists (64 bucket counts, one
    list of all of the band's strips per bucket)."""
    from repo_b200 import _native as nat
    for nt in (1, 7, 1536):
        assert nat.call("cs_unit_lists_size", nt) == 4 * (64 + 64 * 4 * nt)
        assert nat.call("cs_raster_workspace_size", nt) == 256 + 4 * 4 * nt


def test_entry_validation_messages_match_the_reference():
    """Size checks run before any device work, with the reference's messages
    (cubic_splatting.py:3158-3205, cubic_polyline_splatting.py:1365-1400), and
    a scene without primitives is the background (no device needed)."""
    import torch

    import manbo
    fill = manbo.ops.render_cubic_fill_splat_tilelang
    stroke = manbo.ops.render_cubic_polyline_splat_tilelang
    g, p = 6, 3
    cn = torch.zeros(g, 4, 2)
    offs = torch.tensor([0, 2, 4, 6], dtype=torch.int32)
    col, op, dep, bg = torch.zeros(p, 3), torch.ones(p), torch.arange(p).float(), torch.ones(3)
    base = (cn, offs, col, op, dep, 32, 48, 16, 16, bg)
    cases = [
        (dict(colors=torch.zeros(2, 3)), "colors first dim must match primitive count \\(3\\), got 2"),
        (dict(opacities=torch.ones(4)), "opacities size must match primitive count \\(3\\), got 4"),
        (dict(depths=torch.ones(1)), "depths size must match primitive count \\(3\\), got 1"),
    ]
    for repl, msg in cases:
        args = list(base)
        for k, v in repl.items():
            args[{"colors": 2, "opacities": 3, "depths": 4}[k]] = v
        with pytest.raises(ValueError, match=msg):
            fill(*args)
    with pytest.raises(ValueError, match="fill_rules size must match primitive count \\(3\\), got 2"):
        fill(*base, fill_rules=torch.ones(2, dtype=torch.int32))
    with pytest.raises(ValueError, match="aa_widths size must match primitive count \\(3\\), got 2"):
        fill(*base, aa_widths=torch.ones(2))
    sw = torch.ones(p)
    with pytest.raises(ValueError, match="stroke_widths size must match primitive count \\(3\\), got 5"):
        stroke(cn, offs, col, op, torch.ones(5), dep, 32, 48, 16, 16, bg)
    # the stroke entry checks stroke widths before depths, as the reference does
    with pytest.raises(ValueError, match="stroke_widths size"):
        stroke(cn, offs, col, op, torch.ones(5), dep[:1], 32, 48, 16, 16, bg)
    with pytest.raises(ValueError, match="flatten_method"):
        fill(*base, flatten_method="bezier-magic")
    # no primitives: the background, [H, W, 3]
    empty = fill(cn[:0], torch.zeros(1, dtype=torch.int32), col[:0], op[:0], dep[:0], 5, 7, 16,
                 16, torch.tensor([0.1, 0.2, 0.3]))
    assert empty.shape == (5, 7, 3) and torch.equal(empty[2, 3], torch.tensor([0.1, 0.2, 0.3]))
    empty = stroke(cn[:0], torch.zeros(1, dtype=torch.int32), col[:0], op[:0], sw[:0], dep[:0],
                   5, 7, 16, 16, torch.tensor([0.1, 0.2, 0.3]))
    assert empty.shape == (5, 7, 3)
