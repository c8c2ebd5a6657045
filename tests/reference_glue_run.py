"""Train the reference's own model glue (manbo.gaussian_trace.GaussianTrace,
cubic fill backend, Adan) for a few steps and print the losses as JSON.

Run as a child process by tests/test_gpu_reference_glue.py:

    python tests/reference_glue_run.py <reference install dir> b200|reference <steps> fill|stroke

With ``b200`` this repository's ``manbo`` comes first on sys.path, so the
reference's glue runs on the B200 kernels (its renderer, MSE, PSNR and Adan
imports resolve here); with ``reference`` the reference's own ``manbo`` and
TileLang kernels run.  Same seed, same target, same model initialisation.
``fill`` trains closed paths (backend ``cubic_fill``), ``stroke`` open cubic
strokes (backend ``cubic``, degree 3).  The reference repository lacks the
``visual_debug`` module its glue imports; a no-op stand-in is supplied to both
runs.
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _visual_debug_stand_in():
    import types
    mod = types.ModuleType("visual_debug")

    class VisualDebugHook:
        def __init__(self, *args, **kwargs):
            pass

        def __getattr__(self, name):
            return lambda *args, **kwargs: None

    mod.VisualDebugHook = VisualDebugHook
    mod.emit_visual_debug = lambda *args, **kwargs: None
    sys.modules["visual_debug"] = mod


def main(ref_dir: str, which: str, steps: int, kind: str) -> None:
    sys.path[:0] = [ROOT, ref_dir] if which == "b200" else [ref_dir]
    _visual_debug_stand_in()
    import torch

    import manbo
    from manbo.gaussian_trace import GaussianTrace

    dev = torch.device("cuda")
    torch.manual_seed(0)
    torch.cuda.manual_seed_all(0)
    h, w = 80, 112
    yy, xx = torch.meshgrid(torch.linspace(-1, 1, h), torch.linspace(-1, 1, w), indexing="ij")
    target = torch.stack([(xx * xx + yy * yy < 0.5).float(), 0.5 + 0.5 * torch.sin(3 * xx),
                          (yy > 0.1).float() * 0.8]).unsqueeze(0).to(dev).contiguous()
    if kind == "fill":
        cfg = dict(mode="closed", bezier_degree=4, renderer_backend="cubic_fill")
    else:
        cfg = dict(mode="unclosed", bezier_degree=3, renderer_backend="cubic")
    model = GaussianTrace(H=h, W=w, BLOCK_W=16, BLOCK_H=16, device=dev, num_curves=24,
                          num_samples=64, lr=1e-2, opt_type="adan",
                          cubic_distance_samples_train=12, cubic_distance_samples_eval=18,
                          cubic_flatten_method="bernstein", **cfg).to(dev)
    losses, psnrs = [], []
    for _ in range(steps):
        loss, p, _img = model.train_step(target, compute_psnr=True)
        losses.append(float(loss))
        psnrs.append(float(p))
    print(json.dumps({"manbo": os.path.dirname(manbo.__file__), "losses": losses,
                      "psnr": psnrs}))


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2], int(sys.argv[3]), sys.argv[4])
