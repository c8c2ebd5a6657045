"""4-connected component labelling with the reference's names and signatures
(manbo/ops/connected_components.py:98-283), on the B200 union-find kernels
(repo_b200.components).

One difference: the reference relaxes labels one sweep per launch and raises
RuntimeError when max_iters sweeps do not converge; the union-find always
converges, so max_iters is only validated and no such error is raised."""
from repo_b200.components import (
    DEFAULT_MAX_ITERS,
    DEFAULT_THREADS,
    connected_components_labels_4 as _labels_4,
    connected_components_with_stats_4 as _with_stats_4,
    select_largest_component_center,
)


def connected_components_labels_4_tilelang(mask, *, max_iters: int = DEFAULT_MAX_ITERS,
                                           threads: int = DEFAULT_THREADS):
    return _labels_4(mask, max_iters=int(max_iters), threads=int(threads))


def connected_components_with_stats_4_tilelang(mask, *, max_iters: int = DEFAULT_MAX_ITERS,
                                               threads: int = DEFAULT_THREADS):
    return _with_stats_4(mask, max_iters=int(max_iters), threads=int(threads))


__all__ = ["connected_components_labels_4_tilelang", "connected_components_with_stats_4_tilelang",
           "select_largest_component_center", "DEFAULT_MAX_ITERS", "DEFAULT_THREADS"]
