"""Host logic of the multi-GPU band layout: the band split and the gradient
all-reduce hook, the latter between two gloo ranks on the CPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from repo_b200.bands import allreduce_hook, balanced_bands


def test_bands_cover_rows_once_and_in_order():
    work = [5, 1, 1, 9, 2, 2, 2, 7, 0, 3, 4]
    for parts in (1, 2, 3, 4, 8, 11):
        bands = balanced_bands(work, parts)
        assert len(bands) == parts
        assert bands[0][0] == 0 and bands[-1][1] == len(work)
        for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
            assert a1 == b0
        assert all(r1 > r0 for r0, r1 in bands), "every band non-empty when rows >= parts"


def test_bands_minimise_the_largest_band():
    work = [1, 1, 1, 1, 10, 1, 1, 1]
    bands = balanced_bands(work, 3)
    loads = [sum(work[a:b]) for a, b in bands]
    assert max(loads) == 10  # the heavy row alone; no split can do better
    brute = min(max(sum(work[:i]), sum(work[i:j]), sum(work[j:]))
                for i in range(1, 7) for j in range(i + 1, 8))
    assert max(loads) == brute


def test_more_parts_than_rows_gives_trailing_empty_bands():
    bands = balanced_bands([3, 4], 4)
    assert bands == [(0, 1), (1, 2), (2, 2), (2, 2)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        # partial gradients of all primitives + [band sse, band mse]
        flat = torch.arange(10, dtype=torch.float32) * (rank + 1)
        allreduce_hook()(flat)
        out[rank] = flat.tolist()
    finally:
        dist.destroy_process_group()


def test_allreduce_hook_sums_band_gradients_across_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world,
                           join=True, start_method="spawn")
        want = (torch.arange(10, dtype=torch.float32) * 3).tolist()
        assert out[0] == want and out[1] == want


def _ssim_rank_main(rank, world, port, bands_px, seed, out):
    import numpy as np

    import oracle
    from repo_b200.bands import band_ssim

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(seed)
        h = bands_px[-1][1]
        img = torch.rand(3, h, 37, generator=g)
        tgt = torch.rand(3, h, 37, generator=g)
        # only this rank's rows are valid: the others are overwritten
        mine = img.clone()
        y0, y1 = bands_px[rank]
        mine[:, :y0] = float("nan")
        mine[:, y1:] = float("nan")

        def plane_means(x, y):
            m = oracle.ssim_map(x.unsqueeze(0).numpy(), y.unsqueeze(0).numpy())
            return torch.from_numpy(m.reshape(3, -1).astype(np.float64).mean(axis=1))
        out[rank] = float(band_ssim(mine, tgt, bands_px, rank, plane_means=plane_means))
        if rank == 0:
            out["full"] = oracle.ssim(img.unsqueeze(0).numpy(), tgt.unsqueeze(0).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bands_px", [[(0, 16), (16, 45)], [(0, 16), (16, 32), (32, 45)],
                                      [(0, 16), (16, 32), (32, 36)]])
def test_band_ssim_matches_whole_image_ssim_across_gloo_ranks(bands_px):
    """Each rank holds only its band's rows; one halo exchange and one
    all-reduce give the whole image's SSIM on every rank (the last case's
    bottom band is shorter than the window and owns no output row)."""
    world = len(bands_px)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_ssim_rank_main, args=(world, _free_port(), bands_px, 5, out),
                           nprocs=world, join=True, start_method="spawn")
        for r in range(world):
            assert abs(out[r] - out["full"]) <= 1e-6, (r, out[r], out["full"])


def test_band_ssim_halo_rows():
    from repo_b200.bands import ssim_halo_rows
    bands = [(0, 16), (16, 32), (32, 36)]
    assert [ssim_halo_rows(bands, i, 36, 11) for i in range(3)] == [10, 4, 0]
    assert ssim_halo_rows([(0, 16), (16, 16)], 1, 16, 11) == 0
    with pytest.raises(ValueError, match="halo"):
        ssim_halo_rows([(0, 16), (16, 20), (20, 48)], 0, 48, 11)


def test_trainer_needs_a_halo_for_ssim_on_a_band():
    from repo_b200 import scenes
    from repo_b200.train import FillTrainer
    sc = scenes.small_fill_scene(1, h=64, w=64, paths=3)
    with pytest.raises(ValueError, match="halo_gather"):
        FillTrainer(sc, torch.device("cpu"), tile_rows=(0, 2))


def _halo_worker(rank, world, port, q):
    import torch.distributed as dist

    from repo_b200.bands import allgather_halo
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        gather = allgather_halo(rank, world)
        send = torch.full((3, 10, 7), float(rank)) + torch.arange(7.0)
        got = gather(send)
        q.put((rank, None if got is None else got.clone().numpy()))
    finally:
        dist.destroy_process_group()


def test_allgather_halo_returns_the_next_ranks_rows():
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    world = 3
    q = ctx.Queue()
    procs = [ctx.Process(target=_halo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world - 1):
        np.testing.assert_array_equal(got[r], np.full((3, 10, 7), float(r + 1)) + np.arange(7.0))
    assert got[world - 1] is None


def test_peer_buffer_layout_is_aligned_and_disjoint():
    from repo_b200.peer import buffer_layout
    for world, n, halo in ((2, 5, (3, 10, 7)), (8, 1_000_003, (3, 10, 2040)), (1, 0, (3, 0, 5))):
        lay = buffer_layout(world, n, halo)
        starts = [lay["flags"], *lay["grads"], lay["halo"]]
        sizes = [2 * world * 4, n * 4, n * 4, lay["halo_elems"] * 4]
        assert all(s % 256 == 0 for s in starts)
        for (a, sa), (b, _) in zip(zip(starts, sizes), zip(starts[1:], sizes[1:])):
            assert a + sa <= b  # regions in order, no overlap
        assert starts[-1] + sizes[-1] <= lay["nbytes"] and lay["nbytes"] % 256 == 0
