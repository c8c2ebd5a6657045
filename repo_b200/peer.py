"""Peer-memory buffers for the band-parallel training step (one process per GPU).

Each rank allocates one symmetric buffer (torch symmetric memory: the same
size on every rank, each rank holding device pointers to all the others'
copies, reached over NVLink / NVSwitch) with this layout, every region
256-byte aligned:

  flags   uint32 [2][world]   slot 0: "my gradients of step t are complete",
                              slot 1: "the first rows of my band for step t
                              are in my halo region"; word [slot][q] is
                              written by rank q
  grads   float32 [2][n]      this rank's flat gradient buffer of even / odd
                              steps ([primitive gradients | sse, mse | SSIM
                              sums]); step t writes buffer t % 2 while the
                              fused kernel of step t clears buffer (t+1) % 2
  halo    float32 [C, R, W]   the first R rows of this rank's band

The kernels behind it (repo_b200/csrc/collective.cu: cs_peer_signal,
cs_peer_wait_copy, cs_allreduce_adam) replace the library all-reduce and
all-gather of the step: every rank reads every rank's gradients through peer
pointers, sums them in rank order and takes the optimiser step, and reads the
next rank's halo rows directly.  All waits are bounded (CS_ERR_TIMEOUT in the
trainer's status word instead of a hang).
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _native as nat

FLAG_GRADS = 0
FLAG_HALO = 1
SPIN_LIMIT = 1 << 22  # polls (each followed by a 64 ns sleep) before a wait gives up


def _align(n: int, a: int = 256) -> int:
    return (int(n) + a - 1) // a * a


def buffer_layout(world: int, n_grad: int, halo_shape: Sequence[int]) -> dict:
    """Byte offsets of the regions of one rank's symmetric buffer (flags,
    gradients of even and odd steps, halo rows), each 256-byte aligned, and
    its total size; the same on every rank."""
    halo_elems = 1
    for v in halo_shape:
        halo_elems *= int(v)
    off = 0
    flags = off
    off += _align(2 * int(world) * 4)
    grads = []
    for _ in range(2):
        grads.append(off)
        off += _align(int(n_grad) * 4)
    halo = off
    off += _align(halo_elems * 4)
    return {"flags": flags, "grads": grads, "halo": halo, "halo_elems": halo_elems,
            "nbytes": off}


class PeerGroup:
    """One symmetric buffer per rank of `group` (collective: every rank
    constructs it with the same sizes)."""

    def __init__(self, group, device: torch.device, n_grad: int, halo_shape: Sequence[int]):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.device = torch.device(device)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.n_grad = int(n_grad)
        self.halo_shape = tuple(int(v) for v in halo_shape)
        lay = buffer_layout(self.world, self.n_grad, self.halo_shape)
        halo_elems = lay["halo_elems"]
        self.off_flags = lay["flags"]
        self.off_grads = list(lay["grads"])
        self.off_halo = lay["halo"]
        self.nbytes = lay["nbytes"]
        self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        if ptrs[self.rank] != self.buf.data_ptr():
            raise RuntimeError("symmetric buffer: the local pointer does not match the tensor")
        i64 = dict(dtype=torch.int64, device=self.device)
        self.flag_ptrs = torch.tensor([p + self.off_flags for p in ptrs], **i64)
        self.grad_ptrs = [torch.tensor([p + o for p in ptrs], **i64) for o in self.off_grads]
        self.halo_ptrs = [p + self.off_halo for p in ptrs]
        self.flags = self.buf[self.off_flags:self.off_flags + 2 * self.world * 4].view(torch.int32)
        self.grads = [self.buf[o:o + self.n_grad * 4].view(torch.float32) for o in self.off_grads]
        self.halo = self.buf[self.off_halo:self.off_halo + halo_elems * 4].view(
            torch.float32).view(self.halo_shape)
        self.ws = torch.zeros((int(nat.call("cs_allreduce_adam_workspace_size")),),
                              dtype=torch.uint8, device=self.device)

    def signal(self, slot: int, epoch: torch.Tensor, only_peer: int = -1) -> None:
        """Store step *epoch + 1 into word [slot][rank] of every rank's flags
        (or of rank only_peer), after the current stream's earlier work."""
        nat.check(nat.call("cs_peer_signal", self.flag_ptrs.data_ptr(), self.rank, self.world,
                           int(slot), epoch.data_ptr(), 1, int(only_peer),
                           nat.stream(self.device)), "cs_peer_signal")

    def wait_copy(self, slot: int, from_rank: int, epoch: torch.Tensor, status: torch.Tensor,
                  src_ptr, src_plane_stride: int, dst: torch.Tensor, dst_offset: int,
                  dst_plane_stride: int, plane_elems: int, planes: int) -> None:
        """Wait (bounded) for rank from_rank's word [slot] to reach *epoch + 1,
        then copy `planes` blocks of plane_elems floats from src_ptr to dst
        (dst_offset floats in)."""
        dptr = dst.data_ptr() + 4 * int(dst_offset) if dst is not None else None
        nat.check(nat.call("cs_peer_wait_copy", self.flags.data_ptr(), int(slot), self.world,
                           int(from_rank), epoch.data_ptr(), 1, SPIN_LIMIT, status.data_ptr(),
                           src_ptr, int(src_plane_stride), dptr, int(dst_plane_stride),
                           int(plane_elems), int(planes), nat.stream(self.device)),
                  "cs_peer_wait_copy")

    def allreduce_adam(self, parity: int, params, exp_avg, exp_avg_sq, n: int, n_first: int,
                       n_tail: int, tail_out, lr, betas, eps, step, status) -> None:
        """One Adam step with the gradients of every rank (buffer `parity`)
        summed in rank order; clears this rank's buffer 1 - parity."""
        nat.check(nat.call("cs_allreduce_adam", self.grad_ptrs[parity].data_ptr(), self.world,
                           params.data_ptr(), exp_avg.data_ptr(), exp_avg_sq.data_ptr(), int(n),
                           int(n_first), int(n_tail), tail_out.data_ptr(),
                           self.grads[1 - parity].data_ptr(), float(lr[0]), float(lr[1]),
                           float(betas[0]), float(betas[1]), float(eps), step.data_ptr(),
                           self.flags.data_ptr(), FLAG_GRADS, SPIN_LIMIT, status.data_ptr(),
                           self.ws.data_ptr(), nat.stream(self.device)), "cs_allreduce_adam")


__all__ = ["PeerGroup", "buffer_layout", "FLAG_GRADS", "FLAG_HALO", "SPIN_LIMIT"]
