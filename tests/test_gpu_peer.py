"""Peer-memory exchange kernels on one GPU (repo_b200/csrc/collective.cu).

With a world of one rank the fused all-reduce + Adam step reads this rank's
own buffer, so it must equal the plain Adam kernel bit for bit.  Waits whose
flag nobody sets run out after their poll limit and record CS_ERR_TIMEOUT in
the status word, leaving their outputs untouched: the failure path is tested
without hanging or faulting anything.  (The cross-GPU path is
tests/test_gpu_peer_multi.py, which needs two GPUs.)
"""
import numpy as np
import pytest
import torch

from repo_b200 import _native as nat

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _ptrs(*tensors):
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device=DEV)


def _adam_inputs(n, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda s=1.0: (torch.randn(n, generator=g) * s).to(DEV)  # noqa: E731
    return mk(), mk(1e-2), mk(1e-2).abs(), mk(1e-3)  # params, m, v, grads


@pytest.mark.parametrize("n", [13824, 13827])  # vector path and scalar path
def test_world_of_one_equals_the_adam_kernel(n):
    p, m, v, g = _adam_inputs(n, 3)
    tail = torch.arange(5, dtype=torch.float32, device=DEV)
    grads = torch.cat([g, tail])  # [gradients | tail]
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    step = torch.tensor([4], dtype=torch.int32, device=DEV)
    step2 = step.clone()
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    clear = torch.ones(n + 5, device=DEV)
    tail_out = torch.zeros(5, device=DEV)
    ws = torch.zeros(256, dtype=torch.uint8, device=DEV)
    st = nat.stream(DEV)
    fptrs = _ptrs(flags)
    nat.check(nat.call("cs_peer_signal", fptrs.data_ptr(), 0, 1, 0, step.data_ptr(), 1, -1, st),
              "cs_peer_signal")
    nat.check(nat.call("cs_allreduce_adam", _ptrs(grads).data_ptr(), 1, p.data_ptr(), m.data_ptr(),
                       v.data_ptr(), n, 5000, 5, tail_out.data_ptr(), clear.data_ptr(), 0.5, 0.01,
                       0.9, 0.999, 1e-8, step.data_ptr(), flags.data_ptr(), 0, 1 << 20,
                       status.data_ptr(), ws.data_ptr(), st), "cs_allreduce_adam")
    adam_ws = torch.zeros(int(nat.call("cs_adam_workspace_size")), dtype=torch.uint8, device=DEV)
    g2 = g.clone()
    nat.check(nat.call("cs_adam_step", p2.data_ptr(), g2.data_ptr(), m2.data_ptr(), v2.data_ptr(),
                       n, 5000, 0.5, 0.01, 0.9, 0.999, 1e-8, step2.data_ptr(), adam_ws.data_ptr(),
                       0, st), "cs_adam_step")
    torch.cuda.synchronize()
    assert int(status) == 0 and int(flags[0]) == 5
    assert torch.equal(p, p2) and torch.equal(m, m2) and torch.equal(v, v2)
    assert int(step) == int(step2) == 5
    assert torch.equal(tail_out, tail) and not clear.any()


def test_wait_without_a_signal_times_out_and_copies_nothing():
    flags = torch.zeros(4, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    epoch = torch.tensor([0], dtype=torch.int32, device=DEV)
    src = torch.arange(64, dtype=torch.float32, device=DEV)
    dst = torch.full((64,), -1.0, device=DEV)
    nat.check(nat.call("cs_peer_wait_copy", flags.data_ptr(), 1, 2, 1, epoch.data_ptr(), 1, 2000,
                       status.data_ptr(), src.data_ptr(), 32, dst.data_ptr(), 32, 32, 2,
                       nat.stream(DEV)), "cs_peer_wait_copy")
    torch.cuda.synchronize()
    assert int(status) == nat.CS_ERR_TIMEOUT
    assert torch.equal(dst, torch.full((64,), -1.0, device=DEV))
    # once the flag holds the step, the same call copies
    flags[1 * 2 + 1] = 1
    status.zero_()
    nat.check(nat.call("cs_peer_wait_copy", flags.data_ptr(), 1, 2, 1, epoch.data_ptr(), 1, 2000,
                       status.data_ptr(), src.data_ptr(), 32, dst.data_ptr(), 32, 32, 2,
                       nat.stream(DEV)), "cs_peer_wait_copy")
    torch.cuda.synchronize()
    assert int(status) == 0 and torch.equal(dst, src)


def test_allreduce_adam_without_all_flags_times_out_and_leaves_params():
    n = 1024
    p, m, v, g = _adam_inputs(n, 5)
    before = p.clone()
    world = 2  # rank 1's flag never arrives
    flags = torch.zeros(2 * world, dtype=torch.int32, device=DEV)
    flags[0] = 1
    step = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ws = torch.zeros(256, dtype=torch.uint8, device=DEV)
    tail_out = torch.zeros(1, device=DEV)
    nat.check(nat.call("cs_allreduce_adam", _ptrs(g, g).data_ptr(), world, p.data_ptr(),
                       m.data_ptr(), v.data_ptr(), n, n, 0, tail_out.data_ptr(), None, 0.5, 0.5,
                       0.9, 0.999, 1e-8, step.data_ptr(), flags.data_ptr(), 0, 2000,
                       status.data_ptr(), ws.data_ptr(), nat.stream(DEV)), "cs_allreduce_adam")
    torch.cuda.synchronize()
    assert int(status) == nat.CS_ERR_TIMEOUT
    assert torch.equal(p, before) and int(step) == 0
    assert int(ws[:4].view(torch.int32)) == 0  # the completion ticket is reset for the next call
