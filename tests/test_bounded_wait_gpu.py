"""Bounded waits of the peer-memory kernels, tested without a GPU fault.

The tensor-parallel all-reduce kernel (``csrc/collectives.cu``) publishes an epoch into every
rank's flag array and waits, with a 2 s limit, until every rank's epoch has arrived in its own. Here
one process plays rank 0 of a 2-rank group whose "peer" buffers are ordinary local allocations:
  * when the peer's flag was set in advance (as a live peer would set it) the kernel completes and
    returns the rank-ordered sum plus the residual;
  * when nothing ever sets the peer's flag the wait runs out, the kernel records
    ``kStatusTimeoutPeer`` (4), skips the reduction and returns, and the context stays usable.
The reference has no device-side waits; its host-side counterparts are the replay-sample deadline
(``accerl_agent/agent_textworld.py:688-706``) and the rollout stop timeout
(``accerl_agent/vllm_fsdp.py:2214``).
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

from accerl_agent_b200 import ops

TIMEOUT_PEER = 4


def _fake_group(n, world=2):
    dev = torch.device("cuda", 0)
    bufs = [torch.randn(2 * n, device=dev).to(torch.bfloat16) for _ in range(world)]
    flags = [torch.zeros(2 * world, dtype=torch.int32, device=dev) for _ in range(world)]
    data_ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    flag_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=dev)
    ctr = torch.zeros(2, dtype=torch.int32, device=dev)
    return bufs, flags, data_ptrs, flag_ptrs, ctr


@pytest.mark.parametrize("slot", [0, 1])
def test_tp_allreduce_completes_when_peer_flag_arrives(slot):
    n = 4096 + 24  # a vector body and a scalar tail
    bufs, flags, dp, fp, ctr = _fake_group(n)
    world = 2
    flags[0][slot * world + 1] = 1  # the peer's epoch 1, already delivered
    residual = torch.randn(n, device="cuda").to(torch.bfloat16)
    out = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(16, dtype=torch.int32, device="cuda")  # private: the shared word stays clean
    ops.native().tp_allreduce(dp, fp, 0, slot, n, n, residual, out, ctr, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    assert int(ctr[0]) == 1 and int(ctr[1]) == 0
    # this rank's epoch was published to both ranks' flag arrays
    assert int(flags[0][slot * world + 0]) == 1 and int(flags[1][slot * world + 0]) == 1
    base = slot * n
    ref = residual.float() + bufs[0][base : base + n].float() + bufs[1][base : base + n].float()
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=2e-2)


def test_tp_allreduce_peer_that_never_signals_times_out():
    n = 8192
    bufs, flags, dp, fp, ctr = _fake_group(n)
    out = torch.full((n,), 7.0, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(16, dtype=torch.int32, device="cuda")  # private: the shared word stays clean
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ops.native().tp_allreduce(dp, fp, 0, 0, n, n, None, out, ctr, status)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status[0]) == TIMEOUT_PEER
    assert 1.5 < dt < 30.0, dt
    # the reduction was skipped, and the device still runs work afterwards
    assert torch.all(out == 7.0)
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    # the wrapper's host check turns the status into an error
    from accerl_agent_b200.parallel.tp_allreduce import TPAllReduce

    fake = TPAllReduce.__new__(TPAllReduce)
    fake.status = status
    with pytest.raises(RuntimeError, match="timed out"):
        fake.check()
