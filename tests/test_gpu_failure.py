"""Failure detection on one GPU without faulting it: a bounded device wait
that runs out must end its kernel with a status the host reads (mapped to
TimeoutError), quickly when the wait budget is short, and leave the context
usable.  The flags below are never raised by anyone."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _wait(flags, G, epoch, status):
    from dsv4attn import _lib
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().dsa_p2p_wait(flags.data_ptr(), G, epoch.data_ptr(), status.data_ptr(), st), "p2p_wait")


@pytest.mark.parametrize("G,raised", [(1, 0), (4, 3)])
def test_peer_flag_wait_times_out_with_status(cuda_dev, G, raised):
    from dsv4attn import ops
    flags = torch.zeros(G, dtype=torch.int32, device=cuda_dev)
    flags[:raised] = 7                                  # some peers arrived, the last never does
    epoch = torch.full((1,), 7, dtype=torch.int32, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    torch.cuda.synchronize()
    prev = ops.set_wait_limit(4_000_000)                 # ~2 ms of SM clock
    try:
        t0 = time.time()
        _wait(flags, G, epoch, status)
        torch.cuda.synchronize()
        dt = time.time() - t0
    finally:
        ops.set_wait_limit(prev)
    assert int(status.item()) == ops.STATUS_TIMEOUT
    assert dt < 1.0, f"the wait took {dt:.3f} s with a ~2 ms budget"
    with pytest.raises(TimeoutError):
        ops.raise_for_status(status, "p2p_wait")
    # the context is still usable
    x = torch.randn(4, 448, device=cuda_dev).to(torch.bfloat16)
    y, _, _ = ops.act_quant_block(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_peer_flag_wait_passes_when_all_arrived(cuda_dev):
    from dsv4attn import ops
    flags = torch.full((3,), 9, dtype=torch.int32, device=cuda_dev)
    epoch = torch.full((1,), 9, dtype=torch.int32, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    _wait(flags, 3, epoch, status)
    ops.raise_for_status(status, "p2p_wait")


def test_wait_limit_roundtrip(cuda_dev):
    from dsv4attn import _lib, ops
    L = _lib.lib()
    prev = ops.set_wait_limit(123456)
    assert L.dsa_get_wait_limit() == 123456
    ops.set_wait_limit(0)
    assert L.dsa_get_wait_limit() == 2_000_000_000
    ops.set_wait_limit(prev)
