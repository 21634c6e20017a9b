"""Device-side bounded wait: a barrier whose peer never arrives must end by itself, leave a status
word for the host and keep the context usable.  The missing peer is a flag that nothing sets."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_wait_expires_and_context_survives():
    from modded_nanogpt_b200.ops import native
    from modded_nanogpt_b200.runtime.health import DeviceWaitTimeout, check_device
    lib = native.lib()
    dev = torch.device("cuda", 0)
    check_device(dev)
    pads = torch.zeros(2, 64, dtype=torch.int32, device=dev)     # pad of "rank 0" and of a rank 1 that never runs
    ptrs = [pads[0].data_ptr(), pads[1].data_ptr()]
    torch.cuda.synchronize()
    t0 = time.time()
    lib.peer_barrier(ptrs, 0, 1, pads)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert 0.5 < dt < 10.0, dt                                   # the wait ran out, by itself
    assert int(pads[0, 0]) == 1 and int(pads[1, 0]) == 1         # our own arrival was published to both pads
    with pytest.raises(DeviceWaitTimeout):
        check_device(dev)
    check_device(dev)                                            # the word is cleared by the read
    x = torch.randn(256, 256, device=dev, dtype=torch.bfloat16)  # the context still runs kernels
    assert torch.isfinite((x @ x).float().sum())
    pads[0, 1] = 2                                               # a peer that did arrive: no timeout
    lib.peer_barrier(ptrs, 0, 2, pads)
    check_device(dev)
