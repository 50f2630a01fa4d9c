"""A bounded device wait that runs out reports through the status word.

One GPU, no peer: the signal barrier is given two "ranks" whose pads are the
same local buffer, so rank 1's flag is a flag that nothing sets. The wait
gives up after its 2 s budget, records the peer-timeout code and returns; the
host reads the code (KernelTimeoutError) and the context stays usable.
"""

import time

import pytest
import torch


@pytest.mark.gpu
def test_unanswered_barrier_times_out_and_reports():
    from representax_b200.ops._ext import KernelTimeoutError, check_status, ext, status

    device = torch.device("cuda", 0)
    check_status(device)  # start clean
    pad = torch.zeros(2, dtype=torch.int32, device=device)
    pads = torch.tensor([pad.data_ptr(), pad.data_ptr()], dtype=torch.int64, device=device)
    started = time.perf_counter()
    ext().signal_barrier(pads, 0, 2, 1, status(device))
    torch.cuda.synchronize()
    waited = time.perf_counter() - started
    assert 1.5 < waited < 30.0
    with pytest.raises(KernelTimeoutError, match="peer wait"):
        check_status(device)
    check_status(device)  # the word was cleared
    x = torch.arange(1024, device=device, dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2  # the context is still usable
