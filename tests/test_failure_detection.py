"""Failure detection without a GPU fault: every spin-wait in the kernels is bounded, and a
wait that runs out records a code in the device status word and lets the kernel return.
Here the cross-GPU barrier waits (on one GPU) for a peer flag that nothing ever sets; the
call must come back after its ~2 s limit with status 60, and the context must stay usable."""
import pytest
import torch


@pytest.mark.gpu
def test_barrier_wait_runs_out_and_reports():
    from dsalt_b200 import _lib as L
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    assert ops.device_status() == 0
    own = torch.zeros(4, dtype=torch.int32, device=dev)
    never_set = torch.zeros(4, dtype=torch.int32, device=dev)  # the "peer": nothing writes it
    table = torch.tensor([own.data_ptr(), never_set.data_ptr()], dtype=torch.int64, device=dev)
    L.call("dsalt_peer_barrier", own.data_ptr(), table.data_ptr(), 2, 0, 1, torch.cuda.current_stream().cuda_stream)
    # the asynchronous read (what ShardedCore queues after every step) sees the code too
    host = torch.zeros(1, dtype=torch.int32).pin_memory()
    L.call("dsalt_device_status_async", host.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(own[0]) == 1          # this rank published its epoch
    assert int(host[0]) == 60
    assert ops.device_status() == 60  # and gave up waiting for the peer
    # the context still works
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    assert ops.device_status() == 0
