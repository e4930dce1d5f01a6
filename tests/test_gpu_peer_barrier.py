"""fpb_peer_barrier on one GPU: a barrier of one rank passes at once and
counts its epochs (and its all-reduce MAX keeps the value); a barrier whose other rank never announces gives up after
its time limit with device error 601, and the context stays usable.  (The
two-rank barrier that passes runs on two GPUs in test_gpu_nsplit_peers.py;
two waiting ranks never share one GPU.)"""
import pytest

pytestmark = pytest.mark.gpu


def _call(N, torch, counter, flags, table, nranks, rank, timeout_ms):
    N.call("fpb_peer_barrier", counter.data_ptr(), flags.data_ptr(), table.data_ptr(), nranks, rank, timeout_ms,
           torch.cuda.current_stream().cuda_stream)


def test_single_rank_passes():
    import torch

    import firepit_b200 as F
    N = F._native
    F.device_error()  # reset
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    for _ in range(3):
        _call(N, torch, counter, flags, table, 1, 0, 1000)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    assert counter.item() == 3 and flags[0].item() == 3


def test_missing_rank_times_out_with_error():
    import torch

    import firepit_b200 as F
    N = F._native
    F.device_error()
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    other = torch.zeros(8, dtype=torch.int32, device="cuda")  # stands for rank 1's flags; rank 1 never runs
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = torch.tensor([flags.data_ptr(), other.data_ptr()], dtype=torch.int64, device="cuda")
    _call(N, torch, counter, flags, table, 2, 0, 50)
    torch.cuda.synchronize()
    assert F.device_error() == 601
    assert other[0].item() == 1  # this rank's announcement reached the other rank's word
    x = torch.ones(4, device="cuda") * 2  # the context is still usable
    assert float(x.sum()) == 8.0
    with pytest.raises(Exception):
        _call(N, torch, counter, flags, table, 2, 2, 50)  # rank outside [0, nranks)


def test_single_rank_all_reduce_max_keeps_value():
    import torch

    import firepit_b200 as F
    N = F._native
    F.device_error()
    flags = torch.zeros(128, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    v = torch.tensor([12345], dtype=torch.int32, device="cuda")
    for _ in range(2):
        N.call("fpb_peer_all_reduce_max", counter.data_ptr(), flags.data_ptr(), table.data_ptr(), 1, 0, v.data_ptr(),
               1000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert F.device_error() == 0
    assert v.item() == 12345 and counter.item() == 2
