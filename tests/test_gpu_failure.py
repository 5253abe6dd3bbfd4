"""Failure detection without a GPU fault: a bounded device wait is made to run out (an mbarrier that
nothing completes) and must report its error status, leaving the context usable for further work."""
import pytest
import torch

from odie_b200 import _lib
from odie_b200.data import device_stratified_ids

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports(cuda):
    lib = _lib.library()
    stream = torch.cuda.current_stream()
    status = torch.full((1,), -1, dtype=torch.int32, device='cuda')
    for limit in (1, 1000):
        status.fill_(-1)
        _lib.check(lib.odie_wait_probe(limit, status.data_ptr(), stream.cuda_stream), 'odie_wait_probe')
        torch.cuda.synchronize()
        assert status.item() == 2, 'the wait on a barrier nothing completes must give up with status 2'
    # the context is still usable: a library kernel and a torch kernel run and give their results
    ids = device_stratified_ids((64, 64), 16, 1, 1)
    assert ids.shape == (16,) and int(ids.max()) < 64 * 64
    assert torch.arange(10, device='cuda').sum().item() == 45
    with pytest.raises(RuntimeError):
        _lib.check(lib.odie_wait_probe(0, status.data_ptr(), stream.cuda_stream), 'odie_wait_probe')
