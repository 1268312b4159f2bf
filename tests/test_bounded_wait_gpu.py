"""Bounded device waits report an error status instead of hanging.

A one-thread kernel waits on a flag that nothing sets, with a short time limit.  The kernel
must give up, record ``kStatusFlagTimeout`` (bit value 2) in the mapped status word and
return, leaving the CUDA context usable for the next launch.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

FLAG_TIMEOUT = 2


def test_flag_wait_times_out_and_context_stays_usable():
    from revpp.ops import ext

    C = ext()
    C.status_read_and_clear()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.flag_wait_probe(flag, 1, 0.2, result)
    torch.cuda.synchronize()
    assert int(result.item()) == -1
    st = C.status_read_and_clear()
    assert st & FLAG_TIMEOUT
    # the context still works
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum().item()) == 2 * 1023 * 1024 / 2


def test_flag_wait_succeeds_when_flag_is_set():
    from revpp.ops import ext

    C = ext()
    C.status_read_and_clear()
    flag = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    result = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.flag_wait_probe(flag, 3, 1.0, result)
    torch.cuda.synchronize()
    assert int(result.item()) == 1
    assert C.status_read_and_clear() == 0
