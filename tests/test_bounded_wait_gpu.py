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


def test_trainer_raises_on_device_wait_timeout():
    """A bounded wait that gave up (here: the probe's flag timeout) makes the next training
    step fail instead of carrying on with incomplete results."""
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import DeviceWaitError, Trainer
    from revpp.ops import ext
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    C = ext()
    dev = torch.device("cuda", 0)
    cfg = GlobalConfig(model="bert", reversible=True, num_hidden_layers=1, hidden_size=128, num_attention_heads=2,
                       max_position_embeddings=128, num_classes=2, autocast_dtype=torch.bfloat16, batch_size=4,
                       microbatch_size=2, num_microbatches=2, lr=1e-4)
    env = EnvContext(world_size=1, rank=0, local_rank=0, device=dev, proc_logger=build_logger("bw", None),
                     node_logger=None, main_logger=None, pg=None, master_rank=0)
    tr = Trainer(cfg, env)
    batch = SyntheticBatches(cfg, 4, 1, seed=0).make(0)
    C.status_read_and_clear()
    tr.train_step(batch)  # clean
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.flag_wait_probe(flag, 1, 0.05, result)
    torch.cuda.synchronize()
    try:
        with pytest.raises(DeviceWaitError):
            tr.train_step(batch)
    finally:
        assert C.status_read_and_clear() & FLAG_TIMEOUT
