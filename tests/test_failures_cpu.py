"""Failure detection on CPU / gloo ranks: a rank that raises or exits and a message that is
dropped make the surviving rank fail with an error within the process-group timeout
instead of waiting forever.  No GPU is involved."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, env_extra, q, extra_args=""):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), REVPP_P2P_HOST_TIMEOUT_S="8", **env_extra)
    import torch

    from revpp.config import build_global_config, parse_args
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.utils.env import build_env
    from revpp.utils.seed import set_seed

    try:
        args = parse_args(("--preset tiny-bert --num-hidden-layers 2 --reversible --par-mode pp --batch-size 8 "
                           "--microbatch-size 2 --num-microbatches 4 --device cpu " + extra_args).split())
        cfg = build_global_config(args)
        env = build_env(cfg, timeout_s=8)
        set_seed(rank)
        tr = Trainer(cfg, env)
        b = SyntheticBatches(cfg, 8, 1, seed=0).make(0)
        t0 = time.time()
        tr.train_step(b if tr.is_first else None)
        q.put((rank, "ok", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error:{type(e).__name__}", 0.0))


def _run(env_extra, timeout=90, extra_args=""):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, env_extra, q, extra_args)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while time.time() < deadline:
        try:
            r, status, _ = q.get(timeout=0.5)
            results[r] = status
        except Exception:  # noqa: BLE001
            pass
        # done when every rank has either reported or exited
        if all(r in results or procs[r].exitcode is not None for r in range(2)):
            break
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    return results, time.time() - t0


def test_clean_run_reports_ok():
    res, _ = _run({})
    assert res == {0: "ok", 1: "ok"}


def test_rank_raises_peer_fails_fast():
    res, dt = _run({"REVPP_FAULT_RAISE_AT": "1:0"})
    assert res.get(1, "").startswith("error:InjectedFault")
    assert res.get(0, "").startswith("error"), res
    assert dt < 80


def test_dropped_message_times_out():
    res, dt = _run({"REVPP_FAULT_DROP_SEND": "fwd0->1:1"})
    assert res.get(1, "").startswith("error"), res
    assert dt < 80


def test_copy_channels_clean_run_and_raising_rank():
    """Over copy channels: a clean step completes; a rank that raises mid-step marks the
    shared abort word, so its peer's next channel wait raises at once instead of waiting
    out the host time limit (8 s here)."""
    res, _ = _run({}, extra_args="--p2p copy")
    assert res == {0: "ok", 1: "ok"}
    res, dt = _run({"REVPP_FAULT_RAISE_AT": "1:1"}, extra_args="--p2p copy")
    assert res.get(1, "").startswith("error:InjectedFault"), res
    assert res.get(0, "").startswith("error:ChannelError"), res
    assert dt < 60


def test_copy_channels_rank_exit_peer_times_out():
    """A rank that exits without a word leaves its peer waiting on a channel until the host
    time limit, which then raises."""
    res, dt = _run({"REVPP_FAULT_EXIT_AT": "0:2"}, extra_args="--p2p copy")
    assert 0 not in res or res[0] != "ok"
    assert res.get(1, "").startswith("error:ChannelError"), res
    assert dt < 80


def test_rank_exit_peer_fails():
    res, dt = _run({"REVPP_FAULT_EXIT_AT": "0:2"})
    assert 0 not in res or res[0] != "ok"
    assert res.get(1, "").startswith("error"), res
    assert dt < 80


def test_trainer_checks_device_status_word(monkeypatch):
    """finish_step reads the device status word and raises on any set bit (a fake read here;
    the GPU test sets a real bit with a timed-out flag wait)."""
    import revpp.ops as ops
    from revpp.config import GlobalConfig
    from revpp.engine import DeviceWaitError, Trainer
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    cfg = GlobalConfig(model="bert", reversible=True, num_hidden_layers=1, hidden_size=32, num_attention_heads=2,
                       max_position_embeddings=16, num_classes=2, autocast_dtype=torch.float32, batch_size=4,
                       microbatch_size=2, num_microbatches=2, lr=1e-4)
    env = EnvContext(world_size=1, rank=0, local_rank=0, device=torch.device("cpu"),
                     proc_logger=build_logger("st", None), node_logger=None, main_logger=None, pg=None,
                     master_rank=0)
    tr = Trainer(cfg, env)
    tr.uses_kernels = True
    word = {"v": 0}
    monkeypatch.setattr(ops, "check_status", lambda clear=True: word["v"])
    tr.check_device_status()  # clean word: no error
    word["v"] = 1
    with pytest.raises(DeviceWaitError):
        tr.check_device_status()
