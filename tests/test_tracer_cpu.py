"""The tracing frontend (pipe_split / SplitPoint / pipeline / Pipe.build_stage): split
stages compose to the original module, and a traced 2-stage pipeline trained with 1F1B
over gloo gives the same loss and gradients as plain autograd."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from revpp.parallel.tracer import SplitPoint, pipe_split, pipeline


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(16, 32)
        self.b = nn.Linear(32, 32)
        self.c = nn.Linear(32, 4)

    def forward(self, x):
        x = torch.relu(self.a(x))
        x = pipe_split(x)
        x = torch.tanh(self.b(x)) + x
        x = pipe_split(x)
        return self.c(x)


def test_markers_split_into_stages_that_compose():
    torch.manual_seed(0)
    net = Net()
    x = torch.randn(5, 16)
    ref = net(x)
    pipe = pipeline(net, (x,))
    assert pipe.num_stages == 3
    y = x
    for st in pipe.stages:
        y = st(y)
    assert torch.allclose(y, ref, atol=1e-6)
    assert torch.allclose(pipe(x), ref, atol=1e-6)
    assert torch.allclose(net(x), ref)  # eager module unchanged after tracing


def test_split_spec_on_submodules():
    torch.manual_seed(0)
    seq = nn.Sequential(nn.Linear(8, 8), nn.GELU(), nn.Linear(8, 8), nn.GELU(), nn.Linear(8, 2))
    x = torch.randn(3, 8)
    ref = seq(x)
    pipe = pipeline(seq, (x,), split_spec={"2": SplitPoint.BEGINNING, "3": SplitPoint.END})
    assert pipe.num_stages == 3
    y = x
    for st in pipe.stages:
        y = st(y)
    assert torch.allclose(y, ref, atol=1e-6)
    with pytest.raises(ValueError):
        pipeline(seq, (x,), split_spec={"0": SplitPoint.END}, split_policy=lambda g: g)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    try:
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from revpp.parallel.p2p import PipeComms, TensorSpec
        from revpp.parallel.schedule import PipelineExecutor

        torch.manual_seed(0)
        seq = nn.Sequential(nn.Linear(16, 32), nn.Tanh(), nn.Linear(32, 32), nn.Tanh(), nn.Linear(32, 3))
        pipe = pipeline(seq, split_spec={"2": SplitPoint.BEGINNING})
        n, mbs = 4, 2
        spec = TensorSpec((mbs, 32), torch.float32)
        st = pipe.build_stage(rank, torch.device("cpu"), mbs, n, in_spec=spec, out_spec=spec)
        comms = PipeComms(rank, 2, 2, 1, torch.device("cpu"), st.fwd_specs(), st.bwd_specs(rank),
                          TensorSpec((n * mbs,), torch.int64))
        ex = PipelineExecutor(st, comms, n, "1f1b")
        g = torch.Generator().manual_seed(1)
        x = torch.randn(n * mbs, 16, generator=g)
        labels = torch.randint(0, 3, (n * mbs,), generator=g)
        losses = ex.step([(c,) for c in torch.chunk(x, n)] if rank == 0 else None, labels if rank == 0 else None)
        grads = {k: p.grad.clone().numpy() for k, p in st.module.named_parameters()}
        loss = float(torch.stack(losses).mean()) if rank == 1 else None
        out = [None, None]
        dist.all_gather_object(out, (loss, grads))
        if rank == 0:
            q.put(("ok", out))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        import traceback

        q.put(("err", traceback.format_exc()))
        raise


def test_traced_pipeline_trains_like_autograd():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    status, out = q.get(timeout=240)
    for p in ps:
        p.join(timeout=60)
    assert status == "ok", out
    torch.manual_seed(0)
    seq = nn.Sequential(nn.Linear(16, 32), nn.Tanh(), nn.Linear(32, 32), nn.Tanh(), nn.Linear(32, 3))
    g = torch.Generator().manual_seed(1)
    x = torch.randn(8, 16, generator=g)
    labels = torch.randint(0, 3, (8,), generator=g)
    losses = [nn.functional.cross_entropy(seq(xc), lc) for xc, lc in zip(torch.chunk(x, 4), torch.chunk(labels, 4))]
    (sum(losses) / 4).backward()
    assert abs(out[1][0] - float(sum(losses) / 4)) < 1e-6
    names = [k for k, _ in seq.named_parameters()]
    got = {**out[0][1], **out[1][1]}
    assert len(got) == len(names)
    ref = {k: p.grad for k, p in seq.named_parameters()}
    # stage submodules keep the original names of the layers they hold
    for k, v in got.items():
        assert torch.allclose(torch.from_numpy(v), ref[k], atol=1e-6), k
