"""Model-level GPU tests: the sm_100a kernel path against the PyTorch autocast path on the
same weights, reconstruction accuracy of the reversible backward, and a full train step."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(H=256, heads=4, layers=2, B=2, S=197, seed=0):
    from revpp.config import GlobalConfig
    from revpp.models.blockmath import KernelMath, TorchMath
    from revpp.models.encoder import EncoderStage
    from revpp.models.params import FlatParams

    torch.manual_seed(seed)
    cfg = GlobalConfig(model="bert", reversible=True, num_hidden_layers=layers, hidden_size=H,
                       num_attention_heads=heads, max_position_embeddings=S, autocast_dtype=torch.bfloat16)
    st = EncoderStage(cfg, 1, 3, layers, "reversible")  # a middle stage: blocks only
    st.to("cuda")
    flat = FlatParams(st, "cuda", want_shadow=True)
    km = KernelMath(flat, torch.bfloat16, heads)
    tm = TorchMath(flat, torch.bfloat16, heads)
    return cfg, st, flat, km, tm


def _rel(a, b):
    return (a.double() - b.double()).norm().item() / max(b.double().norm().item(), 1e-12)


def test_block_forward_matches_torch():
    from revpp.models.reversible import rev_forward

    cfg, st, flat, km, tm = _setup()
    x = torch.randn(2, 197, 256, device="cuda")
    yk = rev_forward(km, st.blocks, x, x.clone())
    yt = rev_forward(tm, st.blocks, x, x.clone())
    for a, b in zip(yk, yt):
        assert _rel(a, b) < 1e-2


def test_reversible_backward_matches_torch_and_reconstructs():
    from revpp.models.reversible import rev_backward, rev_forward

    cfg, st, flat, km, tm = _setup()
    x2 = torch.randn(2, 197, 256, device="cuda")
    x1 = torch.randn(2, 197, 256, device="cuda")
    y2, y1 = rev_forward(km, st.blocks, x2, x1)
    dy2 = torch.randn_like(y2) * 1e-2
    dy1 = torch.randn_like(y1) * 1e-2
    flat.zero_grad()
    (dx2, dx1), (r2, r1) = rev_backward(km, st.blocks, y2, y1, dy2, dy1)
    torch.cuda.synchronize()
    gk = flat.grad.clone()
    # reconstruction: the recomputed F / G match the forward bit for bit, but the fp32
    # add-then-subtract perturbs X2 by an ulp, which can flip bf16 roundings inside F(X2)
    assert _rel(r2, x2) < 1e-3 and _rel(r1, x1) < 1e-3
    flat.zero_grad()
    (tx2, tx1), _ = rev_backward(tm, st.blocks, y2, y1, dy2, dy1)
    torch.cuda.synchronize()
    gt = flat.grad.clone()
    assert _rel(dx2, tx2) < 3e-2 and _rel(dx1, tx1) < 3e-2
    for name, p in zip(flat.names, flat.params):
        o, n, _ = flat._span(p)
        assert _rel(gk[o:o + n], gt[o:o + n]) < 5e-2, name


def test_pareprop_equals_sequential():
    from revpp.models.reversible import rev_backward, rev_forward

    cfg, st, flat, km, tm = _setup(layers=4)
    x = torch.randn(2, 197, 256, device="cuda")
    y2, y1 = rev_forward(km, st.blocks, x, x.clone())
    dy = torch.randn_like(y2) * 1e-2
    flat.zero_grad()
    (a2, a1), (ra2, ra1) = rev_backward(km, st.blocks, y2, y1, dy, dy)
    g_seq = flat.grad.clone()
    flat.zero_grad()
    streams = (torch.cuda.Stream(), torch.cuda.Stream())
    (b2, b1), (rb2, rb1) = rev_backward(km, st.blocks, y2, y1, dy, dy, pareprop=True, streams=streams)
    torch.cuda.synchronize()
    g_par = flat.grad.clone()
    assert torch.equal(ra2, rb2) and torch.equal(ra1, rb1)
    # the attention dQ accumulates with fp32 atomics, whose order varies run to run
    assert _rel(b2, a2) < 1e-3 and _rel(b1, a1) < 1e-3
    assert _rel(g_par, g_seq) < 1e-3


def test_full_train_step_kernels():
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.ops import ext
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    dev = torch.device("cuda", 0)
    cfg = GlobalConfig(model="bert", reversible=True, num_hidden_layers=2, hidden_size=256, num_attention_heads=4,
                       max_position_embeddings=128, autocast_dtype=torch.bfloat16, batch_size=8,
                       microbatch_size=4, num_microbatches=2, lr=1e-3)
    env = EnvContext(1, 0, 0, dev, build_logger("t", None), None, None, None, 0)
    tr = Trainer(cfg, env)
    data = SyntheticBatches(cfg, 8, 1, seed=0)
    b = data.make(0)
    losses = [float(tr.train_step(b)) for _ in range(8)]
    assert all(math.isfinite(l) for l in losses)
    assert losses[-1] < losses[0]  # memorises the fixed batch
    assert ext().status_read_and_clear() == 0


@pytest.mark.parametrize("kind", ["standard", "checkpoint", "inverse"])
def test_other_stage_kinds_train(kind):
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    dev = torch.device("cuda", 0)
    cfg = GlobalConfig(model="vit", reversible=kind == "inverse", inverse=kind == "inverse",
                       checkpointing=kind == "checkpoint", num_hidden_layers=2, hidden_size=256,
                       num_attention_heads=4, img_size=64, patch_size=16, num_classes=10,
                       autocast_dtype=torch.bfloat16, batch_size=8, microbatch_size=4, num_microbatches=2, lr=1e-3)
    env = EnvContext(1, 0, 0, dev, build_logger("t", None), None, None, None, 0)
    tr = Trainer(cfg, env)
    b = SyntheticBatches(cfg, 8, 1, seed=0).make(0)
    losses = [float(tr.train_step(b)) for _ in range(6)]
    assert all(math.isfinite(l) for l in losses)
    assert losses[-1] < losses[0]


def test_full_model_grads_kernels_vs_torch():
    """Whole single-stage model (embedding, 2 reversible blocks, head): one step's gradients
    from the kernel path against PyTorch autocast on the same weights and batch."""
    from revpp.config import GlobalConfig
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.models.blockmath import TorchMath
    from revpp.models.encoder import TorchEmbedHead
    from revpp.utils.env import EnvContext
    from revpp.utils.logger import build_logger

    dev = torch.device("cuda", 0)
    cfg = GlobalConfig(model="bert", reversible=True, num_hidden_layers=2, hidden_size=256, num_attention_heads=4,
                       max_position_embeddings=128, autocast_dtype=torch.bfloat16, batch_size=8,
                       microbatch_size=4, num_microbatches=2, lr=1e-3)
    env = EnvContext(1, 0, 0, dev, build_logger("t", None), None, None, None, 0)
    torch.manual_seed(0)
    tr = Trainer(cfg, env)
    b = SyntheticBatches(cfg, 8, 1, seed=0).make(0)
    inputs = tr.split_inputs(b)
    labels = b["labels"].to(dev)
    tr.flat.zero_grad()
    lk = torch.stack(tr.executor.step(inputs, labels)).mean()
    gk = tr.flat.grad.clone()
    tr.flat.zero_grad()
    tr.stage.math = TorchMath(tr.flat, torch.bfloat16, cfg.num_attention_heads)
    tr.stage.eh = TorchEmbedHead(tr.module, tr.flat, torch.bfloat16)
    lt = torch.stack(tr.executor.step(inputs, labels)).mean()
    gt = tr.flat.grad.clone()
    assert abs(float(lk) - float(lt)) < 2e-2
    for name, p in zip(tr.flat.names, tr.flat.params):
        o, n, _ = tr.flat._span(p)
        assert _rel(gk[o:o + n], gt[o:o + n]) < 6e-2, name
