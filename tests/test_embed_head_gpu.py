"""Embedding / patch-embedding / head kernels against the PyTorch implementation of the
same math on the same weights (fp32 references, bf16 where autocast rounds)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _stage(model, kind="reversible", first=True, last=True, H=256, heads=4, S=128, img=64, classes=10):
    from revpp.config import GlobalConfig
    from revpp.models.embed_head_kernels import KernelEmbedHead
    from revpp.models.encoder import EncoderStage, TorchEmbedHead
    from revpp.models.params import FlatParams

    torch.manual_seed(0)
    cfg = GlobalConfig(model=model, reversible=kind != "standard", inverse=kind == "inverse", num_hidden_layers=1,
                       hidden_size=H, num_attention_heads=heads, max_position_embeddings=S, img_size=img,
                       patch_size=16, num_classes=classes, autocast_dtype=torch.bfloat16)
    nst = 1 if (first and last) else 2
    st = EncoderStage(cfg, 0 if first else 1, nst, 1, kind).to("cuda")
    with torch.no_grad():
        for p in st.parameters():
            p.add_(torch.randn_like(p) * 0.01)
    flat = FlatParams(st, "cuda", want_shadow=True)
    return cfg, st, flat, KernelEmbedHead(st, flat, torch.bfloat16), TorchEmbedHead(st, flat, torch.bfloat16)


def _rel(a, b):
    return (a.double() - b.double()).norm().item() / max(b.double().norm().item(), 1e-12)


def test_bert_embedding_fwd_bwd():
    cfg, st, flat, ke, te = _stage("bert")
    B, S = 3, 128
    ids = torch.randint(0, cfg.vocab_size, (B, S), device="cuda")
    ids[0, :5] = 0  # padding id
    tt = torch.randint(0, 2, (B, S), device="cuda")
    xk = ke.embed_fwd((ids, tt))
    xt = te.embed_fwd((ids, tt))
    assert _rel(xk, xt) < 1e-5
    dx2, dx1 = torch.randn_like(xk), torch.randn_like(xk)
    flat.zero_grad()
    ke.embed_bwd((ids, tt), dx2, dx1)
    gk = flat.grad.clone()
    flat.zero_grad()
    te.embed_bwd((ids, tt), dx2, dx1)
    gt = flat.grad.clone()
    for name, p in zip(flat.names, flat.params):
        if not name.startswith("embeddings"):
            continue
        o, n, _ = flat._span(p)
        assert _rel(gk[o:o + n], gt[o:o + n]) < 1e-4, name


def test_vit_patch_embedding_fwd_bwd():
    cfg, st, flat, ke, te = _stage("vit")
    img = torch.randn(3, 3, 64, 64, device="cuda")
    xk = ke.embed_fwd((img,))
    xt = te.embed_fwd((img,))
    assert xk.shape == xt.shape == (3, 17, 256)
    assert _rel(xk, xt) < 2e-2
    dx = torch.randn_like(xk)
    flat.zero_grad()
    ke.embed_bwd((img,), dx)
    gk = flat.grad.clone()
    flat.zero_grad()
    te.embed_bwd((img,), dx)
    gt = flat.grad.clone()
    for name, p in zip(flat.names, flat.params):
        if not name.startswith("embeddings"):
            continue
        o, n, _ = flat._span(p)
        assert _rel(gk[o:o + n], gt[o:o + n]) < 3e-2, name


# the last case has an ImageNet-sized head (1000 classes) and 20 samples: several class
# chunks and two sample blocks in the input-gradient kernel
@pytest.mark.parametrize("model,kind,single,classes,B", [("bert", "reversible", False, 2, 4),
                                                         ("vit", "reversible", False, 10, 4),
                                                         ("bert", "standard", True, 2, 4),
                                                         ("bert", "inverse", False, 2, 4),
                                                         ("vit", "reversible", False, 1000, 20)])
def test_head_fwd_bwd(model, kind, single, classes, B):
    cfg, st, flat, ke, te = _stage(model, kind=kind, first=False, last=True, classes=classes)
    S, H = cfg.seq_len, 256
    y2 = torch.randn(B, S, H, device="cuda")
    y1 = None if single else torch.randn(B, S, H, device="cuda")
    labels = torch.randint(0, cfg.num_classes, (B,), device="cuda")
    flat.zero_grad()
    lk, logk, dk2, dk1 = ke.head_fwd_bwd(y2, y1, labels, 0.25)
    gk = flat.grad.clone()
    flat.zero_grad()
    lt, logt, dt2, dt1 = te.head_fwd_bwd(y2, y1, labels, 0.25)
    gt = flat.grad.clone()
    assert abs(float(lk) - float(lt)) < 1e-2 * max(1.0, abs(float(lt)))
    assert _rel(logk, logt) < 1e-2
    assert _rel(dk2, dt2) < 3e-2
    if dt1 is not None:
        assert _rel(dk1, dt1) < 3e-2
    for name, p in zip(flat.names, flat.params):
        if not (name.startswith("norm") or name.startswith("head")):
            continue
        o, n, _ = flat._span(p)
        assert _rel(gk[o:o + n], gt[o:o + n]) < 3e-2, name
