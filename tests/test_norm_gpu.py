"""LayerNorm / cast kernels against float64 PyTorch references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from revpp.ops._ext import ext

    return ext()


@pytest.mark.parametrize("M,H", [(1, 128), (37, 768), (1000, 1024), (64, 2048)])
@pytest.mark.parametrize("eps", [1e-5, 1e-6])
def test_layernorm_fwd_bwd(M, H, eps):
    C = _C()
    x = torch.randn(M, H, device="cuda") * 3 + 1
    g = torch.rand(H, device="cuda") + 0.5
    b = torch.randn(H, device="cuda") * 0.1
    yb = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    yf = torch.empty(M, H, device="cuda")
    mean = torch.empty(M, device="cuda")
    rstd = torch.empty(M, device="cuda")
    C.layernorm_fwd(x, g, b, eps, y_bf16=yb, y_f32=yf, mean=mean, rstd=rstd)
    xd = x.double().requires_grad_()
    ref = torch.nn.functional.layer_norm(xd, (H,), g.double(), b.double(), eps)
    assert (yf.double() - ref).abs().max().item() < 1e-4
    assert (yb.double() - ref).abs().max().item() < 3e-2

    dy = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    resid = torch.randn(M, H, device="cuda")
    gd = g.double().requires_grad_()
    bd = b.double().requires_grad_()
    ref = torch.nn.functional.layer_norm(xd, (H,), gd, bd, eps)
    ref.backward(dy.double())
    dgamma = torch.zeros(H, device="cuda")
    dbeta = torch.zeros(H, device="cuda")
    dx = torch.empty(M, H, device="cuda")
    dxb = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    colsum = torch.zeros(H, device="cuda")
    C.layernorm_bwd(dy, x, g, mean, rstd, dgamma=dgamma, dbeta=dbeta, resid=resid, dx_f32=dx, dx_bf16=dxb,
                    colsum=colsum)
    torch.cuda.synchronize()
    want = xd.grad + resid.double()
    assert (dx.double() - want).abs().max().item() < 1e-3 * (1 + want.abs().max().item())
    assert (dxb.double() - want).abs().max().item() < 2e-2 * (1 + want.abs().max().item())
    assert (dgamma.double() - gd.grad).abs().max().item() < 1e-3 * (1 + gd.grad.abs().max().item())
    assert (dbeta.double() - bd.grad).abs().max().item() < 1e-3 * (1 + bd.grad.abs().max().item())
    assert (colsum.double() - want.sum(0)).abs().max().item() < 1e-3 * (1 + want.abs().sum(0).max().item())


@pytest.mark.parametrize("M,N", [(5, 128), (4099, 1024)])
def test_cast_colsum(M, N):
    C = _C()
    x = torch.randn(M, N, device="cuda")
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cs = torch.ones(N, device="cuda")
    C.cast_colsum(x, out=out, colsum=cs)
    torch.cuda.synchronize()
    assert torch.equal(out, x.to(torch.bfloat16))
    assert (cs.double() - (1 + x.double().sum(0))).abs().max().item() < 1e-3
    cs2 = torch.zeros(N, device="cuda")
    C.cast_colsum(out, colsum=cs2)
    torch.cuda.synchronize()
    assert (cs2.double() - out.double().sum(0)).abs().max().item() < 1e-3
