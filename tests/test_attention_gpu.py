"""Flash attention kernels against float64 PyTorch attention of the same bf16 inputs."""
import math
import zlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from revpp.ops._ext import ext

    return ext()


@pytest.fixture(autouse=True)
def _seed(request):
    """Fixed inputs per test case (the tolerances are checked on known data)."""
    torch.manual_seed(zlib.crc32(request.node.name.encode()))


def _ref(qkv, B, S, heads):
    H = heads * 64
    x = qkv.double().view(B, S, 3, heads, 64)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    s = q @ k.transpose(-1, -2) / math.sqrt(64)
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    o = (p @ v).transpose(1, 2).reshape(B * S, H)
    return o, lse


@pytest.mark.parametrize("B,S,heads", [(1, 64, 1), (2, 197, 2), (2, 512, 16), (3, 577, 4), (1, 100, 3)])
def test_attn_fwd_bwd(B, S, heads):
    C = _C()
    H = heads * 64
    qkv = (torch.randn(B * S, 3 * H, device="cuda") * 1.5).to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    C.attn_fwd(qkv, out, lse, B, S, heads)
    torch.cuda.synchronize()
    qd = qkv.double().requires_grad_()
    o_ref, lse_ref = _ref(qd, B, S, heads)
    assert (out.double() - o_ref).abs().max().item() < 2e-2
    assert (lse.double() - lse_ref).abs().max().item() < 2e-3

    dout = torch.randn(B * S, H, device="cuda").to(torch.bfloat16)
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(B * S, H, device="cuda")
    D = torch.empty(B, heads, S, device="cuda")
    C.attn_bwd(qkv, out, dout, lse, dqkv, dq_acc, D, B, S, heads)
    torch.cuda.synchronize()
    o_ref.backward(dout.double())
    g = qd.grad
    err = (dqkv.double() - g).abs().max().item()
    assert err < 3e-2 * (1 + g.abs().max().item()), err
    assert C.status_read_and_clear() == 0


FWD_KERNELS = ["attn_fwd_tc", "attn_fwd_persistent"]


@pytest.mark.parametrize("kernel", FWD_KERNELS)
@pytest.mark.parametrize("B,S,heads", [(1, 64, 1), (2, 197, 2), (2, 512, 16), (3, 577, 4), (1, 100, 3), (1, 150, 2),
                                       (1, 2048, 2), (20, 577, 8), (40, 512, 16)])
def test_attn_fwd_tcgen05(B, S, heads, kernel):
    """tcgen05 forward kernels against float64 attention and against the mma.sync kernel.
    The last two shapes give the persistent kernel several work items per CTA, some with
    a second query tile past the sequence end."""
    C = _C()
    H = heads * 64
    qkv = (torch.randn(B * S, 3 * H, device="cuda") * 1.5).to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    getattr(C, kernel)(qkv, out, lse, B, S, heads)
    out2 = torch.empty_like(out)
    lse2 = torch.empty_like(lse)
    C.attn_fwd(qkv, out2, lse2, B, S, heads)
    torch.cuda.synchronize()
    assert C.status_read_and_clear() == 0
    o_ref, lse_ref = _ref(qkv.double(), B, S, heads)
    # bf16 P (relative 2^-9 per weight) and a bf16 output: 2e-2 plus 0.5 % of the value
    assert ((out.double() - o_ref).abs() - 5e-3 * o_ref.abs()).max().item() < 2e-2
    assert (lse.double() - lse_ref).abs().max().item() < 2e-3
    # two bf16-rounded results: allow a rounding step of the larger outputs
    assert ((out.double() - out2.double()).abs() - 8e-3 * out2.double().abs()).max().item() < 2e-2


# the last three run more work items (key tile, head, sequence) than a B200 has SMs, so the
# persistent backward's CTAs take 2-4 items each: odd and even query-tile counts per item
@pytest.mark.parametrize("B,S,heads", [(1, 64, 1), (2, 197, 2), (2, 512, 16), (3, 577, 4), (1, 100, 3), (1, 1024, 2),
                                       (6, 197, 16), (4, 577, 16), (8, 512, 16)])
def test_attn_bwd_tcgen05(B, S, heads):
    """tcgen05 backward against float64 autograd and against the mma.sync backward."""
    C = _C()
    H = heads * 64
    qkv = (torch.randn(B * S, 3 * H, device="cuda") * 1.5).to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    C.attn_fwd_tc(qkv, out, lse, B, S, heads)
    dout = torch.randn(B * S, H, device="cuda").to(torch.bfloat16)
    dq_acc = torch.empty(B * S, H, device="cuda")
    D = torch.empty(B, heads, S, device="cuda")
    dqkv = torch.empty_like(qkv)
    cs = torch.full((3 * H,), -0.5, device="cuda")
    C.attn_bwd_tc(qkv, out, dout, lse, dqkv, dq_acc, D, B, S, heads, colsum=cs)
    torch.cuda.synchronize()
    ref_cs = dqkv.double().sum(0) - 0.5  # fused bias gradient = column sums of the bf16 dqkv
    assert (cs.double() - ref_cs).abs().max().item() <= 1e-4 * (1 + ref_cs.abs().max().item())
    dqkv2 = torch.empty_like(qkv)
    C.attn_bwd(qkv, out, dout, lse, dqkv2, dq_acc, D, B, S, heads)
    torch.cuda.synchronize()
    assert C.status_read_and_clear() == 0
    qd = qkv.double().requires_grad_()
    o_ref, _ = _ref(qd, B, S, heads)
    o_ref.backward(dout.double())
    g = qd.grad
    scale = 1 + g.abs().max().item()
    assert (dqkv.double() - g).abs().max().item() < 3e-2 * scale
    assert (dqkv.double() - dqkv2.double()).abs().max().item() < 3e-2 * scale


@pytest.mark.parametrize("kernel", FWD_KERNELS)
@pytest.mark.parametrize("B,S,heads", [(1, 512, 2), (2, 577, 1)])
def test_attn_fwd_tcgen05_rising_scores(B, S, heads, kernel):
    """Scores that grow along the keys: the row maximum rises by far more than the
    rescale threshold from one 64-key tile to the next, so the kernel's in-TMEM output
    rescale runs for every row on most tiles."""
    C = _C()
    H = heads * 64
    x = torch.randn(B, S, 3, heads, 64, device="cuda")
    x[:, :, 0] = x[:, :, 0].abs() * 0.5 + 1.0           # positive queries
    ramp = torch.linspace(0.0, 6.0, S, device="cuda").view(1, S, 1, 1)
    x[:, :, 1] = x[:, :, 1].abs() * 0.5 + ramp           # keys growing with position
    qkv = x.reshape(B * S, 3 * H).to(torch.bfloat16)
    out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, heads, S, device="cuda")
    getattr(C, kernel)(qkv, out, lse, B, S, heads)
    torch.cuda.synchronize()
    assert C.status_read_and_clear() == 0
    o_ref, lse_ref = _ref(qkv.double(), B, S, heads)
    # the scores span more than 8 log2 units between the first and last key tiles
    s = qkv.double().view(B, S, 3, heads, 64)
    sc = (s[:, :, 0] * s[:, :, 1]).sum(-1) / 8.0 / math.log(2.0)
    assert (sc[:, -1] - sc[:, 0]).min().item() > 16.0
    assert ((out.double() - o_ref).abs() - 5e-3 * o_ref.abs()).max().item() < 2e-2
    assert ((lse.double() - lse_ref).abs() / lse_ref.abs().clamp(min=1.0)).max().item() < 2e-3

