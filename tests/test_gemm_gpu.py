"""tcgen05 GEMM numerics against a float64 PyTorch reference of the same op."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

EPI_BF16, EPI_GELU, EPI_RESID, EPI_ATOMIC, EPI_DGELU, EPI_F32 = range(6)

SHAPES = [(128, 256, 64), (256, 512, 256), (300, 96, 200), (1000, 1024, 1024), (4096, 3072, 1024)]


def _C():
    from revpp.ops._ext import ext

    return ext()


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def _gelu(x):
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def _close(out, ref, rtol):
    err = (out.double() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= rtol * scale, f"max abs err {err} vs scale {scale}"


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_fwd_bias_bf16(M, N, K, variant):
    C = _C()
    a, b, bias = _rand(M, K), _rand(N, K, scale=0.05), _rand(N, scale=0.1)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm_tc(a, False, b, False, M, N, K, EPI_BF16, out, bias=bias, variant=variant)
    torch.cuda.synchronize()
    assert C.status_read_and_clear() == 0
    ref = a.double() @ b.double().t() + bias.double()
    _close(out, ref, 1e-2)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_fwd_gelu(M, N, K, variant):
    C = _C()
    a, b, bias = _rand(M, K), _rand(N, K, scale=0.05), _rand(N, scale=0.1)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm_tc(a, False, b, False, M, N, K, EPI_GELU, out, bias=bias, aux_out=pre, variant=variant)
    torch.cuda.synchronize()
    u = a.double() @ b.double().t() + bias.double()
    _close(pre, u, 1e-2)
    _close(out, _gelu(pre.double()), 1e-2)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("sign", [1.0, -1.0])
def test_fwd_resid(M, N, K, sign, variant):
    C = _C()
    a, b, bias = _rand(M, K), _rand(N, K, scale=0.05), _rand(N, scale=0.1)
    resid = torch.randn(M, N, device="cuda")
    out = torch.empty(M, N, device="cuda")
    C.gemm_tc(a, False, b, False, M, N, K, EPI_RESID, out, bias=bias, resid=resid, sign=sign, variant=variant)
    torch.cuda.synchronize()
    f = (a.float() @ b.float().t() + bias.float()).to(torch.bfloat16).double()
    ref = resid.double() + sign * f
    # bf16 rounding of f may differ by one ulp from the float reference
    _close(out, ref, 1e-2)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_dgrad_mn(M, N, K, variant):
    """C[M,N] = A[M,K] @ W where W is stored [K, N] (MN-major B)."""
    C = _C()
    a, w = _rand(M, K), _rand(K, N, scale=0.05)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm_tc(a, False, w, True, M, N, K, EPI_BF16, out, variant=variant)
    torch.cuda.synchronize()
    _close(out, a.double() @ w.double(), 1e-2)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_dgelu(M, N, K, variant):
    C = _C()
    a, w = _rand(M, K), _rand(K, N, scale=0.05)
    u = _rand(M, N)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cs = torch.full((N,), 0.25, device="cuda")
    C.gemm_tc(a, False, w, True, M, N, K, EPI_DGELU, out, aux=u, variant=variant, colsum=cs)
    torch.cuda.synchronize()
    ud = u.double()
    dg = 0.5 * (1 + torch.erf(ud / math.sqrt(2))) + ud * torch.exp(-0.5 * ud * ud) / math.sqrt(2 * math.pi)
    dh = (a.double() @ w.double()).to(torch.bfloat16).double()
    _close(out, dh * dg, 2e-2)
    # fused bias gradient: column sums of the bf16 output, added to what colsum held
    ref_cs = out.double().sum(0) + 0.25
    assert (cs.double() - ref_cs).abs().max().item() <= 1e-4 * (1 + ref_cs.abs().max().item())


@pytest.mark.parametrize("variant", [1, 2])
def test_dgelu_colsum_many_tiles(variant):
    """Column sums over many tiles per CTA: contiguous tile runs cross column blocks, so
    the register-held partial sums are flushed mid-kernel as well as at the end."""
    C = _C()
    M, N, K = 8192, 4096, 1024
    a, w = _rand(M, K), _rand(K, N, scale=0.05)
    u = _rand(M, N)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cs = torch.full((N,), -1.0, device="cuda")
    C.gemm_tc(a, False, w, True, M, N, K, EPI_DGELU, out, aux=u, variant=variant, colsum=cs)
    torch.cuda.synchronize()
    ref_cs = out.double().sum(0) - 1.0
    assert (cs.double() - ref_cs).abs().max().item() <= 1e-4 * (1 + ref_cs.abs().max().item())
    ud = u.double()[:256]
    dg = 0.5 * (1 + torch.erf(ud / math.sqrt(2))) + ud * torch.exp(-0.5 * ud * ud) / math.sqrt(2 * math.pi)
    dh = (a[:256].double() @ w.double()).to(torch.bfloat16).double()
    _close(out[:256], dh * dg, 2e-2)
    assert C.status_read_and_clear() == 0


WGRAD_SHAPES = [(128, 256, 64), (256, 512, 256), (96, 160, 197 * 3), (1024, 1024, 1000), (3072, 1024, 4096)]


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,N,K", WGRAD_SHAPES)
@pytest.mark.parametrize("splits", [1, 3])
def test_wgrad_atomic(M, N, K, splits, variant):
    """C[M,N] += A^T B where A stored [K, M] and B stored [K, N] (both MN-major)."""
    C = _C()
    a, b = _rand(K, M), _rand(K, N)
    out = torch.randn(M, N, device="cuda")
    ref = out.double() + a.double().t() @ b.double()
    C.gemm_tc(a, True, b, True, M, N, K, EPI_ATOMIC, out, splits=splits, variant=variant)
    torch.cuda.synchronize()
    _close(out, ref, 1e-4)


@pytest.mark.parametrize("variant", [1, 2])
def test_fwd_f32_persistent_many_tiles(variant):
    C = _C()
    M, N, K = 8192, 4096, 512
    a, b = _rand(M, K), _rand(N, K, scale=0.05)
    out = torch.empty(M, N, device="cuda")
    C.gemm_tc(a, False, b, False, M, N, K, EPI_F32, out, variant=variant)
    torch.cuda.synchronize()
    _close(out, a.float() @ b.float().t(), 1e-4)
    assert C.status_read_and_clear() == 0


def test_bad_stride_raises():
    """A row stride that TMA cannot describe is rejected with an exception, not a crash."""
    C = _C()
    a, b = _rand(200, 300), _rand(200, 96)
    out = torch.zeros(300, 96, device="cuda")
    with pytest.raises(RuntimeError):
        C.gemm_tc(a, True, b, True, 300, 96, 200, EPI_ATOMIC, out)
