"""Race check: kernels launched concurrently on two streams give the same results as the
same launches run one after another (no hidden shared state between launches: tensor
maps, scratch, status words, per-device configuration)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from revpp.ops._ext import ext

    return ext()


def _gemm(C, A, B, out):
    M, K = A.shape
    N = B.shape[0]
    C.gemm_tc(A, False, B, False, M, N, K, 0, out)


def _ln(C, x, g, b, y, mean, rstd):
    C.layernorm_fwd(x, g, b, 1e-5, y_bf16=y, mean=mean, rstd=rstd)


def test_gemm_and_layernorm_two_streams_match_serial():
    C = _C()
    torch.manual_seed(0)
    shapes = [(2048, 1024, 1024), (1024, 3072, 1024)]
    As = [torch.randn(m, k, device="cuda").to(torch.bfloat16) for m, _, k in shapes]
    Bs = [(torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16) for _, n, k in shapes]
    xs = [torch.randn(4096, 1024, device="cuda") for _ in range(2)]
    g = torch.rand(1024, device="cuda") + 0.5
    b = torch.randn(1024, device="cuda")
    ref_g = [torch.empty(m, n, device="cuda", dtype=torch.bfloat16) for m, n, _ in shapes]
    ref_y = [torch.empty(4096, 1024, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    stats = [(torch.empty(4096, device="cuda"), torch.empty(4096, device="cuda")) for _ in range(2)]
    for i in range(2):
        _gemm(C, As[i], Bs[i], ref_g[i])
        _ln(C, xs[i], g, b, ref_y[i], *stats[i])
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for rep in range(5):
        outs_g = [torch.full_like(r, float("nan")) for r in ref_g]
        outs_y = [torch.full_like(r, float("nan")) for r in ref_y]
        st2 = [(torch.empty(4096, device="cuda"), torch.empty(4096, device="cuda")) for _ in range(2)]
        torch.cuda.synchronize()
        for j in range(2):  # interleave launches across the streams, order flipped each repetition
            for i in ((0, 1) if rep % 2 == 0 else (1, 0)):
                with torch.cuda.stream(streams[i]):
                    if j == 0:
                        _gemm(C, As[i], Bs[i], outs_g[i])
                    else:
                        _ln(C, xs[i], g, b, outs_y[i], *st2[i])
        torch.cuda.synchronize()
        for i in range(2):
            assert torch.equal(outs_g[i], ref_g[i]), (rep, i)
            assert torch.equal(outs_y[i], ref_y[i]), (rep, i)
    assert C.status_read_and_clear() == 0


def test_attention_two_streams_match_serial():
    C = _C()
    torch.manual_seed(1)
    B, S, heads = 2, 512, 16
    H = heads * 64
    qkv = [(torch.randn(B * S, 3 * H, device="cuda") * 1.5).to(torch.bfloat16) for _ in range(2)]
    dout = [torch.randn(B * S, H, device="cuda").to(torch.bfloat16) for _ in range(2)]

    def run(i, bufs):
        out, lse, dqkv, dq, D = bufs
        C.attn_fwd_tc(qkv[i], out, lse, B, S, heads)
        C.attn_bwd_tc(qkv[i], out, dout[i], lse, dqkv, dq, D, B, S, heads)

    def alloc():
        return (torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16), torch.empty(B, heads, S, device="cuda"),
                torch.empty(B * S, 3 * H, device="cuda", dtype=torch.bfloat16), torch.empty(B * S, H, device="cuda"),
                torch.empty(B, heads, S, device="cuda"))

    ref = [alloc() for _ in range(2)]
    for i in range(2):
        run(i, ref[i])
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for rep in range(3):
        got = [alloc() for _ in range(2)]
        torch.cuda.synchronize()
        for i in ((0, 1) if rep % 2 == 0 else (1, 0)):
            with torch.cuda.stream(streams[i]):
                run(i, got[i])
        torch.cuda.synchronize()
        for i in range(2):
            assert torch.equal(got[i][0], ref[i][0]) and torch.equal(got[i][1], ref[i][1])  # forward is deterministic
            # dQ uses fp32 atomics: summation order may differ between runs
            d = (got[i][2].float() - ref[i][2].float()).abs().max().item()
            assert d <= 2e-2 * (1 + ref[i][2].float().abs().max().item()), (rep, i, d)
    assert C.status_read_and_clear() == 0
