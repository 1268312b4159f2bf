"""Host-side planning of the kernels, on CPU (the extension loads without a GPU)."""
import pytest
import torch  # noqa: F401  (loads the libraries the extension links against)


def _ext():
    try:
        import revpp._C as C
    except ImportError as e:  # not built in this checkout
        pytest.skip(f"extension not built: {e}")
    return C


def _makespan(M, N, K, s, sms=148):
    pt = -(-M // 256) * -(-N // 256)
    kb = -(-K // 64)
    return -(-pt * s // (sms // 2)) * (-(-kb // s) + 16)


@pytest.mark.parametrize("M,N,K", [(1024, 4096, 32768), (4096, 1024, 32768), (1024, 1024, 32768),
                                   (3072, 1024, 32768), (3072, 1024, 8192), (1024, 1024, 8192)])
def test_wgrad_split_count_minimises_the_makespan(M, N, K):
    C = _ext()
    s = C.gemm_suggest_splits(M, N, K, sms=148)
    assert 1 <= s <= 16 and (s == 1 or -(-K // 64) // s >= 8)
    best = min(_makespan(M, N, K, t) for t in range(1, 17) if t == 1 or -(-K // 64) // t >= 8)
    assert _makespan(M, N, K, s) == best


def test_wgrad_split_counts_of_the_measured_sweep():
    # the best measured split counts at 32768 / 8192 tokens (48 output tiles of 3072 x 1024
    # on 74 SM pairs: one split would idle a third of them)
    C = _ext()
    assert C.gemm_suggest_splits(3072, 1024, 32768, sms=148) == 3
    assert C.gemm_suggest_splits(1024, 4096, 32768, sms=148) == 1
    assert C.gemm_suggest_splits(1024, 1024, 8192, sms=148) == 4
    assert C.gemm_suggest_splits(3072, 1024, 8192, sms=148) == 3
