"""The allocation-free attention backward entry point, called through its exported C symbol.

``revpp_attn_bwd_tc_noalloc`` (csrc/attention_noalloc.h) must give the same gradients as
the allocating entry point ``revpp._C.attn_bwd_tc`` on two calls in a row (the second with
other shapes and inputs, so stale scratch contents from the first would show), allocate
no device memory, and reject problems larger than its fixed scratch array.
"""
import ctypes

import pytest
import torch

SCRATCH_BYTES = 16 << 20
OK, TOO_LARGE = 0, 1


def _lib():
    from revpp import _C  # noqa: F401  (loads torch's libraries first)
    from revpp.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    f = lib.revpp_attn_bwd_tc_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return f


def _alloc_counters():
    st = torch.cuda.memory_stats()
    return (st.get("allocation.all.allocated", 0), st.get("segment.all.allocated", 0),
            st.get("reserved_bytes.all.current", 0))


def _free_unchanged(free_before, tries=5):
    import time

    for _ in range(tries):
        if torch.cuda.mem_get_info()[0] == free_before:
            return True
        time.sleep(0.05)
    return False


def _call(f, qkv, out, dout, lse, dqkv, B, S, heads, status=None):
    err = ctypes.create_string_buffer(512)
    stream = torch.cuda.current_stream().cuda_stream if torch.cuda.is_available() else 0
    rc = f(qkv, out, dout, lse, dqkv, B, S, heads, status, stream, err, len(err))
    return rc, err.value.decode()


def test_rejects_problem_beyond_scratch():
    """Checked before any CUDA call, so it runs without a GPU."""
    f = _lib()
    B, S, heads = 8, 1024, 16  # 32 MiB of dQ accumulator alone
    fake = 1 << 20  # aligned, never dereferenced: the size check comes first
    rc, msg = _call(f, fake, fake, fake, fake, fake, B, S, heads)
    assert rc == TOO_LARGE
    assert "bytes of scratch" in msg and str(SCRATCH_BYTES) in msg


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_point_twice():
    from revpp.ops._ext import ext

    C = ext()
    f = _lib()
    C.status_read_and_clear()
    cases = [(2, 512, 16), (3, 577, 4)]
    prepared = []
    for B, S, heads in cases:
        H = heads * 64
        qkv = (torch.randn(B * S, 3 * H, device="cuda") * 1.5).to(torch.bfloat16)
        out = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(B, heads, S, device="cuda")
        C.attn_fwd_tc(qkv, out, lse, B, S, heads)
        dout = torch.randn(B * S, H, device="cuda").to(torch.bfloat16)
        ref = torch.empty_like(qkv)
        C.attn_bwd_tc(qkv, out, dout, lse, ref, torch.empty(B * S, H, device="cuda"),
                      torch.empty(B, heads, S, device="cuda"), B, S, heads)
        got = torch.full_like(qkv, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        prepared.append((B, S, heads, qkv, out, dout, lse, ref, got, status))
    torch.cuda.synchronize()
    for i, (B, S, heads, qkv, out, dout, lse, ref, got, status) in enumerate(prepared):
        stats_before = _alloc_counters()
        free_before = torch.cuda.mem_get_info()[0]
        rc, msg = _call(f, qkv.data_ptr(), out.data_ptr(), dout.data_ptr(), lse.data_ptr(), got.data_ptr(),
                        B, S, heads, status.data_ptr())
        assert rc == OK, msg
        torch.cuda.synchronize()
        # nothing went through torch's caching allocator
        assert _alloc_counters() == stats_before
        if i > 0:  # the first call may load the module (and with it the scratch array)
            # device-wide free memory also moves with other processes' allocations: a change
            # must persist over a few re-reads to count
            assert _free_unchanged(free_before), "device free memory changed across the call"
        assert int(status.item()) == 0
        assert torch.isfinite(got.float()).all()
        scale = 1 + ref.double().abs().max().item()
        assert (got.double() - ref.double()).abs().max().item() < 3e-2 * scale, (B, S, heads)
    assert C.status_read_and_clear() == 0
