"""dkv_gemm_noalloc (the GEMM whose split-K scratch is a fixed array in the
library) against dkv_gemm (the same GEMM with a caller-provided work buffer).

The fp32 CUDA-core kernel is the one that needs scratch: when it splits K,
its partial tiles and arrival tickets go to the fixed array.  The bf16
tensor-core kernel sums its partials in shared memory, so its no-alloc call
is the same launch as dkv_gemm's.  Both must give bit-identical results.

The file name makes pytest collect it last, so it runs both after every other
GPU test (the shared scratch array then holds stale partials) and alone in a
fresh process (the first call does the device set-up)."""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

LIMIT = 16 << 20      # DKV_GEMM_NOALLOC_SCRATCH_BYTES


def _lib():
    from draftkv import _lib
    _lib.load()
    return _lib


def _epi(L, out, ld, dtype_code):
    e = L.EpilogueS()
    e.kind = L.EPI_STORE
    e.out_f32 = out.data_ptr()
    e.ld_out = ld
    e.act_dtype = dtype_code
    return e


def _weights(L, M, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn((M, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    Wt = L.pack_weight(W)
    return W, Wt, g


def _with_work(L, X, Wt, M, N, K, dtype_code):
    out = torch.zeros((N, M), dtype=torch.float32, device="cuda")
    work = torch.zeros(int(L.load().dkv_gemm_work_bytes(M, N, K, dtype_code)), dtype=torch.uint8, device="cuda")
    e = _epi(L, out, M, dtype_code)
    L.call("dkv_gemm", X.data_ptr(), dtype_code, Wt.data_ptr(), dtype_code, M, N, K, C.byref(e),
           work.data_ptr(), work.numel(), L.stream_ptr())
    return out


def _no_alloc(L, X, Wt, M, N, K, dtype_code):
    out = torch.full((N, M), float("nan"), dtype=torch.float32, device="cuda")
    e = _epi(L, out, M, dtype_code)
    L.call("dkv_gemm_noalloc", X.data_ptr(), dtype_code, Wt.data_ptr(), dtype_code, M, N, K, C.byref(e),
           L.stream_ptr())
    return out


# (M, K, N) bf16 decode shapes, and one with more row tiles x token blocks
# than the fixed array has tickets (no scratch is involved either way).
@pytest.mark.parametrize("M,K,N", [(4096, 4096, 36), (1024, 1536, 100), (384, 576, 5), (16384, 256, 2100)])
def test_no_alloc_bf16_gemm_matches_dkv_gemm_twice(M, K, N):
    """Bit-identical to dkv_gemm (a caller may mix the two and keep the
    verify-row == decode-row identity), and within 1e-4 of a torch fp32
    product."""
    L = _lib()
    W, Wt, g = _weights(L, M, K, M + K)
    for call in range(2):     # two calls in a row, different inputs
        X = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
        want = _with_work(L, X, Wt, M, N, K, L.BF16)
        got = _no_alloc(L, X, Wt, M, N, K, L.BF16)
        torch.cuda.synchronize()
        code = C.c_uint32(0)
        L.call("dkv_device_error", C.byref(code), L.stream_ptr())
        assert code.value == 0
        assert torch.equal(got, want), f"call {call}: max diff {(got - want).abs().max().item()}"
        torch.testing.assert_close(got, X.float() @ W.float().t(), rtol=1e-4, atol=1e-4, msg=f"call {call}")


# (M, K, N) fp32 shapes whose K is split (3 and 4 ways): the partial tiles
# and tickets live in the fixed array
@pytest.mark.parametrize("M,K,N", [(1024, 1536, 9), (512, 768, 37)])
def test_no_alloc_f32_gemm_matches_dkv_gemm_twice(M, K, N):
    """Two calls in a row (the array keeps the previous call's partials and
    must be re-armed): bit-identical to dkv_gemm, within 1e-4 of torch fp32."""
    L = _lib()
    g = torch.Generator(device="cuda").manual_seed(M)
    W = torch.randn((M, K), generator=g, device="cuda") * 0.05
    for call in range(2):
        X = torch.randn((N, K), generator=g, device="cuda")
        want = _with_work(L, X, W, M, N, K, L.F32)
        got = _no_alloc(L, X, W, M, N, K, L.F32)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: max diff {(got - want).abs().max().item()}"
        torch.testing.assert_close(got, X @ W.t(), rtol=1e-4, atol=1e-4, msg=f"call {call}")


def test_no_alloc_rejects_shapes_beyond_the_fixed_scratch():
    L = _lib()
    M, K, N = 4096, 4096, 320
    # the fp32 kernel's split-K partials: 80 token blocks x 32 row tiles x 4
    # K splits x a 4 x 132 fp32 tile, ~22 MB
    need = 80 * 32 * 4 * 4 * 132 * 4
    assert need > LIMIT + (1 << 20)
    x = torch.zeros(16, dtype=torch.float32, device="cuda")     # never read: rejected before launch
    out = torch.zeros(16, dtype=torch.float32, device="cuda")
    e = _epi(L, out, M, L.F32)
    rc = L.load().dkv_gemm_noalloc(x.data_ptr(), L.F32, x.data_ptr(), L.F32, M, N, K, C.byref(e),
                                   L.stream_ptr())
    assert rc == L.EINVAL
    assert b"fixed array" in L.load().dkv_last_error()
