"""Kernel-level parity on the GPU, through the C ABI, against the CPU oracle.

Bit-exact where the work is integer / byte / index work (quantization codes,
scales, packed bytes, kept slot sets); within an fp32 tolerance written in each
test for floating point.
"""

import ctypes as C
import json

import numpy as np
import pytest

import oracle
from oracle.caches import OracleComp
from draftkv.config import CompressionConfig
from draftkv.weights import round_bf16
from tests.golden.make_golden import QUANT_CASES

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def lib():
    from draftkv import _lib
    return _lib


@pytest.fixture(scope="module")
def quant_npz(golden_dir):
    return np.load(golden_dir / "quantize.npz")


# ------------------------------------------------------------------ K1
@pytest.mark.parametrize("cid", [c for _, c in QUANT_CASES])
@pytest.mark.parametrize("bits", [2, 3, 4, 8, 16])
def test_quantize_matches_reference_bit_for_bit(quant_npz, cid, bits):
    from draftkv import quantize
    x = quant_npz[f"x{cid}"]
    got = quantize(x, bits)
    want = quant_npz[f"deq{cid}_b{bits}"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_codes_scale_lo_bit_exact(bits):
    from draftkv import quantize_codes
    rng = np.random.default_rng(bits)
    x = (rng.standard_normal((300, 2, 128)) * rng.uniform(0.1, 30.0, (300, 2, 1))).astype(np.float32)
    x[3] = 0.5        # constant vectors: scale clamps to 1e-8
    codes, scale, lo, deq = quantize_codes(x, bits)
    rc, rs, rl, rd = oracle.quant_codes(x, bits)
    assert np.array_equal(codes, rc)
    assert np.array_equal(scale.view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(lo.view(np.uint32), rl.view(np.uint32))
    assert np.array_equal(deq.view(np.uint32), rd.view(np.uint32))


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("k_order", [1, 0])
@pytest.mark.parametrize("src_dtype", ["f32", "bf16"])
def test_packed_storage_bytes(d, bits, k_order, src_dtype):
    L = lib()
    rng = np.random.default_rng(d * 10 + bits)
    x = round_bf16(rng.standard_normal((97, d)).astype(np.float32) * 3)
    tdt = torch.float32 if src_dtype == "f32" else torch.bfloat16
    src = torch.from_numpy(x).to("cuda", tdt)
    codes = torch.zeros((97, d * bits // 8), dtype=torch.uint8, device="cuda")
    sl = torch.zeros((97, d // 64, 2), dtype=torch.int16, device="cuda")
    L.call("dkv_quantize_pack", src.data_ptr(), L.F32 if src_dtype == "f32" else L.BF16, 97, d, bits, k_order,
           codes.data_ptr(), sl.data_ptr(), L.stream_ptr())
    rc, rs, rl, _ = oracle.quant_codes(x, bits)
    want = oracle.pack_codes(rc[:, :d], bits, k_order=bool(k_order))
    assert np.array_equal(codes.cpu().numpy(), want)
    got_sl = sl.cpu().numpy().view(np.float16)
    assert np.array_equal(got_sl[:, :, 0], rs.astype(np.float16))
    assert np.array_equal(got_sl[:, :, 1], rl.astype(np.float16))


# ------------------------------------------------------------- K6 / K7
def _dev_comp(cfg, n_layers=2, n_kv=2, d=64, cap=64):
    from draftkv import CompressedKVCache
    return CompressedKVCache(n_layers, cfg, n_kv=n_kv, d_head=d, dtype=np.float32, capacity=cap)


@pytest.mark.parametrize("cap", [64, 60000])   # positions staged in shared memory / read from global memory
def test_eviction_trace_matches_reference(golden_dir, cap):
    """Replays the reference trace (append + note_attention, truncation) on the
    device cache: kept positions exact after every step, scores to fp32."""
    states = json.loads((golden_dir / "evict_trace.json").read_text())["states"]
    comp = _dev_comp(CompressionConfig(bits=4, keep_frac=0.5, sink=2, recent=4), cap=cap)
    rng = np.random.default_rng(7)
    pos = 0
    for step, want in enumerate(states):
        n_rows = 1 if step % 7 else 3
        for L in range(2):
            k = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            v = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            comp.append(L, k, v, np.arange(pos, pos + n_rows))
            n_live = len(comp.read(L)[2])
            probs = rng.random((1, 2, n_live)).astype(np.float32)
            probs /= probs.sum(-1, keepdims=True)
            comp.note_attention(L, probs)
        pos += n_rows
        if step % 9 == 8:
            pos -= 2
            comp.truncate(pos)
        assert comp.seen_positions == want["seen"], step
        for L in range(2):
            p, s = comp.scores(L)
            assert p.tolist() == want["pos"][L], (step, L)
            np.testing.assert_allclose(s, want["score"][L], rtol=2e-6, atol=1e-6)


def _filled_full(n, n_layers=2, n_kv=2, d=64, seed=0, dtype=np.float32):
    from draftkv import FullKVCache
    full = FullKVCache(n_layers, n_kv, d, dtype, capacity=max(n, 16))
    ref = oracle.OracleFull(n_layers)
    rng = np.random.default_rng(seed)
    for L in range(n_layers):
        k = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
        v = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
        full.append(L, k, v, np.arange(n))
        ref.append(L, k, v, np.arange(n))
    return full, ref


@pytest.mark.parametrize("cfg", [CompressionConfig(4, 0.5), CompressionConfig(2, 0.25, 4, 8),
                                 CompressionConfig(8, 1.0), CompressionConfig(3, 0.5, 0, 16),
                                 CompressionConfig(16, 0.25)], ids=lambda c: c.label() + f"-s{c.sink}r{c.recent}")
def test_sync_from_zero_keeps_the_reference_slots(cfg):
    full, ref = _filled_full(150)
    comp = _dev_comp(cfg, cap=256)
    rcomp = OracleComp(2, cfg)
    assert comp.sync_from(full, 0) == rcomp.sync_from(ref, 0)
    assert comp.seen_positions == rcomp.seen
    for L in range(2):
        k, v, p = comp.read(L)
        assert p.tolist() == rcomp.pos[L]
        rk = np.stack(rcomp.k[L])
        rv = np.stack(rcomp.v[L])
        # fp16 storage of (scale, lo) against the reference's fp32: half a step
        tol = 0.51 * (np.abs(rk).max() / ((1 << cfg.bits) - 1) if cfg.bits < 16 else 1e-6) + 1e-3
        assert np.abs(k - rk).max() <= tol
        assert np.abs(v - rv).max() <= 0.51 * (np.abs(rv).max() / ((1 << cfg.bits) - 1) if cfg.bits < 16 else 1e-6) + 1e-3


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bits", [2, 3, 4, 8, 16])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rebuild_bytes_match_reference_packing(d, bits, dtype):
    """The rebuild's codes, (scale, lo) and raw 16-bit vectors, byte for byte
    against the reference quantizer packed in the storage order."""
    n, n_kv = 150, 2
    full, ref = _filled_full(n, n_kv=n_kv, d=d, seed=bits, dtype=dtype)
    from draftkv import CompressedKVCache
    comp = CompressedKVCache(2, CompressionConfig(bits, 1.0), n_kv=n_kv, d_head=d, dtype=dtype, capacity=256)
    comp.sync_from(full, 0)
    torch.cuda.synchronize()
    for L in range(2):
        rk, rv, _ = ref.read(L)                                    # [n][n_kv][d]
        for name, x, k_order in (("k", rk, True), ("v", rv, False)):
            codes = comp.code_rows(name, L)[:, :n].cpu().numpy()                  # [n_kv][n][bytes]
            sl = getattr(comp, name + "_sl")[0, L, :, :n].cpu().numpy().view(np.float16)
            for h in range(n_kv):
                if bits == 16:
                    order = oracle.quant.fragment_order(d) if k_order else np.arange(d)
                    raw = np.ascontiguousarray(x[:, h, order], dtype=np.float32)
                    want = (raw.astype(np.float32).view(np.uint8).reshape(n, -1) if dtype == "f32" else
                            (raw.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
                            .reshape(n, -1))
                    assert np.array_equal(codes[h][:, :want.shape[1]], want), (L, name, h)
                    continue
                rc, rs, rl, _ = oracle.quant_codes(x[:, h], bits)
                want = oracle.pack_codes(rc[:, :d], bits, k_order=k_order)
                assert np.array_equal(codes[h][:, :want.shape[1]], want), (L, name, h)
                assert np.array_equal(sl[h][:, :, 0], rs.astype(np.float16)), (L, name, h)
                assert np.array_equal(sl[h][:, :, 1], rl.astype(np.float16)), (L, name, h)


def test_resync_rewrites_the_suffix():
    """Reference tests/test_lossless.py:60-77 on the device cache."""
    full, ref = _filled_full(120)
    comp = _dev_comp(CompressionConfig(8, 1.0), cap=256)
    comp.sync_from(full, 0)
    assert comp.length == full.length
    comp.truncate(10)
    assert comp.length == 10
    rows = comp.sync_from(full, 10)
    assert rows == (120 - 10) * 2
    assert comp.length == 120


def test_resync_with_eviction_matches_reference():
    cfg = CompressionConfig(4, 0.5, 2, 6)
    full, ref = _filled_full(80)
    comp = _dev_comp(cfg, cap=128)
    rcomp = OracleComp(2, cfg)
    comp.sync_from(full, 0)
    rcomp.sync_from(ref, 0)
    rng = np.random.default_rng(3)
    for it in range(6):
        for L in range(2):
            n = len(rcomp.pos[L])
            probs = rng.random((1, 2, n)).astype(np.float32)
            comp.note_attention(L, probs)
            rcomp.note_attention(L, probs)
        cut = 80 - 3 * (it + 1)
        comp.truncate(cut)
        rcomp.truncate(cut)
        assert comp.sync_from(full, cut) == rcomp.sync_from(ref, cut)
        for L in range(2):
            assert comp.read(L)[2].tolist() == rcomp.pos[L], (it, L)


def test_only_changed_layers_are_rebuilt():
    """Reference tests/test_adaptive.py:130-153 on the device cache."""
    full, _ = _filled_full(64, n_layers=3)
    a, b = CompressionConfig(2, 0.25), CompressionConfig(8, 1.0)
    comp = _dev_comp([a, a, a], n_layers=3, cap=128)
    comp.sync_from(full, 0)
    before = [comp.read(L)[0].copy() for L in range(3)]
    rows = comp.rebuild_layers(full, [1], [a, b, a])
    assert rows == 64 and comp.cfgs[1] == b
    for L in range(3):
        same = comp.read(L)[0].shape == before[L].shape and np.array_equal(comp.read(L)[0], before[L])
        assert same == (L != 1), L


# ------------------------------------------------------------------- K4
def _gemm(x, w_tiled, M, N, K, kind, dtype_code, out=None, ld=None, work=None):
    L = lib()
    if work is None:
        work = torch.zeros(int(L.load().dkv_gemm_work_bytes(M, N, K, dtype_code)), dtype=torch.uint8, device="cuda")
    e = L.EpilogueS()
    e.kind = kind
    e.out_f32 = out.data_ptr()
    e.ld_out = ld
    e.act_dtype = dtype_code
    L.call("dkv_gemm", x.data_ptr(), dtype_code, w_tiled.data_ptr(), dtype_code, M, N, K, C.byref(e),
           work.data_ptr(), work.numel(), L.stream_ptr())
    return work


@pytest.mark.parametrize("M,K", [(256, 128), (384, 576), (1024, 1536)])
def test_bf16_gemm_matches_torch_and_is_batch_invariant(M, K):
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(M + K)
    W = (torch.randn((M, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    Wt = L.pack_weight(W)
    X = torch.randn((1100, K), generator=g, device="cuda").to(torch.bfloat16)
    ref = X.float() @ W.float().t()
    outs = {}
    for N in (1, 5, 37, 64, 100, 300, 1100):    # token tiles of 16 .. 64, 128 and 256
        out = torch.zeros((N, M), dtype=torch.float32, device="cuda")
        _gemm(X[:N].contiguous(), Wt, M, N, K, L.EPI_STORE, L.BF16, out=out, ld=M)
        torch.testing.assert_close(out, ref[:N], rtol=1e-4, atol=1e-4)
        outs[N] = out
    for N in (5, 37, 64, 100, 300, 1100):     # token 0's column is bit-identical whatever N
        assert torch.equal(outs[N][0], outs[1][0])
    assert torch.equal(outs[100][:64], outs[64])
    assert torch.equal(outs[1100][:300], outs[300])


@pytest.mark.parametrize("M,K", [(4096, 4096), (1024, 512)])
@pytest.mark.parametrize("N", [4, 36, 600])
def test_fused_rmsnorm_epilogues(M, K, N):
    """The two halves of the RMSNorm fused into the bf16 GEMM (llama.py:93-94).
    Output side (RESADD): h_new = h + X W^T + b, xn = bf16(h_new * w) and the
    sums of h_new^2 over each 128-row tile, against torch fp32.  Input side
    (STORE) on those: Y = (xn W2^T) / rms(h_new) + b2 per token.  Both
    shapes run the split-K cluster reduction (4096 x 4096) and the unsplit
    kernel (1024 x 512); a token's results do not depend on N."""
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(M + N)
    W = (torch.randn((M, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    X = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
    h0 = torch.randn((N, M), generator=g, device="cuda") * 3
    b = torch.randn(M, generator=g, device="cuda") * 0.1
    wn = torch.rand(M, generator=g, device="cuda") + 0.5
    W2 = (torch.randn((256, M), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    b2 = torch.randn(256, generator=g, device="cuda") * 0.1
    eps = 1e-5
    Wt, W2t = L.pack_weight(W), L.pack_weight(W2)
    work = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    ld = N + 3
    h = h0.clone()
    xn = torch.zeros((N, M), dtype=torch.bfloat16, device="cuda")
    part = torch.full((M // 128, ld), -1.0, device="cuda")
    e = L.EpilogueS()
    e.kind = L.EPI_RESADD
    e.bias = b.data_ptr()
    e.out_f32 = h.data_ptr()
    e.ld_out = M
    e.act_dtype = L.BF16
    e.norm_out_part = part.data_ptr()
    e.norm_out_x = xn.data_ptr()
    e.norm_out_w = wn.data_ptr()
    e.norm_ld = ld
    L.call("dkv_gemm", X.data_ptr(), L.BF16, Wt.data_ptr(), L.BF16, M, N, K, C.byref(e), work.data_ptr(),
           work.numel(), L.stream_ptr())
    torch.cuda.synchronize()
    h_ref = h0 + (X.float() @ W.float().t() + b)
    torch.testing.assert_close(h, h_ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(xn.float(), (h * wn).to(torch.bfloat16).float(), rtol=0, atol=0)
    sq = (h * h).view(N, M // 128, 128).sum(-1).t()
    torch.testing.assert_close(part[:, :N], sq, rtol=1e-5, atol=1e-5)
    assert torch.all(part[:, N:] == -1.0)
    out = torch.zeros((N, 256), device="cuda")
    e2 = L.EpilogueS()
    e2.kind = L.EPI_STORE
    e2.bias = b2.data_ptr()
    e2.out_f32 = out.data_ptr()
    e2.ld_out = 256
    e2.act_dtype = L.BF16
    e2.norm_in_part = part.data_ptr()
    e2.norm_n_part = M // 128
    e2.norm_ld = ld
    e2.norm_dm = M
    e2.norm_eps = eps
    L.call("dkv_gemm", xn.data_ptr(), L.BF16, W2t.data_ptr(), L.BF16, 256, N, M, C.byref(e2), work.data_ptr(),
           work.numel(), L.stream_ptr())
    torch.cuda.synchronize()
    inv = 1.0 / torch.sqrt((h * h).mean(-1, keepdim=True) + eps)
    ref = (xn.float() @ W2.float().t()) * inv + b2
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    # the same tokens at N = 1: bit-identical rows
    if N > 1:
        h1 = h0[:1].clone()
        xn1 = torch.zeros((1, M), dtype=torch.bfloat16, device="cuda")
        part1 = torch.zeros((M // 128, 1), device="cuda")
        e.out_f32, e.norm_out_x, e.norm_out_part, e.norm_ld = h1.data_ptr(), xn1.data_ptr(), part1.data_ptr(), 1
        L.call("dkv_gemm", X[:1].contiguous().data_ptr(), L.BF16, Wt.data_ptr(), L.BF16, M, 1, K, C.byref(e),
               work.data_ptr(), work.numel(), L.stream_ptr())
        torch.cuda.synchronize()
        assert torch.equal(h1[0], h[0]) and torch.equal(xn1[0], xn[0]) and torch.equal(part1[:, 0], part[:, 0])


def test_fused_rmsnorm_rejects_f32_and_wrong_kinds():
    L = lib()
    lib_ = L.load()
    x = torch.zeros((4, 256), device="cuda")
    w = torch.zeros((128, 256), device="cuda")
    out = torch.zeros((4, 128), device="cuda")
    part = torch.zeros((2, 4), device="cuda")
    work = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    e = L.EpilogueS()
    e.kind = L.EPI_STORE
    e.out_f32 = out.data_ptr()
    e.ld_out = 128
    e.norm_in_part = part.data_ptr()
    e.norm_n_part, e.norm_ld, e.norm_dm = 2, 4, 256
    rc = lib_.dkv_gemm(x.data_ptr(), L.F32, w.data_ptr(), L.F32, 128, 4, 256, C.byref(e), work.data_ptr(),
                       work.numel(), L.stream_ptr())
    assert rc != 0 and b"bf16" in lib_.dkv_last_error()
    e2 = L.EpilogueS()
    e2.kind = L.EPI_STORE
    e2.out_f32 = out.data_ptr()
    e2.ld_out = 128
    e2.norm_out_x = out.data_ptr()
    rc = lib_.dkv_gemm(x.data_ptr(), L.BF16, w.data_ptr(), L.BF16, 128, 4, 256, C.byref(e2), work.data_ptr(),
                       work.numel(), L.stream_ptr())
    assert rc != 0 and b"RESADD" in lib_.dkv_last_error()


def test_f32_gemm_matches_torch():
    L = lib()
    M, K = 256, 192
    g = torch.Generator(device="cuda").manual_seed(1)
    W = torch.randn((M, K), generator=g, device="cuda")
    X = torch.randn((9, K), generator=g, device="cuda")
    out = torch.zeros((9, M), device="cuda")
    _gemm(X, W, M, 9, K, L.EPI_STORE, L.F32, out=out, ld=M)
    torch.testing.assert_close(out, X @ W.t(), rtol=1e-5, atol=1e-4)


# ------------------------------------------------------------- K2
@pytest.mark.parametrize("bits", [2, 3, 4, 8, 16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_draft_attention_and_mass(bits, d, dtype):
    """Drafter attention (T = 1) over the quantized slot cache vs a torch fp32
    reference on the read-back (dequantized) entries, and the attention mass
    folded into the slot scores (compress.py:144-151 + llama.py:213-216).
    Tolerances: output 2e-2 of the output scale (f16 / bf16 operands), mass
    1e-3 absolute + 3e-2 relative (bf16 queries of the 16-bit arm carry ~1%
    probability error)."""
    from draftkv import CompressedKVCache
    L = lib()
    B, n_kv, G, n = 2, 2, 4, 900
    full_pages = -(-n // 16)
    from draftkv import FullKVCache
    full = FullKVCache(1, n_kv, d, dtype, capacity=n + 16, batch=B)
    rng = np.random.default_rng(bits * 7 + d)
    for b in range(B):
        full.ensure(b, n)
    k = round_bf16(rng.standard_normal((B, n, n_kv, d)).astype(np.float32))
    v = round_bf16(rng.standard_normal((B, n, n_kv, d)).astype(np.float32))
    src = torch.from_numpy(np.stack([k, v], axis=3)).to("cuda", torch.float32 if dtype == "f32" else torch.bfloat16)
    p0 = torch.zeros((B,), dtype=torch.int32, device="cuda")
    L.call("dkv_full_write", full.struct(), full.dims(), 0, src.data_ptr(), n, p0.data_ptr(), None, L.stream_ptr())
    for b in range(B):
        full.set_length(b, n)
    comp = CompressedKVCache(1, CompressionConfig(bits, 0.5, 4, 32), n_kv=n_kv, d_head=d, dtype=dtype,
                             capacity=n + 8, batch=B)
    comp.sync_from(full, 0)
    # give the slots distinct scores, then evict a few more through a resync
    comp.score_t.copy_(torch.rand_like(comp.score_t))
    q = torch.from_numpy(rng.standard_normal((B, n_kv * G, d)).astype(np.float32) * 2).cuda()
    qpos = torch.full((B,), n, dtype=torch.int32, device="cuda")
    out = torch.zeros((B, n_kv * G * d), dtype=torch.float32, device="cuda")
    dims = comp.dims()
    work = torch.zeros(int(L.load().dkv_attn_work_bytes(dims, G, 1, 16, 512, comp.cap)), dtype=torch.uint8,
                       device="cuda")
    before = comp.score_t.clone()
    L.call("dkv_attn_comp", comp.struct(), dims, 0, G, q.data_ptr(), qpos.data_ptr(), out.data_ptr(), L.F32,
           work.data_ptr(), work.numel(), L.stream_ptr())
    after = comp.score_t.clone()
    for b in range(B):
        kk, vv, pp = comp.read(0, b)
        pos_all = comp.pos_t[b, 0].cpu().numpy()
        kt = torch.from_numpy(kk).cuda().repeat_interleave(G, dim=1)
        vt = torch.from_numpy(vv).cuda().repeat_interleave(G, dim=1)
        s = torch.einsum("hd,khd->hk", q[b], kt) / np.sqrt(d)
        pr = torch.softmax(s, -1)
        ref = torch.einsum("hk,khd->hd", pr, vt).reshape(-1)
        scale = ref.abs().max().item()
        assert (out[b] - ref).abs().max().item() <= 2e-2 * scale, b
        mass = pr.reshape(n_kv, G, -1).sum(dim=(0, 1)).cpu().numpy()        # per live entry, position order
        live = np.nonzero(pos_all >= 0)[0]
        live = live[np.argsort(pos_all[live], kind="stable")]
        got = (after[b, 0] - before[b, 0]).cpu().numpy()[live]
        np.testing.assert_allclose(got, mass, atol=1e-3, rtol=3e-2)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("d", [64, 128])
def test_draft_attention_keep_whole_skips_scores(bits, d):
    """A layer kept whole (keep 1.0) never evicts, so the tensor-core drafter
    kernel does not fold the attention mass into the slot scores: the output
    still matches a torch fp32 reference on the read-back entries (2e-2 of
    the output scale, f16 operands) and the scores are left as they were."""
    from draftkv import CompressedKVCache, FullKVCache
    L = lib()
    B, n_kv, G, n = 2, 2, 4, 700
    full = FullKVCache(1, n_kv, d, "bf16", capacity=n + 16, batch=B)
    rng = np.random.default_rng(bits * 11 + d)
    for b in range(B):
        full.ensure(b, n)
    k = round_bf16(rng.standard_normal((B, n, n_kv, d)).astype(np.float32))
    v = round_bf16(rng.standard_normal((B, n, n_kv, d)).astype(np.float32))
    src = torch.from_numpy(np.stack([k, v], axis=3)).to("cuda", torch.bfloat16)
    p0 = torch.zeros((B,), dtype=torch.int32, device="cuda")
    L.call("dkv_full_write", full.struct(), full.dims(), 0, src.data_ptr(), n, p0.data_ptr(), None, L.stream_ptr())
    for b in range(B):
        full.set_length(b, n)
    comp = CompressedKVCache(1, CompressionConfig(bits, 1.0), n_kv=n_kv, d_head=d, dtype="bf16",
                             capacity=n + 8, batch=B)
    comp.sync_from(full, 0)
    comp.score_t.copy_(torch.rand_like(comp.score_t))
    q = torch.from_numpy(rng.standard_normal((B, n_kv * G, d)).astype(np.float32) * 2).cuda()
    qpos = torch.full((B,), n, dtype=torch.int32, device="cuda")
    out = torch.zeros((B, n_kv * G * d), dtype=torch.float32, device="cuda")
    dims = comp.dims()
    work = torch.zeros(int(L.load().dkv_attn_work_bytes(dims, G, 1, 16, 512, comp.cap)), dtype=torch.uint8,
                       device="cuda")
    before = comp.score_t.clone()
    L.call("dkv_attn_comp", comp.struct(), dims, 0, G, q.data_ptr(), qpos.data_ptr(), out.data_ptr(), L.F32,
           work.data_ptr(), work.numel(), L.stream_ptr())
    assert torch.equal(comp.score_t, before)
    for b in range(B):
        kk, vv, _ = comp.read(0, b)
        kt = torch.from_numpy(kk).cuda().repeat_interleave(G, dim=1)
        vt = torch.from_numpy(vv).cuda().repeat_interleave(G, dim=1)
        s_ = torch.einsum("hd,khd->hk", q[b], kt) / np.sqrt(d)
        ref = torch.einsum("hk,khd->hd", torch.softmax(s_, -1), vt).reshape(-1)
        assert (out[b] - ref).abs().max().item() <= 2e-2 * ref.abs().max().item(), b


# ------------------------------------------------------------- K3
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("G", [1, 4])
@pytest.mark.parametrize("d", [64, 128])
def test_full_attention_matches_torch_and_decode(dtype, G, d):
    """Causal GQA attention over the paged cache vs a torch fp32 reference
    (fp32 cache: 2e-5; bf16 cache through the tensor-core kernel, whose q and
    p operands are bf16: 1e-2); the T-row verify result equals T separate
    decode calls bit for bit."""
    from draftkv import PagedKVCache
    L = lib()
    n_kv, n = 2, 700
    code = L.F32 if dtype == "f32" else L.BF16
    # 160 pages: 20 splits of 128 keys, past the merge's static 16 (the
    # tensor-core kernel stages the split weights in its drained ring)
    cache = PagedKVCache(1, n_kv, d, 16, 160, dtype, batch=1)
    rng = np.random.default_rng(G)
    k = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    v = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    cache.append(0, k, v, np.arange(n))
    T = 6
    p0 = n - T
    q = torch.from_numpy(rng.standard_normal((T, n_kv * G, d)).astype(np.float32)).cuda()
    pos0 = torch.tensor([p0], dtype=torch.int32, device="cuda")
    dims = cache.dims()
    work = torch.zeros(int(L.load().dkv_attn_work_bytes(dims, G, T, cache.capacity_tokens, 128, 0)),
                       dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, n_kv * G * d), dtype=torch.float32, device="cuda")
    L.call("dkv_attn_full", cache.struct(), dims, 0, G, T, q.data_ptr(), pos0.data_ptr(), out.data_ptr(), L.F32,
           128, work.data_ptr(), work.numel(), L.stream_ptr())
    # reference
    kk = torch.from_numpy(k).cuda().repeat_interleave(G, dim=1)
    vv = torch.from_numpy(v).cuda().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->qhk", q, kk) / np.sqrt(d)
    mask = torch.arange(n, device="cuda")[None, :] > (p0 + torch.arange(T, device="cuda"))[:, None]
    s = s.masked_fill(mask[:, None, :], float("-inf"))
    ref = torch.einsum("qhk,khd->qhd", torch.softmax(s, -1), vv).reshape(T, -1)
    tol = 2e-5 if dtype == "f32" else 1e-2
    torch.testing.assert_close(out, ref, rtol=tol, atol=tol)
    for t in range(T):
        o1 = torch.zeros((1, n_kv * G * d), dtype=torch.float32, device="cuda")
        pt = torch.tensor([p0 + t], dtype=torch.int32, device="cuda")
        L.call("dkv_attn_full", cache.struct(), dims, 0, G, 1, q[t:t + 1].contiguous().data_ptr(), pt.data_ptr(),
               o1.data_ptr(), L.F32, 128, work.data_ptr(), work.numel(), L.stream_ptr())
        assert torch.equal(o1[0], out[t]), t


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("G", [1, 4])
@pytest.mark.parametrize("n,T,split", [(700, 700, 3648), (1000, 37, 256), (4100, 300, 1024), (40000, 300, 128)])
def test_prefill_attention_matches_torch(d, G, n, T, split):
    """The tcgen05 prefill kernel (more than 64 query rows, bf16 pool in
    device memory): causal GQA attention of T new tokens at positions
    n-T..n-1 against a float64 reference, at most 2e-2 per element and 1e-3
    on average.  q * scale * log2 e and p are bf16 operands: in these cases
    that rounding alone (modelled in float64 with the kernel's 128-key tiles,
    splits and lazy rescale) moves single outputs by up to 1.24e-2 and the
    mean by 2.5e-4 to 5.8e-4.  Cases: a whole 700-token prompt (ragged last
    row block, one split), 37 tokens over 1000 keys in 256-key splits (rows
    whose split starts past their position), 300 tokens over 4100 keys, and
    over 40000 keys (the prompt kernel's splits are at least 16384 keys: 3
    splits merged, through the weights staged in the drained ring); every
    context ends inside a page whose unused rows hold NaN."""
    from draftkv import PagedKVCache
    L = lib()
    n_kv = 2
    cache = PagedKVCache(1, n_kv, d, 16, (n + 15) // 16 + 4, "bf16", batch=1)
    cache.k_pool.fill_(float("nan"))
    cache.v_pool.fill_(float("nan"))
    rng = np.random.default_rng(n + G + d)
    k = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    v = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    cache.append(0, k, v, np.arange(n))
    p0 = n - T
    q = torch.from_numpy(rng.standard_normal((T, n_kv * G, d)).astype(np.float32) * 2).cuda()
    pos0 = torch.tensor([p0], dtype=torch.int32, device="cuda")
    dims = cache.dims()
    work = torch.zeros(int(L.load().dkv_attn_work_bytes(dims, G, T, cache.capacity_tokens, split, 0)),
                       dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, n_kv * G * d), dtype=torch.float32, device="cuda")
    kk = torch.from_numpy(k).cuda().repeat_interleave(G, dim=1).double()
    vv = torch.from_numpy(v).cuda().repeat_interleave(G, dim=1).double()
    mask = torch.arange(n, device="cuda")[None, :] > (p0 + torch.arange(T, device="cuda"))[:, None]
    s = torch.einsum("qhd,khd->qhk", q.double(), kk) / np.sqrt(d)
    s = s.masked_fill(mask[:, None, :], float("-inf"))
    ref = torch.einsum("qhk,khd->qhd", torch.softmax(s, -1), vv).reshape(T, -1).float()
    for _ in range(2):       # the second launch reuses the tickets the first one reset
        out.zero_()
        L.call("dkv_attn_full", cache.struct(), dims, 0, G, T, q.data_ptr(), pos0.data_ptr(), out.data_ptr(), L.F32,
               split, work.data_ptr(), work.numel(), L.stream_ptr())
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out, ref, rtol=2e-2, atol=2e-2)
        assert (out - ref).abs().mean().item() <= 1e-3
    code = C.c_uint32(0)
    L.call("dkv_device_error", C.byref(code), L.stream_ptr())
    assert code.value == 0


def test_drafter_capacity_is_whole_tiles():
    """The tensor-core drafter kernel copies 16-slot tiles: every capacity the
    cache allocates (initial and grown) is a multiple of 16."""
    from draftkv import CompressedKVCache
    comp = CompressedKVCache(2, CompressionConfig(4, 0.5), n_kv=2, d_head=64, dtype="bf16", capacity=1000)
    comp.materialize(2, 64, "bf16") if hasattr(comp, "materialize") else None
    assert comp.cap % 16 == 0 and comp.cap >= 1000
    comp._grow(2049)
    assert comp.cap % 16 == 0 and comp.cap >= 2049


def test_full_attention_reads_pages_anywhere_in_a_large_pool():
    """Pages far into a large pool (ids above 2^31 elements / page size, as a
    32-layer, 4-sequence, 32k-context pool has) are read correctly by the
    copy-engine path: T = 1 attention over 40 pages of ids 139900.. against a
    torch fp32 reference (1e-2, bf16 operands)."""
    from draftkv import PagedKVCache
    L = lib()
    n_kv, d, G, n = 8, 128, 4, 640
    cache = PagedKVCache(1, n_kv, d, 16, 140000, "bf16", batch=1, max_blocks_per_seq=64)
    pages = list(range(139900, 139900 + n // 16 + 1))
    cache.block_tables[0][0] = list(pages)
    for i, p in enumerate(pages):
        cache.table_host[0, 0, i] = p
    cache._dirty = True
    rng = np.random.default_rng(5)
    k = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    v = round_bf16(rng.standard_normal((n, n_kv, d)).astype(np.float32))
    src = torch.from_numpy(np.stack([k, v], axis=2)).to("cuda", torch.bfloat16)
    p0 = torch.zeros((1,), dtype=torch.int32, device="cuda")
    L.call("dkv_full_write", cache.struct(), cache.dims(), 0, src.data_ptr(), n, p0.data_ptr(), None, L.stream_ptr())
    cache.set_length(0, n)
    q = torch.from_numpy(rng.standard_normal((1, n_kv * G, d)).astype(np.float32)).cuda()
    pos0 = torch.tensor([n - 1], dtype=torch.int32, device="cuda")
    dims = cache.dims()
    work = torch.zeros(int(L.load().dkv_attn_work_bytes(dims, G, 1, cache.capacity_tokens, 128, 0)),
                       dtype=torch.uint8, device="cuda")
    out = torch.zeros((1, n_kv * G * d), dtype=torch.float32, device="cuda")
    L.call("dkv_attn_full", cache.struct(), dims, 0, G, 1, q.data_ptr(), pos0.data_ptr(), out.data_ptr(), L.F32,
           128, work.data_ptr(), work.numel(), L.stream_ptr())
    kk = torch.from_numpy(k).cuda().repeat_interleave(G, dim=1)
    vv = torch.from_numpy(v).cuda().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->qhk", q, kk) / np.sqrt(d)
    ref = torch.einsum("qhk,khd->qhd", torch.softmax(s, -1), vv).reshape(1, -1)
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
