// Tensor-core attention over the paged full cache (bf16): verify, baseline
// decode and prefill chunks.  Replaces draftkv/llama.py:202-219 /
// draftkv/gpt2.py:197-207 over FullKVCache / PagedKVCache.
//
// Prefill chunks (> 64 query rows): one CTA per (key split, KV head, sequence
// x row block); 4 warps.  K/V pages of the split stream through a
// double-buffered, XOR-swizzled shared-memory tile of 64 keys with cp.async;
// warp w owns query rows [16w, 16w+16) of the CTA (rows = token x GQA head)
// and runs S = Q K^T and O += P V with mma.sync.m16n8k16 (bf16 in, fp32
// accumulate) and a per-row online softmax.  Decode and verify (<= 64 rows)
// take attn_kq_kernel below, whose tiles the copy engine (TMA) fetches one
// page at a time when the pool is in device memory.
// The CTA partials merge in split order (split_merge), so a row's result does
// not depend on how many rows share the launch: verify row i equals the
// one-token decode at that position bit for bit.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "attn_common.cuh"

namespace dkv {

uint32_t* device_error_word();

DKV_DEV uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

DKV_DEV void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

DKV_DEV void ldsm4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}
DKV_DEV void ldsm4t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}
DKV_DEV void cpasync16(void* smem, const void* gmem, bool pred) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(pred ? 16 : 0));
}

constexpr int kTcKT = 64;          // keys per tile
constexpr int kTcThreads = 128;    // 4 warps x 16 query rows

// swizzled element offset of (key, 16-byte chunk) in a [keys][D] bf16 tile
template <int D>
DKV_DEV int swz(int key, int chunk) {
    return key * D + ((chunk ^ (key & 7)) << 3);
}

template <int D>
__global__ void __launch_bounds__(kTcThreads) attn_full_tc_kernel(AttnArgs a) {
    constexpr int DC = D / 8;      // 16-byte chunks per key row
    constexpr int KS = D / 16;     // k16 steps over d
    extern __shared__ __align__(128) uint8_t tsm[];
    __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(tsm);        // [2][KT][D]
    __nv_bfloat16* Vs = Ks + 2 * kTcKT * D;                             // [2][KT][D]
    float* ms = reinterpret_cast<float*>(Vs + 2 * kTcKT * D);          // [kAttnRB]
    float* ls = ms + kAttnRB;

    const int s = blockIdx.x, h = blockIdx.y;
    const int b = blockIdx.z / a.n_rb, rb = blockIdx.z % a.n_rb;
    const int G = a.group, T = a.T;
    const int r0 = rb * kAttnRB;
    const int R = min(kAttnRB, T * G - r0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qr = lane >> 2, qc = lane & 3;
    const int qbase = a.qpos0[b];
    const int n_keys = qbase + T;
    const int k0 = s * a.split;
    const int k1 = min(n_keys, k0 + a.split);
    const size_t bl = (size_t)b * a.n_layers + a.layer;
    const int HQ = a.n_kv * G;
    const KeySrc& src = a.src;
    const __nv_bfloat16* kpool = reinterpret_cast<const __nv_bfloat16*>(src.k_pool);
    const __nv_bfloat16* vpool = reinterpret_cast<const __nv_bfloat16*>(src.v_pool);
    const bool active = warp * 16 < R;

    // ---- Q fragments of this warp's 16 rows (bf16, rows >= R are zero)
    uint32_t qf[KS][4];
    {
        const int rA = warp * 16 + qr, rB = rA + 8;
        const float* qa = nullptr;
        const float* qb = nullptr;
        if (rA < R) {
            const int t = (r0 + rA) / G, g = (r0 + rA) % G;
            qa = a.q + (((size_t)b * T + t) * HQ + h * G + g) * D;
        }
        if (rB < R) {
            const int t = (r0 + rB) / G, g = (r0 + rB) % G;
            qb = a.q + (((size_t)b * T + t) * HQ + h * G + g) * D;
        }
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int d0 = kk * 16 + 2 * qc;
            qf[kk][0] = qa ? pack_bf16(qa[d0], qa[d0 + 1]) : 0u;
            qf[kk][1] = qb ? pack_bf16(qb[d0], qb[d0 + 1]) : 0u;
            qf[kk][2] = qa ? pack_bf16(qa[d0 + 8], qa[d0 + 9]) : 0u;
            qf[kk][3] = qb ? pack_bf16(qb[d0 + 8], qb[d0 + 9]) : 0u;
        }
    }
    // query positions of the two rows this thread accumulates
    const int rowA = warp * 16 + qr, rowB = rowA + 8;
    const int qpA = qbase + (r0 + rowA) / G, qpB = qbase + (r0 + rowB) / G;

    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

    const int ntiles = k1 > k0 ? (k1 - k0 + kTcKT - 1) / kTcKT : 0;
    auto load_tile = [&](int buf, int t0) {
        __nv_bfloat16* kd = Ks + buf * kTcKT * D;
        __nv_bfloat16* vd = Vs + buf * kTcKT * D;
        for (int i = threadIdx.x; i < kTcKT * DC; i += kTcThreads) {
            const int key = i / DC, ch = i % DC;
            const int kp = t0 + key;
            const bool ok = kp < k1;
            size_t off = 0;
            if (ok) {
                const int page = __ldg(src.page_table + bl * src.max_pages + (kp >> src.page_shift));
                off = ((((size_t)page * a.n_kv + h) << src.page_shift) + (kp & (src.page_size - 1))) * D + ch * 8;
            }
            cpasync16(kd + swz<D>(key, ch), kpool + off, ok);
            cpasync16(vd + swz<D>(key, ch), vpool + off, ok);
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };

    if (ntiles > 0) load_tile(0, k0);
    for (int it = 0; it < ntiles; ++it) {
        const int t0 = k0 + it * kTcKT;
        if (it + 1 < ntiles) {
            load_tile((it + 1) & 1, t0 + kTcKT);
            asm volatile("cp.async.wait_group 1;\n" ::);
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::);
        }
        __syncthreads();
        if (active) {
            const __nv_bfloat16* kt = Ks + (it & 1) * kTcKT * D;
            const __nv_bfloat16* vt = Vs + (it & 1) * kTcKT * D;
            // ---- S = Q K^T over 64 keys (8 n8 tiles)
            float sc[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
            const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b0, b1, b2, b3;
                    const int key = np * 16 + (mi >> 1) * 8 + ri;
                    ldsm4(b0, b1, b2, b3, kt + swz<D>(key, 2 * kk + (mi & 1)));
                    mma_bf16_16816(sc[2 * np], qf[kk], b0, b1);
                    mma_bf16_16816(sc[2 * np + 1], qf[kk], b2, b3);
                }
            }
            // ---- scale, causal / range mask, online softmax (rows A and B)
            float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = t0 + 8 * j + 2 * qc + (e & 1);
                    const int qp = e < 2 ? qpA : qpB;
                    float v = sc[j][e] * a.scale;
                    if (key >= k1 || key > qp) v = -INFINITY;
                    sc[j][e] = v;
                }
                mxA = fmaxf(mxA, fmaxf(sc[j][0], sc[j][1]));
                mxB = fmaxf(mxB, fmaxf(sc[j][2], sc[j][3]));
            }
            mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
            mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
            mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
            mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
            const float nmA = fmaxf(mA, mxA), nmB = fmaxf(mB, mxB);
            const float alA = nmA == -INFINITY ? 1.f : expf(mA - nmA);
            const float alB = nmB == -INFINITY ? 1.f : expf(mB - nmB);
            float sumA = 0.f, sumB = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float nm = e < 2 ? nmA : nmB;
                    const float p = sc[j][e] == -INFINITY ? 0.f : expf(sc[j][e] - nm);
                    sc[j][e] = p;
                }
                sumA += sc[j][0] + sc[j][1];
                sumB += sc[j][2] + sc[j][3];
            }
            sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
            sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
            sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
            sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
            lA = lA * alA + sumA;
            lB = lB * alB + sumB;
            mA = nmA;
            mB = nmB;
#pragma unroll
            for (int j = 0; j < D / 8; ++j) {
                o[j][0] *= alA;
                o[j][1] *= alA;
                o[j][2] *= alB;
                o[j][3] *= alB;
            }
            // ---- O += P V (4 k16 steps over the 64 keys)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t pa[4];
                pa[0] = pack_bf16(sc[2 * ks][0], sc[2 * ks][1]);
                pa[1] = pack_bf16(sc[2 * ks][2], sc[2 * ks][3]);
                pa[2] = pack_bf16(sc[2 * ks + 1][0], sc[2 * ks + 1][1]);
                pa[3] = pack_bf16(sc[2 * ks + 1][2], sc[2 * ks + 1][3]);
#pragma unroll
                for (int dp = 0; dp < D / 16; ++dp) {
                    uint32_t b0, b1, b2, b3;
                    const int key = ks * 16 + (mi & 1) * 8 + ri;
                    ldsm4t(b0, b1, b2, b3, vt + swz<D>(key, 2 * dp + (mi >> 1)));
                    mma_bf16_16816(o[2 * dp], pa, b0, b1);
                    mma_bf16_16816(o[2 * dp + 1], pa, b2, b3);
                }
            }
        }
        __syncthreads();
    }

    // ---- partials (rows < R), then the split merge
    const int PS = D + 2;
    const size_t bhr = ((size_t)b * a.n_kv + h) * a.n_rb + rb;
    float* mypart = a.part + ((bhr * a.n_splits + s) * kAttnRB) * PS;
    if (active) {
        if (rowA < R) {
#pragma unroll
            for (int j = 0; j < D / 8; ++j) {
                mypart[rowA * PS + 2 + 8 * j + 2 * qc] = o[j][0];
                mypart[rowA * PS + 2 + 8 * j + 2 * qc + 1] = o[j][1];
            }
            if (qc == 0) {
                mypart[rowA * PS] = mA;
                mypart[rowA * PS + 1] = lA;
            }
        }
        if (rowB < R) {
#pragma unroll
            for (int j = 0; j < D / 8; ++j) {
                mypart[rowB * PS + 2 + 8 * j + 2 * qc] = o[j][2];
                mypart[rowB * PS + 2 + 8 * j + 2 * qc + 1] = o[j][3];
            }
            if (qc == 0) {
                mypart[rowB * PS] = mB;
                mypart[rowB * PS + 1] = lB;
            }
        }
    }
    split_merge(a, bhr, b, h, R, r0, ms, ls);
}

// ---------------------------------------------------------------------------
// Up to 64 query rows (decode, verify): keys are the MMA rows.  S^T = K Q^T
// with A = 16 keys of K (ldmatrix from the swizzled tile) and B = Q^T (8 query
// rows as columns); O^T += V^T P^T with A = V^T (ldmatrix.trans) and
// B = P^T (movmatrix of the S accumulators); the softmax sum comes from one
// more product with a row of ones.  Warp (kg, rt) takes keys [16kg, 16kg+16)
// of every 64-key tile and query rows [8rt, 8rt+8); the 4 key groups merge in
// a fixed order, so a row's arithmetic does not depend on how many rows share
// the launch: verify rows equal decode rows bit for bit.  Scores are kept in
// log2 units (log2 e folded into the query scale); partials store the max in
// natural units for the split merge.
//
// Tiles come through a 3-deep ring of 64-key slots.  With the pool in device
// memory (TMA = true) thread 0 fetches a tile with one 4-D tensor copy per
// (page, K or V, 64 dims) -- 16 copies of 2 KB for d = 128 -- completing on
// the slot's mbarrier, in the copy engine's 128-byte swizzle; keys past the
// split's end get zero V rows.  With the pool in pinned host memory
// (configuration 5) every thread issues 16-byte cp.async copies.
constexpr int kKqKG = 4;
constexpr int kKqNST = 3;
// Query rows per CTA: at most 2 row tiles (8 warps, no register spills, two
// CTAs per SM); more rows (a verify of gamma + 1 tokens x the GQA group) take
// more CTAs per (split, head), whose tiles the later ones mostly find in L2.
// A row's arithmetic is the same in any CTA.
constexpr int kKqRows = 16;
// Page ids a CTA stages in shared memory (splits of up to 8192 keys; longer
// splits look each page up in global memory).
constexpr int kKqSplitPages = 512;

template <int D>
size_t kq_smem(int RT) {
    const size_t ring = (size_t)kKqNST * 2 * kTcKT * D * 2;
    const size_t merge = (size_t)RT * kKqKG * 8 * (D + 2) * sizeof(float);
    return (ring > merge ? ring : merge) + 1024;      // + alignment slack
}

DKV_DEV uint32_t movm_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}

// Element offset of (key, 16-byte chunk) in a 64-key K or V tile.  TMA
// tiles: [d/64 halves][64 keys][64 dims], 128-byte rows with the chunk XOR
// (key % 8) that the copy engine's swizzle writes; cp.async tiles: [64][d]
// with the same XOR on the low chunk bits (both conflict-free for ldmatrix).
template <int D, bool TMA>
DKV_DEV int kv_off(int key, int chunk) {
    if constexpr (TMA)
        return (chunk >> 3) * (kTcKT * 64) + key * 64 + (((chunk & 7) ^ (key & 7)) << 3);
    else
        return swz<D>(key, chunk);
}

template <int D, int MAXT, bool TMA>
__global__ void __launch_bounds__(MAXT, 2) attn_kq_kernel(const __grid_constant__ KvMaps maps, AttnArgs a) {
    constexpr int DC = D / 8;      // 16-byte chunks per key row
    constexpr int KS = D / 16;     // k16 steps over d
    constexpr int PS = D + 2;
    constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
    extern __shared__ __align__(128) uint8_t tsm_raw[];
    // 1024-byte aligned base (the 128-byte swizzle of the copy engine)
    uint8_t* tsm = tsm_raw + ((1024u - (smem_u32(tsm_raw) & 1023u)) & 1023u);
    __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(tsm);      // [NST][K 64xD | V 64xD]
    __shared__ float ms[kAttnRB], ls[kAttnRB];
    __shared__ __align__(8) uint64_t full_bar[kKqNST];
    // page ids of this CTA's key split, staged once (copy-engine path): the
    // producer thread then issues a tile's copies without a global load
    __shared__ int32_t split_pages[kKqSplitPages];
    if (TMA && threadIdx.x == 0) {
        for (int i = 0; i < kKqNST; ++i) mbar_init(&full_bar[i], 1);
        fence_async_shared();
    }
    if (TMA) __syncthreads();    // the barriers are initialised before anyone waits on them
    pdl_trigger();
    pdl_wait();         // queries and the new cache rows come from the previous kernel

    const int s = blockIdx.x, h = blockIdx.y;
    const int b = blockIdx.z / a.n_rb, rb = blockIdx.z % a.n_rb;
    const int G = a.group, T = a.T;
    const int rbase = rb * kKqRows;                 // this CTA's rows: rbase .. rbase + R - 1
    const int R = min(kKqRows, T * G - rbase);
    const int nthreads = blockDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kg = warp % kKqKG, rt = warp / kKqKG;
    const int qr = lane >> 2, qc = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const int qbase = a.qpos0[b];
    const int n_keys = qbase + T;
    const int k0 = s * a.split;
    const int k1 = min(n_keys, k0 + a.split);
    const size_t bl = (size_t)b * a.n_layers + a.layer;
    const int HQ = a.n_kv * G;
    const KeySrc& src = a.src;
    const __nv_bfloat16* kpool = reinterpret_cast<const __nv_bfloat16*>(src.k_pool);
    const __nv_bfloat16* vpool = reinterpret_cast<const __nv_bfloat16*>(src.v_pool);
    const int32_t* ptab = src.page_table + bl * src.max_pages;

    // ---- Q^T fragments: column = query row 8rt + qr (rows >= R are zero)
    uint32_t qb[KS][2];
    {
        const int r = rt * 8 + qr;
        const int gr = rbase + r;                   // row of the launch
        const float* qv = r < R ? a.q + (((size_t)b * T + gr / G) * HQ + h * G + gr % G) * D : nullptr;
        const float sc = a.scale * kLog2e;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int d0 = kk * 16 + 2 * qc;
            qb[kk][0] = qv ? pack_bf16(qv[d0] * sc, qv[d0 + 1] * sc) : 0u;
            qb[kk][1] = qv ? pack_bf16(qv[d0 + 8] * sc, qv[d0 + 9] * sc) : 0u;
        }
    }
    // this thread's S columns: rows 8rt + 2qc (0) and 8rt + 2qc + 1 (1)
    const int r0 = rbase + rt * 8 + 2 * qc;
    const int qp0 = qbase + r0 / G, qp1 = qbase + (r0 + 1) / G;

    float m0 = -INFINITY, m1 = -INFINITY;
    float c2[4] = {0.f, 0.f, 0.f, 0.f};
    float oacc[KS][4];                 // O^T: rows d = 16md + qr (+8), cols query rows 2qc, 2qc+1
#pragma unroll
    for (int md = 0; md < KS; ++md) oacc[md][0] = oacc[md][1] = oacc[md][2] = oacc[md][3] = 0.f;
    const uint32_t ones = qr == 0 ? 0x3F803F80u : 0u;     // bf16 ones in row 0 of the sum product

    const int ntiles = k1 > k0 ? (k1 - k0 + kTcKT - 1) / kTcKT : 0;
    const int psh = src.page_shift, pmask = src.page_size - 1;     // power-of-two pages (host-checked)
    const int n_split_pages = k1 > k0 ? (k1 - k0 + 15) / 16 : 0;
    const bool staged = TMA && n_split_pages <= kKqSplitPages;
    if (staged) {
        for (int i = threadIdx.x; i < n_split_pages; i += nthreads) split_pages[i] = __ldg(ptab + (k0 >> 4) + i);
        __syncthreads();
    }
    auto load_tile = [&](int slot, int t0) {
        __nv_bfloat16* kd = ring + (size_t)slot * 2 * kTcKT * D;
        __nv_bfloat16* vd = kd + kTcKT * D;
        if constexpr (TMA) {
            // one thread: per 16-key page with a live key, D/64 boxes of K
            // and of V; pages wholly past the split's last key are skipped
            if (threadIdx.x == 0) {
                const int np = min(kTcKT / 16, (k1 - t0 + 15) / 16);
                mbar_expect_tx(&full_bar[slot], (uint32_t)np * 2 * (D / 64) * (16 * 64 * 2));
                for (int j = 0; j < np; ++j) {
                    const int page = staged ? split_pages[((t0 - k0) >> 4) + j] : __ldg(ptab + ((t0 >> 4) + j));
#pragma unroll
                    for (int x = 0; x < D / 64; ++x) {
                        tma_load_4d(kd + x * (kTcKT * 64) + j * 16 * 64, &maps.k, x * 64, 0, h, page, &full_bar[slot]);
                        tma_load_4d(vd + x * (kTcKT * 64) + j * 16 * 64, &maps.v, x * 64, 0, h, page, &full_bar[slot]);
                    }
                }
            }
        } else {
#pragma unroll 4
            for (int i = threadIdx.x; i < kTcKT * DC; i += nthreads) {
                const int key = i / DC, ch = i % DC;
                const int kp = t0 + key;
                const bool ok = kp < k1;
                size_t off = 0;
                if (ok) {
                    const int page = __ldg(ptab + (kp >> psh));
                    off = ((((size_t)page * a.n_kv + h) << psh) + (kp & pmask)) * D + ch * 8;
                }
                cpasync16(kd + swz<D>(key, ch), kpool + off, ok);
                cpasync16(vd + swz<D>(key, ch), vpool + off, ok);
            }
        }
    };
    bool ok_all = true;
#pragma unroll
    for (int i = 0; i < kKqNST - 1; ++i) {
        if (i < ntiles) load_tile(i, k0 + i * kTcKT);
        if constexpr (!TMA) asm volatile("cp.async.commit_group;\n" ::);
    }
    for (int it = 0; it < ntiles; ++it) {
        const int t0 = k0 + it * kTcKT;
        const int slot = it % kKqNST;
        if (it + kKqNST - 1 < ntiles) load_tile((it + kKqNST - 1) % kKqNST, t0 + (kKqNST - 1) * kTcKT);
        const __nv_bfloat16* kt = ring + (size_t)slot * 2 * kTcKT * D;
        const __nv_bfloat16* vt = kt + kTcKT * D;
        if constexpr (TMA) {
            ok_all = mbar_wait(&full_bar[slot], (uint32_t)((it / kKqNST) & 1), a.err) && ok_all;
            if (t0 + kTcKT > k1) {
                // keys past the split's end: the rest of the last page holds
                // whatever the pool held there, and whole pages were not
                // copied; their probabilities are zero, so zero their V rows
                // (0 x NaN would not be 0)
                __nv_bfloat16* vz = const_cast<__nv_bfloat16*>(vt);
                for (int i = threadIdx.x; i < (t0 + kTcKT - k1) * DC; i += nthreads) {
                    const int key = k1 - t0 + i / DC, ch = i % DC;
                    *reinterpret_cast<uint4*>(vz + kv_off<D, true>(key, ch)) = make_uint4(0u, 0u, 0u, 0u);
                }
                __syncthreads();
            }
        } else {
            asm volatile("cp.async.commit_group;\n" ::);
            asm volatile("cp.async.wait_group %0;\n" ::"n"(kKqNST - 1));
            __syncthreads();
        }
        // ---- S^T: rows keys 16kg + qr (+8), columns query rows
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            uint32_t af[4];
            ldsm4(af[0], af[1], af[2], af[3], kt + kv_off<D, TMA>(kg * 16 + (mi & 1) * 8 + ri, 2 * kk + (mi >> 1)));
            mma_bf16_16816(sc, af, qb[kk][0], qb[kk][1]);
        }
        // ---- causal / range mask
        const int kpa = t0 + kg * 16 + qr, kpb = kpa + 8;
        if (kpa >= k1 || kpa > qp0) sc[0] = -INFINITY;
        if (kpa >= k1 || kpa > qp1) sc[1] = -INFINITY;
        if (kpb >= k1 || kpb > qp0) sc[2] = -INFINITY;
        if (kpb >= k1 || kpb > qp1) sc[3] = -INFINITY;
        // ---- online softmax (base 2) of the two rows over the 16 keys
        float t0m = fmaxf(sc[0], sc[2]), t1m = fmaxf(sc[1], sc[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            t0m = fmaxf(t0m, __shfl_xor_sync(0xffffffffu, t0m, off));
            t1m = fmaxf(t1m, __shfl_xor_sync(0xffffffffu, t1m, off));
        }
        {
            const float n0 = fmaxf(m0, t0m), n1 = fmaxf(m1, t1m);
            if (!__all_sync(0xffffffffu, n0 == m0 && n1 == m1)) {
                const float al0 = n0 == -INFINITY ? 1.f : exp2f(m0 - n0);
                const float al1 = n1 == -INFINITY ? 1.f : exp2f(m1 - n1);
#pragma unroll
                for (int md = 0; md < KS; ++md) {
                    oacc[md][0] *= al0;
                    oacc[md][1] *= al1;
                    oacc[md][2] *= al0;
                    oacc[md][3] *= al1;
                }
                c2[0] *= al0;
                c2[1] *= al1;
                m0 = n0;
                m1 = n1;
            }
        }
        const float p0 = sc[0] == -INFINITY ? 0.f : exp2f(sc[0] - m0);
        const float p1 = sc[1] == -INFINITY ? 0.f : exp2f(sc[1] - m1);
        const float p2 = sc[2] == -INFINITY ? 0.f : exp2f(sc[2] - m0);
        const float p3 = sc[3] == -INFINITY ? 0.f : exp2f(sc[3] - m1);
        const uint32_t pb0 = movm_trans(pack_bf16(p0, p1)), pb1 = movm_trans(pack_bf16(p2, p3));
        {
            const uint32_t a2[4] = {ones, 0u, ones, 0u};
            mma_bf16_16816(c2, a2, pb0, pb1);
        }
        // ---- O^T += V^T P^T
#pragma unroll
        for (int md = 0; md < KS; ++md) {
            uint32_t va[4];
            ldsm4t(va[0], va[1], va[2], va[3], vt + kv_off<D, TMA>(kg * 16 + (mi >> 1) * 8 + ri, 2 * md + (mi & 1)));
            mma_bf16_16816(oacc[md], va, pb0, pb1);
        }
        __syncthreads();          // the ring slot is refilled next
    }
    if constexpr (TMA) {
        if (!ok_all && threadIdx.x == 0) {
            // a copy never completed: wait (bounded) for any still in flight
            // before the shared memory is reused
            for (int it = max(0, ntiles - kKqNST); it < ntiles; ++it)
                mbar_wait(&full_bar[it % kKqNST], (uint32_t)((it / kKqNST) & 1), nullptr);
        }
    } else {
        asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();

    // ---- merge the 4 key groups of each row (fixed order) into the split partial
    const float l0 = __shfl_sync(0xffffffffu, c2[0], qc);
    const float l1 = __shfl_sync(0xffffffffu, c2[1], qc);
    float* mrg = reinterpret_cast<float*>(tsm);          // [RT][KG][8 rows][D + 2]
    {
        float* mine = mrg + ((size_t)(rt * kKqKG + kg) * 8) * PS;
#pragma unroll
        for (int md = 0; md < KS; ++md) {
            const int d0 = 16 * md + qr;
            mine[(2 * qc) * PS + 2 + d0] = oacc[md][0];
            mine[(2 * qc + 1) * PS + 2 + d0] = oacc[md][1];
            mine[(2 * qc) * PS + 2 + d0 + 8] = oacc[md][2];
            mine[(2 * qc + 1) * PS + 2 + d0 + 8] = oacc[md][3];
        }
        if (qr == 0) {
            mine[(2 * qc) * PS] = m0;
            mine[(2 * qc) * PS + 1] = l0;
            mine[(2 * qc + 1) * PS] = m1;
            mine[(2 * qc + 1) * PS + 1] = l1;
        }
    }
    __syncthreads();
    const size_t bhr = ((size_t)b * a.n_kv + h) * a.n_rb + rb;
    float* mypart = a.part + ((bhr * a.n_splits + s) * kAttnRB) * PS;
    for (int i = threadIdx.x; i < R * (D + 1); i += nthreads) {
        const int r = i / (D + 1), e = i % (D + 1);      // e == D: the row's (max, sum)
        const float* g0 = mrg + ((size_t)((r / 8) * kKqKG) * 8 + r % 8) * PS;
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < kKqKG; ++q) M = fmaxf(M, g0[(size_t)q * 8 * PS]);
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < kKqKG; ++q) {
            const float mq = g0[(size_t)q * 8 * PS];
            if (mq != -INFINITY) acc += g0[(size_t)q * 8 * PS + (e == D ? 1 : 2 + e)] * exp2f(mq - M);
        }
        if (e == D) {
            mypart[(size_t)r * PS] = M == -INFINITY ? -INFINITY : M * kLn2;
            mypart[(size_t)r * PS + 1] = acc;
        } else {
            mypart[(size_t)r * PS + 2 + e] = acc;
        }
    }
    // the drained ring holds the merge's per-(row, split) weights
    split_merge(a, bhr, b, h, R, rbase, ms, ls, ok_all ? reinterpret_cast<float*>(tsm) : nullptr,
                (int)(kKqNST * 2 * kTcKT * D * 2 / 4));
}

template <int D>
size_t full_tc_smem() {
    return (size_t)4 * kTcKT * D * 2 + 2 * kAttnRB * sizeof(float);
}

template <int D, int MAXT, bool TMA>
cudaError_t launch_kq(const KvMaps& maps, const AttnArgs& a, dim3 grid, int threads, cudaStream_t st) {
    const cudaError_t e = allow_smem_max_once<attn_kq_kernel<D, MAXT, TMA>>();
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_kq_kernel<D, MAXT, TMA>, grid, dim3(threads), kq_smem<D>((threads / 32) / kKqKG), st,
                      maps, a);
}

int encode_bf16_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box);

// Tensor maps of a device-resident pool with 16-row pages (cached per pool);
// false when the pool is elsewhere (pinned host memory: the cp.async path).
bool kv_maps(const KeySrc& src, int n_kv, int d, KvMaps* out) {
    struct Entry {
        const void* k;
        const void* v;
        int n_kv, d, n_pages;
        bool ok;
        KvMaps maps;
    };
    static std::mutex mu;
    static Entry cache[32];
    static int n = 0, next = 0;
    if (src.page_size != 16 || (d != 64 && d != 128) || src.n_pages <= 0) return false;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i) {
        const Entry& e = cache[i];
        if (e.k == src.k_pool && e.v == src.v_pool && e.n_kv == n_kv && e.d == d && e.n_pages == src.n_pages) {
            *out = e.maps;
            return e.ok;
        }
    }
    Entry e{src.k_pool, src.v_pool, n_kv, d, src.n_pages, false, {}};
    cudaPointerAttributes ak, av;
    const bool dev = cudaPointerGetAttributes(&ak, src.k_pool) == cudaSuccess &&
                     cudaPointerGetAttributes(&av, src.v_pool) == cudaSuccess && ak.type == cudaMemoryTypeDevice &&
                     av.type == cudaMemoryTypeDevice;
    cudaGetLastError();
    if (dev) {
        // the view spans exactly the pool's pages (the copy engine zero-fills
        // anything outside a view's bounds)
        const uint64_t dims[4] = {(uint64_t)d, 16, (uint64_t)n_kv, (uint64_t)src.n_pages};
        const uint64_t strides[3] = {(uint64_t)d * 2, (uint64_t)16 * d * 2, (uint64_t)16 * d * 2 * n_kv};
        const uint32_t box[4] = {64, 16, 1, 1};
        const uint32_t box8[4] = {64, 16, 1, 8};
        e.ok = encode_bf16_map(&e.maps.k, src.k_pool, 4, dims, strides, box) == DKV_OK &&
               encode_bf16_map(&e.maps.v, src.v_pool, 4, dims, strides, box) == DKV_OK &&
               encode_bf16_map(&e.maps.k8, src.k_pool, 4, dims, strides, box8) == DKV_OK &&
               encode_bf16_map(&e.maps.v8, src.v_pool, 4, dims, strides, box8) == DKV_OK;
    }
    cache[next] = e;
    next = (next + 1) % 32;
    n = n < 32 ? n + 1 : 32;
    *out = e.maps;
    return e.ok;
}

int attn_full_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, int max_keys, cudaStream_t st,
                 bool* handled);
int attn_prefill_tc(AttnArgs& a, dkv_dims dims, const KvMaps& maps, void* work, size_t work_bytes, int max_keys,
                    cudaStream_t st);
int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled);

constexpr size_t kAttnTicketsTc = 16384;   // same fixed ticket region as the generic kernel

int attn_full_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, int max_keys, cudaStream_t st,
                 bool* handled) {
    *handled = false;
    if (a.src.dtype != DKV_BF16 || (dims.d != 64 && dims.d != 128) || a.split % kTcKT != 0) return DKV_OK;
    if (a.src.page_shift < 0) return DKV_OK;     // pages of any other size: generic kernel
    const int R = a.T * a.group;
    if (R > kAttnRB && ((uintptr_t)a.q & 15) == 0) {
        // prefill chunks over a device-resident pool: the tcgen05 kernel
        KvMaps pm;
        if (kv_maps(a.src, dims.n_kv, dims.d, &pm)) {
            DKV_TRY(attn_prefill_tc(a, dims, pm, work, work_bytes, max_keys, st));
            *handled = true;
            return DKV_OK;
        }
    }
    // more than 64 rows (a prompt chunk over a host-resident pool): splits of
    // at least kPromptMinSplit keys, as the tcgen05 prefill kernel takes (the
    // forward's scratch is sized for that)
    if (R > kAttnRB && a.split < kPromptMinSplit) a.split = kPromptMinSplit;
    a.n_rb = R <= kAttnRB ? (R + kKqRows - 1) / kKqRows : (R + kAttnRB - 1) / kAttnRB;
    a.n_splits = (max_keys + a.split - 1) / a.split;
    if (a.n_splits < 1) a.n_splits = 1;
    const size_t n_tk = (size_t)dims.batch * dims.n_kv * a.n_rb;
    DKV_REQUIRE(n_tk + dims.batch <= kAttnTicketsTc, "attention: batch x heads x row blocks too large");
    Arena ar(work, work_bytes);
    unsigned* tk = ar.take<unsigned>(kAttnTicketsTc);
    a.tickets = tk;
    a.fold_tickets = tk ? tk + n_tk : nullptr;
    a.part = ar.take<float>(n_tk * a.n_splits * kAttnRB * (dims.d + 2));
    a.sbuf = nullptr;
    DKV_REQUIRE(a.part && a.tickets, "attention: work buffer too small (%zu bytes)", work_bytes);
    dim3 grid(a.n_splits, dims.n_kv, dims.batch * a.n_rb);
    ProfScope ps(DKV_PROF_ATTN_FULL, 0.0, st);
    if (R <= kAttnRB) {
        const int RT = (std::min(R, kKqRows) + 7) / 8;
        const int threads = 32 * kKqKG * RT;
        KvMaps maps;
        const bool tma = kv_maps(a.src, dims.n_kv, dims.d, &maps);
        a.err = device_error_word();
        cudaError_t e = cudaSuccess;
        if (tma)
            e = dims.d == 128 ? launch_kq<128, 256, true>(maps, a, grid, threads, st)
                              : launch_kq<64, 256, true>(maps, a, grid, threads, st);
        else
            e = dims.d == 128 ? launch_kq<128, 256, false>(maps, a, grid, threads, st)
                              : launch_kq<64, 256, false>(maps, a, grid, threads, st);
        DKV_CUDA(e);
        *handled = true;
        return DKV_OK;
    }
    if (dims.d == 128) {
        DKV_CUDA(allow_smem_max_once<attn_full_tc_kernel<128>>());
        attn_full_tc_kernel<128><<<grid, kTcThreads, full_tc_smem<128>(), st>>>(a);
    } else {
        DKV_CUDA(allow_smem_max_once<attn_full_tc_kernel<64>>());
        attn_full_tc_kernel<64><<<grid, kTcThreads, full_tc_smem<64>(), st>>>(a);
    }
    DKV_LAUNCHED();
    *handled = true;
    return DKV_OK;
}

}  // namespace dkv
