// Prefill attention on the fifth-generation tensor cores: a chunk's query
// rows attend causally to the paged full cache (bf16, 16-key pages in device
// memory).  Replaces the attention of the prompt forward (draftkv/engine.py:
// 133-134 running draftkv/llama.py:202-219 over every prompt position).
//
// One CTA per (sequence, KV head, key split, block of 256 query rows: query
// tiles A and B of 128), rows = token x GQA head as in the other attention
// kernels; 10 warps, one CTA per SM:
//   warp 8 -- producer: per 128-key tile, one copy of 128 keys x 64 dims
//     when the tile's 8 pages are consecutive in the pool (ascending, or
//     descending for a tile no row masks), else 8 lanes issue one page each
//     (16 keys x 64 dims, 2 KB; one copy engine serves the SM at ~90 cycles a
//     2 KB box, so fewer, larger boxes are faster); 128-byte swizzle, 2-deep
//     K and V rings; pages wholly past the CTA's last key are read past the
//     pool view (zeros).  K_j is copied once S_A(j-2) and S_B(j-2) have read
//     its slot, V_{j-1} once the P V products of tile j - 3 have;
//   warp 9 -- TMEM allocation; lane 0 issues the MMAs.  Per key tile j and
//     query tile t: O_t += P_t(j-1) V(j-1) (M 128, N d, K 128 keys; P in
//     TMEM, V read in place through an MN-major descriptor), then S_t(j) =
//     Q_t K_j^T (M 128, N 128, K = d; Q and K in shared memory) over the
//     same TMEM columns -- MMAs run in issue order, so P_t(j-1) is read
//     first.  One query tile's products run on the tensor core while the
//     other tile's softmax works;
//   warps 0-3 (tile A) and 4-7 (tile B) -- softmax, one query row a thread
//     (TMEM lane = row): first the row of Q (bf16) into shared memory, then
//     per key tile the row's 128 scores (tcgen05.ld), causal mask, running
//     max, exp2, and bf16 P back into TMEM over the scores.  S_t(j) completes
//     after P_t(j-1) V(j-1), so O_t is up to date when the scores arrive; it
//     is rescaled in TMEM only when the row max grows by more than 8 (log2
//     units): a stale max leaves O / l exact and keeps every P below 2^8.
// Two softmax warps on each scheduler hide each other's dependent latency
// (one warp a scheduler ran at 762 TF/s on the C4 prompt's last chunk).
// At the end the O rows (tcgen05.ld) go to the split partials, merged in
// split order as in the other attention kernels.  Scores are in log2 units
// (log2 e folded into the query scale).  Every mbarrier wait is bounded
// (error word 0x80); after a failed wait the CTA waits (bounded) for its
// copies and MMAs in flight before it frees shared and tensor memory.
#include "attn_common.cuh"
#include "tcgen05.cuh"

namespace dkv {

uint32_t* device_error_word();

constexpr int kPfTile = 128;          // query rows per tile (MMA M, TMEM lanes)
constexpr int kPfRows = 256;          // query rows per CTA: tiles A and B
constexpr int kPfKeys = 128;          // keys per tile
constexpr int kPfThreads = 320;       // 8 softmax warps (4 a query tile), producer, MMA
constexpr int kPfNst = 2;             // K and V ring depth
constexpr int kPfTmemCols = 512;      // per query tile t: S at 256 t (P over its first 64 columns), O at 256 t + 128
constexpr int kPfSplitPages = 1024;   // page ids staged in shared memory
constexpr float kPfRescale = 8.f;     // lazy-rescale threshold (log2 units)

// Shared memory (from a 1024-byte aligned base): Q of tiles A and B
// [2][d/64][128 rows][64], K slots [2][d/64][128 keys][64], V slots (same
// arrangement); every 128 x 64 block in the 128-byte swizzle (row r at
// r * 128 bytes, its 16-byte unit u at u ^ (r % 8)).
template <int D>
struct PfGeo {
    static constexpr int CH = D / 64;
    static constexpr int QT = CH * 16384;        // one query tile
    static constexpr int KVB = CH * 16384;       // one K (or V) tile
    static constexpr int K0 = 2 * QT;            // first K slot
    static constexpr int V0 = K0 + kPfNst * KVB; // first V slot
    static constexpr size_t SMEM = (size_t)V0 + kPfNst * KVB + 1024;
};

DKV_DEV uint32_t pf_pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
DKV_DEV float pf_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}
DKV_DEV float pf_max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// two fp32 lanes in one 64-bit register, and the sm_100 packed add / subtract
DKV_DEV uint64_t pf_pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
DKV_DEV void pf_unpack2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(v));
}
DKV_DEV uint64_t pf_add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
DKV_DEV uint64_t pf_sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
DKV_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// D (TMEM) += A (TMEM: row i in lane i, two bf16 a 32-bit column) . B (shared)
DKV_DEV void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_tc_kernel(const __grid_constant__ KvMaps maps, AttnArgs a) {
    using Geo = PfGeo<D>;
    constexpr int PS = D + 2;
    constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
    extern __shared__ uint8_t pf_raw[];
    uint8_t* sm = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t k_full[kPfNst], k_empty[kPfNst], v_full[kPfNst], v_empty[kPfNst];
    __shared__ __align__(8) uint64_t s_full[2], p_full[2], o_done, drain;
    __shared__ uint32_t tmem_slot;
    __shared__ float ms[kPfRows], ls[kPfRows];
    __shared__ int32_t pages_s[kPfSplitPages];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // one linear grid, row block fastest: the row blocks of a (sequence,
    // head, split) run together and read each K/V tile through L2
    const int rb = (int)(blockIdx.x % a.n_rb);
    const int s = (int)(blockIdx.x / a.n_rb % a.n_splits);
    const int h = (int)(blockIdx.x / a.n_rb / a.n_splits % a.n_kv);
    const int b = (int)(blockIdx.x / a.n_rb / a.n_splits / a.n_kv);
    const int G = a.group, T = a.T;
    const int r0 = rb * kPfRows;
    const int R = min(kPfRows, T * G - r0);
    const int HQ = a.n_kv * G;
    const size_t bhr = ((size_t)b * a.n_kv + h) * a.n_rb + rb;
    const int wcap = (Geo::V0 + kPfNst * Geo::KVB) / 4;     // floats of the rings (the merge's scratch)

    pdl_trigger();
    pdl_wait();      // the queries and the chunk's cache rows come from earlier kernels
    const int qbase = a.qpos0[b];
    const int n_keys = qbase + T;
    const int k0 = s * a.split;                         // a multiple of 128
    const int tmax = (r0 + R - 1) / G;                  // this CTA's last token
    const int kend = min(min(n_keys, k0 + a.split), qbase + tmax + 1);
    const int ntiles = kend > k0 ? (kend - k0 + kPfKeys - 1) / kPfKeys : 0;
    if (ntiles == 0) {
        // no key of this split is visible to these rows (early prompt
        // chunks leave most splits of a long pool empty): empty partials and
        // the merge ticket only
        for (int r = threadIdx.x; r < R; r += blockDim.x) {
            float* mypart = a.part + ((bhr * a.n_splits + s) * kPfRows + r) * PS;
            mypart[0] = -INFINITY;
            mypart[1] = 0.f;
        }
        split_merge<kPfRows>(a, bhr, b, h, R, r0, ms, ls, reinterpret_cast<float*>(sm), wcap);
        return;
    }

    if (threadIdx.x == 0) {
        for (int i = 0; i < kPfNst; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 128);
        }
        mbar_init(&o_done, 1);
        mbar_init(&drain, 1);
        fence_barrier_init();
        fence_async_shared();
    }
    if (warp == 9) tmem_alloc(&tmem_slot, kPfTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const int32_t* ptab = a.src.page_table + ((size_t)b * a.n_layers + a.layer) * a.src.max_pages;
    const int npg = (kend - k0 + 15) / 16;
    const bool staged = npg <= kPfSplitPages;

    bool ok = true;
    int issued_k = 0, issued_v = 0;    // producer: tiles whose K / V copies were issued
    if (warp == 8) {
        // ---------------- producer: the split's page ids, then per tile j the
        // copies of K_j and of V_{j-1}; lane p issues page p's boxes (one
        // lane's copies issue ~125 cycles apart), lane 0 arms the barrier
        if (staged) {
            for (int i = lane; i < npg; i += 32) pages_s[i] = __ldg(ptab + (k0 >> 4) + i);
            __syncwarp();
        }
        const bool live = lane < kPfKeys / 16;
        // keys below kfree are live for every row of the CTA (no mask)
        const int kfree = min(qbase + r0 / G + 1, kend);
        auto issue = [&](int j, bool v) {
            const int slot = j % kPfNst;
            uint8_t* dst = sm + (v ? Geo::V0 : Geo::K0) + slot * Geo::KVB;
            uint64_t* bar = v ? &v_full[slot] : &k_full[slot];
            if (lane == 0) mbar_expect_tx(bar, (uint32_t)Geo::KVB);
            __syncwarp();
            const int key = k0 + j * kPfKeys + 16 * lane;
            const int page = live ? (key < kend ? (staged ? pages_s[(key - k0) >> 4] : __ldg(ptab + (key >> 4)))
                                                : a.src.n_pages)
                                  : 0;
            const int first = __shfl_sync(0xffffffffu, page, 0);
            const bool unmasked = k0 + (j + 1) * kPfKeys <= kfree;
            if (__all_sync(0xffffffffu, !live || page == first + lane)) {
                // the tile's 8 pages are consecutive in the pool: one copy of
                // 128 keys per 64 dims (pages past the pool read zeros)
                if (lane == 0)
#pragma unroll
                    for (int x = 0; x < Geo::CH; ++x)
                        tma_load_4d(dst + x * 16384, v ? &maps.v8 : &maps.k8, x * 64, 0, h, first, bar);
            } else if (unmasked && __all_sync(0xffffffffu, !live || page == first - lane)) {
                // consecutive in descending order (the block pool hands out
                // its free list last-in first-out): one copy from the lowest
                // page puts the 16-key blocks in reverse order.  K and V get
                // the same order, so S, P and V stay consistent, and the max
                // and sum do not depend on order: only for tiles no row masks
                if (lane == 0)
#pragma unroll
                    for (int x = 0; x < Geo::CH; ++x)
                        tma_load_4d(dst + x * 16384, v ? &maps.v8 : &maps.k8, x * 64, 0, h, first - 7, bar);
            } else if (live) {
#pragma unroll
                for (int x = 0; x < Geo::CH; ++x)
                    tma_load_4d(dst + x * 16384 + lane * 2048, v ? &maps.v : &maps.k, x * 64, 0, h, page, bar);
            }
        };
        for (int j = 0; j <= ntiles; ++j) {
            if (j < ntiles) {
                // slot j % 2 was last read by S_A(j-2) and S_B(j-2)
                if (j >= kPfNst && !__all_sync(0xffffffffu, mbar_wait(&k_empty[j % kPfNst],
                                                                      (uint32_t)((j / kPfNst - 1) & 1), a.err))) {
                    ok = false;
                    break;
                }
                issue(j, false);
                issued_k = j + 1;
            }
            if (j >= 1) {
                const int i = j - 1;     // slot i % 2 was last read by the P V products of tile i - 2
                if (i >= kPfNst && !__all_sync(0xffffffffu, mbar_wait(&v_empty[i % kPfNst],
                                                                      (uint32_t)((i / kPfNst - 1) & 1), a.err))) {
                    ok = false;
                    break;
                }
                issue(i, true);
                issued_v = i + 1;
            }
        }
    } else if (warp == 9) {
        // ---------------- MMA issuer (the warp waits together, lane 0 issues).
        // Per key tile j and query tile t (A = 0, B = 1): P_t(j-1) V(j-1),
        // then S_t(j) over the same TMEM columns (MMAs run in issue order, so
        // P_t(j-1) is read first), so one tile's product runs on the tensor
        // core while the other tile's softmax works
        const uint32_t q_s = smem_u32(sm), k_s0 = smem_u32(sm + Geo::K0), v_s0 = smem_u32(sm + Geo::V0);
        constexpr uint32_t idS = tc_idesc_n(kPfKeys, false), idO = tc_idesc_n(D, true);
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, a.err));
        };
        // V of tile i in place (the rest of a ragged last page zeroed)
        auto v_ready = [&](int i) -> bool {
            const int slot = i % kPfNst;
            if (!wait_all(&v_full[slot], (uint32_t)((i / kPfNst) & 1))) return false;
            const int t0 = k0 + i * kPfKeys;
            if (kend - t0 < kPfKeys && (kend & 15) != 0) {
                // the rest of the last page holds whatever the pool held
                // there: zero those V rows (their P is 0, but 0 x NaN is not)
                uint8_t* vd = sm + Geo::V0 + slot * Geo::KVB;
                const int z0 = kend - t0, z1 = (z0 + 15) & ~15;
                for (int e = lane; e < (z1 - z0) * (D / 8); e += 32) {
                    const int key = z0 + e / (D / 8), u = e % (D / 8);
                    *reinterpret_cast<uint4*>(vd + (u >> 3) * 16384 + key * 128 + (((u & 7) ^ (key & 7)) << 4)) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
                fence_async_shared();
                __syncwarp();
            }
            return true;
        };
        auto issue_pv = [&](int t, int i) {
            const uint32_t v_s = v_s0 + (i % kPfNst) * Geo::KVB;
            const uint32_t base = tmem + (uint32_t)(t * 256);
#pragma unroll
            for (int ks = 0; ks < kPfKeys / 16; ++ks)
                tc_mma_ts(base + 128, base + ks * 8, sw128_desc_mn(v_s + ks * 2048, 16384), idO,
                          (i | ks) != 0 ? 1u : 0u);
        };
        auto issue_s = [&](int t, int j) {
            const uint32_t k_s = k_s0 + (j % kPfNst) * Geo::KVB;
            const uint32_t qt = q_s + t * Geo::QT;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
                tc_mma_i(tmem + (uint32_t)(t * 256), sw128_desc(qt + (kk >> 2) * 16384 + (kk & 3) * 32),
                         sw128_desc(k_s + (kk >> 2) * 16384 + (kk & 3) * 32), idS, kk != 0 ? 1u : 0u);
            tc_commit(&s_full[t]);
        };
        named_sync(1, 288);      // Q is in shared memory
        for (int j = 0; j < ntiles && ok; ++j) {
            if (!wait_all(&k_full[j % kPfNst], (uint32_t)((j / kPfNst) & 1))) {
                ok = false;
                break;
            }
            if (j >= 1 && !v_ready(j - 1)) {
                ok = false;
                break;
            }
            for (int t = 0; t < 2; ++t) {
                if (j >= 1 && !wait_all(&p_full[t], (uint32_t)((j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    if (j >= 1) issue_pv(t, j - 1);
                    issue_s(t, j);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) {
                tc_commit(&k_empty[j % kPfNst]);               // S_A(j), S_B(j) read K_j
                if (j >= 1) tc_commit(&v_empty[(j - 1) % kPfNst]);     // both P V of tile j - 1 read V_{j-1}
            }
            __syncwarp();
        }
        if (ok) {
            const int i = ntiles - 1;
            if (!v_ready(i)) ok = false;
            for (int t = 0; t < 2 && ok; ++t) {
                if (!wait_all(&p_full[t], (uint32_t)(i & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) issue_pv(t, i);
                __syncwarp();
            }
            if (ok && lane == 0) tc_commit(&o_done);
            __syncwarp();
        }
    } else {
        // ---------------- softmax: query tile t (warps 4t .. 4t + 3), row rt
        // of the tile = TMEM lane rt; CTA row cr = 128 t + rt
        const int t = warp >> 2, rt = threadIdx.x & 127, cr = t * kPfTile + rt;
        const uint32_t lanes = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t sb = lanes + (uint32_t)(t * 256), ob = sb + 128;     // S (P over it), O
        {
            // the row of Q in shared memory: bf16 of q * scale * log2 e, the
            // tile's 128-byte swizzle; rows >= R zero
            const float sc = a.scale * kLog2e;
            const float* qrow =
                cr < R ? a.q + (((size_t)b * T + (r0 + cr) / G) * HQ + h * G + (r0 + cr) % G) * D : nullptr;
            uint8_t* qt = sm + t * Geo::QT;
#pragma unroll 4
            for (int u = 0; u < D / 8; ++u) {
                float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
                if (qrow) {
                    x0 = __ldg(reinterpret_cast<const float4*>(qrow + 8 * u));
                    x1 = __ldg(reinterpret_cast<const float4*>(qrow + 8 * u + 4));
                }
                *reinterpret_cast<uint4*>(qt + (u >> 3) * 16384 + rt * 128 + (((u & 7) ^ (rt & 7)) << 4)) =
                    make_uint4(pf_pack(x0.x * sc, x0.y * sc), pf_pack(x0.z * sc, x0.w * sc),
                               pf_pack(x1.x * sc, x1.y * sc), pf_pack(x1.z * sc, x1.w * sc));
            }
            fence_async_shared();
            named_sync(1, 288);      // with the MMA warp
        }
        const int qp = cr < R ? qbase + (r0 + cr) / G : kend - 1;   // padding rows see every key
        const int lim = min(qp, kend - 1);                          // this row's last key
        float m = -INFINITY, l = 0.f;
        for (int j = 0; j < ntiles; ++j) {
            // S_t(j) done: and with it P_t(j-1) V(j-1), issued before it
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], (uint32_t)(j & 1), a.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int lc = lim - (k0 + j * kPfKeys);                  // last live column
            // pass 1: the row max, 32 scores at a time (8 chains of
            // three-input max)
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t sr[32];
                tmem_ld32(sb + c * 32, sr);
                tmem_wait_ld();
                if (lc < kPfKeys - 1) {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (c * 32 + e > lc) sr[e] = __float_as_uint(-INFINITY);
                }
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const int k = 2 * c + (e >> 4);
                    mx[k] = pf_max3(mx[k], __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]));
                }
            }
            const float mn = fmaxf(m, pf_max3(pf_max3(mx[0], mx[1], mx[2]), pf_max3(mx[3], mx[4], mx[5]),
                                              fmaxf(mx[6], mx[7])));
            float alpha = 1.f;
            if (m == -INFINITY || mn > m + kPfRescale) {
                alpha = m == -INFINITY ? 0.f : pf_ex2(m - mn);
                m = mn;
            }
            const float msub = m == -INFINITY ? 0.f : m;
            // pass 2, 64 scores at a time: exp2(s - m) two at a time (packed
            // subtract and sum), bf16 P into the 32 columns those scores
            // held first (P block k over S columns 32k .. 32k + 31, read in
            // this pass or the one before)
            const uint64_t mm = pf_pack2(msub, msub);
            uint64_t sum2[2] = {0ull, 0ull};
            uint32_t sr[2][32];
#pragma unroll 1
            for (int k = 0; k < 2; ++k) {
                tmem_ld32(sb + 64 * k, sr[0]);
                tmem_ld32(sb + 64 * k + 32, sr[1]);
                tmem_wait_ld();
                uint32_t pk[32];
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const int c = 2 * k + h2;
                    if (lc < kPfKeys - 1) {
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (c * 32 + e > lc) sr[h2][e] = __float_as_uint(-INFINITY);
                    }
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        float d0, d1;
                        pf_unpack2(pf_sub2(pf_pack2(__uint_as_float(sr[h2][e]), __uint_as_float(sr[h2][e + 1])), mm),
                                   d0, d1);
                        const float p0 = pf_ex2(d0), p1 = pf_ex2(d1);
                        sum2[h2] = pf_add2(sum2[h2], pf_pack2(p0, p1));
                        pk[h2 * 16 + e / 2] = pf_pack(p0, p1);
                    }
                }
                tmem_st32(sb + 32 * k, pk);
            }
            float a0, a1, a2, a3;
            pf_unpack2(sum2[0], a0, a1);
            pf_unpack2(sum2[1], a2, a3);
            l = l * alpha + ((a0 + a1) + (a2 + a3));
            if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
                // O_t holds P_t(j-1) V(j-1) (S_t(j) completed after it) and
                // P_t(j) V(j) waits for this tile's P
#pragma unroll 1
                for (int c0 = 0; c0 < D; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(ob + c0, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tmem_st32(ob + c0, o);
                }
            }
            tmem_wait_st();      // P_t(j) is in TMEM (and any rescaled O)
            tc_fence_before();
            mbar_arrive(&p_full[t]);
        }
        if (ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(&o_done, 0u, a.err));
            tc_fence_after();
        }
        // ---- this split's partial row: (max in natural units, sum, O)
        float* mypart = a.part + ((bhr * a.n_splits + s) * kPfRows + cr) * PS;
        const bool live = ok && m != -INFINITY;
        if (__all_sync(0xffffffffu, ok)) {
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 32) {
                uint32_t o[32];
                tmem_ld32(ob + c0, o);
                tmem_wait_ld();
                if (live && cr < R) {
#pragma unroll
                    for (int e = 0; e < 32; e += 2)
                        *reinterpret_cast<float2*>(mypart + 2 + c0 + e) =
                            make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1]));
                }
            }
        }
        if (cr < R) {
            mypart[0] = live ? m * kLn2 : -INFINITY;
            mypart[1] = live ? l : 0.f;
        }
    }

    // ---- teardown: one verdict for the CTA; after a failure wait (bounded)
    // for the copies and MMAs still in flight
    const bool all_ok = __syncthreads_and(ok) != 0;
    if (!all_ok) {
        if (warp == 8 && lane == 0) {
            for (int j = max(0, issued_k - kPfNst); j < issued_k; ++j)
                mbar_wait(&k_full[j % kPfNst], (uint32_t)((j / kPfNst) & 1), nullptr);
            for (int j = max(0, issued_v - kPfNst); j < issued_v; ++j)
                mbar_wait(&v_full[j % kPfNst], (uint32_t)((j / kPfNst) & 1), nullptr);
        }
        if (warp == 9 && lane == 0) {
            tc_commit(&drain);     // arrives once every MMA issued so far has completed
            mbar_wait(&drain, 0u, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, kPfTmemCols);
    }
    // after a failure (error word set) every row of this split is empty, and
    // the merge still runs so that the tickets stay consistent; the drained
    // rings hold the merge's per-(row, split) weights
    split_merge<kPfRows>(a, bhr, b, h, R, r0, ms, ls, all_ok ? reinterpret_cast<float*>(sm) : nullptr, wcap);
}

// Host: the prefill launch of dkv_attn_full (rows > 64, bf16 pool in device
// memory with 16-key pages, d 64 or 128, 16-byte aligned queries).  Splits
// of the key range: the caller's split rounded up to 128 keys, at least
// kPromptMinSplit (the decode-time split -- 1792 keys for one sequence at 64k --
// leaves a CTA a dozen tiles against its fixed costs and the merge of the
// last one 37 splits to read: 348 TF/s there.  Measured on B200: 8192-key
// splits 863 TF/s on 4 x 32k and 924 on 1 x 64k with 2048-token chunks,
// 16384-key splits 882 and 997); partials and tickets come from the
// attention work buffer.
int attn_prefill_tc(AttnArgs& a, dkv_dims dims, const KvMaps& maps, void* work, size_t work_bytes, int max_keys,
                    cudaStream_t st) {
    const int R = a.T * a.group;
    a.split = std::max(kPromptMinSplit, (a.split + kPfKeys - 1) / kPfKeys * kPfKeys);
    a.n_rb = (R + kPfRows - 1) / kPfRows;
    a.n_splits = std::max(1, (max_keys + a.split - 1) / a.split);
    const size_t n_tk = (size_t)dims.batch * dims.n_kv * a.n_rb;
    constexpr size_t kTickets = 16384;     // the fixed ticket region at the start of the work buffer
    DKV_REQUIRE(n_tk + dims.batch <= kTickets, "attention: batch x heads x row blocks too large");
    Arena ar(work, work_bytes);
    a.tickets = ar.take<unsigned>(kTickets);
    a.fold_tickets = a.tickets ? a.tickets + n_tk : nullptr;
    a.part = ar.take<float>(n_tk * a.n_splits * kPfRows * (dims.d + 2));
    a.sbuf = nullptr;
    a.err = device_error_word();
    DKV_REQUIRE(a.part && a.tickets, "attention: work buffer too small (%zu bytes)", work_bytes);
    dim3 grid((unsigned)(n_tk * a.n_splits));
    ProfScope ps(DKV_PROF_ATTN_FULL, 0.0, st);
    cudaError_t e;
    if (dims.d == 128) {
        e = allow_smem_max_once<attn_prefill_tc_kernel<128>>();
        if (e == cudaSuccess)
            e = launch_pdl(attn_prefill_tc_kernel<128>, grid, dim3(kPfThreads), PfGeo<128>::SMEM, st, maps, a);
    } else {
        e = allow_smem_max_once<attn_prefill_tc_kernel<64>>();
        if (e == cudaSuccess)
            e = launch_pdl(attn_prefill_tc_kernel<64>, grid, dim3(kPfThreads), PfGeo<64>::SMEM, st, maps, a);
    }
    DKV_CUDA(e);
    return DKV_OK;
}

}  // namespace dkv
