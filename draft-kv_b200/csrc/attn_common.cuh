// Arguments and the split merge shared by the attention kernels.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace dkv {

struct KeySrc {
    // full cache
    const void* k_pool;
    const void* v_pool;
    const int32_t* page_table;
    int page_size, max_pages, dtype;
    int n_pages;             // pages in the pool (the bounds of the copy-engine view)
    int page_shift;          // log2(page_size), or -1 when page_size is not a power of two
    // drafter cache
    const uint8_t* k_codes;
    const uint8_t* v_codes;
    const uint16_t* k_sl;
    const uint16_t* v_sl;
    const int32_t* cpos;
    const int32_t* meta;
    int cap, cb_max, bits;
    bool comp;
};

struct AttnArgs {
    KeySrc src;
    int n_layers, n_kv, d, layer, group, T, batch;
    const float* q;          // [batch*T][n_kv*group][d]
    const int32_t* qpos0;    // [batch]
    void* out;
    int out_dtype;
    int split;               // keys (full) or slots (drafter) per split
    int n_splits;
    int n_rb;                // query row blocks per (sequence, head)
    float scale;
    // scratch
    float* part;             // [batch][n_kv][n_rb][n_splits][kAttnRB][d + 2]
    unsigned* tickets;       // [batch][n_kv][n_rb]  (+ [batch] head tickets for the fold)
    float* sbuf;             // drafter: raw scores [batch][n_kv][group][cap]
    float* mass;             // drafter: [batch][n_layers][n_kv][cap]
    int note_mass;           // drafter: fold the attention mass into the slot scores
    float* score;            // drafter: [batch][n_layers][cap]
    unsigned* fold_tickets;  // [batch]
    uint32_t* err;           // device error word (bounded waits of the copy-engine path)
};

constexpr int kAttnRB = 64;   // query rows (token x group head) per CTA
// Keys per split, at least, of bf16 attention over more than kAttnRB query
// rows (prompt chunks: no row of theirs is compared with a decode row): the
// tcgen05 prefill kernel and the host-pool fallback take it, and the
// forward's work buffer is sized for it
constexpr int kPromptMinSplit = 16384;

// Tensor maps of the K and V pools for the copy-engine-fed kernels: 4-D views
// {d, 16 page rows, n_kv, n_pages} with 128-byte swizzle; k / v copy a box of
// {64, 16, 1, 1} (one page's 16 keys of one head, 64 dims), k8 / v8 a box of
// {64, 16, 1, 8} (8 consecutive pages: 128 keys in one copy).
struct KvMaps {
    CUtensorMap k, v, k8, v8;
};
// The cached maps of a device-resident pool with 16-row pages; false when the
// pool is elsewhere (pinned host memory) or has pages of another size.
bool kv_maps(const KeySrc& src, int n_kv, int d, KvMaps* out);

// One box of a 4-D tensor map into this CTA's shared memory (no multicast),
// completing on `bar`.  Coordinates past the view's bounds read zeros.
DKV_DEV void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];\n" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// After a CTA has stored its partial rows (m, l, unnormalised O) for split s
// of (sequence, head, row block) `bhr`, the last CTA to arrive merges every
// split in split order (splits with no live key skipped), writes the output
// rows and returns true with the merged max / sum in ms / ls (R rows).
// The merge order is fixed, so a row's result is the same whatever the number
// of rows or splits that share the launch.  RB: the row stride of a split's
// partial block (the launch's rows per CTA).  wbuf / wcap: shared memory
// the caller no longer needs (its drained ring), floats; without it the
// weights of up to 16 splits go to a static array.
template <int RB = kAttnRB>
DKV_DEV bool split_merge(const AttnArgs& a, size_t bhr, int b, int h, int R, int r0, float* ms, float* ls,
                         float* wbuf = nullptr, int wcap = 0) {
    const int d = a.d, G = a.group, T = a.T, PS = d + 2, HQ = a.n_kv * G;
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (threadIdx.x == 0) {
        unsigned* tk = a.tickets + bhr;
        const unsigned prev = atomicAdd(tk, 1u);
        is_last = prev == (unsigned)(a.n_splits - 1);
        if (is_last) *tk = 0u;
    }
    __syncthreads();
    if (!is_last) return false;
    __threadfence();
    const float* parts = a.part + (bhr * a.n_splits) * RB * PS;
    // per (row, split) weight exp(m_q - M), -1 for a split with no live key;
    // with up to kMergeW splits the weights sit in shared memory and the
    // partials of several elements are loaded at once (the same products in
    // the same split order as the one-element loop, so the same bits)
    constexpr int kMergeW = 16;
    __shared__ float wq_s[RB * kMergeW];
    const int ns = a.n_splits;
    const bool big = wbuf && ns > kMergeW && (long long)ns * RB <= wcap;
    float* wq = big ? wbuf : wq_s;
    const int wst = big ? ns : kMergeW;       // row stride of wq
    const bool staged = (big || ns <= kMergeW) && d % 2 == 0;
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        float M = -INFINITY, L = 0.f;
        if (staged) {
            // splits in groups of kMergeW, each group's loads issued together:
            // the max first, then the weights and the sum in split order
            for (int q0 = 0; q0 < ns; q0 += kMergeW) {
                float mq[kMergeW];
#pragma unroll
                for (int k = 0; k < kMergeW; ++k)
                    mq[k] = q0 + k < ns ? __ldcg(parts + ((size_t)(q0 + k) * RB + r) * PS) : -INFINITY;
#pragma unroll
                for (int k = 0; k < kMergeW; ++k) M = fmaxf(M, mq[k]);
            }
            for (int q0 = 0; q0 < ns; q0 += kMergeW) {
                float mq[kMergeW], lq[kMergeW];
#pragma unroll
                for (int k = 0; k < kMergeW; ++k) {
                    const int q = q0 + k;
                    mq[k] = q < ns ? __ldcg(parts + ((size_t)q * RB + r) * PS) : -INFINITY;
                    lq[k] = q < ns ? __ldcg(parts + ((size_t)q * RB + r) * PS + 1) : 0.f;
                }
#pragma unroll
                for (int k = 0; k < kMergeW; ++k) {
                    if (q0 + k >= ns) break;
                    if (mq[k] == -INFINITY) {
                        wq[r * wst + q0 + k] = -1.f;
                        continue;
                    }
                    const float w = expf(mq[k] - M);
                    wq[r * wst + q0 + k] = w;
                    L += lq[k] * w;
                }
            }
        } else {
            for (int q = 0; q < ns; ++q) M = fmaxf(M, __ldcg(parts + ((size_t)q * RB + r) * PS));
            for (int q = 0; q < ns; ++q) {
                const float mq = __ldcg(parts + ((size_t)q * RB + r) * PS);
                if (mq == -INFINITY) continue;
                L += __ldcg(parts + ((size_t)q * RB + r) * PS + 1) * expf(mq - M);
            }
        }
        ms[r] = M;
        ls[r] = L;
    }
    __syncthreads();
    if (staged) {
        // element pairs (e, e + 1), kMergeP of them a thread, kMergeQ splits
        // at a time: their kMergeP x kMergeQ loads are issued together, then
        // each element is summed over the splits in split order (128-row
        // blocks: eight pairs a thread, one split at a time -- measured on
        // B200, prefill attention at batch 4 x 32k: 716 TF/s, 640 with four
        // splits at a time; up to 64 rows: two pairs, eight splits at a
        // time, within the decode kernels' 128 registers)
        constexpr int kMergeP = RB >= 128 ? 8 : 2, kMergeQ = RB >= 128 ? 1 : 8;
        const int npairs = R * d / 2;
        for (int p0 = threadIdx.x; p0 < npairs; p0 += kMergeP * blockDim.x) {
            float2 acc[kMergeP];
            int rr[kMergeP], ee[kMergeP];
#pragma unroll
            for (int u = 0; u < kMergeP; ++u) {
                const int pi = p0 + u * blockDim.x;
                rr[u] = pi < npairs ? 2 * pi / d : -1;
                ee[u] = pi < npairs ? 2 * pi % d : 0;
                acc[u] = make_float2(0.f, 0.f);
            }
            for (int q0 = 0; q0 < ns; q0 += kMergeQ) {
                float2 v[kMergeQ][kMergeP];
                float w[kMergeQ][kMergeP];
#pragma unroll
                for (int k = 0; k < kMergeQ; ++k)
#pragma unroll
                    for (int u = 0; u < kMergeP; ++u) {
                        const int q = q0 + k;
                        w[k][u] = (q < ns && rr[u] >= 0) ? wq[rr[u] * wst + (q < ns ? q : 0)] : -1.f;
                        v[k][u] = w[k][u] >= 0.f ? __ldcg(reinterpret_cast<const float2*>(
                                                       parts + ((size_t)q * RB + rr[u]) * PS + 2 + ee[u]))
                                                 : make_float2(0.f, 0.f);
                    }
#pragma unroll
                for (int k = 0; k < kMergeQ; ++k)
#pragma unroll
                    for (int u = 0; u < kMergeP; ++u)
                        if (w[k][u] >= 0.f) {
                            acc[u].x += v[k][u].x * w[k][u];
                            acc[u].y += v[k][u].y * w[k][u];
                        }
            }
#pragma unroll
            for (int u = 0; u < kMergeP; ++u) {
                if (rr[u] < 0) continue;
                const int r = rr[u], e = ee[u];
                const float L = ls[r];
                const int t = (r0 + r) / G, g = (r0 + r) % G;
                const size_t o = (((size_t)b * T + t) * HQ + h * G + g) * d + e;
                store_from_f32(a.out, a.out_dtype, o, L > 0.f ? acc[u].x / L : 0.f);
                store_from_f32(a.out, a.out_dtype, o + 1, L > 0.f ? acc[u].y / L : 0.f);
            }
        }
    } else {
        for (int i = threadIdx.x; i < R * d; i += blockDim.x) {
            const int r = i / d, e = i % d;
            const float M = ms[r];
            float acc = 0.f;
            for (int q = 0; q < ns; ++q) {
                const float mq = __ldcg(parts + ((size_t)q * RB + r) * PS);
                if (mq == -INFINITY) continue;
                acc += __ldcg(parts + ((size_t)q * RB + r) * PS + 2 + e) * expf(mq - M);
            }
            const float o = ls[r] > 0.f ? acc / ls[r] : 0.f;
            const int t = (r0 + r) / G, g = (r0 + r) % G;
            store_from_f32(a.out, a.out_dtype, (((size_t)b * T + t) * HQ + h * G + g) * d + e, o);
        }
    }
    __syncthreads();
    return true;
}

}  // namespace dkv
