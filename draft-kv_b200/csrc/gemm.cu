// K4 weight-streaming GEMM (Y = X W^T) and K4e fused epilogues.
//
// Replaces the projections of draftkv/llama.py:187-225 (x @ W.T, SwiGLU :222,
// tied head :224-225, RoPE :197-198 with _rope :164-172) and
// draftkv/gpt2.py:191-213 (Conv1D x @ W + b, gelu_new :126-127, tied head).
//
// Decode-time GEMMs have few tokens (N = batch x (gamma+1) <= 64 per CTA)
// and stream every weight byte once, so the kernel is organised around the
// weight stream: weights are stored in a tiled layout where one warp-wide
// 16-byte load per k-step yields exactly the mma.m16n8k16 A fragments
// (512 contiguous bytes per warp per k-step), weight rows ride on M and the
// tokens on N ("swap-AB").  Tokens are staged in shared memory in 128-wide k
// chunks and fed through ldmatrix.
//
// Determinism / batch invariance: the split of K across CTAs (S) depends
// only on (M, K) and the device, partial sums are reduced in a fixed order
// (bf16: by the CTAs of a thread-block cluster through distributed shared
// memory; fp32 and the no-alloc entry: by the last CTA of each row tile,
// atomic ticket, no spin), and a token's column never depends on the other
// columns, so a token's output is bit-identical whether it is computed with
// 1 or 64 other tokens.  This is what makes the verify pass reproduce plain
// decoding exactly.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dkv {

constexpr int kTileM = 128;     // weight rows per CTA (8 warps x 16)
constexpr int kChunkK = 256;    // k elements per staged X chunk
constexpr int kChunkSteps = kChunkK / 16;   // k16 steps per chunk = weight prefetch depth
constexpr int kTileStride = 132;  // smem row stride (floats) of the result tile [n][m]
// Split-K tickets occupy a fixed region at the start of every GEMM work
// buffer, so consecutive calls of any shape see them zero (each launch
// resets the tickets it used).
constexpr size_t kGemmTickets = 65536;

struct EpiArgs {
    int kind;
    const float* bias;
    float* out_f32;
    void* act;
    int act_dtype, ld_out, M_real;
    int n_heads, n_kv, d_head, tokens_per_seq;
    const int32_t* pos0;
    const float* rope_cos;
    const float* rope_sin;
    float* q_out;
    void* kv_stage;
    int model_dtype;
    // full cache target
    void* k_pool;
    void* v_pool;
    const int32_t* page_table;
    int page_size, max_pages, layer, n_layers;
};

DKV_DEV float gelu_new(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))  (gpt2.py:126-127)
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

DKV_DEV float silu(float x) { return x / (1.0f + expf(-x)); }

// Applies the epilogue to the tile T[n][m] (n < nb valid tokens starting at
// n0), token rows [j0, j1) of it (all rows when j1 < 0).
DKV_DEV void run_epilogue(const EpiArgs& e, const float* T, int mtile, int n0, int nb, int j0 = 0, int j1 = -1) {
    const int m0 = mtile * kTileM;
    if (j1 < 0) j1 = nb;
    const int total = kTileM * (j1 - j0);
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int i = idx % kTileM, j = j0 + idx / kTileM;
        const int m = m0 + i, n = n0 + j;
        const float acc = T[j * kTileStride + i];
        switch (e.kind) {
            case DKV_EPI_STORE:
                if (m < e.M_real) e.out_f32[(size_t)n * e.ld_out + m] = acc + (e.bias ? e.bias[m] : 0.f);
                break;
            case DKV_EPI_RESADD:
                if (m < e.M_real) e.out_f32[(size_t)n * e.ld_out + m] += acc + (e.bias ? e.bias[m] : 0.f);
                break;
            case DKV_EPI_GELU:
                if (m < e.M_real)
                    store_from_f32(e.act, e.act_dtype, (size_t)n * e.ld_out + m,
                                   gelu_new(acc + (e.bias ? e.bias[m] : 0.f)));
                break;
            case DKV_EPI_SWIGLU:
                if (i < 64) {
                    const float g = acc + (e.bias ? e.bias[m] : 0.f);
                    const float u = T[j * kTileStride + i + 64] + (e.bias ? e.bias[m + 64] : 0.f);
                    const int col = mtile * 64 + i;
                    if (col < e.M_real) store_from_f32(e.act, e.act_dtype, (size_t)n * e.ld_out + col, silu(g) * u);
                }
                break;
            case DKV_EPI_QKV: {
                const int D = e.d_head, HD = e.n_heads * D, KD = e.n_kv * D;
                if (m >= HD + 2 * KD) break;
                const int b = n / e.tokens_per_seq, t = n % e.tokens_per_seq;
                const int p = e.pos0[b] + t;
                const int sec = m < HD ? 0 : (m < HD + KD ? 1 : 2);
                const int mm = sec == 0 ? m : (sec == 1 ? m - HD : m - HD - KD);
                const int head = mm / D, dd = mm % D;
                float val = acc + (e.bias ? e.bias[m] : 0.f);
                if (sec < 2 && e.rope_cos) {
                    const int hd = D / 2;
                    const int pair = dd < hd ? i + hd : i - hd;
                    const float other = T[j * kTileStride + pair] + (e.bias ? e.bias[m0 + pair] : 0.f);
                    const int f = dd < hd ? dd : dd - hd;
                    const float cs = e.rope_cos[(size_t)p * hd + f], sn = e.rope_sin[(size_t)p * hd + f];
                    // x*cos + rotate_half(x)*sin, rotate_half = [-x2, x1]
                    val = dd < hd ? val * cs - other * sn : val * cs + other * sn;
                }
                if (sec == 0) {
                    e.q_out[(size_t)n * HD + mm] = val;
                } else if (e.kv_stage) {
                    const size_t o = (((size_t)n * e.n_kv + head) * 2 + (sec - 1)) * D + dd;
                    store_from_f32(e.kv_stage, e.model_dtype, o, val);
                } else {
                    const int page = e.page_table[((size_t)b * e.n_layers + e.layer) * e.max_pages + p / e.page_size];
                    const size_t o = (((size_t)page * e.n_kv + head) * e.page_size + (p % e.page_size)) * D + dd;
                    store_from_f32(sec == 1 ? e.k_pool : e.v_pool, e.model_dtype, o, val);
                }
                break;
            }
            default:
                break;
        }
    }
}

// Split-K finish: every CTA of a row tile leaves its partial tile; the last to
// arrive sums them in split order and runs the epilogue.
DKV_DEV void finish_tile(const EpiArgs& e, float* tile, int nbc, int mtile, int mtiles, int nblk_idx, int S,
                         int s, int n0, int nb, float* ws, unsigned* tickets) {
    const int tile_floats = nbc * kTileStride;
    if (S > 1) {
        float* mine = ws + (((size_t)nblk_idx * mtiles + mtile) * S + s) * tile_floats;
        for (int i = threadIdx.x; i < tile_floats; i += blockDim.x) mine[i] = tile[i];
        __threadfence();
        __syncthreads();
        __shared__ int is_last;
        if (threadIdx.x == 0) {
            unsigned* tk = tickets + (size_t)nblk_idx * mtiles + mtile;
            const unsigned prev = atomicAdd(tk, 1u);
            is_last = prev == (unsigned)(S - 1);
            if (is_last) *tk = 0u;   // self-reset for the next launch
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        const float* base = ws + (((size_t)nblk_idx * mtiles + mtile) * S) * tile_floats;
        for (int i = threadIdx.x; i < tile_floats; i += blockDim.x) {
            float acc = __ldcg(base + i);
            for (int q = 1; q < S; ++q) acc += __ldcg(base + (size_t)q * tile_floats + i);
            tile[i] = acc;
        }
        __syncthreads();
    }
    run_epilogue(e, tile, mtile, n0, nb);
}

struct GemmArgs {
    const void* x;      // [N][K] bf16 or f32
    const void* w;      // tiled bf16 or row-major f32
    int M, N, K, S;
    float* ws;
    unsigned* tickets;
    uint32_t* err;      // device error word (bounded waits)
    EpiArgs epi;
};

DKV_DEV void mma_bf16(float (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

DKV_DEV void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
DKV_DEV void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(a));
}

DKV_DEV void cp_async16(void* smem, const void* gmem, bool pred) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    const int n = pred ? 16 : 0;   // zero-fill when out of range
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
DKV_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
DKV_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// X chunk row stride in bf16 elements (128 + 8 padding: conflict-free ldmatrix)
constexpr int kXStride = kChunkK + 8;

constexpr int kWChunkBytes = kChunkSteps * 512;   // one warp's weights for one X chunk

// Weight stages per warp: deeper for few tokens (small X chunks).
template <int NT>
__host__ __device__ constexpr int gemm_stages() {
    return NT <= 2 ? 3 : 2;
}
template <int NT>
__host__ __device__ constexpr size_t gemm_smem() {
    return (size_t)2 * 8 * NT * kXStride * 2 + (size_t)8 * gemm_stages<NT>() * kWChunkBytes + 8 * 8 * sizeof(uint64_t);
}

template <int NT>   // number of n8 token tiles per CTA (tokens = 8*NT)
__global__ void __launch_bounds__(256) gemm_bf16_kernel(GemmArgs g) {
    extern __shared__ __align__(128) uint8_t gsm[];
    constexpr int NB = 8 * NT;
    constexpr int NST = gemm_stages<NT>();
    uint16_t* xs = reinterpret_cast<uint16_t*>(gsm);          // [2][NB][kXStride]
    uint8_t* wst = gsm + (size_t)2 * NB * kXStride * 2;       // [8 warps][NST][kWChunkBytes]
    uint64_t* bars = reinterpret_cast<uint64_t*>(wst + (size_t)8 * NST * kWChunkBytes);   // [8][NST]
    const int mtiles = g.M / kTileM;
    const int mtile = blockIdx.x % mtiles, s = blockIdx.x / mtiles;
    const int nblk = blockIdx.y, n0 = nblk * 64;
    const int KT = g.K / 16;
    const int kt0 = (int)((long long)s * KT / g.S), kt1 = (int)((long long)(s + 1) * KT / g.S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t* X = reinterpret_cast<const uint16_t*>(g.x);
    const int nsteps = kt1 - kt0;
    const int nchunks = (nsteps + kChunkSteps - 1) / kChunkSteps;
    // this warp's weight stream: 16 rows x [kt0, kt1) is one contiguous byte range
    const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(g.w) + ((size_t)(mtile * 8 + warp) * KT + kt0) * 512;
    uint8_t* my_st = wst + (size_t)warp * NST * kWChunkBytes;
    uint64_t* my_bar = bars + warp * NST;
    auto issue = [&](int ch) {    // lane 0 only
        const int steps = min(kChunkSteps, nsteps - ch * kChunkSteps);
        const uint32_t bytes = (uint32_t)steps * 512u;
        uint64_t* bar = my_bar + (ch % NST);
        mbar_expect_tx(bar, bytes);
        bulk_g2s(my_st + (size_t)(ch % NST) * kWChunkBytes, wsrc + (size_t)ch * kWChunkBytes, bytes, bar);
    };
    pdl_trigger();
    if (lane == 0) {
        for (int i = 0; i < NST; ++i) mbar_init(my_bar + i, 1);
        fence_async_shared();
        for (int ch = 0; ch < NST && ch < nchunks; ++ch) issue(ch);
    }
    __syncwarp();
    // the weights do not depend on earlier kernels; activations, outputs,
    // split-K partials and tickets do
    pdl_wait();

    // X chunk loader: rows n0..n0+NB-1, k range [k_lo, k_lo + 128)
    auto load_chunk = [&](int buf, int k_lo) {
        uint16_t* dst = xs + buf * NB * kXStride;
        for (int i = threadIdx.x; i < NB * (kChunkK / 8); i += blockDim.x) {
            const int r = i / (kChunkK / 8), c8 = i % (kChunkK / 8);
            const int n = n0 + r, k = k_lo + c8 * 8;
            const bool ok = n < g.N && k < kt1 * 16;
            cp_async16(dst + r * kXStride + c8 * 8, ok ? (const void*)(X + (size_t)n * g.K + k) : (const void*)X, ok);
        }
        cp_async_commit();
    };

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

    bool ok_all = true;
    if (nchunks > 0) load_chunk(0, kt0 * 16);
    for (int ch = 0; ch < nchunks; ++ch) {
        if (ch + 1 < nchunks) {
            load_chunk((ch + 1) & 1, (kt0 + (ch + 1) * kChunkSteps) * 16);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint16_t* xb = xs + (ch & 1) * NB * kXStride;
        const bool ready = mbar_wait(my_bar + (ch % NST), (uint32_t)((ch / NST) & 1), g.err);
        ok_all = ok_all && ready;
        const uint4* wa = reinterpret_cast<const uint4*>(my_st + (size_t)(ch % NST) * kWChunkBytes) + lane;
#pragma unroll
        for (int i = 0; i < kChunkSteps; ++i) {
            const int kt = kt0 + ch * kChunkSteps + i;
            if (kt < kt1 && ready) {
                const uint4 a = wa[i * 32];
                const int kc = i * 16;   // k offset within chunk
#pragma unroll
                for (int j = 0; j + 1 < NT; j += 2) {
                    uint32_t b0, b1, b2, b3;
                    const int mi = lane >> 3, r = lane & 7;
                    const uint16_t* p = xb + (8 * j + (mi >= 2 ? 8 : 0) + r) * kXStride + kc + (mi & 1) * 8;
                    ldsm_x4(b0, b1, b2, b3, p);
                    mma_bf16(acc[j], a, b0, b1);
                    mma_bf16(acc[j + 1], a, b2, b3);
                }
                if (NT & 1) {
                    uint32_t b0, b1;
                    const int mi = (lane >> 3) & 1, r = lane & 7;
                    const uint16_t* p = xb + (8 * (NT - 1) + r) * kXStride + kc + mi * 8;
                    ldsm_x2(b0, b1, p);
                    mma_bf16(acc[NT - 1], a, b0, b1);
                }
            }
        }
        // this stage is consumed: refill it with chunk ch + NST
        __syncwarp();
        if (lane == 0 && ch + NST < nchunks && ok_all) {
            fence_async_shared();
            issue(ch + NST);
        }
        __syncthreads();
    }
    if (!ok_all && lane == 0) {
        // a copy never completed: wait (bounded) for any still in flight
        // before the shared memory is reused or released
        for (int ch = max(0, nchunks - NST); ch < nchunks; ++ch)
            mbar_wait(my_bar + (ch % NST), (uint32_t)((ch / NST) & 1), nullptr);
    }
    __syncthreads();

    // result tile T[n][m] in shared memory (reuses the X buffers)
    float* tile = reinterpret_cast<float*>(gsm);
    {
        const int r = lane >> 2, c = lane & 3;
        const int mrow = warp * 16 + r;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int n = 8 * j + 2 * c;
            tile[n * kTileStride + mrow] = acc[j][0];
            tile[(n + 1) * kTileStride + mrow] = acc[j][1];
            tile[n * kTileStride + mrow + 8] = acc[j][2];
            tile[(n + 1) * kTileStride + mrow + 8] = acc[j][3];
        }
    }
    __syncthreads();
    const int nb = min(NB, g.N - n0);
    finish_tile(g.epi, tile, NB, mtile, mtiles, nblk, g.S, s, n0, nb, g.ws, g.tickets);
}

// ---------------------------------------------------------------------------
// Clustered split-K schedule (every bf16 dkv_gemm call).
//
// The S CTAs that split one row tile's K range form a thread-block cluster.
// After its k range each CTA leaves its partial tile in its own shared
// memory; every CTA then sums the S partials of its share of the token rows
// in rank order through distributed shared memory (no global round trip, no
// ticket: the tail of a split GEMM is one cluster barrier and a few KB of
// DSMEM reads) and applies the epilogue to those rows.  Clusters are
// persistent over row tiles (tile = cluster id + i x clusters) and a CTA's
// weight ring runs on across its tiles, so a GEMM with more row tiles than
// SMs has no relaunch gap between waves.  S depends on (M, K) only and the
// partials are summed in a fixed order, so a token's output does not depend
// on the other tokens of the call.
template <int NT>   // number of n8 token tiles per CTA (tokens = 8*NT)
__global__ void __launch_bounds__(256, 1) gemm_bf16_cl_kernel(GemmArgs g) {
    extern __shared__ __align__(128) uint8_t gsm[];
    constexpr int NB = 8 * NT;
    constexpr int NST = gemm_stages<NT>();
    uint16_t* xs = reinterpret_cast<uint16_t*>(gsm);          // [2][NB][kXStride]
    uint8_t* wst = gsm + (size_t)2 * NB * kXStride * 2;       // [8 warps][NST][kWChunkBytes]
    uint64_t* bars = reinterpret_cast<uint64_t*>(wst + (size_t)8 * NST * kWChunkBytes);   // [8][NST]
    cg::cluster_group cluster = cg::this_cluster();
    const int S = g.S;
    const int s = S > 1 ? (int)cluster.block_rank() : 0;
    const int cid = blockIdx.x / S, ncl = gridDim.x / S;
    const int mtiles = g.M / kTileM;
    const int nblk = blockIdx.y, n0 = nblk * 64;
    const int KT = g.K / 16;
    const int kt0 = (int)((long long)s * KT / S), kt1 = (int)((long long)(s + 1) * KT / S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t* X = reinterpret_cast<const uint16_t*>(g.x);
    const int nsteps = kt1 - kt0;
    const int nchunks = (nsteps + kChunkSteps - 1) / kChunkSteps;
    const int my_tiles = cid < mtiles ? (mtiles - 1 - cid) / ncl + 1 : 0;
    const int total = my_tiles * nchunks;        // ring units of this CTA
    uint8_t* my_st = wst + (size_t)warp * NST * kWChunkBytes;
    uint64_t* my_bar = bars + warp * NST;
    // ring unit i: chunk i % nchunks of row tile cid + (i / nchunks) ncl; this
    // warp's 16 weight rows over the chunk are one contiguous byte range
    auto issue = [&](int i) {    // lane 0 only
        const int tile = cid + (i / nchunks) * ncl, ch = i % nchunks;
        const int steps = min(kChunkSteps, nsteps - ch * kChunkSteps);
        const uint32_t bytes = (uint32_t)steps * 512u;
        uint64_t* bar = my_bar + (i % NST);
        mbar_expect_tx(bar, bytes);
        bulk_g2s(my_st + (size_t)(i % NST) * kWChunkBytes,
                 reinterpret_cast<const uint8_t*>(g.w) +
                     ((size_t)(tile * 8 + warp) * KT + kt0 + (size_t)ch * kChunkSteps) * 512,
                 bytes, bar);
    };
    pdl_trigger();
    if (lane == 0) {
        for (int i = 0; i < NST; ++i) mbar_init(my_bar + i, 1);
        fence_async_shared();
        for (int i = 0; i < NST && i < total; ++i) issue(i);
    }
    __syncwarp();
    // the weights do not depend on earlier kernels; activations and outputs do
    pdl_wait();

    // X chunk loader: rows n0..n0+NB-1, k range [k_lo, k_lo + 256) within [kt0, kt1)
    auto load_chunk = [&](int buf, int k_lo) {
        uint16_t* dst = xs + buf * NB * kXStride;
        for (int i = threadIdx.x; i < NB * (kChunkK / 8); i += blockDim.x) {
            const int r = i / (kChunkK / 8), c8 = i % (kChunkK / 8);
            const int n = n0 + r, k = k_lo + c8 * 8;
            const bool ok = n < g.N && k < kt1 * 16;
            cp_async16(dst + r * kXStride + c8 * 8, ok ? (const void*)(X + (size_t)n * g.K + k) : (const void*)X, ok);
        }
        cp_async_commit();
    };

    const int nb = min(NB, g.N - n0);
    // this CTA's token rows of each tile's epilogue
    const int j0 = s * nb / S, j1 = (s + 1) * nb / S;
    bool ok_all = true;
    int i = 0;
    for (int ti = 0; ti < my_tiles; ++ti) {
        const int mtile = cid + ti * ncl;
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        if (nchunks > 0) load_chunk(0, kt0 * 16);
        for (int ch = 0; ch < nchunks; ++ch, ++i) {
            if (ch + 1 < nchunks) {
                load_chunk((ch + 1) & 1, (kt0 + (ch + 1) * kChunkSteps) * 16);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
            const uint16_t* xb = xs + (ch & 1) * NB * kXStride;
            const bool ready = mbar_wait(my_bar + (i % NST), (uint32_t)((i / NST) & 1), g.err);
            ok_all = ok_all && ready;
            const uint4* wa = reinterpret_cast<const uint4*>(my_st + (size_t)(i % NST) * kWChunkBytes) + lane;
#pragma unroll
            for (int st = 0; st < kChunkSteps; ++st) {
                const int kt = kt0 + ch * kChunkSteps + st;
                if (kt < kt1 && ready) {
                    const uint4 a = wa[st * 32];
                    const int kc = st * 16;   // k offset within chunk
#pragma unroll
                    for (int j = 0; j + 1 < NT; j += 2) {
                        uint32_t b0, b1, b2, b3;
                        const int mi = lane >> 3, r = lane & 7;
                        const uint16_t* p = xb + (8 * j + (mi >= 2 ? 8 : 0) + r) * kXStride + kc + (mi & 1) * 8;
                        ldsm_x4(b0, b1, b2, b3, p);
                        mma_bf16(acc[j], a, b0, b1);
                        mma_bf16(acc[j + 1], a, b2, b3);
                    }
                    if (NT & 1) {
                        uint32_t b0, b1;
                        const int mi = (lane >> 3) & 1, r = lane & 7;
                        const uint16_t* p = xb + (8 * (NT - 1) + r) * kXStride + kc + mi * 8;
                        ldsm_x2(b0, b1, p);
                        mma_bf16(acc[NT - 1], a, b0, b1);
                    }
                }
            }
            // this stage is consumed: refill it with ring unit i + NST
            __syncwarp();
            if (lane == 0 && i + NST < total && ok_all) {
                fence_async_shared();
                issue(i + NST);
            }
            __syncthreads();
        }

        // ---- partial tile T[n][m] in the X buffers (both consumed)
        float* tile = reinterpret_cast<float*>(gsm);
        {
            const int r = lane >> 2, c = lane & 3;
            const int mrow = warp * 16 + r;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int n = 8 * j + 2 * c;
                tile[n * kTileStride + mrow] = acc[j][0];
                tile[(n + 1) * kTileStride + mrow] = acc[j][1];
                tile[n * kTileStride + mrow + 8] = acc[j][2];
                tile[(n + 1) * kTileStride + mrow + 8] = acc[j][3];
            }
        }
        if (S > 1) {
            cluster.sync();
            // rows [j0, j1): sum of the S partials in rank order, in place (the
            // other CTAs read only their own rows of this tile)
            for (int e = threadIdx.x; e < (j1 - j0) * kTileM; e += blockDim.x) {
                const int o = (j0 + e / kTileM) * kTileStride + e % kTileM;
                float v = cluster.map_shared_rank(tile, 0)[o];
                for (int q = 1; q < S; ++q) v += cluster.map_shared_rank(tile, q)[o];
                tile[o] = v;
            }
        }
        __syncthreads();
        run_epilogue(g.epi, tile, mtile, n0, nb, j0, j1);
        // the next tile's X chunks overwrite this tile: every CTA of the
        // cluster has read its rows of it
        if (S > 1) cluster.sync();
        else __syncthreads();
    }
    if (!ok_all && lane == 0) {
        // a copy never completed: wait (bounded) for any still in flight
        // before the shared memory is released
        for (int u = max(0, total - NST); u < total; ++u)
            mbar_wait(my_bar + (u % NST), (uint32_t)((u / NST) & 1), nullptr);
    }
}

// fp32 weights [M][K] row-major, CUDA cores.  Warp w owns 16 weight rows of
// the tile; lanes split k in float4 steps; 4 tokens per CTA; warp sums
// reduced in a fixed butterfly.
constexpr int kF32Tok = 4;
constexpr int kF32Chunk = 256;

__global__ void __launch_bounds__(256) gemm_f32_kernel(GemmArgs g) {
    extern __shared__ __align__(16) uint8_t gsm[];
    float* xs = reinterpret_cast<float*>(gsm);   // [kF32Tok][kF32Chunk]
    const int mtiles = g.M / kTileM;
    const int mtile = blockIdx.x % mtiles, s = blockIdx.x / mtiles;
    const int nblk = blockIdx.y, n0 = nblk * kF32Tok;
    const int KT = g.K / 16;
    const int k0 = (int)((long long)s * KT / g.S) * 16, k1 = (int)((long long)(s + 1) * KT / g.S) * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* X = reinterpret_cast<const float*>(g.x);
    const float* W = reinterpret_cast<const float*>(g.w);
    float acc[16][kF32Tok];
#pragma unroll
    for (int r = 0; r < 16; ++r)
#pragma unroll
        for (int t = 0; t < kF32Tok; ++t) acc[r][t] = 0.f;

    for (int kc = k0; kc < k1; kc += kF32Chunk) {
        const int kl = min(kF32Chunk, k1 - kc);
        __syncthreads();
        for (int i = threadIdx.x; i < kF32Tok * kF32Chunk; i += blockDim.x) {
            const int t = i / kF32Chunk, k = i % kF32Chunk;
            const int n = n0 + t;
            xs[i] = (n < g.N && k < kl) ? X[(size_t)n * g.K + kc + k] : 0.f;
        }
        __syncthreads();
        for (int k4 = lane; k4 * 4 < kl; k4 += 32) {
            float4 xv[kF32Tok];
#pragma unroll
            for (int t = 0; t < kF32Tok; ++t) xv[t] = *reinterpret_cast<const float4*>(xs + t * kF32Chunk + k4 * 4);
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const int m = mtile * kTileM + warp * 16 + r;
                const float4 w = __ldcs(reinterpret_cast<const float4*>(W + (size_t)m * g.K + kc) + k4);
#pragma unroll
                for (int t = 0; t < kF32Tok; ++t)
                    acc[r][t] += w.x * xv[t].x + w.y * xv[t].y + w.z * xv[t].z + w.w * xv[t].w;
            }
        }
    }
    __syncthreads();
    float* tile = reinterpret_cast<float*>(gsm);
#pragma unroll
    for (int r = 0; r < 16; ++r)
#pragma unroll
        for (int t = 0; t < kF32Tok; ++t) {
            const float v = warp_sum(acc[r][t]);
            if (lane == 0) tile[t * kTileStride + warp * 16 + r] = v;
        }
    __syncthreads();
    const int nb = min(kF32Tok, g.N - n0);
    finish_tile(g.epi, tile, kF32Tok, mtile, mtiles, nblk, g.S, s, n0, nb, g.ws, g.tickets);
}

// Tiles W [M][K] bf16 into the A-fragment layout [M/16][K/16][32][8].
__global__ void pack_weight_kernel(const uint16_t* __restrict__ w, int M, int K, uint16_t* __restrict__ out) {
    const size_t total = (size_t)M * K;
    for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int e = o & 7;
        const int lane = (o >> 3) & 31;
        const size_t tk = o >> 8;           // (mt16 * KT + kt)
        const int KT = K / 16;
        const int kt = (int)(tk % KT);
        const int mt = (int)(tk / KT);
        const int reg = e >> 1, el = e & 1;
        const int r = lane >> 2, c = lane & 3;
        const int row = mt * 16 + r + ((reg & 1) ? 8 : 0);
        const int col = kt * 16 + 2 * c + ((reg & 2) ? 8 : 0) + el;
        out[o] = w[(size_t)row * K + col];
    }
}

// K split S for an (M, K) GEMM.  One CTA per SM is resident (the weight
// stages fill shared memory), and a launch of decode-sized GEMMs is bound by
// per-CTA latency as much as by bandwidth, so S fills at most one wave of 148
// SMs with few, long CTAs: S = floor(128 / row tiles), capped at 4 and at the
// number of 256-wide k chunks (measured on B200: 4096 x 4096 is fastest at
// S = 4, 6144 x 4096 at S = 2, 28672 x 4096 and the 128256-row head at S = 1).
// S depends on (M, K) only -- never on the token count -- which keeps every
// token's reduction order fixed.
uint32_t* device_error_word();

int choose_split(int M, int K) {
    const int mtiles = M / kTileM > 0 ? M / kTileM : 1;
    const int max_s = K / kChunkK > 0 ? K / kChunkK : 1;
    int S = 128 / mtiles;
    S = S < 1 ? 1 : (S > 4 ? 4 : S);
    return S < max_s ? S : max_s;
}

// Clusters of S CTAs of gemm_bf16_cl_kernel<NT> that can be resident at once
// on the current device (one CTA per SM; clusters do not span GPCs).
template <int NT>
int cl_active(int S) {
    static int cache[64][9] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || S < 1 || S > 8) return 0;
    if (cache[dev][S] == 0) {
        if (allow_smem_max(gemm_bf16_cl_kernel<NT>) != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S * 148);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = gemm_smem<NT>();
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_cl_kernel<NT>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return 0;
        }
        cache[dev][S] = n;
    }
    return cache[dev][S];
}

// Clusters launched for mtiles row tiles when act fit at once: one per row
// tile up to two waves, persistent clusters over more row tiles (no gap
// between the waves of the 1002-tile head).
int cl_count(int mtiles, int act) { return mtiles <= 2 * act ? mtiles : act; }

// Launches the clustered kernel: ncl clusters of S CTAs per token block,
// with programmatic dependent launch.
template <typename Kern>
cudaError_t launch_cl(Kern kern, int ncl, int S, int nblk, size_t smem, cudaStream_t st, const GemmArgs& g) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ncl * S, nblk);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = S;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = S > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, g);
}

// K split S of the clustered schedule for an (M, K) GEMM: the S in 1..8 (at
// most the number of 256-wide k chunks) that minimises the modelled time of
// one CTA in k steps, rounds x (ceil(KT / S) + 32), where rounds = row tiles
// per cluster with as many clusters as fit at once and 32 k steps charge the
// end of a row tile (barriers, partial sums, epilogue: the weight ring runs
// dry meanwhile; measured on B200, ~2 us), plus 8 k steps per extra partial
// summed.  The residency used is that of the one-token-tile kernel, so S
// depends on (M, K) and the device only -- never on the token count.
int choose_split_cl(int M, int K) {
    const int mtiles = M / kTileM > 0 ? M / kTileM : 1;
    const int KT = K / 16;
    const int max_s = std::max(1, std::min(8, K / kChunkK));
    int best = 1;
    double best_cost = 0.0;
    for (int S = 1; S <= max_s; ++S) {
        const int act = cl_active<1>(S);
        if (act <= 0) continue;
        const int ncl = std::min(mtiles, act);
        const int rounds = (mtiles + ncl - 1) / ncl;
        const double cost = (double)rounds * ((KT + S - 1) / S + 32) + 8.0 * (S - 1);
        if (S == 1 || cost < best_cost - 1e-9) {
            best = S;
            best_cost = cost;
        }
    }
    return best;
}

}  // namespace dkv

using namespace dkv;

namespace dkv {
EpiArgs make_epi(const dkv_epilogue* e, int M_real);
}

dkv::EpiArgs dkv::make_epi(const dkv_epilogue* e, int M_real) {
    EpiArgs a{};
    a.kind = e->kind;
    a.bias = e->bias;
    a.out_f32 = e->out_f32;
    a.act = e->act;
    a.act_dtype = e->act_dtype;
    a.ld_out = e->ld_out;
    a.M_real = M_real;
    a.n_heads = e->n_heads;
    a.n_kv = e->n_kv;
    a.d_head = e->d_head;
    a.tokens_per_seq = e->tokens_per_seq > 0 ? e->tokens_per_seq : 1;
    a.pos0 = e->pos0;
    a.rope_cos = e->rope_cos;
    a.rope_sin = e->rope_sin;
    a.q_out = e->q_out;
    a.kv_stage = e->kv_stage;
    a.model_dtype = e->act_dtype;
    a.layer = e->layer;
    a.n_layers = e->n_layers;
    if (e->full) {
        a.k_pool = e->full->k_pool;
        a.v_pool = e->full->v_pool;
        a.page_table = e->full->page_table;
        a.page_size = e->full->page_size;
        a.max_pages = e->full->max_pages;
        a.model_dtype = e->full->dtype;
    }
    return a;
}

extern "C" size_t dkv_gemm_work_bytes(int M, int N, int K, int w_dtype) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int mtiles = (M + kTileM - 1) / kTileM;
    const int S = choose_split(mtiles * kTileM, K);
    const int tok = w_dtype == DKV_F32 ? kF32Tok : 64;
    const int nblk = (N + tok - 1) / tok;
    const size_t tile = (size_t)tok * kTileStride * sizeof(float);
    size_t b = kGemmTickets * sizeof(unsigned);
    // bf16: the split-K partials stay in the clusters' shared memory
    if (w_dtype == DKV_F32 && S > 1) b += (size_t)nblk * mtiles * S * tile;
    return b + 256;
}

extern "C" int dkv_pack_weight(const uint16_t* w, int M, int K, uint16_t* tiled, void* stream) {
    DKV_REQUIRE(w && tiled && M > 0 && K > 0, "dkv_pack_weight args");
    DKV_REQUIRE(M % 16 == 0 && K % 16 == 0, "dkv_pack_weight: M, K must be multiples of 16 (M=%d K=%d)", M, K);
    pack_weight_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(w, M, K, tiled);
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" int dkv_gemm(const void* x, int x_dtype, const void* w, int w_dtype, int M, int N, int K,
                        const dkv_epilogue* epi, void* work, size_t work_bytes, void* stream) {
    DKV_REQUIRE(x && w && epi && M > 0 && N >= 0 && K > 0, "dkv_gemm: bad arguments");
    DKV_REQUIRE(x_dtype == w_dtype, "dkv_gemm: x and w dtypes must match");
    DKV_REQUIRE(M % kTileM == 0, "dkv_gemm: M (%d) must be padded to a multiple of 128", M);
    DKV_REQUIRE(K % 16 == 0, "dkv_gemm: K (%d) must be a multiple of 16", K);
    if (N == 0) return DKV_OK;
    const int mtiles = M / kTileM;
    const bool f32 = w_dtype == DKV_F32;
    const int S = f32 ? choose_split(M, K) : choose_split_cl(M, K);
    const int tok = f32 ? kF32Tok : 64;
    const int nblk = (N + tok - 1) / tok;
    DKV_REQUIRE((size_t)nblk * mtiles <= kGemmTickets, "dkv_gemm: too many row tiles x token blocks");
    Arena ar(work, work_bytes);
    GemmArgs g;
    g.x = x;
    g.w = w;
    g.M = M;
    g.N = N;
    g.K = K;
    g.S = S;
    g.tickets = ar.take<unsigned>(kGemmTickets);
    const size_t tile_floats = (size_t)tok * kTileStride;
    // bf16 partials stay in the clusters' shared memory
    g.ws = f32 && S > 1 ? ar.take<float>((size_t)nblk * mtiles * S * tile_floats) : nullptr;
    DKV_REQUIRE(g.tickets && (!f32 || S == 1 || g.ws), "dkv_gemm: work buffer too small (%zu bytes, need %zu)",
                work_bytes, dkv_gemm_work_bytes(M, N, K, w_dtype));
    // columns written: m < min(M, ld_out) (the head is padded to 128 rows;
    // SwiGLU writes d_ff = ld_out columns from 2*d_ff rows)
    int M_real = M;
    if (epi->kind != DKV_EPI_QKV) {
        DKV_REQUIRE(epi->ld_out > 0, "dkv_gemm: ld_out required");
        M_real = std::min(M, epi->ld_out);
    }
    g.epi = make_epi(epi, M_real);
    if (epi->kind == DKV_EPI_QKV) {
        DKV_REQUIRE(epi->q_out && epi->pos0 && epi->d_head > 0 && kTileM % epi->d_head == 0,
                    "dkv_gemm QKV: q_out/pos0 required and d_head must divide 128");
        DKV_REQUIRE(epi->kv_stage || (epi->full && epi->full->k_pool), "dkv_gemm QKV: no K/V destination");
    }
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid(mtiles * S, nblk);
    // algorithmic bytes: the weights once, the activations in and out
    const double elem = w_dtype == DKV_F32 ? 4.0 : 2.0;
    ProfScope ps(DKV_PROF_GEMM, (double)M_real * K * elem + (double)N * K * elem + (double)N * M_real * 4.0, st);
    if (w_dtype == DKV_F32) {
        const size_t smem = std::max((size_t)kF32Tok * kF32Chunk * 4, (size_t)kF32Tok * kTileStride * 4);
        gemm_f32_kernel<<<grid, 256, smem, st>>>(g);
        DKV_LAUNCHED();
        return DKV_OK;
    }
    const int nt = std::min(8, (std::min(N, 64) + 7) / 8);
    g.err = device_error_word();
    // the result tile [NB][kTileStride] reuses the X staging buffers, which
    // are larger, so the bf16 kernel's shared memory is gemm_smem<NT>().
    // Unsplit GEMMs of at most two waves take the plain kernel (one CTA per
    // row tile, the same arithmetic): measured on B200, the clustered kernel
    // streams the 224-tile gate/up projection ~10% slower even when launched
    // without clusters.
#define DKV_GEMM_CASE(NTV)                                                              \
    case NTV: {                                                                         \
        const int act = cl_active<NTV>(S);                                              \
        DKV_REQUIRE(act > 0, "dkv_gemm: no resident cluster of %d CTAs", S);            \
        const int ncl = cl_count(mtiles, act);                                          \
        if (S == 1 && ncl == mtiles) {                                                  \
            DKV_CUDA(allow_smem_max_once<gemm_bf16_kernel<NTV>>());                     \
            DKV_CUDA(launch_pdl(gemm_bf16_kernel<NTV>, grid, dim3(256), gemm_smem<NTV>(), st, g)); \
        } else {                                                                        \
            DKV_CUDA(launch_cl(gemm_bf16_cl_kernel<NTV>, ncl, S, nblk, gemm_smem<NTV>(), st, g)); \
        }                                                                               \
        break;                                                                          \
    }
    switch (nt) {
        DKV_GEMM_CASE(1)
        DKV_GEMM_CASE(2)
        DKV_GEMM_CASE(3)
        DKV_GEMM_CASE(4)
        DKV_GEMM_CASE(5)
        DKV_GEMM_CASE(6)
        DKV_GEMM_CASE(7)
        DKV_GEMM_CASE(8)
        default:
            return DKV_EINVAL;
    }
#undef DKV_GEMM_CASE
    DKV_LAUNCHED();
    return DKV_OK;
}

// ---------------------------------------------------------------------------
// dkv_gemm_noalloc: the same GEMM for callers that cannot allocate.
//
// Some callers cannot hand the library a work buffer: code that runs where
// device allocation is unavailable or forbidden (inside an allocator hook or
// an out-of-memory handler, a host that preallocated its whole HBM pool up
// front, a plugin whose framework owns every allocation).  For them the
// split-K partial tiles and the arrival tickets live in one fixed array
// compiled into this library, so the call needs nothing but its inputs and
// outputs.  The array costs DKV_GEMM_NOALLOC_SCRATCH_BYTES of device memory
// on every GPU that loads the library, held until the process exits.
//
// The first call on a device does that device's set-up (finds the array's
// device address and raises the kernels' shared-memory limit).  Make that
// first call outside any stream capture.  Every call on a device shares the
// one array: two calls whose kernels overlap on the GPU (different streams,
// no ordering between them) race on it and give wrong results; calls on one
// stream, or otherwise ordered, are safe.
#include <mutex>

namespace dkv {
namespace {

constexpr size_t kNoAllocBytes = DKV_GEMM_NOALLOC_SCRATCH_BYTES;
constexpr size_t kNoAllocTicketBytes = 16384;   // 4096 (row tile, token block) tickets
constexpr int kNoAllocMaxDevices = 64;

// In host code this name only stands for the device array; its device
// address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices] = {};

template <int NT>
cudaError_t noalloc_attr() {
    return allow_smem_max(gemm_bf16_kernel<NT>);
}

// Returns the current device's scratch address, doing the set-up on the first
// call for that device.
int noalloc_scratch(unsigned char** out) {
    int dev = 0;
    DKV_CUDA(cudaGetDevice(&dev));
    DKV_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "dkv_gemm_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        DKV_CUDA(cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch));
        DKV_REQUIRE(p && ((uintptr_t)p & 255) == 0, "dkv_gemm_noalloc: scratch array not 256-byte aligned");
        DKV_CUDA(noalloc_attr<1>());
        DKV_CUDA(noalloc_attr<2>());
        DKV_CUDA(noalloc_attr<3>());
        DKV_CUDA(noalloc_attr<4>());
        DKV_CUDA(noalloc_attr<5>());
        DKV_CUDA(noalloc_attr<6>());
        DKV_CUDA(noalloc_attr<7>());
        DKV_CUDA(noalloc_attr<8>());
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return DKV_OK;
}

template <int NT>
void noalloc_launch(const GemmArgs& g, dim3 grid, cudaStream_t st) {
    gemm_bf16_kernel<NT><<<grid, 256, gemm_smem<NT>(), st>>>(g);
}

}  // namespace
}  // namespace dkv

extern "C" int dkv_gemm_noalloc(const void* x, int x_dtype, const void* w, int w_dtype, int M, int N, int K,
                                const dkv_epilogue* epi, void* stream) {
    DKV_REQUIRE(x && w && epi && M > 0 && N >= 0 && K > 0, "dkv_gemm_noalloc: bad arguments");
    DKV_REQUIRE(x_dtype == w_dtype, "dkv_gemm_noalloc: x and w dtypes must match");
    DKV_REQUIRE(w_dtype == DKV_BF16 || w_dtype == DKV_F32, "dkv_gemm_noalloc: dtype must be bf16 or f32");
    DKV_REQUIRE(M % kTileM == 0, "dkv_gemm_noalloc: M (%d) must be padded to a multiple of 128", M);
    DKV_REQUIRE(K % 16 == 0, "dkv_gemm_noalloc: K (%d) must be a multiple of 16", K);
    int M_real = M;
    if (epi->kind != DKV_EPI_QKV) {
        DKV_REQUIRE(epi->ld_out > 0, "dkv_gemm_noalloc: ld_out required");
        M_real = std::min(M, epi->ld_out);
    } else {
        DKV_REQUIRE(epi->q_out && epi->pos0 && epi->d_head > 0 && kTileM % epi->d_head == 0,
                    "dkv_gemm_noalloc QKV: q_out/pos0 required and d_head must divide 128");
        DKV_REQUIRE(epi->kv_stage || (epi->full && epi->full->k_pool), "dkv_gemm_noalloc QKV: no K/V destination");
    }
    if (N == 0) return DKV_OK;
    const int mtiles = M / kTileM;
    // the same K split as dkv_gemm, so both sum the same partials in the same
    // order and give bit-identical results
    const int S = w_dtype == DKV_F32 ? choose_split(M, K) : choose_split_cl(M, K);
    const int tok = w_dtype == DKV_F32 ? kF32Tok : 64;
    const int nblk = (N + tok - 1) / tok;
    const size_t tickets = (size_t)nblk * mtiles;
    const size_t partial_bytes = S > 1 ? tickets * S * tok * kTileStride * sizeof(float) : 0;
    // an unsplit launch touches neither the tickets nor the partials
    DKV_REQUIRE(S == 1 || tickets * sizeof(unsigned) <= kNoAllocTicketBytes,
                "dkv_gemm_noalloc: %zu row tiles x token blocks exceed the %zu tickets of the fixed scratch "
                "(use dkv_gemm with a work buffer)", tickets, kNoAllocTicketBytes / sizeof(unsigned));
    DKV_REQUIRE(partial_bytes <= kNoAllocBytes - kNoAllocTicketBytes,
                "dkv_gemm_noalloc: M=%d N=%d K=%d needs %zu bytes of split-K scratch, the fixed array holds %zu "
                "(use dkv_gemm with a work buffer)", M, N, K, partial_bytes, kNoAllocBytes - kNoAllocTicketBytes);
    unsigned char* scratch = nullptr;
    DKV_TRY(noalloc_scratch(&scratch));
    cudaStream_t st = (cudaStream_t)stream;
    // The array keeps whatever the previous call left; the tickets must start
    // at zero (a launch that stopped early can leave one raised).
    if (S > 1) DKV_CUDA(cudaMemsetAsync(scratch, 0, tickets * sizeof(unsigned), st));
    GemmArgs g;
    g.x = x;
    g.w = w;
    g.M = M;
    g.N = N;
    g.K = K;
    g.S = S;
    g.tickets = reinterpret_cast<unsigned*>(scratch);
    g.ws = S > 1 ? reinterpret_cast<float*>(scratch + kNoAllocTicketBytes) : nullptr;
    g.epi = make_epi(epi, M_real);
    dim3 grid(mtiles * S, nblk);
    if (w_dtype == DKV_F32) {
        const size_t smem = std::max((size_t)kF32Tok * kF32Chunk * 4, (size_t)kF32Tok * kTileStride * 4);
        gemm_f32_kernel<<<grid, 256, smem, st>>>(g);
        DKV_LAUNCHED();
        return DKV_OK;
    }
    g.err = device_error_word();
    DKV_REQUIRE(g.err, "dkv_gemm_noalloc: device error word unavailable");
    switch (std::min(8, (std::min(N, 64) + 7) / 8)) {
        case 1: noalloc_launch<1>(g, grid, st); break;
        case 2: noalloc_launch<2>(g, grid, st); break;
        case 3: noalloc_launch<3>(g, grid, st); break;
        case 4: noalloc_launch<4>(g, grid, st); break;
        case 5: noalloc_launch<5>(g, grid, st); break;
        case 6: noalloc_launch<6>(g, grid, st); break;
        case 7: noalloc_launch<7>(g, grid, st); break;
        default: noalloc_launch<8>(g, grid, st); break;
    }
    DKV_LAUNCHED();
    return DKV_OK;
}
