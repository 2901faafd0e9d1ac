// Shared by the weight-streaming GEMM kernels: the epilogue arguments and the
// fused epilogues (K4e) applied to a finished [token][row] result tile.
//
// Replaces the elementwise tails of the projections in draftkv/llama.py:
// 187-225 (RoPE :197-198 with _rope :164-172, SwiGLU :222, residual adds)
// and draftkv/gpt2.py:191-213 (Conv1D bias, gelu_new :126-127).
#pragma once

#include "common.cuh"

namespace dkv {

constexpr int kTileM = 128;       // weight rows per CTA
constexpr int kTileStride = 132;  // smem row stride (floats) of the result tile [n][m]

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
    // fused RMSNorm (tensor-core kernel only): the input side scales token
    // n's accumulators by 1 / sqrt(sum_t norm_in_part[t][n] / norm_dm + eps);
    // the output side (RESADD) also writes bf16(h_new * norm_out_w) and the
    // per-128-row sums of h_new^2
    const float* norm_in_part;
    int norm_n_part, norm_ld, norm_dm;
    float norm_eps;
    float* norm_out_part;
    void* norm_out_x;
    const float* norm_out_w;
};

DKV_DEV float gelu_new(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))  (gpt2.py:126-127)
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

DKV_DEV float silu(float x) { return x / (1.0f + expf(-x)); }

constexpr int kEpiU = 8;    // token rows a thread keeps in flight in the epilogue

// Applies the epilogue to the tile T[n][m] (n < nb valid tokens starting at
// n0), token rows [j0, j1) of it (all rows when j1 < 0).  Thread t owns row
// t % 128 of the tile and every (blockDim.x / 128)-th token row from
// t / 128; each pass reads kEpiU token rows of the tile before it writes,
// so the global loads and stores of a pass are in flight together.
// `inv` (shared memory, indexed by token row, or null) scales the
// accumulators (the input side of a fused RMSNorm).  With e.norm_out_x a
// RESADD also writes bf16(h_new * norm_out_w) and leaves h_new^2 (0 past
// M_real) in T for epi_norm_partials.
DKV_DEV void run_epilogue(const EpiArgs& e, float* T, int mtile, int n0, int nb, int j0 = 0, int j1 = -1,
                          const float* inv = nullptr, int tid = -1, int nthr = -1) {
    const int m0 = mtile * kTileM;
    if (j1 < 0) j1 = nb;
    if (tid < 0) {      // all threads of the CTA take part (else threads tid < nthr do)
        tid = threadIdx.x;
        nthr = blockDim.x;
    }
    const int i = tid & (kTileM - 1), jstep = nthr / kTileM;
    const int m = m0 + i;
    const bool col_ok = m < e.M_real;
    // the bias of this row (rows past the written columns have none; QKV and
    // SwiGLU rows are checked in their cases)
    const float bm = (e.bias && col_ok && e.kind != DKV_EPI_QKV && e.kind != DKV_EPI_SWIGLU) ? e.bias[m] : 0.f;
    for (int jb = j0 + tid / kTileM; jb < j1; jb += kEpiU * jstep) {
        float acc[kEpiU];
#pragma unroll
        for (int u = 0; u < kEpiU; ++u) {
            const int j = jb + u * jstep;
            acc[u] = j < j1 ? T[j * kTileStride + i] * (inv ? inv[j] : 1.f) : 0.f;
        }
        switch (e.kind) {
            case DKV_EPI_STORE:
#pragma unroll
                for (int u = 0; u < kEpiU; ++u) {
                    const int j = jb + u * jstep;
                    if (j < j1 && col_ok) e.out_f32[(size_t)(n0 + j) * e.ld_out + m] = acc[u] + bm;
                }
                break;
            case DKV_EPI_RESADD: {
                float hv[kEpiU];
#pragma unroll
                for (int u = 0; u < kEpiU; ++u) {
                    const int j = jb + u * jstep;
                    hv[u] = (j < j1 && col_ok) ? e.out_f32[(size_t)(n0 + j) * e.ld_out + m] : 0.f;
                }
                const float wn = (e.norm_out_x && col_ok) ? e.norm_out_w[m] : 0.f;
#pragma unroll
                for (int u = 0; u < kEpiU; ++u) {
                    const int j = jb + u * jstep;
                    if (j >= j1) continue;
                    const float nh = hv[u] + (acc[u] + bm);
                    if (col_ok) e.out_f32[(size_t)(n0 + j) * e.ld_out + m] = nh;
                    if (e.norm_out_x) {
                        if (col_ok) store_from_f32(e.norm_out_x, DKV_BF16, (size_t)(n0 + j) * e.ld_out + m, nh * wn);
                        T[j * kTileStride + i] = col_ok ? nh * nh : 0.f;
                    }
                }
                break;
            }
            case DKV_EPI_GELU:
#pragma unroll
                for (int u = 0; u < kEpiU; ++u) {
                    const int j = jb + u * jstep;
                    if (j < j1 && col_ok)
                        store_from_f32(e.act, e.act_dtype, (size_t)(n0 + j) * e.ld_out + m, gelu_new(acc[u] + bm));
                }
                break;
            case DKV_EPI_SWIGLU:
                if (i < 64 && mtile * 64 + i < e.M_real) {
                    // rows m (gate) and m + 64 (up) make column mtile * 64 + i
                    const int col = mtile * 64 + i;
                    const float bg = e.bias ? e.bias[m] : 0.f;
                    const float bu = e.bias ? e.bias[m + 64] : 0.f;
#pragma unroll
                    for (int u = 0; u < kEpiU; ++u) {
                        const int j = jb + u * jstep;
                        if (j >= j1) continue;
                        const float g = acc[u] + bg;
                        const float up = T[j * kTileStride + i + 64] * (inv ? inv[j] : 1.f) + bu;
                        store_from_f32(e.act, e.act_dtype, (size_t)(n0 + j) * e.ld_out + col, silu(g) * up);
                    }
                }
                break;
            case DKV_EPI_QKV: {
                const int D = e.d_head, HD = e.n_heads * D, KD = e.n_kv * D;
                if (m >= HD + 2 * KD) break;
                const int sec = m < HD ? 0 : (m < HD + KD ? 1 : 2);
                const int mm = sec == 0 ? m : (sec == 1 ? m - HD : m - HD - KD);
                const int head = mm / D, dd = mm % D;
                const int hd = D / 2;
                const int pair = dd < hd ? i + hd : i - hd;
                const float bp = e.bias ? e.bias[m0 + pair] : 0.f;
                const int f = dd < hd ? dd : dd - hd;
                const float bq = e.bias ? e.bias[m] : 0.f;
#pragma unroll
                for (int u = 0; u < kEpiU; ++u) {
                    const int j = jb + u * jstep;
                    if (j >= j1) continue;
                    const int n = n0 + j;
                    const int b = n / e.tokens_per_seq, t = n % e.tokens_per_seq;
                    const int p = e.pos0[b] + t;
                    float val = acc[u] + bq;
                    if (sec < 2 && e.rope_cos) {
                        const float other = T[j * kTileStride + pair] * (inv ? inv[j] : 1.f) + bp;
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
                        const int page =
                            e.page_table[((size_t)b * e.n_layers + e.layer) * e.max_pages + p / e.page_size];
                        const size_t o = (((size_t)page * e.n_kv + head) * e.page_size + (p % e.page_size)) * D + dd;
                        store_from_f32(sec == 1 ? e.k_pool : e.v_pool, e.model_dtype, o, val);
                    }
                }
                break;
            }
            default:
                break;
        }
    }
}

// Input side of a fused RMSNorm: inv[j] for token rows j0 <= j < j1 of the
// tile, summing the partials in part order (thread tid takes rows j0 + tid,
// j0 + tid + nthr, ...: a 256-token tile has two rows a thread; the caller
// syncs).
DKV_DEV void epi_token_inv(const EpiArgs& e, int n0, int j0, int j1, float* inv, int tid = -1, int nthr = -1) {
    if (tid < 0) {
        tid = threadIdx.x;
        nthr = blockDim.x;
    }
    for (int j = j0 + tid; j < j1; j += nthr) {
        const float* p = e.norm_in_part + n0 + j;
        float s = 0.f;
        int t = 0;
        for (; t + 4 <= e.norm_n_part; t += 4) {
            const float a = p[(size_t)t * e.norm_ld], b = p[(size_t)(t + 1) * e.norm_ld];
            const float c = p[(size_t)(t + 2) * e.norm_ld], d = p[(size_t)(t + 3) * e.norm_ld];
            s = (((s + a) + b) + c) + d;
        }
        for (; t < e.norm_n_part; ++t) s += p[(size_t)t * e.norm_ld];
        inv[j] = 1.0f / sqrtf(s / (float)e.norm_dm + e.norm_eps);
    }
}

// Output side: after run_epilogue left h_new^2 in T and the CTA synced, the
// sum over the tile's 128 rows for token rows [j0, j1) goes to
// norm_out_part[mtile][n] (4 rows a lane in row order, then a butterfly:
// the same order for every token and launch).
DKV_DEV void epi_norm_partials(const EpiArgs& e, const float* T, int mtile, int n0, int j0, int j1, int tid = -1,
                               int nthr = -1) {
    if (tid < 0) {
        tid = threadIdx.x;
        nthr = blockDim.x;
    }
    const int warp = tid >> 5, lane = tid & 31, nw = nthr >> 5;
    for (int j = j0 + warp; j < j1; j += nw) {
        const float* r = T + j * kTileStride;
        float v = ((r[lane] + r[lane + 32]) + r[lane + 64]) + r[lane + 96];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) e.norm_out_part[(size_t)mtile * e.norm_ld + n0 + j] = v;
    }
}

// Host: kernel epilogue arguments from the C-ABI description.
EpiArgs make_epi(const dkv_epilogue* e, int M_real);

}  // namespace dkv
