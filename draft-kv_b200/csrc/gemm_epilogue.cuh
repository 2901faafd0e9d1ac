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

// Host: kernel epilogue arguments from the C-ABI description.
EpiArgs make_epi(const dkv_epilogue* e, int M_real);

}  // namespace dkv
