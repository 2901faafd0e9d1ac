// Whole-decoder forward pass: the native runtime loop over layers.
//
// Replaces draftkv/llama.py:175-225 (LlamaLike.forward) and
// draftkv/gpt2.py:182-213 (GPT2.forward).  The layer loop runs here, in C++,
// so one call launches every kernel of a forward and the sequence can be
// captured into one CUDA graph per (shape, config).
#include <algorithm>

#include "attn_common.cuh"

namespace dkv {
size_t forward_work(const dkv_model* m, int batch, int T, int max_ctx, int comp_cap, size_t* attn_bytes,
                    size_t* gemm_bytes);
int norm_prep(const float* h, int N, int dm, const float* w, void* x, float* part, int ld, cudaStream_t st);
int gemm_entry(const void* x, int x_dtype, const void* w, int w_dtype, int M, int N, int K, const dkv_epilogue* epi,
               void* work, size_t work_bytes, void* stream, bool fill);

// RMSNorm fused into the GEMMs (bf16 Llama-family models): the norm before
// the QKV, gate/up and head projections costs no launch of its own.
bool fused_norm(const dkv_model* m) {
    return m->arch == DKV_ARCH_LLAMA && m->dtype == DKV_BF16 && m->d_model % 128 == 0;
}
}

using namespace dkv;

static int round128(int x) { return (x + 127) / 128 * 128; }

size_t dkv::forward_work(const dkv_model* m, int batch, int T, int max_ctx, int comp_cap, size_t* attn_bytes,
                         size_t* gemm_bytes) {
    const int N = batch * T;
    const int elem = m->dtype == DKV_F32 ? 4 : 2;
    const int HD = m->n_heads * m->d_head, KD = m->n_kv * m->d_head;
    const int dff_act = m->d_ff;
    size_t g = 0;
    g = std::max(g, dkv_gemm_work_bytes(round128(HD + 2 * KD), N, m->d_model, m->dtype));
    g = std::max(g, dkv_gemm_work_bytes(round128(m->d_model), N, HD, m->dtype));
    g = std::max(g, dkv_gemm_work_bytes(round128(m->arch == DKV_ARCH_LLAMA ? 2 * m->d_ff : m->d_ff), N, m->d_model,
                                        m->dtype));
    g = std::max(g, dkv_gemm_work_bytes(round128(m->d_model), N, m->d_ff, m->dtype));
    g = std::max(g, dkv_gemm_work_bytes(m->vocab_pad, N, m->d_model, m->dtype));
    dkv_dims dims{m->n_layers, m->n_kv, m->d_head, batch};
    // attention scratch: up to 64 query rows (decode, verify) at the model's
    // split; more rows (prompt chunks) in bf16 take splits of at least
    // kPromptMinSplit keys, far fewer partials
    const int G = m->n_heads / m->n_kv;
    const int sk = m->split_keys > 0 ? m->split_keys : 512;
    size_t a = dkv_attn_work_bytes(dims, G, std::min(T, std::max(1, 64 / G)), max_ctx, sk, comp_cap);
    if (T * G > 64) {
        const int sk_rows = m->dtype == DKV_BF16 ? std::max(kPromptMinSplit, (sk + 127) / 128 * 128) : sk;
        a = std::max(a, dkv_attn_work_bytes(dims, G, T, max_ctx, sk_rows, comp_cap));
    }
    if (attn_bytes) *attn_bytes = a;
    if (gemm_bytes) *gemm_bytes = g;
    size_t b = 0;
    b += align_up((size_t)N * m->d_model * 4, 256);                  // h
    b += align_up((size_t)N * std::max(m->d_model, HD) * elem, 256);  // x / attn out
    b += align_up((size_t)N * dff_act * elem, 256);                  // act
    b += align_up((size_t)N * HD * 4, 256);                          // q
    b += align_up((size_t)N * KD * 2 * elem, 256);                   // kv stage
    if (fused_norm(m)) {
        b += align_up((size_t)N * m->d_model * 2, 256);              // bf16(h * w) of the next norm
        b += align_up((size_t)(m->d_model / 128) * N * 4, 256);      // its per-row-tile sums of squares
    }
    return b + align_up(g, 256) + align_up(a, 256) + 4096;
}

extern "C" size_t dkv_forward_work_bytes(const dkv_model* m, int batch, int T, int max_ctx, int comp_cap) {
    if (!m) return 0;
    return forward_work(m, batch, T, max_ctx, comp_cap, nullptr, nullptr);
}

extern "C" int dkv_forward(const dkv_model* m, const dkv_full_cache* full, const dkv_comp_cache* comp,
                           const dkv_step* st, void* stream) {
    DKV_REQUIRE(m && st && m->layers && st->tokens && st->pos0, "dkv_forward: bad arguments");
    DKV_REQUIRE(comp || (full && full->k_pool && full->page_table),
                "dkv_forward: a full-cache forward needs the full cache");
    DKV_REQUIRE(m->n_heads % m->n_kv == 0, "dkv_forward: n_heads %% n_kv != 0");
    DKV_REQUIRE(!comp || st->T == 1, "dkv_forward: draft steps have T == 1");
    DKV_REQUIRE(st->max_T >= st->T && st->T >= 0, "dkv_forward: T %d > max_T %d", st->T, st->max_T);
    DKV_REQUIRE(!full || m->dtype == full->dtype, "dkv_forward: model and cache dtypes differ");
    const int N = st->batch * st->T;
    if (N == 0) return DKV_OK;
    const int dm = m->d_model, D = m->d_head, H = m->n_heads, KV = m->n_kv;
    const int HD = H * D, KD = KV * D;
    const int elem = m->dtype == DKV_F32 ? 4 : 2;
    const bool llama = m->arch == DKV_ARCH_LLAMA;
    size_t attn_bytes = 0, gemm_bytes = 0;
    // the arena layout depends on (batch, max_T, max_ctx, cap) only, so the
    // ticket regions stay at fixed offsets across calls with different T
    const size_t need = forward_work(m, st->batch, st->max_T, st->max_ctx, comp ? comp->cap : 0, &attn_bytes,
                                     &gemm_bytes);
    DKV_REQUIRE(st->work && st->work_bytes >= need, "dkv_forward: work buffer %zu < %zu bytes", st->work_bytes, need);
    const size_t NM = (size_t)st->batch * st->max_T;
    Arena ar(st->work, st->work_bytes);
    uint8_t* gwork = ar.take<uint8_t>(gemm_bytes);
    uint8_t* awork = ar.take<uint8_t>(attn_bytes);
    float* h = ar.take<float>(NM * dm);
    uint8_t* x = ar.take<uint8_t>(NM * std::max(dm, HD) * elem);
    uint8_t* act = ar.take<uint8_t>(NM * m->d_ff * elem);
    float* q = ar.take<float>(NM * HD);
    uint8_t* stage = ar.take<uint8_t>(NM * KD * 2 * elem);
    DKV_REQUIRE(h && x && act && q && stage && gwork && awork, "dkv_forward: arena");
    dkv_dims dims{m->n_layers, KV, D, st->batch};
    const int group = H / KV;
    // fused RMSNorm: xn = bf16(h * w) of the next norm and its partial sums
    // of squares, written by the previous residual GEMM (by norm_prep for
    // the first layer) and divided out by the GEMM that reads xn
    const bool fused = fused_norm(m);
    uint8_t* xn = fused ? ar.take<uint8_t>(NM * dm * 2) : nullptr;
    float* npart = fused ? ar.take<float>((size_t)(dm / 128) * NM) : nullptr;
    DKV_REQUIRE(!fused || (xn && npart), "dkv_forward: arena");
    auto norm_in = [&](dkv_epilogue& e) {
        if (!fused) return;
        e.norm_in_part = npart;
        e.norm_n_part = dm / 128;
        e.norm_ld = (int)NM;
        e.norm_dm = dm;
        e.norm_eps = m->eps;
    };
    auto norm_out = [&](dkv_epilogue& e, const float* w_next) {
        if (!fused) return;
        e.norm_out_part = npart;
        e.norm_out_x = xn;
        e.norm_out_w = w_next;
        e.norm_ld = (int)NM;
    };
    const uint8_t* xin = fused ? xn : x;    // what the normed projections read

    const int M_qkv = round128(HD + 2 * KD), M_up = round128(llama ? 2 * m->d_ff : m->d_ff);

    auto qkv_epi = [&](int L) {
        const dkv_layer& ly = m->layers[L];
        dkv_epilogue e{};
        e.kind = DKV_EPI_QKV;
        e.bias = ly.b_qkv;
        e.act_dtype = m->dtype;
        e.n_heads = H;
        e.n_kv = KV;
        e.d_head = D;
        e.tokens_per_seq = st->T;
        e.pos0 = st->pos0;
        e.rope_cos = llama ? m->rope_cos : nullptr;
        e.rope_sin = llama ? m->rope_sin : nullptr;
        e.q_out = q;
        e.kv_stage = comp ? stage : nullptr;
        e.full = full;
        e.layer = L;
        e.n_layers = m->n_layers;
        norm_in(e);
        return e;
    };
    auto o_epi = [&](int L) {
        dkv_epilogue e{};
        e.kind = DKV_EPI_RESADD;
        e.bias = m->layers[L].b_o;
        e.out_f32 = h;
        e.ld_out = dm;
        e.act_dtype = m->dtype;
        norm_out(e, m->layers[L].n2_w);
        return e;
    };
    auto up_epi = [&](int L) {
        dkv_epilogue e{};
        e.kind = llama ? DKV_EPI_SWIGLU : DKV_EPI_GELU;
        e.bias = m->layers[L].b_up;
        e.act = act;
        e.act_dtype = m->dtype;
        e.ld_out = m->d_ff;
        norm_in(e);
        return e;
    };
    auto down_epi = [&](int L) {
        dkv_epilogue e{};
        e.kind = DKV_EPI_RESADD;
        e.bias = m->layers[L].b_down;
        e.out_f32 = h;
        e.ld_out = dm;
        e.act_dtype = m->dtype;
        norm_out(e, L + 1 < m->n_layers ? m->layers[L + 1].n1_w : m->nf_w);
        return e;
    };
    auto head_epi = [&]() {
        dkv_epilogue e{};
        e.kind = DKV_EPI_STORE;
        e.out_f32 = st->logits;
        e.ld_out = m->vocab;
        e.act_dtype = m->dtype;
        norm_in(e);
        return e;
    };

    // the prompt forward (no logits): its rows feed only the cache, so each
    // projection takes the K split that fills the GPU for this many tokens
    const bool prompt = st->logits == nullptr;
    auto gemm = [&](const void* xa, const void* w, int M, int K, const dkv_epilogue* e) {
        return dkv::gemm_entry(xa, m->dtype, w, m->dtype, M, N, K, e, gwork, gemm_bytes, stream, prompt);
    };
    DKV_TRY(dkv_embed(m->tok_emb, m->dtype, m->pos_emb, st->tokens, st->tok_stride, st->batch, st->T, st->pos0, dm,
                      m->vocab, m->max_pos, h, stream));
    if (fused) DKV_TRY(norm_prep(h, N, dm, m->layers[0].n1_w, xn, npart, (int)NM, (cudaStream_t)stream));
    for (int L = 0; L < m->n_layers; ++L) {
        const dkv_layer& ly = m->layers[L];
        if (!fused) DKV_TRY(dkv_norm(h, N, dm, llama ? 0 : 1, ly.n1_w, ly.n1_b, m->eps, x, m->dtype, stream));
        const dkv_epilogue e = qkv_epi(L);
        DKV_TRY(gemm(xin, ly.w_qkv, M_qkv, dm, &e));
        if (comp) {
            DKV_TRY(dkv_comp_append(comp, full, dims, L, 1, stage, m->dtype, 1, st->pos0, nullptr, nullptr, L == 0 ? 1 : 0,
                                    stream));
            DKV_TRY(dkv_attn_comp(comp, dims, L, group, q, st->pos0, x, m->dtype, awork, attn_bytes, stream));
        } else {
            DKV_TRY(dkv_attn_full(full, dims, L, group, st->T, q, st->pos0, x, m->dtype, m->split_keys, awork,
                                  attn_bytes, stream));
        }
        const dkv_epilogue eo = o_epi(L);
        DKV_TRY(gemm(x, ly.w_o, round128(dm), HD, &eo));
        if (!fused) DKV_TRY(dkv_norm(h, N, dm, llama ? 0 : 1, ly.n2_w, ly.n2_b, m->eps, x, m->dtype, stream));
        const dkv_epilogue eu = up_epi(L);
        DKV_TRY(gemm(xin, ly.w_up, M_up, dm, &eu));
        const dkv_epilogue ed = down_epi(L);
        DKV_TRY(gemm(act, ly.w_down, round128(dm), m->d_ff, &ed));
    }
    if (!st->logits) return DKV_OK;        // prefill: the cache is written, no logits wanted
    if (!fused) DKV_TRY(dkv_norm(h, N, dm, llama ? 0 : 1, m->nf_w, m->nf_b, m->eps, x, m->dtype, stream));
    const dkv_epilogue eh = head_epi();
    DKV_TRY(dkv_gemm(xin, m->dtype, m->w_head, m->dtype, m->vocab_pad, N, dm, &eh, gwork, gemm_bytes, stream));
    return DKV_OK;
}
