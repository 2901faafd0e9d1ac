// Attention over the full (verify / baseline) and the drafter cache.
//
// Replaces, per layer, draftkv/llama.py:202-219 and draftkv/gpt2.py:197-207:
// the query is appended before attention (a token attends to itself), keys
// with position > query position are masked, softmax(q k^T / sqrt(d)) v, GQA
// by sharing each KV head across its query group.  On the drafter cache it
// also produces the attention mass of draftkv/compress.py:144-151
// (note_attention), summed over the GQA group (draftkv/llama.py:213-216) and
// folded into the slot scores in a fixed order.
//
// This file holds the generic CUDA-core kernel (fp32 math, any key source);
// it serves fp32 models and shapes the tensor-core kernels do not cover.
#include "common.cuh"

#include "attn_common.cuh"

namespace dkv {

DKV_DEV float deq_code(const uint8_t* codes, const uint16_t* sl, int d, int bits, bool k_order, int e, int raw) {
    int p = e;
    if (k_order) {
        const int q4 = d >> 2;
        const int j = e >> 4, w = e & 15;
        const int c = (w & 7) >> 1;
        const int r = (w & 1) | ((w >> 3) << 1);
        p = c * q4 + 4 * j + r;
    }
    if (bits == 16) return load_as_f32(codes, raw, p);
    uint32_t qv;
    if (bits == 8) {
        qv = codes[p];
    } else if (bits == 4 || bits == 2) {
        const int per = 32 / bits;
        const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[p / per];
        const int i = (p % per) >> 1;
        qv = (w >> ((p & 1) ? 16 + bits * i : bits * i)) & ((1u << bits) - 1);
    } else {
        const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[p / 16];
        const int i = (p % 16) >> 1;
        const uint32_t lo2 = (w >> ((p & 1) ? 16 + 2 * i : 2 * i)) & 3u;
        const uint16_t u = reinterpret_cast<const uint16_t*>(codes + d / 4)[p / 16];
        qv = lo2 | (((u >> ((p & 1) ? 8 + i : i)) & 1u) << 2);
    }
    const int g = e >> 6;
    return (float)qv * half_bits_to_f32(sl[2 * g]) + half_bits_to_f32(sl[2 * g + 1]);
}

constexpr int kGenKT = 32;     // keys per tile
constexpr int kGenThreads = 128;
constexpr int kGenRB = kAttnRB;   // query rows per CTA

// smem: Q[R][d] | K[KT][d+1] | V[KT][d+1] | P[R][KT] | m[R] l[R] a[R] | O[R][d] | kp[KT]
// Rows (query token x group head) are processed in blocks of at most kGenRB
// per CTA (grid z = batch x row blocks); a row's result does not depend on
// which block it lands in.
__global__ void __launch_bounds__(kGenThreads) attn_generic_kernel(AttnArgs a) {
    extern __shared__ float sm[];
    const int s = blockIdx.x, h = blockIdx.y;
    const int b = blockIdx.z / a.n_rb, rb = blockIdx.z % a.n_rb;
    const int d = a.d, G = a.group, T = a.T;
    const int r0 = rb * kGenRB;
    const int R = min(kGenRB, T * G - r0);   // rows of this CTA; row r is global row r0 + r
    const KeySrc& src = a.src;
    float* Qs = sm;
    float* Ks = Qs + R * d;
    float* Vs = Ks + kGenKT * (d + 1);
    float* Ps = Vs + kGenKT * (d + 1);
    float* ms = Ps + R * kGenKT;
    float* ls = ms + R;
    float* as = ls + R;
    float* Os = as + R;
    int* kp = reinterpret_cast<int*>(Os + R * d);

    const int qbase = a.qpos0[b];
    int n_keys;
    size_t bl = (size_t)b * a.n_layers + a.layer;
    if (src.comp) n_keys = src.meta[bl * 4 + 0];
    else n_keys = qbase + T;
    const int k0 = s * a.split;
    const int k1 = min(n_keys, k0 + a.split);
    const int HQ = a.n_kv * G;

    for (int i = threadIdx.x; i < R * d; i += blockDim.x) {
        const int r = i / d, e = i % d;
        const int t = (r0 + r) / G, g = (r0 + r) % G;
        Qs[i] = a.q[(((size_t)b * T + t) * HQ + h * G + g) * d + e];
        Os[i] = 0.f;
    }
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        ms[r] = -INFINITY;
        ls[r] = 0.f;
    }
    __syncthreads();

    for (int kt = k0; kt < k1; kt += kGenKT) {
        const int nk = min(kGenKT, k1 - kt);
        // keys / values of this tile, dequantized to fp32
        for (int i = threadIdx.x; i < kGenKT * d; i += blockDim.x) {
            const int j = i / d, e = i % d;
            float kvv = 0.f, vvv = 0.f;
            if (j < nk) {
                const int key = kt + j;
                if (src.comp) {
                    if (src.cpos[bl * src.cap + key] >= 0) {
                        const size_t vh = (bl * a.n_kv + h) * (size_t)src.cap;
                        const size_t vi = vh + key;
                        const int raw = src.cb_max >= d * 4 ? DKV_F32 : DKV_BF16;
                        const size_t co = vh * src.cb_max + (size_t)key * code_row_bytes(d, src.bits, raw);
                        kvv = deq_code(src.k_codes + co, src.k_sl + vi * (d / 64) * 2, d, src.bits, true, e, raw);
                        vvv = deq_code(src.v_codes + co, src.v_sl + vi * (d / 64) * 2, d, src.bits, false, e, raw);
                    }
                } else {
                    const int page = src.page_table[bl * src.max_pages + key / src.page_size];
                    const size_t o = (((size_t)page * a.n_kv + h) * src.page_size + key % src.page_size) * d + e;
                    kvv = load_as_f32(src.k_pool, src.dtype, o);
                    vvv = load_as_f32(src.v_pool, src.dtype, o);
                }
            }
            Ks[j * (d + 1) + e] = kvv;
            Vs[j * (d + 1) + e] = vvv;
        }
        for (int j = threadIdx.x; j < kGenKT; j += blockDim.x) {
            int p = -1;
            if (j < nk) p = src.comp ? src.cpos[bl * src.cap + kt + j] : kt + j;
            kp[j] = p;
        }
        __syncthreads();
        // scores
        for (int i = threadIdx.x; i < R * kGenKT; i += blockDim.x) {
            const int r = i / kGenKT, j = i % kGenKT;
            const int qp = qbase + (r0 + r) / G;
            float sc = -INFINITY;
            if (kp[j] >= 0 && kp[j] <= qp) {
                float acc = 0.f;
                const float* qr = Qs + r * d;
                const float* kr = Ks + j * (d + 1);
                for (int e = 0; e < d; ++e) acc = fmaf(qr[e], kr[e], acc);
                sc = acc * a.scale;
            }
            Ps[i] = sc;
            if (a.sbuf && j < nk)
                a.sbuf[(((size_t)b * a.n_kv + h) * G + ((r0 + r) % G)) * src.cap + kt + j] = sc;
        }
        __syncthreads();
        // online softmax per row (sequential over the tile: order fixed)
        for (int r = threadIdx.x; r < R; r += blockDim.x) {
            float mx = ms[r];
            for (int j = 0; j < kGenKT; ++j) mx = fmaxf(mx, Ps[r * kGenKT + j]);
            const float alpha = (mx == -INFINITY) ? 1.f : expf(ms[r] - mx);
            float sum = 0.f;
            for (int j = 0; j < kGenKT; ++j) {
                const float sc = Ps[r * kGenKT + j];
                const float p = sc == -INFINITY ? 0.f : expf(sc - mx);
                Ps[r * kGenKT + j] = p;
                sum += p;
            }
            ls[r] = ls[r] * alpha + sum;
            ms[r] = mx;
            as[r] = alpha;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < R * d; i += blockDim.x) {
            const int r = i / d, e = i % d;
            float acc = Os[i] * as[r];
            for (int j = 0; j < kGenKT; ++j) acc = fmaf(Ps[r * kGenKT + j], Vs[j * (d + 1) + e], acc);
            Os[i] = acc;
        }
        __syncthreads();
    }

    // ---- partials, then the last split of (b, h) merges in split order
    const int PS = d + 2;
    const size_t bhr = ((size_t)b * a.n_kv + h) * a.n_rb + rb;     // (sequence, head, row block)
    float* mypart = a.part + ((bhr * a.n_splits + s) * kGenRB) * PS;
    for (int i = threadIdx.x; i < R * d; i += blockDim.x) mypart[(i / d) * PS + 2 + (i % d)] = Os[i];
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
        mypart[r * PS + 0] = ms[r];
        mypart[r * PS + 1] = ls[r];
    }
    if (!split_merge(a, bhr, b, h, R, r0, ms, ls)) return;
    if (!a.sbuf) return;
    // ---- drafter: attention mass per slot for this head (sum over the group)
    __shared__ int is_last;
    float* mass_h = a.mass + (bl * a.n_kv + h) * (size_t)src.cap;
    for (int slot = threadIdx.x; slot < n_keys; slot += blockDim.x) {
        float mval = 0.f;
        for (int g = 0; g < G; ++g) {
            const float sc = __ldcg(a.sbuf + (((size_t)b * a.n_kv + h) * G + g) * src.cap + slot);
            if (sc != -INFINITY && ls[g] > 0.f) mval += expf(sc - ms[g]) / ls[g];
        }
        mass_h[slot] = mval;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* tk = a.fold_tickets + b;
        const unsigned prev = atomicAdd(tk, 1u);
        is_last = prev == (unsigned)(a.n_kv - 1);
        if (is_last) *tk = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float* sc_row = a.score + bl * src.cap;
    const float* mass_l = a.mass + bl * a.n_kv * (size_t)src.cap;
    for (int slot = threadIdx.x; slot < n_keys; slot += blockDim.x) {
        if (src.cpos[bl * src.cap + slot] < 0) continue;
        float add = 0.f;
        for (int hh = 0; hh < a.n_kv; ++hh) add += __ldcg(mass_l + (size_t)hh * src.cap + slot);
        sc_row[slot] += add;
    }
}

size_t generic_smem(int R, int d) {
    return sizeof(float) * ((size_t)R * d * 2 + 2 * kGenKT * (d + 1) + (size_t)R * kGenKT + 3 * R) + kGenKT * 4 + 64;
}

KeySrc full_src(const dkv_full_cache* f) {
    KeySrc k{};
    k.k_pool = f->k_pool;
    k.v_pool = f->v_pool;
    k.page_table = f->page_table;
    k.page_size = f->page_size;
    k.page_shift = -1;
    for (int sh = 0; sh < 31; ++sh)
        if ((1 << sh) == f->page_size) k.page_shift = sh;
    k.max_pages = f->max_pages;
    k.n_pages = f->n_pages;
    k.dtype = f->dtype;
    k.comp = false;
    return k;
}

KeySrc comp_src(const dkv_comp_cache* c, int layer) {
    KeySrc k{};
    k.k_codes = c->k_codes;
    k.v_codes = c->v_codes;
    k.k_sl = c->k_sl;
    k.v_sl = c->v_sl;
    k.cpos = c->pos;
    k.meta = c->meta;
    k.cap = c->cap;
    k.cb_max = c->cb_max;
    k.bits = c->bits[layer];
    k.comp = true;
    return k;
}

}  // namespace dkv

using namespace dkv;

// Tickets (split merge per (b, head), head fold per b) sit at a fixed region
// at the start of every attention work buffer; launches reset what they use.
constexpr size_t kAttnTickets = 16384;

static size_t attn_scratch(int batch, int n_kv, int n_splits, int R, int d, int cap, int group, bool comp) {
    // row blocks: up to 64 rows the tensor-core kernel takes 16 rows a CTA
    // (each block keeps a 64-row partial stride); beyond that the prefill
    // kernel takes 256 rows a CTA (counted as four 64-row blocks, which also
    // covers the 64-row kernels)
    const int n_rb = comp ? (R + kGenRB - 1) / kGenRB
                          : (R <= kGenRB ? (R + 15) / 16 : 4 * ((R + 4 * kGenRB - 1) / (4 * kGenRB)));
    size_t b = kAttnTickets * sizeof(unsigned);
    b += align_up((size_t)batch * n_kv * n_rb * n_splits * kGenRB * (d + 2) * sizeof(float), 256);
    if (comp) b += align_up((size_t)batch * n_kv * group * cap * sizeof(float), 256);
    return b + 1024;
}

extern "C" size_t dkv_attn_work_bytes(dkv_dims dims, int group, int T, int max_ctx, int split_keys, int comp_cap) {
    const int sk = split_keys > 0 ? split_keys : 512;
    const int n_splits_full = (max_ctx + sk - 1) / sk;
    size_t full = attn_scratch(dims.batch, dims.n_kv, n_splits_full > 0 ? n_splits_full : 1, T * group, dims.d, 0,
                               group, false);
    size_t comp = 0;
    if (comp_cap > 0) {
        const int ns = (comp_cap + sk - 1) / sk;
        comp = attn_scratch(dims.batch, dims.n_kv, ns, group, dims.d, comp_cap, group, true);
    }
    return full > comp ? full : comp;
}

static int launch_generic(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, int max_keys, bool comp,
                          cudaStream_t st) {
    const int R = a.T * a.group;
    a.n_rb = (R + kGenRB - 1) / kGenRB;
    DKV_REQUIRE(!comp || a.n_rb == 1, "drafter attention: group %d > %d", a.group, kGenRB);
    a.n_splits = (max_keys + a.split - 1) / a.split;
    if (a.n_splits < 1) a.n_splits = 1;
    const size_t n_tk = (size_t)dims.batch * dims.n_kv * a.n_rb;
    DKV_REQUIRE(n_tk + dims.batch <= kAttnTickets, "attention: batch x heads x row blocks too large");
    Arena ar(work, work_bytes);
    unsigned* tk = ar.take<unsigned>(kAttnTickets);
    a.tickets = tk;
    a.fold_tickets = tk ? tk + n_tk : nullptr;
    a.part = ar.take<float>(n_tk * a.n_splits * kGenRB * (dims.d + 2));
    a.sbuf = comp ? ar.take<float>((size_t)dims.batch * dims.n_kv * a.group * a.src.cap) : nullptr;
    DKV_REQUIRE(a.part && a.tickets && a.fold_tickets && (!comp || a.sbuf),
                "attention: work buffer too small (%zu bytes)", work_bytes);
    const size_t smem = generic_smem(R < kGenRB ? R : kGenRB, dims.d);
    DKV_REQUIRE(smem <= 220 * 1024, "attention: %zu bytes of shared memory", smem);
    DKV_CUDA(allow_smem_max_once<attn_generic_kernel>());
    dim3 grid(a.n_splits, dims.n_kv, dims.batch * a.n_rb);
    {
        ProfScope ps(comp ? DKV_PROF_ATTN_COMP : DKV_PROF_ATTN_FULL, 0.0, st);
        attn_generic_kernel<<<grid, kGenThreads, smem, st>>>(a);
    }
    DKV_LAUNCHED();
    return DKV_OK;
}

namespace dkv {
int attn_full_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, int max_keys, cudaStream_t st,
                 bool* handled);
int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled,
                 uint32_t* comp_tickets, int raw_dtype);
}

extern "C" int dkv_attn_full(const dkv_full_cache* full, dkv_dims dims, int layer, int group, int T, const float* q,
                             const int32_t* pos0, void* out, int out_dtype, int split_keys, void* work,
                             size_t work_bytes, void* stream) {
    DKV_REQUIRE(full && full->k_pool && full->page_table && q && pos0 && out, "dkv_attn_full args");
    DKV_REQUIRE(layer >= 0 && layer < dims.n_layers && group >= 1 && T >= 1, "dkv_attn_full: layer/group/T");
    AttnArgs a{};
    a.src = full_src(full);
    a.n_layers = dims.n_layers;
    a.n_kv = dims.n_kv;
    a.d = dims.d;
    a.layer = layer;
    a.group = group;
    a.T = T;
    a.batch = dims.batch;
    a.q = q;
    a.qpos0 = pos0;
    a.out = out;
    a.out_dtype = out_dtype;
    a.split = split_keys > 0 ? split_keys : 512;
    a.scale = 1.0f / sqrtf((float)dims.d);
    const int max_keys = full->max_pages * full->page_size;
    bool handled = false;
    DKV_TRY(attn_full_tc(a, dims, work, work_bytes, max_keys, (cudaStream_t)stream, &handled));
    if (handled) return DKV_OK;
    return launch_generic(a, dims, work, work_bytes, max_keys, false, (cudaStream_t)stream);
}

extern "C" int dkv_attn_comp(const dkv_comp_cache* comp, dkv_dims dims, int layer, int group, const float* q,
                             const int32_t* qpos, void* out, int out_dtype, void* work, size_t work_bytes,
                             void* stream) {
    DKV_REQUIRE(comp && comp->pos && comp->meta && comp->mass && comp->score && comp->bits && q && qpos && out,
                "dkv_attn_comp args");
    DKV_REQUIRE(layer >= 0 && layer < dims.n_layers && group >= 1, "dkv_attn_comp: layer/group");
    AttnArgs a{};
    a.src = comp_src(comp, layer);
    a.n_layers = dims.n_layers;
    a.n_kv = dims.n_kv;
    a.d = dims.d;
    a.layer = layer;
    a.group = group;
    a.T = 1;
    a.batch = dims.batch;
    a.q = q;
    a.qpos0 = qpos;
    a.out = out;
    a.out_dtype = out_dtype;
    a.split = 512;
    a.scale = 1.0f / sqrtf((float)dims.d);
    a.mass = comp->mass;
    a.score = comp->score;
    // A layer kept whole (keep >= 1) never evicts, and a configuration switch
    // rebuilds the drafter cache at zero scores, so its accumulated mass is
    // never read: the tensor-core kernel skips it (the generic kernel, for
    // fp32 16-bit entries, still folds it).
    a.note_mass = !(comp->keep && comp->keep[layer] >= 1.0);
    bool handled = false;
    // 16-bit entries are stored in the model dtype: 4-byte elements mean fp32
    const int raw_dtype = comp->cb_max >= dims.d * 4 ? DKV_F32 : DKV_BF16;
    DKV_TRY(attn_comp_tc(a, dims, work, work_bytes, (cudaStream_t)stream, &handled, comp->tickets, raw_dtype));
    if (handled) return DKV_OK;
    return launch_generic(a, dims, work, work_bytes, comp->cap, true, (cudaStream_t)stream);
}
