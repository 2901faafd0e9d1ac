// Embedding, normalisation, and K5 sampling / acceptance.
//
//   embedding + learned positions   draftkv/gpt2.py:186, draftkv/llama.py:180
//   RMSNorm                         draftkv/llama.py:93-94
//   LayerNorm                       draftkv/gpt2.py:120-123
//   _probs / _sample                draftkv/engine.py:36-42, :101-106
//   acceptance, bonus, residual     draftkv/engine.py:188-213
#include "common.cuh"

namespace dkv {

__global__ void embed_kernel(const void* emb, int emb_dtype, const void* pos_emb, const int32_t* tokens,
                             int tok_stride, int T, const int32_t* pos0, int dm, float* h, int vocab, int max_pos,
                             uint32_t* err) {
    const int n = blockIdx.x;
    const int b = n / T, t = n % T;
    int tok = tokens[(size_t)b * tok_stride + t];
    int p = pos0 ? pos0[b] + t : t;
    // ids / positions outside the tables are reported, never read
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, 0x100u);
        tok = 0;
    }
    if (pos_emb && (p < 0 || p >= max_pos)) {
        if (threadIdx.x == 0) atomicOr(err, 0x200u);
        p = 0;
    }
    for (int i = threadIdx.x; i < dm; i += blockDim.x) {
        float v = load_as_f32(emb, emb_dtype, (size_t)tok * dm + i);
        if (pos_emb) v += load_as_f32(pos_emb, emb_dtype, (size_t)p * dm + i);
        h[(size_t)n * dm + i] = v;
    }
}

// One CTA per row; block reductions in a fixed order.
__global__ void norm_kernel(const float* __restrict__ h, int dm, int layernorm, const float* __restrict__ w,
                            const float* __restrict__ bias, float eps, void* x, int x_dtype) {
    __shared__ float red[32];
    const int n = blockIdx.x;
    const float* row = h + (size_t)n * dm;
    if (layernorm) {
        float s = 0.f;
        for (int i = threadIdx.x; i < dm; i += blockDim.x) s += row[i];
        const float mu = block_sum(s, red) / (float)dm;
        float v = 0.f;
        for (int i = threadIdx.x; i < dm; i += blockDim.x) {
            const float z = row[i] - mu;
            v += z * z;
        }
        const float var = block_sum(v, red) / (float)dm;
        const float inv = 1.0f / sqrtf(var + eps);
        for (int i = threadIdx.x; i < dm; i += blockDim.x)
            store_from_f32(x, x_dtype, (size_t)n * dm + i, (row[i] - mu) * inv * w[i] + (bias ? bias[i] : 0.f));
    } else {
        float s = 0.f;
        for (int i = threadIdx.x; i < dm; i += blockDim.x) s += row[i] * row[i];
        const float ms = block_sum(s, red) / (float)dm;
        const float inv = 1.0f / sqrtf(ms + eps);
        for (int i = threadIdx.x; i < dm; i += blockDim.x)
            store_from_f32(x, x_dtype, (size_t)n * dm + i, row[i] * inv * w[i]);
    }
}

// Register-resident variant (dm % 4 == 0, dm <= 256 * 4 * kNormV): the row
// is read once as float4 into registers, reduced once (twice for LayerNorm,
// from registers) and written; no second pass over global memory.
constexpr int kNormV = 8;       // float4s a thread holds (dm <= 8192)

__global__ void __launch_bounds__(256) norm_reg_kernel(const float* __restrict__ h, int dm, int layernorm,
                                                       const float* __restrict__ w, const float* __restrict__ bias,
                                                       float eps, void* x, int x_dtype) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x;
    const float4* row = reinterpret_cast<const float4*>(h + (size_t)n * dm);
    const int n4 = dm >> 2;
    float4 v[kNormV];
#pragma unroll
    for (int k = 0; k < kNormV; ++k) {
        const int i = threadIdx.x + k * 256;
        v[k] = i < n4 ? __ldg(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mu = 0.f;
    if (layernorm) {
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < kNormV; ++k) sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        mu = block_sum(sum, red) / (float)dm;
    }
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < kNormV; ++k) {
        if (threadIdx.x + k * 256 < n4) {
            const float a = v[k].x - mu, b = v[k].y - mu, c = v[k].z - mu, d = v[k].w - mu;
            sq += (a * a + b * b) + (c * c + d * d);
        }
    }
    const float inv = 1.0f / sqrtf(block_sum(sq, red) / (float)dm + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
    for (int k = 0; k < kNormV; ++k) {
        const int i = threadIdx.x + k * 256;
        if (i >= n4) continue;
        const float4 g = __ldg(w4 + i);
        const float4 bb = b4 ? __ldg(b4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float o0 = (v[k].x - mu) * inv * g.x + bb.x, o1 = (v[k].y - mu) * inv * g.y + bb.y;
        const float o2 = (v[k].z - mu) * inv * g.z + bb.z, o3 = (v[k].w - mu) * inv * g.w + bb.w;
        const size_t o = (size_t)n * dm + 4 * (size_t)i;
        if (x_dtype == DKV_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(x) + o) = make_float4(o0, o1, o2, o3);
        } else {
            __nv_bfloat162 p0 = __floats2bfloat162_rn(o0, o1), p1 = __floats2bfloat162_rn(o2, o3);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&p0);
            pk.y = *reinterpret_cast<uint32_t*>(&p1);
            *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(x) + o) = pk;
        }
    }
}

// ------------------------------------------------------------------ sampling
struct ArgMax {
    float v;
    int i;
};
DKV_DEV ArgMax better(ArgMax a, ArgMax b) {
    // larger value wins, ties -> lower index (numpy argmax returns the first)
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}
DKV_DEV ArgMax block_argmax(ArgMax m, ArgMax* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgMax t{__shfl_xor_sync(0xffffffffu, m.v, o), __shfl_xor_sync(0xffffffffu, m.i, o)};
        m = better(m, t);
    }
    __syncthreads();
    if (lane == 0) red[wid] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgMax r = red[0];
        for (int w = 1; w < nw; ++w) r = better(r, red[w]);
        red[0] = r;
    }
    __syncthreads();
    return red[0];
}

// Row argmax; 16-byte aligned rows are read as float4, four loads in flight
// a thread (the result does not depend on the scan order: larger value, then
// lower index).
DKV_DEV ArgMax row_argmax(const float* row, int V, ArgMax* red) {
    ArgMax m{-INFINITY, 0x7fffffff};
    int tail = 0;
    if (((uintptr_t)row & 15u) == 0) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        const int V4 = V >> 2, bd = blockDim.x;
        int i = threadIdx.x;
        for (; i + 3 * bd < V4; i += 4 * bd) {
            float4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = __ldg(r4 + i + u * bd);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = 4 * (i + u * bd);
                m = better(m, ArgMax{q[u].x, e});
                m = better(m, ArgMax{q[u].y, e + 1});
                m = better(m, ArgMax{q[u].z, e + 2});
                m = better(m, ArgMax{q[u].w, e + 3});
            }
        }
        for (; i < V4; i += bd) {
            const float4 q = __ldg(r4 + i);
            m = better(m, ArgMax{q.x, 4 * i});
            m = better(m, ArgMax{q.y, 4 * i + 1});
            m = better(m, ArgMax{q.z, 4 * i + 2});
            m = better(m, ArgMax{q.w, 4 * i + 3});
        }
        tail = 4 * V4;
    }
    for (int i = tail + threadIdx.x; i < V; i += blockDim.x) m = better(m, ArgMax{row[i], i});
    return block_argmax(m, red);
}

// sum of exp((l - mx) / T) in double, fixed order
DKV_DEV double row_expsum(const float* row, int V, float mx, double invT, double* redd) {
    double s = 0.0;
#pragma unroll 4
    for (int i = threadIdx.x; i < V; i += blockDim.x) s += exp(((double)__ldg(row + i) - (double)mx) * invT);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    s = warp_sum_d(s);
    __syncthreads();
    if (lane == 0) redd[wid] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < nw; ++w) t += redd[w];
        redd[0] = t;
    }
    __syncthreads();
    return redd[0];
}

// Inverse-CDF draw over weights w(i) (non-negative, any scale) whose sum is
// `total`: first i with prefix(i) > u*total, scanning in blocks of blockDim.
template <typename WFn>
DKV_DEV int draw_index(WFn wfn, int V, double total, double u, double* redd, int* found) {
    const double target = u * total;
    double carry = 0.0;
    constexpr int kNone = 0x7fffffff;
    if (threadIdx.x == 0) *found = kNone;   // lowered by atomicMin on a hit
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int last_pos = -1;
    for (int base = 0; base < V; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const double wv = i < V ? wfn(i) : 0.0;
        if (i < V && wv > 0.0) last_pos = i;
        // inclusive scan of wv across the block (warp scan + warp offsets)
        double x = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double t = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += t;
        }
        if (lane == 31) redd[wid] = x;
        __syncthreads();
        if (threadIdx.x == 0) {
            double run = 0.0;
            for (int w = 0; w < nw; ++w) {
                double t = redd[w];
                redd[w] = run;
                run += t;
            }
            redd[nw] = run;
        }
        __syncthreads();
        const double incl = carry + redd[wid] + x;
        const bool hit = i < V && wv > 0.0 && incl > target;
        if (hit) atomicMin(found, i);
        carry += redd[nw];
        __syncthreads();
        if (*found != kNone) break;
    }
    // rounding can leave the target just above the final prefix: take the
    // last index with positive weight
    const bool none = *found == kNone;
    __syncthreads();
    if (none) {
        if (threadIdx.x == 0) *found = -1;
        __syncthreads();
        int lp = last_pos;
        for (int o = 16; o > 0; o >>= 1) lp = max(lp, __shfl_xor_sync(0xffffffffu, lp, o));
        if (lane == 0) atomicMax(found, lp);
        __syncthreads();
    }
    const int r = *found;
    __syncthreads();
    return r < 0 ? 0 : r;
}

constexpr int kRowThreads = 512;   // threads of the per-row sampling / acceptance CTAs

// One CTA per row: argmax (T <= 0) or a draw from softmax(l / T).
__global__ void __launch_bounds__(kRowThreads) sample_kernel(const float* logits, int V, float temperature, uint64_t seed, const uint64_t* counter,
                              int32_t* tokens, int tok_stride) {
    __shared__ ArgMax red[32];
    __shared__ double redd[33];
    __shared__ int found;
    const int r = blockIdx.x;
    const float* row = logits + (size_t)r * V;
    const ArgMax am = row_argmax(row, V, red);
    int tok = am.i;
    if (temperature > 0.f) {
        const double invT = 1.0 / (double)temperature;
        const double tot = row_expsum(row, V, am.v, invT, redd);
        const double u = philox_uniform(seed, counter ? *counter : 0ull, 0x5A3Du, (uint32_t)r);
        const float mx = am.v;
        tok = draw_index([&](int i) { return exp(((double)row[i] - (double)mx) * invT); }, V, tot, u, redd, &found);
    }
    if (threadIdx.x == 0) tokens[(size_t)r * tok_stride] = tok;
}

// --------------------------------------------------------------- acceptance
// Phase 1: one CTA per (row, sequence) computes argmax, max and the exp-sum
// of verify rows (gamma+1) and of draft rows (gamma, T > 0 only), plus the
// row's value at the drafted token.
struct RowStat {
    float mx;
    int arg;
    double sum;     // sum exp((l - mx)/T)
    float at_tok;   // logit at the drafted token (verify row i / draft row i)
};

struct AcceptArgs {
    const float* verify;   // [batch][gamma+1][V]
    const float* draft;    // [gamma][batch][V]
    int batch, gamma, V;
    float temperature;
    uint64_t seed;
    const uint64_t* counter;
    int32_t* vtok;
    int vstride;
    int32_t* base_pos;
    int32_t* accepted;
    int32_t* next;
    int32_t* rs_pos0;
    int32_t* rs_rows;
    int32_t* rs_trunc;
    const int32_t* active;
    RowStat* stats;        // [batch][2*gamma+1]
    unsigned* tickets;     // [batch]
};

DKV_DEV double p_of(const RowStat& s, float l, double invT) {
    return exp(((double)l - (double)s.mx) * invT) / s.sum;
}

__global__ void __launch_bounds__(kRowThreads) accept_kernel(AcceptArgs a) {
    __shared__ ArgMax red[32];
    __shared__ double redd[33];
    __shared__ int found, is_last;
    const int b = blockIdx.y, row = blockIdx.x;   // rows: [0, gamma] verify, [gamma+1, 2gamma] draft
    const int G = a.gamma, V = a.V;
    const bool sampling = a.temperature > 0.f;
    const double invT = sampling ? 1.0 / (double)a.temperature : 0.0;
    const int n_rows = sampling ? 2 * G + 1 : G + 1;
    if (row >= n_rows) return;
    const float* lrow = row <= G ? a.verify + ((size_t)b * (G + 1) + row) * V
                                 : a.draft + ((size_t)(row - G - 1) * a.batch + b) * V;
    const ArgMax am = row_argmax(lrow, V, red);
    RowStat st;
    st.mx = am.v;
    st.arg = am.i;
    st.sum = sampling ? row_expsum(lrow, V, am.v, invT, redd) : 0.0;
    const int di = row <= G ? row : row - G - 1;      // draft index this row is compared at
    st.at_tok = di < G ? lrow[a.vtok[(size_t)b * a.vstride + 1 + di]] : 0.f;
    if (threadIdx.x == 0) a.stats[(size_t)b * (2 * G + 1) + row] = st;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.tickets + b, 1u);
        is_last = prev == (unsigned)(n_rows - 1);
        if (is_last) a.tickets[b] = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // ---- phase 2 (last CTA of sequence b): accepted count and next token
    const RowStat* S = a.stats + (size_t)b * (2 * G + 1);
    const uint64_t ctr = a.counter ? *a.counter : 0ull;
    __shared__ int sh_k, sh_next;
    if (threadIdx.x == 0) {
        int k = 0;
        for (int i = 0; i < G; ++i) {
            const int d = a.vtok[(size_t)b * a.vstride + 1 + i];
            bool ok;
            if (!sampling) {
                ok = S[i].arg == d;
            } else {
                const double p = p_of(S[i], S[i].at_tok, invT);
                const double q = p_of(S[G + 1 + i], S[G + 1 + i].at_tok, invT);
                const double ratio = q > 0.0 ? p / q : 0.0;
                const double u = philox_uniform(a.seed, ctr, 0xACCEu, (uint32_t)(b * 64 + i));
                ok = u < (ratio < 1.0 ? ratio : 1.0);
            }
            if (!ok) break;
            ++k;
        }
        sh_k = k;
        sh_next = S[k].arg;
    }
    __syncthreads();
    const int k = sh_k;
    if (sampling) {
        const float* vrow = a.verify + ((size_t)b * (G + 1) + k) * V;
        const RowStat pv = S[k];
        const double u = philox_uniform(a.seed, ctr, 0xB0A5u, (uint32_t)b);
        int tok;
        if (k == G) {
            tok = draw_index([&](int i) { return p_of(pv, vrow[i], invT); }, V, 1.0, u, redd, &found);
        } else {
            const float* qrow = a.draft + ((size_t)k * a.batch + b) * V;
            const RowStat qs = S[G + 1 + k];
            auto resid = [&](int i) {
                const double r = p_of(pv, vrow[i], invT) - p_of(qs, qrow[i], invT);
                return r > 0.0 ? r : 0.0;
            };
            // total of the residual (fixed order)
            double part = 0.0;
            for (int i = threadIdx.x; i < V; i += blockDim.x) part += resid(i);
            part = warp_sum_d(part);
            __syncthreads();
            if ((threadIdx.x & 31) == 0) redd[threadIdx.x >> 5] = part;
            __syncthreads();
            if (threadIdx.x == 0) {
                double t = 0.0;
                for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += redd[w];
                redd[32] = t;
            }
            __syncthreads();
            const double tot = redd[32];
            __syncthreads();
            if (tot > 0.0)
                tok = draw_index(resid, V, tot, u, redd, &found);
            else
                tok = draw_index([&](int i) { return p_of(pv, vrow[i], invT); }, V, 1.0, u, redd, &found);
        }
        if (threadIdx.x == 0) sh_next = tok;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const bool act = a.active ? a.active[b] != 0 : true;
        const int nxt = sh_next;
        a.accepted[b] = k;
        a.next[b] = nxt;
        const int old = a.base_pos[b];
        if (a.rs_pos0) a.rs_pos0[b] = old;
        if (a.rs_rows) a.rs_rows[b] = act ? k + 1 : 0;
        if (a.rs_trunc) a.rs_trunc[b] = old;
        if (act) {
            a.vtok[(size_t)b * a.vstride + 1 + k] = nxt;   // emitted stream: drafts[0..k) + next
            a.vtok[(size_t)b * a.vstride] = nxt;           // pending token of the next round
            a.base_pos[b] = old + k + 1;
        }
    }
}

}  // namespace dkv

using namespace dkv;

namespace dkv {
uint32_t* device_error_word();
}

extern "C" int dkv_embed(const void* emb, int emb_dtype, const void* pos_emb, const int32_t* tokens, int tok_stride,
                         int batch, int T, const int32_t* pos0, int dm, int vocab, int max_pos, float* h,
                         void* stream) {
    DKV_REQUIRE(emb && tokens && h && batch >= 0 && T >= 0 && dm > 0 && vocab > 0, "dkv_embed args");
    if (batch * T == 0) return DKV_OK;
    ProfScope ps(DKV_PROF_EMBED, 0.0, (cudaStream_t)stream);
    embed_kernel<<<batch * T, 256, 0, (cudaStream_t)stream>>>(emb, emb_dtype, pos_emb, tokens, tok_stride, T, pos0,
                                                               dm, h, vocab, max_pos, device_error_word());
    DKV_LAUNCHED();
    return DKV_OK;
}

// First half of a fused RMSNorm (the forward's first layer; later ones come
// out of the residual GEMM's epilogue): x[n][m] = bf16(h[n][m] * w[m]) and
// part[t * ld + n] = sum of h[n][m]^2 over the 128 columns m of tile t, in
// the order of the GEMM epilogue (4 columns a lane, then a butterfly).  The
// GEMM that reads x divides by the rms.  One CTA of 4 warps per token.
__global__ void __launch_bounds__(128) norm_prep_kernel(const float* __restrict__ h, int dm,
                                                        const float* __restrict__ w, uint16_t* __restrict__ x,
                                                        float* __restrict__ part, int ld) {
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* row = h + (size_t)n * dm;
    for (int t = warp; t < dm / 128; t += 4) {
        const float* r = row + t * 128;
        const float a = r[lane], b = r[lane + 32], c = r[lane + 64], d = r[lane + 96];
        float v = ((a * a + b * b) + c * c) + d * d;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) part[(size_t)t * ld + n] = v;
        const float* wt = w + t * 128;
        uint16_t* xt = x + (size_t)n * dm + t * 128;
        xt[lane] = f32_to_bf16_bits(a * wt[lane]);
        xt[lane + 32] = f32_to_bf16_bits(b * wt[lane + 32]);
        xt[lane + 64] = f32_to_bf16_bits(c * wt[lane + 64]);
        xt[lane + 96] = f32_to_bf16_bits(d * wt[lane + 96]);
    }
}

namespace dkv {
int norm_prep(const float* h, int N, int dm, const float* w, void* x, float* part, int ld, cudaStream_t st) {
    DKV_REQUIRE(h && w && x && part && dm % 128 == 0 && ld >= N, "norm_prep args");
    if (N == 0) return DKV_OK;
    ProfScope ps(DKV_PROF_NORM, (double)N * dm * 6.0, st);
    DKV_CUDA(launch_pdl(norm_prep_kernel, dim3(N), dim3(128), 0, st, h, dm, w, reinterpret_cast<uint16_t*>(x), part,
                        ld));
    DKV_LAUNCHED();
    return DKV_OK;
}
}  // namespace dkv

extern "C" int dkv_norm(const float* h, int N, int dm, int layernorm, const float* w, const float* b, float eps,
                        void* x, int x_dtype, void* stream) {
    DKV_REQUIRE(h && w && x && N >= 0 && dm > 0, "dkv_norm args");
    if (N == 0) return DKV_OK;
    ProfScope ps(DKV_PROF_NORM, (double)N * dm * (4.0 + (x_dtype == DKV_F32 ? 4.0 : 2.0)), (cudaStream_t)stream);
    const bool aligned = ((uintptr_t)h % 16 == 0) && ((uintptr_t)w % 16 == 0) && (!b || (uintptr_t)b % 16 == 0) &&
                         ((uintptr_t)x % 16 == 0);
    if (dm % 4 == 0 && dm <= 256 * 4 * kNormV && aligned)
        DKV_CUDA(launch_pdl(norm_reg_kernel, dim3(N), dim3(256), 0, (cudaStream_t)stream, h, dm, layernorm, w, b,
                            eps, x, x_dtype));
    else
        norm_kernel<<<N, 256, 0, (cudaStream_t)stream>>>(h, dm, layernorm, w, b, eps, x, x_dtype);
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" size_t dkv_sample_work_bytes(int rows, int V) {
    (void)V;
    // rows = batch; stats for up to 2*63+1 rows per sequence
    return align_up((size_t)rows * sizeof(unsigned), 256) + align_up((size_t)rows * 127 * sizeof(RowStat), 256) + 512;
}

extern "C" int dkv_sample(const float* logits, int rows, int V, float temperature, uint64_t seed,
                          const uint64_t* counter, int32_t* tokens, int tok_stride, void* work, size_t work_bytes,
                          void* stream) {
    (void)work;
    (void)work_bytes;
    DKV_REQUIRE(logits && tokens && rows >= 0 && V > 0, "dkv_sample args");
    if (rows == 0) return DKV_OK;
    ProfScope ps(DKV_PROF_SAMPLE, (double)rows * V * 4.0, (cudaStream_t)stream);
    sample_kernel<<<rows, kRowThreads, 0, (cudaStream_t)stream>>>(logits, V, temperature, seed, counter, tokens,
                                                                   tok_stride);
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" int dkv_accept(const float* verify, const float* draft_logits, int batch, int gamma, int V,
                          float temperature, uint64_t seed, const uint64_t* counter, int32_t* vtok, int vstride,
                          int32_t* base_pos, int32_t* accepted, int32_t* next, int32_t* rs_pos0, int32_t* rs_rows,
                          int32_t* rs_trunc, const int32_t* active, void* work, size_t work_bytes, void* stream) {
    DKV_REQUIRE(verify && vtok && base_pos && accepted && next && batch > 0 && gamma >= 0 && V > 0, "dkv_accept args");
    DKV_REQUIRE(vstride >= gamma + 2, "dkv_accept: vstride %d < gamma+2", vstride);
    DKV_REQUIRE(temperature <= 0.f || gamma == 0 || draft_logits, "dkv_accept: sampling needs the draft logits");
    DKV_REQUIRE(gamma <= 63, "dkv_accept: gamma <= 63");
    Arena ar(work, work_bytes);
    AcceptArgs a;
    a.verify = verify;
    a.draft = draft_logits;
    a.batch = batch;
    a.gamma = gamma;
    a.V = V;
    a.temperature = temperature;
    a.seed = seed;
    a.counter = counter;
    a.vtok = vtok;
    a.vstride = vstride;
    a.base_pos = base_pos;
    a.accepted = accepted;
    a.next = next;
    a.rs_pos0 = rs_pos0;
    a.rs_rows = rs_rows;
    a.rs_trunc = rs_trunc;
    a.active = active;
    a.tickets = ar.take<unsigned>(batch);            // fixed offset: tickets first
    a.stats = ar.take<RowStat>((size_t)batch * (2 * gamma + 1));
    DKV_REQUIRE(a.stats && a.tickets, "dkv_accept: work buffer too small");
    const int rows = temperature > 0.f ? 2 * gamma + 1 : gamma + 1;
    ProfScope ps(DKV_PROF_ACCEPT, (double)batch * rows * V * 4.0, (cudaStream_t)stream);
    accept_kernel<<<dim3(rows, batch), kRowThreads, 0, (cudaStream_t)stream>>>(a);
    DKV_LAUNCHED();
    return DKV_OK;
}
