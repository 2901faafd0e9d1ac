// K1 quantize / pack, K6 evict, K7 truncate + resync + rebuild of the drafter
// cache, and plain writes / reads of the full cache.
//
// Reference behaviour followed (aabhimittal/Draft-KV):
//   quantize              draftkv/compress.py:21-46
//   CompressedKVCache     draftkv/compress.py:95-241  (append :122-133,
//                         budget :154-157, _evict :159-179, truncate :181-188,
//                         sync_from :190-207, rebuild_layers :209-230)
//   FullKVCache / paged   draftkv/compress.py:49-92, draftkv/paged.py:76-177
#include "common.cuh"

namespace dkv {

// --------------------------------------------------------------------------
// Exact group quantization of one 64-wide group held by a warp: lane l owns
// elements 64g+l and 64g+32+l (zero beyond d, as numpy pads).  All ops are
// IEEE round-to-nearest without contraction, reproducing numpy bit for bit.
struct GroupQ {
    float lo, scale;
};

DKV_DEV GroupQ group_params(float a, float b, int bits) {
    float lo = warp_min(fminf(a, b));
    float hi = warp_max(fmaxf(a, b));
    float levels = (float)((1 << bits) - 1);
    float scale = __fdiv_rn(__fsub_rn(hi, lo), levels);
    scale = fmaxf(scale, 1e-8f);
    return {lo, scale};
}

DKV_DEV float code_of(float x, GroupQ g, int bits) {
    float q = rintf(__fdiv_rn(__fsub_rn(x, g.lo), g.scale));
    q = fminf(fmaxf(q, 0.f), (float)((1 << bits) - 1));
    return q;
}

DKV_DEV float deq_of(float q, GroupQ g) { return __fadd_rn(__fmul_rn(q, g.scale), g.lo); }

// One warp per (row, group).
__global__ void quantize_exact_kernel(const float* __restrict__ x, int64_t rows, int d, int bits,
                                      uint8_t* __restrict__ codes, float* __restrict__ scale,
                                      float* __restrict__ lo, float* __restrict__ deq) {
    const int ng = (d + 63) / 64;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows * ng) return;
    const int64_t r = warp / ng;
    const int g = (int)(warp % ng);
    const int e0 = 64 * g + lane, e1 = e0 + 32;
    float a = e0 < d ? x[r * d + e0] : 0.f;
    float b = e1 < d ? x[r * d + e1] : 0.f;
    if (bits >= 16) {
        if (deq) {
            if (e0 < d) deq[r * d + e0] = a;
            if (e1 < d) deq[r * d + e1] = b;
        }
        return;
    }
    GroupQ gq = group_params(a, b, bits);
    float qa = code_of(a, gq, bits), qb = code_of(b, gq, bits);
    if (codes) {
        codes[r * ng * 64 + e0] = (uint8_t)qa;
        codes[r * ng * 64 + e1] = (uint8_t)qb;
    }
    if (lane == 0) {
        if (scale) scale[r * ng + g] = gq.scale;
        if (lo) lo[r * ng + g] = gq.lo;
    }
    if (deq) {
        if (e0 < d) deq[r * d + e0] = deq_of(qa, gq);
        if (e1 < d) deq[r * d + e1] = deq_of(qb, gq);
    }
}

// --------------------------------------------------------------------------
// Storage order of the drafter cache (stated with the bit layouts in
// include/draftkv_b200.h): K vectors in the tensor-core fragment order, V
// vectors in element order.  Storage position p of a K vector holds element
// 16j + 2c + (r & 1) + 8 (r >> 1) for quad c = p / (d/4), k-step j and r = p % 4.
DKV_DEV int storage_elem(int p, int d, bool k_order) {
    if (!k_order) return p;
    const int q4 = d >> 2;
    const int c = p / q4, rem = p - c * q4;
    const int j = rem >> 2, r = rem & 3;
    return 16 * j + 2 * c + (r & 1) + ((r >> 1) << 3);
}

// Quantizes and packs one d-element vector with one warp.  `src` is read
// through load_as_f32 (element stride 1).  `scratch` holds d bytes (warp
// private).  Writes cb = d*bits/8 bytes of codes and d/64 (scale, lo) fp16
// pairs; bits == 16 stores the raw elements (in `raw_dtype`) instead.
DKV_DEV void quant_pack_vector(const void* src, int src_dtype, size_t src_off, int d, int bits,
                               bool k_order, uint8_t* __restrict__ dst_codes,
                               uint16_t* __restrict__ dst_sl, int raw_dtype,
                               uint8_t* scratch) {
    const int lane = threadIdx.x & 31;
    if (bits == 16) {
        for (int p = lane; p < d; p += 32) {
            float v = load_as_f32(src, src_dtype, src_off + storage_elem(p, d, k_order));
            store_from_f32(dst_codes, raw_dtype, p, v);
        }
        return;
    }
    const int ng = d >> 6;
    for (int g = 0; g < ng; ++g) {
        const int e0 = 64 * g + lane, e1 = e0 + 32;
        float a = load_as_f32(src, src_dtype, src_off + e0);
        float b = load_as_f32(src, src_dtype, src_off + e1);
        GroupQ gq = group_params(a, b, bits);
        scratch[e0] = (uint8_t)code_of(a, gq, bits);
        scratch[e1] = (uint8_t)code_of(b, gq, bits);
        if (lane == 0) {
            dst_sl[2 * g] = f32_to_half_bits(gq.scale);
            dst_sl[2 * g + 1] = f32_to_half_bits(gq.lo);
        }
    }
    __syncwarp();
    uint32_t* out = reinterpret_cast<uint32_t*>(dst_codes);
    if (bits == 8) {
        for (int w = lane; w < d / 4; w += 32) {
            uint32_t v = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) v |= (uint32_t)scratch[storage_elem(4 * w + i, d, k_order)] << (8 * i);
            out[w] = v;
        }
    } else if (bits == 4 || bits == 2) {
        const int per = 32 / bits, half = per / 2;
        for (int w = lane; w < d / per; w += 32) {
            uint32_t v = 0;
            for (int i = 0; i < half; ++i) {
                v |= (uint32_t)scratch[storage_elem(per * w + 2 * i, d, k_order)] << (bits * i);
                v |= (uint32_t)scratch[storage_elem(per * w + 2 * i + 1, d, k_order)] << (16 + bits * i);
            }
            out[w] = v;
        }
    } else {  // 3 bit: plane A (low 2 bits, 2-bit layout) then plane B (high bit)
        for (int w = lane; w < d / 16; w += 32) {
            uint32_t v = 0;
            for (int i = 0; i < 8; ++i) {
                v |= ((uint32_t)scratch[storage_elem(16 * w + 2 * i, d, k_order)] & 3u) << (2 * i);
                v |= ((uint32_t)scratch[storage_elem(16 * w + 2 * i + 1, d, k_order)] & 3u) << (16 + 2 * i);
            }
            out[w] = v;
        }
        uint16_t* units = reinterpret_cast<uint16_t*>(dst_codes + d / 4);
        for (int u = lane; u < d / 16; u += 32) {
            uint32_t v = 0;
            for (int i = 0; i < 8; ++i) {
                v |= ((uint32_t)scratch[storage_elem(16 * u + 2 * i, d, k_order)] >> 2) << i;
                v |= ((uint32_t)scratch[storage_elem(16 * u + 2 * i + 1, d, k_order)] >> 2) << (8 + i);
            }
            units[u] = (uint16_t)v;
        }
    }
    __syncwarp();
}

// --------------------------------------------------------------------------
// Lane-sliced quantize + pack (d % 64 == 0): each lane owns 16 consecutive
// elements 16j..16j+15 of a vector (j = lane index within the vector's d/16
// lanes), so a 64-element group is 4 neighbouring lanes and every packed
// word is assembled in registers, OR-combined across the 2 or 4 lanes that
// share it.  Same bytes as quant_pack_vector.
//
// Codes: q = clip(rint((x - lo) / scale)).  The quotient is first taken as
// (x - lo) * RN(1/scale): its distance from the correctly rounded quotient is
// below 4.6e-5 for quotients <= 255 (two fp32 roundings of relative 2^-24
// each on the product, one on the quotient), so rint of the two agrees unless
// the product lies within 1e-4 of a half-integer; only then is the IEEE
// division evaluated.
DKV_DEV void slice_group_params(const float (&x)[16], int bits, float* lo_out, float* scale_out) {
    float lo = x[0], hi = x[0];
#pragma unroll
    for (int i = 1; i < 16; ++i) {
        lo = fminf(lo, x[i]);
        hi = fmaxf(hi, x[i]);
    }
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, 1));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, 1));
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, 2));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, 2));
    const float levels = (float)((1 << bits) - 1);
    *lo_out = lo;
    *scale_out = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), levels), 1e-8f);
}

DKV_DEV uint32_t slice_code(float x, float lo, float scale, float rs, float qmax) {
    const float num = __fsub_rn(x, lo);
    const float t = __fmul_rn(num, rs);
    float q = rintf(t);
    if (fabsf(t - q) > 0.4999f) q = rintf(__fdiv_rn(num, scale));
    q = fminf(fmaxf(q, 0.f), qmax);
    return (uint32_t)q;
}

DKV_DEV void st_u32(uint8_t* p, uint32_t v) { *reinterpret_cast<uint32_t*>(p) = v; }

// x: this lane's 16 elements (as f32); j: lane index within the vector.
// Lanes of a warp must all call this together (shuffles); `active` = false
// lanes compute on their (arbitrary) x and store nothing.  raw_dtype is the
// storage dtype of 16-bit vectors.
DKV_DEV void quant_pack_slice(const float (&x)[16], int j, int d, int bits, bool k_order, bool active,
                              uint8_t* __restrict__ dst, uint16_t* __restrict__ dst_sl, int raw_dtype) {
    const int q4 = d >> 2;     // elements (storage positions) per quad segment in K order
    if (bits == 16) {
        if (!active) return;
        if (k_order) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int P = c * q4 + 4 * j;
                store_from_f32(dst, raw_dtype, P + 0, x[2 * c]);
                store_from_f32(dst, raw_dtype, P + 1, x[2 * c + 1]);
                store_from_f32(dst, raw_dtype, P + 2, x[2 * c + 8]);
                store_from_f32(dst, raw_dtype, P + 3, x[2 * c + 9]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) store_from_f32(dst, raw_dtype, 16 * j + i, x[i]);
        }
        return;
    }
    float lo, scale;
    slice_group_params(x, bits, &lo, &scale);
    const float rs = __frcp_rn(scale);
    const float qmax = (float)((1 << bits) - 1);
    uint32_t q[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = slice_code(x[i], lo, scale, rs, qmax);
    if (active && (j & 3) == 0) {
        dst_sl[2 * (j >> 2)] = f32_to_half_bits(scale);
        dst_sl[2 * (j >> 2) + 1] = f32_to_half_bits(lo);
    }
    if (!k_order) {
        // element order: this lane owns whole words (2-bit: one word, 3-bit:
        // one plane-A word and one plane-B unit, 4-bit: two words, 8-bit: four)
        if (bits == 8) {
            if (active) {
#pragma unroll
                for (int w = 0; w < 4; ++w)
                    st_u32(dst + 16 * j + 4 * w, q[4 * w] | (q[4 * w + 1] << 8) | (q[4 * w + 2] << 16) | (q[4 * w + 3] << 24));
            }
        } else if (bits == 4) {
            if (active) {
#pragma unroll
                for (int w = 0; w < 2; ++w) {
                    uint32_t v = 0;
#pragma unroll
                    for (int i = 0; i < 4; ++i) v |= (q[8 * w + 2 * i] << (4 * i)) | (q[8 * w + 2 * i + 1] << (16 + 4 * i));
                    st_u32(dst + 8 * j + 4 * w, v);
                }
            }
        } else {   // 2 or 3 bits: plane A in the 2-bit layout
            uint32_t v = 0, u = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v |= ((q[2 * i] & 3u) << (2 * i)) | ((q[2 * i + 1] & 3u) << (16 + 2 * i));
                u |= ((q[2 * i] >> 2) << i) | ((q[2 * i + 1] >> 2) << (8 + i));
            }
            if (active) {
                st_u32(dst + 4 * j, v);
                if (bits == 3) reinterpret_cast<uint16_t*>(dst + d / 4)[j] = (uint16_t)u;
            }
        }
        return;
    }
    // fragment order: quad c's codes of this lane are elements 2c, 2c+1,
    // 2c+8, 2c+9 at storage positions P = c*q4 + 4j + {0,1,2,3}
    if (bits == 8) {
        if (active) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                st_u32(dst + c * q4 + 4 * j, q[2 * c] | (q[2 * c + 1] << 8) | (q[2 * c + 8] << 16) | (q[2 * c + 9] << 24));
        }
    } else if (bits == 4) {
        // a word holds 8 positions = lanes j (even) and j+1; position k of
        // the word sits at bits 4*(k>>1) (+16 if k odd)
        const int h = j & 1;
        uint32_t piece[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            piece[c] = (q[2 * c] << (8 * h)) | (q[2 * c + 1] << (16 + 8 * h)) | (q[2 * c + 8] << (4 + 8 * h)) |
                       (q[2 * c + 9] << (20 + 8 * h));
            piece[c] |= __shfl_xor_sync(0xffffffffu, piece[c], 1);
        }
        if (active) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * h + cc;
                st_u32(dst + (c * q4 + 4 * (j & ~1)) / 2, piece[c]);
            }
        }
    } else {   // 2 or 3 bits: a plane-A word / plane-B unit holds 16 positions = 4 lanes
        const int m = j & 3;
        uint32_t pa[4], pb[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t a0 = q[2 * c], a1 = q[2 * c + 1], a2 = q[2 * c + 8], a3 = q[2 * c + 9];
            pa[c] = ((a0 & 3u) << (4 * m)) | ((a1 & 3u) << (16 + 4 * m)) | ((a2 & 3u) << (4 * m + 2)) |
                    ((a3 & 3u) << (18 + 4 * m));
            pb[c] = ((a0 >> 2) << (2 * m)) | ((a1 >> 2) << (8 + 2 * m)) | ((a2 >> 2) << (2 * m + 1)) |
                    ((a3 >> 2) << (9 + 2 * m));
            pa[c] |= __shfl_xor_sync(0xffffffffu, pa[c], 1);
            pa[c] |= __shfl_xor_sync(0xffffffffu, pa[c], 2);
            if (bits == 3) {
                pb[c] |= __shfl_xor_sync(0xffffffffu, pb[c], 1);
                pb[c] |= __shfl_xor_sync(0xffffffffu, pb[c], 2);
            }
        }
        if (active) {
            uint32_t wa = pa[0], wb = pb[0];
#pragma unroll
            for (int c = 1; c < 4; ++c)
                if (m == c) {
                    wa = pa[c];
                    wb = pb[c];
                }
            const int P = m * q4 + 4 * (j & ~3);      // first position of the word (quad c = m)
            st_u32(dst + P / 4, wa);
            if (bits == 3) reinterpret_cast<uint16_t*>(dst + d / 4)[P / 16] = (uint16_t)wb;
        }
    }
}

// Loads this lane's 16 elements (offset `off` + 16j of a row) as f32.
DKV_DEV void load_slice(const void* src, int dtype, size_t off, float (&x)[16]) {
    if (dtype == DKV_F32) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + off);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = __ldg(p + i);
            x[4 * i] = v.x;
            x[4 * i + 1] = v.y;
            x[4 * i + 2] = v.z;
            x[4 * i + 3] = v.w;
        }
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + off);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 v = __ldg(p + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                x[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
                x[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
    }
}

// Dequantizes element e of a stored vector (test read-back path).
DKV_DEV float dequant_elem(const uint8_t* codes, const uint16_t* sl, int d, int bits, bool k_order,
                           int e, int raw_dtype) {
    // find the storage position p holding element e
    int p = e;
    if (k_order) {
        const int q4 = d >> 2;
        const int j = e >> 4, w = e & 15;
        const int c = (w & 7) >> 1;
        const int r = (w & 1) | ((w >> 3) << 1);
        p = c * q4 + 4 * j + r;
    }
    if (bits == 16) return load_as_f32(codes, raw_dtype, p);
    uint32_t q;
    if (bits == 8) {
        q = codes[p];
    } else if (bits == 4 || bits == 2) {
        const int per = 32 / bits;
        const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[p / per];
        const int i = (p % per) >> 1;
        const int sh = (p & 1) ? 16 + bits * i : bits * i;
        q = (w >> sh) & ((1u << bits) - 1);
    } else {
        const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[p / 16];
        const int i = (p % 16) >> 1;
        const int sh = (p & 1) ? 16 + 2 * i : 2 * i;
        const uint32_t lo2 = (w >> sh) & 3u;
        const uint16_t u = reinterpret_cast<const uint16_t*>(codes + d / 4)[p / 16];
        const int sh1 = (p & 1) ? 8 + i : i;
        q = lo2 | (((u >> sh1) & 1u) << 2);
    }
    const int g = e >> 6;
    float scale = half_bits_to_f32(sl[2 * g]), lo = half_bits_to_f32(sl[2 * g + 1]);
    return (float)q * scale + lo;
}

// d % 64 == 0: d/16 lanes per row (lane-sliced packer).
__global__ void quantize_pack_slice_kernel(const void* src, int src_dtype, int64_t rows, int d, int bits,
                                           bool k_order, uint8_t* codes, uint16_t* sl) {
    const int lpv = d >> 4, vpw = 32 / lpv;
    const int lane = threadIdx.x & 31;
    const int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x - lane) / 32 * vpw;
    const int64_t r = base + lane / lpv;
    const int j = lane % lpv;
    if (base >= rows) return;                 // uniform per warp
    const bool active = r < rows;
    const int64_t rr = active ? r : base;
    const int elem = src_dtype == DKV_F32 ? 4 : 2;
    const int cb = bits == 16 ? d * elem : d * bits / 8;
    float x[16];
    load_slice(src, src_dtype, (size_t)rr * d + 16 * j, x);
    quant_pack_slice(x, j, d, bits, k_order, active, codes + rr * cb, sl + rr * (d / 64) * 2, src_dtype);
}

// --------------------------------------------------------------------------
// Drafter cache addressing.
struct CompView {
    uint8_t* k_codes;
    uint8_t* v_codes;
    uint16_t* k_sl;
    uint16_t* v_sl;
    int32_t* pos;
    float* score;
    int32_t* meta;
    int32_t* seen;
    int cap, cb_max, n_layers, n_kv, d;

    DKV_DEV size_t bl(int b, int L) const { return (size_t)b * n_layers + L; }
    DKV_DEV size_t vec(int b, int L, int h, int slot) const {
        return ((bl(b, L) * n_kv + h) * (size_t)cap + slot);
    }
    // byte offset of a vector's codes: the (b, L, h) region of cap x cb_max
    // bytes holds rows of kb = code_row_bytes(...) bytes, densely
    DKV_DEV size_t code_off(int b, int L, int h, int slot, int kb) const {
        return (bl(b, L) * n_kv + h) * (size_t)cap * cb_max + (size_t)slot * kb;
    }
};

struct FullView {
    const void* k_pool;
    const void* v_pool;
    const int32_t* page_table;
    int page_size, max_pages, dtype, n_layers, n_kv, d;

    DKV_DEV size_t elem(int b, int L, int h, int p) const {
        const int page = page_table[((size_t)b * n_layers + L) * max_pages + p / page_size];
        return (((size_t)page * n_kv + h) * page_size + (p % page_size)) * (size_t)d;
    }
};

struct LayerCfgs {
    int n;
    int bits[128];
    int sink[128];
    int recent[128];
    double keep[128];
};

DKV_DEV int budget_of(double keep, int seen, int sink, int recent) {
    const int s = seen > 1 ? seen : 1;
    const int k = (int)rint(keep * (double)s);   // python round(): half to even
    return k > sink + recent ? k : sink + recent;
}

// k-th smallest (0-based) of 64-bit keys over the slots that `pred` accepts,
// by 8-bit radix passes.  All threads of the block call it.
template <typename KeyFn>
DKV_DEV unsigned long long block_select_kth(int hwm, int k, int key_bits, KeyFn key_of,
                                            unsigned* hist, unsigned long long* shared_prefix,
                                            int* shared_k) {
    if (threadIdx.x == 0) {
        *shared_prefix = 0ull;
        *shared_k = k;
    }
    unsigned long long mask = 0ull;
    for (int shift = key_bits - 8; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const unsigned long long prefix = *shared_prefix;
        for (int s = threadIdx.x; s < hwm; s += blockDim.x) {
            unsigned long long key;
            if (key_of(s, &key) && (key & mask) == prefix)
                atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int kk = *shared_k;
            unsigned cum = 0;
            int bin = 0;
            for (; bin < 256; ++bin) {
                if (cum + hist[bin] > (unsigned)kk) break;
                cum += hist[bin];
            }
            *shared_prefix = prefix | ((unsigned long long)bin << shift);
            *shared_k = kk - (int)cum;
        }
        mask |= 255ull << shift;
        __syncthreads();
    }
    return *shared_prefix;
}

// Finds the k-th (1-based) set bit of a 1024-bit map (32 words) with warp 0;
// returns the bit index, or -1 when fewer than k bits are set.
DKV_DEV int kth_set_bit(const uint32_t* bm, int k) {
    const int lane = threadIdx.x & 31;
    int c = __popc(bm[lane]);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (total < k) return -1;
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= k);
    const int wl = __ffs(hit) - 1;
    const int before = __shfl_sync(0xffffffffu, incl - c, wl);
    int need = k - before;
    uint32_t w = bm[wl];
    int bit = -1;
    for (int i = 0; i < 32; ++i) {
        if ((w >> i) & 1u) {
            if (--need == 0) {
                bit = i;
                break;
            }
        }
    }
    return wl * 32 + bit;
}

struct AppendArgs {
    CompView c;
    FullView f;
    const void* src;
    int src_dtype, rows_stride, src_rows_max, raw_dtype;
    const int32_t* pos0;
    const int32_t* n_rows;
    const int32_t* trunc;
    int advance_seen, layer0;
    int stage_pos;          // the slot positions are staged in shared memory
    uint32_t* err;
    LayerCfgs cfg;
};

constexpr int kAppendThreads = 512;
constexpr int kAppendMaxRows = 1024;

// One CTA per (layer, sequence): truncate, append + quantize, evict.
__global__ void __launch_bounds__(kAppendThreads) comp_append_kernel(AppendArgs a) {
    extern __shared__ uint8_t ap_smem[];
    __shared__ int slot_list[kAppendMaxRows];
    __shared__ uint32_t bm_lo[32], bm_hi[32];
    __shared__ __align__(16) unsigned hist[256];   // also read as 64-bit warp partials
    __shared__ unsigned long long sh_prefix;
    __shared__ int sh_k, sh_hwm, sh_n, sh_pmax, sh_plo, sh_phi, sh_free;
    __shared__ unsigned long long sh_min;
    __shared__ int red_i[32];

    pdl_trigger();
    pdl_wait();         // the rows to append come from the previous kernel
    const int li = blockIdx.x, b = blockIdx.y;
    const int L = a.layer0 + li;
    const CompView& c = a.c;
    const int bits = a.cfg.bits[li], sink = a.cfg.sink[li], recent = a.cfg.recent[li];
    const double keep = a.cfg.keep[li];
    const size_t bl = c.bl(b, L);
    int32_t* pos = c.pos + bl * c.cap;
    float* score = c.score + bl * c.cap;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;

    int hwm = c.meta[bl * 4 + 0];
    const int live0 = c.meta[bl * 4 + 1];
    const int trunc = a.trunc ? a.trunc[b] : -1;
    const int R = a.n_rows ? a.n_rows[b] : a.src_rows_max;
    const int p0 = a.pos0 ? a.pos0[b] : 0;
    if (R > kAppendMaxRows || R > a.src_rows_max) {
        if (tid == 0) atomicOr(a.err, 0x10u);
        return;
    }
    // seen: clipped by truncation, advanced to the last appended position + 1
    int seen = c.seen[b];
    if (trunc >= 0 && trunc < seen) seen = trunc;
    if (a.advance_seen && R > 0 && p0 + R > seen) seen = p0 + R;

    // quantize + pack the R new rows into slot_list[0..R) (one warp per K or V vector)
    const int d = c.d;
    auto quantize_rows = [&]() {
        uint8_t* scratch = ap_smem + wid * d;
        const int n_vec = R * c.n_kv * 2;
        const int kb = code_row_bytes(d, bits, a.raw_dtype);
        for (int v = wid; v < n_vec; v += nw) {
            const int r = v / (2 * c.n_kv);
            const int h = (v / 2) % c.n_kv;
            const bool is_k = (v & 1) == 0;
            const int slot = slot_list[r];
            const size_t vi = c.vec(b, L, h, slot);
            uint8_t* dst = (is_k ? c.k_codes : c.v_codes) + c.code_off(b, L, h, slot, kb);
            uint16_t* sl = (is_k ? c.k_sl : c.v_sl) + vi * (d / 64) * 2;
            if (a.src) {
                const size_t off = ((((size_t)b * a.rows_stride + r) * c.n_kv + h) * 2 + (is_k ? 0 : 1)) * d;
                quant_pack_vector(a.src, a.src_dtype, off, d, bits, is_k, dst, sl, a.raw_dtype, scratch);
            } else {
                const size_t off = a.f.elem(b, L, h, p0 + r);
                quant_pack_vector(is_k ? a.f.k_pool : a.f.v_pool, a.f.dtype, off, d, bits, is_k, dst, sl,
                                  a.raw_dtype, scratch);
            }
        }
    };

    // ---- fast path: nothing to truncate, no hole below hwm and keep >= 1
    // (the budget, max(keep * seen, sink + recent), is never below the live
    // count, so nothing is evicted): the rows go to hwm.. and the counts
    // advance by R, exactly what the general path below computes then
    if (trunc < 0 && live0 == hwm && keep >= 1.0) {
        if (hwm + R > c.cap) {
            if (tid == 0) atomicOr(a.err, 0x20u);
            return;
        }
        for (int r = tid; r < R; r += blockDim.x) slot_list[r] = hwm + r;
        __syncthreads();
        quantize_rows();
        for (int r = tid; r < R; r += blockDim.x) {
            pos[hwm + r] = p0 + r;
            score[hwm + r] = 0.f;
        }
        if (tid == 0) {
            c.meta[bl * 4 + 0] = hwm + R;
            c.meta[bl * 4 + 1] = live0 + R;
            if (L == 0 && a.advance_seen) c.seen[b] = seen;
        }
        return;
    }

    // positions of the slot array, staged in shared memory when they fit
    // (every pass below reads them; writes go to both copies)
    int32_t* spos = reinterpret_cast<int32_t*>(ap_smem + (size_t)nw * c.d);
    int32_t* P = a.stage_pos ? spos : pos;
    if (a.stage_pos) {
        // int4 copies, four in flight a thread (pos is 64-byte aligned: cap % 16 == 0)
        const int n4 = (hwm + 3) >> 2, bd = blockDim.x;
        const int4* g4 = reinterpret_cast<const int4*>(pos);
        int4* s4 = reinterpret_cast<int4*>(spos);
        int i = tid;
        for (; i + 3 * bd < n4; i += 4 * bd) {
            int4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcg(g4 + i + u * bd);
#pragma unroll
            for (int u = 0; u < 4; ++u) s4[i + u * bd] = v[u];
        }
        for (; i < n4; i += bd) s4[i] = __ldcg(g4 + i);
        __syncthreads();
    }
    auto setp = [&](int s, int v) {
        pos[s] = v;
        if (a.stage_pos) spos[s] = v;
    };
    if (trunc >= 0) {
        for (int s = tid; s < hwm; s += blockDim.x)
            if (P[s] >= trunc) setp(s, -1);
    }
    __syncthreads();

    // ---- slots for the R new rows: the lowest R empty slots in slot order,
    // then extend hwm.  Warp w counts the empty slots of its contiguous
    // segment; after one barrier each warp knows how many precede it and
    // emits its share in order (rows of 32 slots, ballots, no more barriers).
    {
        const int seg = ((hwm + nw - 1) / nw + 31) / 32 * 32;
        const int w0 = min(hwm, wid * seg), w1 = min(hwm, w0 + seg);
        int cnt = 0;
        if (R > 0) {
            for (int base = w0; base < w1; base += 32) {
                const int s = base + lane;
                cnt += __popc(__ballot_sync(0xffffffffu, s < w1 && P[s] < 0));
            }
        }
        if (lane == 0) red_i[wid] = cnt;
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < nw; ++w) {
            before += w < wid ? red_i[w] : 0;
            total += red_i[w];
        }
        if (cnt > 0 && before < R) {
            int idx = before;
            for (int base = w0; base < w1 && idx < R; base += 32) {
                const int s = base + lane;
                const bool empty = s < w1 && P[s] < 0;
                const unsigned ball = __ballot_sync(0xffffffffu, empty);
                const int my = idx + __popc(ball & ((1u << lane) - 1u));
                if (empty && my < R) slot_list[my] = s;
                idx += __popc(ball);
            }
        }
        if (tid == 0) {
            int f = min(R, total);
            int h2 = hwm;
            while (f < R) slot_list[f++] = h2++;
            sh_hwm = h2;
        }
        __syncthreads();
    }
    hwm = sh_hwm;
    if (hwm > c.cap) {
        if (tid == 0) atomicOr(a.err, 0x20u);
        return;
    }

    // ---- quantize + pack the new rows
    quantize_rows();
    for (int r = tid; r < R; r += blockDim.x) {
        setp(slot_list[r], p0 + r);
        score[slot_list[r]] = 0.f;
    }
    __syncthreads();

    if (R > 0) {
        // ---- eviction (compress.py:159-179)
        for (int i = tid; i < 32; i += blockDim.x) {
            bm_lo[i] = 0;
            bm_hi[i] = 0;
        }
        __syncthreads();
        int n_loc = 0, pmax_loc = -1;
        for (int s = tid; s < hwm; s += blockDim.x) {
            const int p = P[s];
            if (p >= 0) {
                ++n_loc;
                pmax_loc = max(pmax_loc, p);
                if (p < 1024) atomicOr(&bm_lo[p >> 5], 1u << (p & 31));
            }
        }
        n_loc = warp_sum_i(n_loc);
        pmax_loc = warp_max_i(pmax_loc);
        if (lane == 0) red_i[wid] = n_loc;
        __syncthreads();
        if (tid == 0) {
            int t = 0;
            for (int w = 0; w < nw; ++w) t += red_i[w];
            sh_n = t;
        }
        __syncthreads();
        if (lane == 0) red_i[wid] = pmax_loc;
        __syncthreads();
        if (tid == 0) {
            int t = -1;
            for (int w = 0; w < nw; ++w) t = max(t, red_i[w]);
            sh_pmax = t;
        }
        __syncthreads();
        const int n = sh_n, pmax = sh_pmax;
        const int budget = budget_of(keep, seen, sink, recent);
        bool do_evict = n > budget && recent > 0 && recent < n;
        if (do_evict) {
            // sink-th lowest position
            if (wid == 0) {
                int plo = -1;
                if (sink > 0) {
                    plo = kth_set_bit(bm_lo, sink);
                    if (plo < 0) plo = -2;   // fall back to a radix select
                }
                if (lane == 0) sh_plo = plo;
            }
            // recent-th highest position, from a window below pmax
            for (int s = tid; s < hwm; s += blockDim.x) {
                const int p = P[s];
                if (p >= 0 && pmax - p < 1024) atomicOr(&bm_hi[(pmax - p) >> 5], 1u << ((pmax - p) & 31));
            }
            __syncthreads();
            if (wid == 0) {
                int o = kth_set_bit(bm_hi, recent);
                if (lane == 0) sh_phi = o < 0 ? -2 : pmax - o;
            }
            __syncthreads();
            if (sh_plo == -2) {
                auto key = [&](int s, unsigned long long* k) {
                    const int p = P[s];
                    *k = (unsigned long long)(uint32_t)p;
                    return p >= 0;
                };
                unsigned long long v = block_select_kth(hwm, sink - 1, 32, key, hist, &sh_prefix, &sh_k);
                if (tid == 0) sh_plo = (int)v;
                __syncthreads();
            }
            if (sh_phi == -2) {
                auto key = [&](int s, unsigned long long* k) {
                    const int p = P[s];
                    *k = (unsigned long long)(uint32_t)p;
                    return p >= 0;
                };
                unsigned long long v = block_select_kth(hwm, n - recent, 32, key, hist, &sh_prefix, &sh_k);
                if (tid == 0) sh_phi = (int)v;
                __syncthreads();
            }
            const int plo = sh_plo, phi = sh_phi;
            int fr = 0;
            for (int s = tid; s < hwm; s += blockDim.x) {
                const int p = P[s];
                fr += (p > plo && p < phi) ? 1 : 0;
            }
            fr = warp_sum_i(fr);
            __syncthreads();
            if (lane == 0) red_i[wid] = fr;
            __syncthreads();
            if (tid == 0) {
                int t = 0;
                for (int w = 0; w < nw; ++w) t += red_i[w];
                sh_free = t;
            }
            __syncthreads();
            const int drop = min(n - budget, sh_free);
            auto free_key = [&](int s, unsigned long long* k) {
                const int p = P[s];
                *k = ((unsigned long long)__float_as_uint(score[s]) << 32) | (uint32_t)p;
                return p > plo && p < phi;
            };
            if (drop > 0 && drop <= 8) {
                for (int it = 0; it < drop; ++it) {
                    unsigned long long best = ~0ull;
                    {
                        // 4 slots a thread per step (float4 scores), two steps of loads in flight
                        const int n4 = (hwm + 3) >> 2, bd = blockDim.x;
                        const float4* sc4 = reinterpret_cast<const float4*>(score);
                        auto take = [&](int s, float sv) {
                            if (s < hwm) {
                                const int p = P[s];
                                if (p > plo && p < phi) {
                                    const unsigned long long k =
                                        ((unsigned long long)__float_as_uint(sv) << 32) | (uint32_t)p;
                                    if (k < best) best = k;
                                }
                            }
                        };
                        int i = tid;
                        for (; i + bd < n4; i += 2 * bd) {
                            const float4 v0 = __ldcg(sc4 + i), v1 = __ldcg(sc4 + i + bd);
                            take(4 * i, v0.x);
                            take(4 * i + 1, v0.y);
                            take(4 * i + 2, v0.z);
                            take(4 * i + 3, v0.w);
                            take(4 * (i + bd), v1.x);
                            take(4 * (i + bd) + 1, v1.y);
                            take(4 * (i + bd) + 2, v1.z);
                            take(4 * (i + bd) + 3, v1.w);
                        }
                        for (; i < n4; i += bd) {
                            const float4 v0 = __ldcg(sc4 + i);
                            take(4 * i, v0.x);
                            take(4 * i + 1, v0.y);
                            take(4 * i + 2, v0.z);
                            take(4 * i + 3, v0.w);
                        }
                    }
                    best = warp_min_u64(best);
                    __syncthreads();
                    if (lane == 0) reinterpret_cast<unsigned long long*>(hist)[wid] = best;
                    __syncthreads();
                    if (tid == 0) {
                        unsigned long long m = ~0ull;
                        for (int w = 0; w < nw; ++w) {
                            unsigned long long t = reinterpret_cast<unsigned long long*>(hist)[w];
                            m = t < m ? t : m;
                        }
                        sh_min = m;
                    }
                    __syncthreads();
                    const unsigned long long m = sh_min;
                    if (m != ~0ull) {
                        // live positions are unique: the key's low word names the slot
                        const int pm = (int)(uint32_t)m;
                        for (int s = tid; s < hwm; s += blockDim.x)
                            if (P[s] == pm) setp(s, -1);
                    }
                    __syncthreads();
                }
            } else if (drop > 8) {
                const unsigned long long thr = block_select_kth(hwm, drop - 1, 64, free_key, hist, &sh_prefix, &sh_k);
                __syncthreads();
                for (int s = tid; s < hwm; s += blockDim.x) {
                    unsigned long long k;
                    if (free_key(s, &k) && k <= thr) setp(s, -1);
                }
                __syncthreads();
            }
        }
    }
    // ---- shrink hwm to the last live slot, recount
    __syncthreads();
    int last = -1, cnt = 0;
    for (int s = tid; s < hwm; s += blockDim.x)
        if (P[s] >= 0) {
            last = max(last, s);
            ++cnt;
        }
    last = warp_max_i(last);
    cnt = warp_sum_i(cnt);
    __syncthreads();
    if (lane == 0) {
        red_i[wid] = last;
    }
    __syncthreads();
    if (tid == 0) {
        int t = -1;
        for (int w = 0; w < nw; ++w) t = max(t, red_i[w]);
        sh_hwm = t + 1;
    }
    __syncthreads();
    if (lane == 0) red_i[wid] = cnt;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int w = 0; w < nw; ++w) t += red_i[w];
        c.meta[bl * 4 + 0] = sh_hwm;
        c.meta[bl * 4 + 1] = t;
        if (L == 0 && a.advance_seen) c.seen[b] = seen;
        else if (L == 0 && trunc >= 0) c.seen[b] = seen;
    }
}

// Rebuild: clear the layer and refill it from the full cache with the rows
// that survive eviction when every score is zero (sink rows + newest rows).
struct RebuildArgs {
    CompView c;
    FullView f;
    const int32_t* ctx;
    uint32_t* err;
    int raw_dtype, advance_seen, rows_per_cta;
    int layer_ids[128];
    LayerCfgs cfg;
};

DKV_DEV void rebuild_plan(const RebuildArgs& a, int li, int b, int* kept, int* gap_at, int* gap_len,
                          int* seen_out) {
    const int n = a.ctx[b];
    int seen = a.c.seen[b];
    if (a.advance_seen && n > seen) seen = n;
    const int sink = a.cfg.sink[li], recent = a.cfg.recent[li];
    const int budget = budget_of(a.cfg.keep[li], seen, sink, recent);
    *seen_out = seen;
    if (n <= budget || recent <= 0) {
        *kept = n;
        *gap_at = n;
        *gap_len = 0;
        return;
    }
    const int s0 = min(sink, n);
    const int n_drop = n - budget;
    *kept = n - n_drop;
    *gap_at = s0;
    *gap_len = n_drop;
}

__global__ void comp_rebuild_kernel(RebuildArgs a) {
    extern __shared__ uint8_t rb_smem[];
    const int li = blockIdx.y, b = blockIdx.z;
    const int L = a.layer_ids[li];
    const CompView& c = a.c;
    int kept, gap_at, gap_len, seen;
    rebuild_plan(a, li, b, &kept, &gap_at, &gap_len, &seen);
    const size_t bl = c.bl(b, L);
    const int bits = a.cfg.bits[li];
    if (kept > c.cap) {   // the caller sized the slot array too small: report, write nothing
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.err, 0x20u);
        return;
    }
    // every chunk of [0, cap) is visited: live slots get their position,
    // the rest are cleared (no CTA depends on the old high-water mark)
    const int r0 = blockIdx.x * a.rows_per_cta;
    if (r0 >= c.cap) return;
    const int r1 = min(r0 + a.rows_per_cta, c.cap);
    const int wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int s = r0 + threadIdx.x; s < r1; s += blockDim.x) {
        if (s < kept) {
            c.pos[bl * c.cap + s] = s < gap_at ? s : s + gap_len;
            c.score[bl * c.cap + s] = 0.f;
        } else {
            c.pos[bl * c.cap + s] = -1;
        }
    }
    const int d = c.d;
    const int rq1 = min(r1, kept);
    const int n_vec = (rq1 > r0 ? rq1 - r0 : 0) * c.n_kv * 2;
    uint8_t* scratch = rb_smem + wid * d;
    for (int v = wid; v < n_vec; v += nw) {
        const int s = r0 + v / (2 * c.n_kv);
        const int h = (v / 2) % c.n_kv;
        const bool is_k = (v & 1) == 0;
        const int p = s < gap_at ? s : s + gap_len;
        const size_t vi = c.vec(b, L, h, s);
        quant_pack_vector(is_k ? a.f.k_pool : a.f.v_pool, a.f.dtype, a.f.elem(b, L, h, p), d, bits, is_k,
                          (is_k ? c.k_codes : c.v_codes) + c.code_off(b, L, h, s, code_row_bytes(d, bits, a.raw_dtype)),
                          (is_k ? c.k_sl : c.v_sl) + vi * (d / 64) * 2, a.raw_dtype, scratch);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        c.meta[bl * 4 + 0] = kept;
        c.meta[bl * 4 + 1] = kept;
    }
}

// Rebuild for d % 64 == 0: same plan and slot assignment as
// comp_rebuild_kernel; vectors are quantized lane-sliced, d/16 lanes per
// vector, consecutive vectors of a warp being consecutive slots of one
// (head, K/V) so the loads stream whole rows of the paged cache.  Two vector
// groups are loaded before either is packed.
__global__ void __launch_bounds__(256) comp_rebuild_slice_kernel(RebuildArgs a) {
    const int li = blockIdx.y, b = blockIdx.z;
    const int L = a.layer_ids[li];
    const CompView& c = a.c;
    int kept, gap_at, gap_len, seen;
    rebuild_plan(a, li, b, &kept, &gap_at, &gap_len, &seen);
    const size_t bl = c.bl(b, L);
    const int bits = a.cfg.bits[li];
    if (kept > c.cap) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.err, 0x20u);
        return;
    }
    const int r0 = blockIdx.x * a.rows_per_cta;
    if (r0 >= c.cap) return;
    const int r1 = min(r0 + a.rows_per_cta, c.cap);
    for (int s = r0 + threadIdx.x; s < r1; s += blockDim.x) {
        if (s < kept) {
            c.pos[bl * c.cap + s] = s < gap_at ? s : s + gap_len;
            c.score[bl * c.cap + s] = 0.f;
        } else {
            c.pos[bl * c.cap + s] = -1;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        c.meta[bl * 4 + 0] = kept;
        c.meta[bl * 4 + 1] = kept;
    }
    const int d = c.d, lpv = d >> 4, vpw = 32 / lpv;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int sub = lane / lpv, j = lane % lpv;
    const int rq1 = min(r1, kept);
    const int nslot = rq1 > r0 ? rq1 - r0 : 0;
    const int n_vec = nslot * c.n_kv * 2;
    const int sl_stride = (d / 64) * 2;
    for (int base = wid * vpw; base < n_vec; base += 2 * nw * vpw) {     // uniform per warp
        float x[2][16];
        int vix[2];
        bool act[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int v = base + u * nw * vpw + sub;
            act[u] = v < n_vec;
            vix[u] = act[u] ? v : base;
            const int s = r0 + vix[u] % nslot, hk = vix[u] / nslot;
            const bool is_k = hk < c.n_kv;
            const int h = is_k ? hk : hk - c.n_kv;
            const int p = s < gap_at ? s : s + gap_len;
            load_slice(is_k ? a.f.k_pool : a.f.v_pool, a.f.dtype, a.f.elem(b, L, h, p) + 16 * j, x[u]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (base + u * nw * vpw >= n_vec) break;           // uniform per warp
            const int s = r0 + vix[u] % nslot, hk = vix[u] / nslot;
            const bool is_k = hk < c.n_kv;
            const int h = is_k ? hk : hk - c.n_kv;
            const size_t vi = c.vec(b, L, h, s);
            quant_pack_slice(x[u], j, d, bits, is_k, act[u],
                             (is_k ? c.k_codes : c.v_codes) + c.code_off(b, L, h, s, code_row_bytes(d, bits, a.raw_dtype)),
                             (is_k ? c.k_sl : c.v_sl) + vi * sl_stride, a.raw_dtype);
        }
    }
}

// seen update after a rebuild (one thread per sequence)
__global__ void comp_seen_kernel(int32_t* seen, const int32_t* ctx, int batch, int advance, int trunc_zero) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= batch) return;
    int s = seen[b];
    if (trunc_zero) s = 0;
    if (advance && ctx[b] > s) s = ctx[b];
    seen[b] = s;
}

// Read-back (tests): every slot of [0, n_slots) in slot order, dequantized,
// with its position (-1 = empty) and score; the caller sorts by position.
__global__ void comp_read_kernel(CompView c, int b, int L, int bits, int raw_dtype, int n_slots,
                                 float* k, float* v, int32_t* pos_out, float* score_out) {
    const int slot = blockIdx.x;
    if (slot >= n_slots) return;
    const size_t bl = c.bl(b, L);
    const int p = c.pos[bl * c.cap + slot];
    if (threadIdx.x == 0) {
        pos_out[slot] = p;
        if (score_out) score_out[slot] = c.score[bl * c.cap + slot];
    }
    const int d = c.d;
    for (int t = threadIdx.x; t < c.n_kv * d; t += blockDim.x) {
        const int h = t / d, e = t % d;
        const size_t vi = c.vec(b, L, h, slot);
        float kv = 0.f, vv = 0.f;
        if (p >= 0) {
            const size_t co = c.code_off(b, L, h, slot, code_row_bytes(d, bits, raw_dtype));
            kv = dequant_elem(c.k_codes + co, c.k_sl + vi * (d / 64) * 2, d, bits, true, e, raw_dtype);
            vv = dequant_elem(c.v_codes + co, c.v_sl + vi * (d / 64) * 2, d, bits, false, e, raw_dtype);
        }
        k[((size_t)slot * c.n_kv + h) * d + e] = kv;
        v[((size_t)slot * c.n_kv + h) * d + e] = vv;
    }
}

// ------------------------------------------------------------------ full cache
__global__ void full_write_kernel(FullView f, int L, const void* src, int rows, const int32_t* pos0,
                                  const int32_t* n_rows) {
    const int b = blockIdx.y, r = blockIdx.x;
    const int nr = n_rows ? n_rows[b] : rows;
    if (r >= nr) return;
    const int p = pos0[b] + r;
    for (int t = threadIdx.x; t < f.n_kv * f.d * 2; t += blockDim.x) {
        const int kv = t / (f.n_kv * f.d);
        const int h = (t / f.d) % f.n_kv, e = t % f.d;
        const size_t si = ((((size_t)b * rows + r) * f.n_kv + h) * 2 + kv) * f.d + e;
        const float val = load_as_f32(src, f.dtype, si);
        store_from_f32(const_cast<void*>(kv ? f.v_pool : f.k_pool), f.dtype, f.elem(b, L, h, p) + e, val);
    }
}

__global__ void full_read_kernel(FullView f, int b, int L, int n, void* dst) {
    const int r = blockIdx.x;
    if (r >= n) return;
    for (int t = threadIdx.x; t < f.n_kv * f.d * 2; t += blockDim.x) {
        const int kv = t / (f.n_kv * f.d);
        const int h = (t / f.d) % f.n_kv, e = t % f.d;
        const float val = load_as_f32(kv ? f.v_pool : f.k_pool, f.dtype, f.elem(b, L, h, r) + e);
        store_from_f32(dst, f.dtype, (((size_t)r * f.n_kv + h) * 2 + kv) * f.d + e, val);
    }
}

// --------------------------------------------------------------------------
// host side
CompView comp_view(const dkv_comp_cache* c, dkv_dims dims) {
    CompView v;
    v.k_codes = c->k_codes;
    v.v_codes = c->v_codes;
    v.k_sl = c->k_sl;
    v.v_sl = c->v_sl;
    v.pos = c->pos;
    v.score = c->score;
    v.meta = c->meta;
    v.seen = c->seen;
    v.cap = c->cap;
    v.cb_max = c->cb_max;
    v.n_layers = dims.n_layers;
    v.n_kv = dims.n_kv;
    v.d = dims.d;
    return v;
}

FullView full_view(const dkv_full_cache* f, dkv_dims dims) {
    FullView v;
    v.k_pool = f ? f->k_pool : nullptr;
    v.v_pool = f ? f->v_pool : nullptr;
    v.page_table = f ? f->page_table : nullptr;
    v.page_size = f ? f->page_size : 16;
    v.max_pages = f ? f->max_pages : 0;
    v.dtype = f ? f->dtype : DKV_BF16;
    v.n_layers = dims.n_layers;
    v.n_kv = dims.n_kv;
    v.d = dims.d;
    return v;
}

uint32_t* device_error_word();

}  // namespace dkv

using namespace dkv;

extern "C" int dkv_quantize(const float* x, int64_t rows, int d, int bits, uint8_t* codes,
                            float* scale, float* lo, float* deq, void* stream) {
    DKV_REQUIRE(x != nullptr && rows >= 0 && d > 0, "dkv_quantize: bad arguments");
    DKV_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 8 || bits == 16,
                "dkv_quantize: unsupported bits=%d", bits);
    if (rows == 0) return DKV_OK;
    const int ng = (d + 63) / 64;
    const int64_t warps = rows * ng;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    quantize_exact_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(x, rows, d, bits, codes,
                                                                                  scale, lo, deq);
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" int dkv_quantize_pack(const void* src, int src_dtype, int64_t rows, int d, int bits,
                                 int k_order, uint8_t* codes, uint16_t* sl, void* stream) {
    DKV_REQUIRE(src && codes && sl && rows >= 0, "dkv_quantize_pack: bad arguments");
    DKV_REQUIRE(d % 64 == 0 && d <= 256, "dkv_quantize_pack: d must be 64, 128 or 256 (got %d)", d);
    DKV_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 8 || bits == 16, "bad bits %d", bits);
    if (rows == 0) return DKV_OK;
    const int rows_per_block = 8 * (32 / (d >> 4));     // 8 warps
    quantize_pack_slice_kernel<<<(unsigned)((rows + rows_per_block - 1) / rows_per_block), 256, 0,
                                 (cudaStream_t)stream>>>(src, src_dtype, rows, d, bits, k_order != 0, codes, sl);
    DKV_LAUNCHED();
    return DKV_OK;
}

static int fill_cfgs(const dkv_comp_cache* c, const int32_t* layers, int n_sel, int layer0, int d, int raw_elem,
                     LayerCfgs* out) {
    DKV_REQUIRE(n_sel > 0 && n_sel <= 128, "at most 128 layers per call (got %d)", n_sel);
    DKV_REQUIRE(c->bits && c->keep && c->sink && c->recent, "per-layer config arrays are required");
    out->n = n_sel;
    for (int i = 0; i < n_sel; ++i) {
        const int L = layers ? layers[i] : layer0 + i;
        const int bits = c->bits[L];
        DKV_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 8 || bits == 16, "layer %d: bits %d", L, bits);
        const int cb = bits == 16 ? d * raw_elem : d * bits / 8;
        DKV_REQUIRE(cb <= c->cb_max, "layer %d: %d-bit vectors need %d bytes > cb_max %d", L, bits, cb, c->cb_max);
        DKV_REQUIRE(c->keep[L] > 0.0 && c->keep[L] <= 1.0, "layer %d: keep %f", L, c->keep[L]);
        DKV_REQUIRE(c->sink[L] >= 0 && c->recent[L] >= 0, "layer %d: sink/recent", L);
        out->bits[i] = bits;
        out->keep[i] = c->keep[L];
        out->sink[i] = c->sink[L];
        out->recent[i] = c->recent[L];
    }
    return DKV_OK;
}

static int check_comp(const dkv_comp_cache* c, dkv_dims dims, int raw_elem) {
    DKV_REQUIRE(c && c->k_codes && c->v_codes && c->k_sl && c->v_sl && c->pos && c->score && c->meta &&
                    c->seen,
                "drafter cache pointers must be set");
    DKV_REQUIRE(dims.d % 64 == 0 && dims.d <= 256, "head dim %d unsupported (64/128/256)", dims.d);
    (void)raw_elem;   // per-layer widths are checked against cb_max in fill_cfgs
    DKV_REQUIRE(c->cb_max >= dims.d * 2 / 8, "cb_max %d below the 2-bit width", c->cb_max);
    DKV_REQUIRE(c->cap > 0, "cap must be positive");
    return DKV_OK;
}

extern "C" int dkv_comp_append(const dkv_comp_cache* comp, const dkv_full_cache* full, dkv_dims dims,
                               int layer0, int n_layer_sel, const void* src, int src_dtype, int rows_stride,
                               const int32_t* pos0, const int32_t* n_rows, const int32_t* trunc,
                               int advance_seen, void* stream) {
    const int raw_dtype = full ? full->dtype : src_dtype;
    DKV_TRY(check_comp(comp, dims, raw_dtype == DKV_F32 ? 4 : 2));
    DKV_REQUIRE(layer0 >= 0 && layer0 + n_layer_sel <= dims.n_layers, "layer range");
    DKV_REQUIRE(rows_stride >= 0 && rows_stride <= kAppendMaxRows, "rows_stride %d > %d", rows_stride,
                kAppendMaxRows);
    DKV_REQUIRE(rows_stride == 0 || src != nullptr || (full && full->k_pool && full->page_table),
                "dkv_comp_append: rows to append but no row source");
    AppendArgs a;
    a.c = comp_view(comp, dims);
    a.f = full_view(full, dims);
    a.src = src;
    a.src_dtype = src_dtype;
    a.rows_stride = rows_stride;
    a.src_rows_max = rows_stride;
    a.raw_dtype = raw_dtype;
    a.pos0 = pos0;
    a.n_rows = n_rows;
    a.trunc = trunc;
    a.advance_seen = advance_seen;
    a.layer0 = layer0;
    a.err = device_error_word();
    DKV_TRY(fill_cfgs(comp, nullptr, n_layer_sel, layer0, dims.d, raw_dtype == DKV_F32 ? 4 : 2, &a.cfg));
    // quantization scratch, plus the slot positions when they fit
    DKV_CUDA(allow_smem_max_once<comp_append_kernel>());
    size_t smem_cap = 0;
    {
        int dev = 0, optin = 0;
        DKV_CUDA(cudaGetDevice(&dev));
        DKV_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        cudaFuncAttributes fa;
        DKV_CUDA(cudaFuncGetAttributes(&fa, comp_append_kernel));
        smem_cap = (size_t)optin - fa.sharedSizeBytes;
    }
    size_t smem = (kAppendThreads / 32) * dims.d;
    a.stage_pos = smem + (size_t)comp->cap * sizeof(int32_t) <= smem_cap;
    if (a.stage_pos) smem += (size_t)comp->cap * sizeof(int32_t);
    dim3 grid(n_layer_sel, dims.batch);
    ProfScope ps(DKV_PROF_APPEND, 0.0, (cudaStream_t)stream);
    DKV_CUDA(launch_pdl(comp_append_kernel, grid, dim3(kAppendThreads), smem, (cudaStream_t)stream, a));
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" int dkv_comp_rebuild(const dkv_comp_cache* comp, const dkv_full_cache* full, dkv_dims dims,
                                const int32_t* layers, int n_sel, const int32_t* ctx, int advance_seen,
                                void* stream) {
    DKV_REQUIRE(full && full->k_pool && full->page_table, "rebuild needs the full cache");
    DKV_TRY(check_comp(comp, dims, full->dtype == DKV_F32 ? 4 : 2));
    DKV_REQUIRE(layers && ctx, "layers / ctx required");
    RebuildArgs a;
    a.c = comp_view(comp, dims);
    a.f = full_view(full, dims);
    a.ctx = ctx;
    a.err = device_error_word();
    a.raw_dtype = full->dtype;
    a.advance_seen = advance_seen;
    a.rows_per_cta = 64;
    DKV_TRY(fill_cfgs(comp, layers, n_sel, 0, dims.d, full->dtype == DKV_F32 ? 4 : 2, &a.cfg));
    for (int i = 0; i < n_sel; ++i) {
        DKV_REQUIRE(layers[i] >= 0 && layers[i] < dims.n_layers, "layer id %d", layers[i]);
        a.layer_ids[i] = layers[i];
    }
    const int warps = 8;
    dim3 grid((comp->cap + a.rows_per_cta - 1) / a.rows_per_cta, n_sel, dims.batch);
    {
        ProfScope ps(DKV_PROF_REBUILD, 0.0, (cudaStream_t)stream);
        if (dims.d % 64 == 0 && dims.d <= 512)
            comp_rebuild_slice_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(a);
        else
            comp_rebuild_kernel<<<grid, warps * 32, warps * dims.d, (cudaStream_t)stream>>>(a);
    }
    DKV_LAUNCHED();
    // the layer-0 rebuild advances `seen` (compress.py:131-132); done after all
    // CTAs read it, in stream order
    bool has0 = false;
    for (int i = 0; i < n_sel; ++i) has0 |= layers[i] == 0;
    if (has0 && advance_seen) {
        comp_seen_kernel<<<(dims.batch + 127) / 128, 128, 0, (cudaStream_t)stream>>>(comp->seen, ctx, dims.batch,
                                                                                     1, 0);
        DKV_LAUNCHED();
    }
    return DKV_OK;
}

extern "C" int dkv_comp_read(const dkv_comp_cache* comp, dkv_dims dims, int b, int layer, int max_n,
                             float* k, float* v, int32_t* pos, float* score, int* n_out, void* stream) {
    DKV_REQUIRE(comp && k && v && pos && n_out && comp->bits, "dkv_comp_read: bad arguments");
    DKV_REQUIRE(b >= 0 && b < dims.batch && layer >= 0 && layer < dims.n_layers, "dkv_comp_read: index");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t bl = (size_t)b * dims.n_layers + layer;
    int meta[4];
    DKV_CUDA(cudaMemcpyAsync(meta, comp->meta + bl * 4, sizeof(meta), cudaMemcpyDeviceToHost, st));
    DKV_CUDA(cudaStreamSynchronize(st));
    const int hwm = meta[0];
    *n_out = hwm;
    DKV_REQUIRE(hwm <= max_n, "dkv_comp_read: %d slots > max_n %d", hwm, max_n);
    if (hwm == 0) return DKV_OK;
    const int raw_dtype = comp->cb_max >= dims.d * 4 ? DKV_F32 : DKV_BF16;
    comp_read_kernel<<<hwm, 256, 0, st>>>(comp_view(comp, dims), b, layer, comp->bits[layer], raw_dtype, hwm, k,
                                          v, pos, score);
    DKV_LAUNCHED();
    DKV_CUDA(cudaStreamSynchronize(st));
    return DKV_OK;
}

extern "C" int dkv_full_write(const dkv_full_cache* full, dkv_dims dims, int layer, const void* src, int rows,
                              const int32_t* pos0, const int32_t* n_rows, void* stream) {
    DKV_REQUIRE(full && full->k_pool && full->v_pool && full->page_table && src && pos0, "dkv_full_write args");
    DKV_REQUIRE(layer >= 0 && layer < dims.n_layers && rows >= 0, "dkv_full_write: layer/rows");
    if (rows == 0) return DKV_OK;
    FullView f = full_view(full, dims);
    full_write_kernel<<<dim3(rows, dims.batch), 256, 0, (cudaStream_t)stream>>>(f, layer, src, rows, pos0, n_rows);
    DKV_LAUNCHED();
    return DKV_OK;
}

extern "C" int dkv_full_read(const dkv_full_cache* full, dkv_dims dims, int b, int layer, int n, void* dst,
                             void* stream) {
    DKV_REQUIRE(full && full->k_pool && dst && n >= 0, "dkv_full_read args");
    if (n == 0) return DKV_OK;
    FullView f = full_view(full, dims);
    full_read_kernel<<<n, 256, 0, (cudaStream_t)stream>>>(f, b, layer, n, dst);
    DKV_LAUNCHED();
    return DKV_OK;
}
