// Tensor-core drafter attention over the quantized slot cache (T = 1).
//
// Replaces, for a draft step, draftkv/llama.py:202-219 with cache =
// CompressedKVCache (read :135-142) plus note_attention
// (draftkv/compress.py:144-151) summed over the GQA group
// (draftkv/llama.py:213-216).
//
// One thread-block cluster of CS CTAs per (sequence, KV head); CTA r of the
// cluster takes a contiguous 1/CS of the live slot range.  Its 8 warps walk
// 16-slot tiles:
//   S^T = Q K^T  with mma.m16n8k16: A = the group's queries (rows = heads,
//                padded to 16), B = K read straight from the packed codes
//                -- the K storage order puts each thread's fragment elements
//                in one contiguous segment, so codes go register-direct to
//                f16 (c, exact), and per group s = scale*S + lo*sum(q);
//   O^T += V^T P^T  with V dequantized to f16 (c*scale + lo) in a per-warp
//                swizzled shared tile read by ldmatrix.trans, and P from the
//                S^T accumulators.
// Raw scores stay in shared memory; after an online-softmax merge across the
// warps, the cluster exchanges (max, sum) through distributed shared memory,
// each CTA writes its share of the output and the exact attention mass of its
// slots, and the last of the n_kv clusters to finish a slot range folds the
// per-head masses into the slot scores in head order (atomic ticket, no wait).
#include <cooperative_groups.h>

#include "attn_common.cuh"

namespace cg = cooperative_groups;

namespace dkv {

DKV_DEV uint32_t pk_f16(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
DKV_DEV uint32_t pk_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

template <bool BF>
DKV_DEV void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if (BF) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

DKV_DEV void ldsm4t_(uint32_t (&r)[4], const void* p) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s));
}

// half2 of two integer codes (exact small integers).
DKV_DEV uint32_t codes_to_h2(uint32_t pair_bits) {
    const uint32_t biased = pair_bits | 0x64006400u;               // 1024 + c in each f16 lane
    __half2 v = *reinterpret_cast<const __half2*>(&biased);
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
    v = __hsub2(v, k1024);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Code pair q (0-based, pairs of consecutive storage positions) of a packed
// segment held in registers.  `w` holds the segment's 32-bit words; for 3 bits
// `w` holds plane-A words and `u` plane-B 16-bit units.
template <int BITS>
DKV_DEV uint32_t pair_bits(const uint32_t* w, const uint16_t* u, int q) {
    if (BITS == 4) return (w[q >> 2] >> (4 * (q & 3))) & 0x000F000Fu;
    if (BITS == 2) return (w[q >> 3] >> (2 * (q & 7))) & 0x00030003u;
    if (BITS == 8) {
        const uint32_t x = w[q >> 1];
        return (q & 1) ? (((x >> 16) & 0xFFu) | ((x >> 8) & 0xFF0000u)) : ((x & 0xFFu) | ((x << 8) & 0xFF0000u));
    }
    // 3 bits
    const uint32_t lo2 = (w[q >> 3] >> (2 * (q & 7))) & 0x00030003u;
    const uint32_t un = u[q >> 3];
    const uint32_t x = (un & 0xFFu) | ((un & 0xFF00u) << 8);
    const uint32_t hb = (x >> (q & 7)) & 0x00010001u;
    return lo2 | (hb << 2);
}

constexpr int kDraftWarps = 8;
constexpr int kDraftThreads = kDraftWarps * 32;

struct DraftArgs {
    AttnArgs a;
    int cs;                 // cluster size (CTAs per (sequence, head))
    int chunk_cap;          // slots per CTA the shared memory holds
    int raw_dtype;          // dtype of 16-bit entries
    uint32_t* tickets;      // comp->tickets [batch][n_layers][64]
    uint32_t* err;
};

// Segment of quad c of a packed vector: bytes [c*D*BITS/32, ...), plus for 3
// bits the plane-B units at D/4 + c*D/32.
template <int D, int BITS>
DKV_DEV void load_k_segment(const uint8_t* vec, int c, uint32_t* w, uint16_t* u) {
    if (BITS == 16) {
        const uint4* p = reinterpret_cast<const uint4*>(vec + c * (D / 2));
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            const uint4 v = __ldg(p + i);
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    } else if (BITS == 3) {
        const uint32_t* pa = reinterpret_cast<const uint32_t*>(vec + c * (D / 16));
#pragma unroll
        for (int i = 0; i < D / 64; ++i) w[i] = __ldg(pa + i);
        const uint16_t* pb = reinterpret_cast<const uint16_t*>(vec + D / 4 + c * (D / 32));
#pragma unroll
        for (int i = 0; i < D / 64; ++i) u[i] = __ldg(pb + i);
    } else {
        constexpr int SEGB = D * BITS / 32;     // bytes per quad segment
        const uint32_t* p = reinterpret_cast<const uint32_t*>(vec + c * SEGB);
#pragma unroll
        for (int i = 0; i < SEGB / 4; ++i) w[i] = __ldg(p + i);
    }
}

template <int D, int BITS>
__global__ void __launch_bounds__(kDraftThreads) attn_draft_tc_kernel(DraftArgs da) {
    constexpr bool RAW = BITS == 16;
    constexpr int KS = D / 16;              // k16 steps over d
    constexpr int NG = D / 64;              // quantization groups
    constexpr int SEGW = RAW ? D / 8 : (BITS == 3 ? D / 64 : D * BITS / 128);   // words per quad segment
    const AttnArgs& a = da.a;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.y, b = blockIdx.z;
    const int G = a.group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qr = lane >> 2, qc = lane & 3;
    const KeySrc& src = a.src;
    const size_t bl = (size_t)b * a.n_layers + a.layer;
    const int hwm = src.meta[bl * 4 + 0];
    const int per = (hwm + da.cs - 1) / da.cs;
    const int chunk = (per + 15) / 16 * 16;
    const int s0 = min(rank * chunk, hwm), s1 = min(s0 + chunk, hwm);
    const int qpos = a.qpos0[b];
    const int HQ = a.n_kv * G;

    extern __shared__ __align__(128) uint8_t dsm[];
    float* sbuf = reinterpret_cast<float*>(dsm);                            // [G][chunk_cap]
    uint16_t* vtile = reinterpret_cast<uint16_t*>(sbuf + (size_t)G * da.chunk_cap);   // [warps][16][D]
    float* cta_m = reinterpret_cast<float*>(vtile + kDraftWarps * 16 * D);  // [8]
    float* cta_l = cta_m + 8;                                               // [8]
    float* cta_o = cta_l + 8;                                               // [8][D]
    float* glob_m = cta_o + 8 * D;                                          // [8]
    float* glob_l = glob_m + 8;                                             // [8]
    uint16_t* vt = vtile + warp * 16 * D;

    if (chunk > da.chunk_cap) {       // host sized the launch; never expected
        if (threadIdx.x == 0) atomicOr(da.err, 0x40u);
    }

    // ---- queries of head qr (rows >= G and the upper 8 rows are zero)
    const bool qrow = qr < G;
    const float* qv = a.q + ((size_t)b * HQ + h * G + (qrow ? qr : 0)) * D;
    uint32_t qa[KS][4];
    float qsum[NG] = {};
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        const int d0 = kk * 16 + 2 * qc;
        float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
        if (qrow) {
            x0 = qv[d0] * a.scale;
            x1 = qv[d0 + 1] * a.scale;
            x2 = qv[d0 + 8] * a.scale;
            x3 = qv[d0 + 9] * a.scale;
        }
        if (RAW && src.dtype == DKV_BF16) {
            qa[kk][0] = pk_bf16(x0, x1);
            qa[kk][2] = pk_bf16(x2, x3);
        } else {
            qa[kk][0] = pk_f16(x0, x1);
            qa[kk][2] = pk_f16(x2, x3);
            // sum of the f16-rounded scaled queries per group (for the lo term)
            const __half2 h01 = *reinterpret_cast<__half2*>(&qa[kk][0]);
            const __half2 h23 = *reinterpret_cast<__half2*>(&qa[kk][2]);
            qsum[kk / 4] += __low2float(h01) + __high2float(h01) + __low2float(h23) + __high2float(h23);
        }
        qa[kk][1] = 0u;
        qa[kk][3] = 0u;
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 1);
        qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 2);
    }

    float m_run = -INFINITY, l_run = 0.f;    // stats of head qr
    float oacc[KS][4];                       // O^T: rows d = 16md + qr (+8), cols heads 2qc, 2qc+1
#pragma unroll
    for (int md = 0; md < KS; ++md) oacc[md][0] = oacc[md][1] = oacc[md][2] = oacc[md][3] = 0.f;

    const uint8_t* kbase = src.k_codes + (bl * a.n_kv + h) * (size_t)src.cap * src.cb_max;
    const uint8_t* vbase = src.v_codes + (bl * a.n_kv + h) * (size_t)src.cap * src.cb_max;
    const uint16_t* ksl = src.k_sl + (bl * a.n_kv + h) * (size_t)src.cap * NG * 2;
    const uint16_t* vsl = src.v_sl + (bl * a.n_kv + h) * (size_t)src.cap * NG * 2;
    const int32_t* cpos = src.cpos + bl * src.cap;

    const int first_tile = s0 / 16;
    const int n_tiles = s1 > s0 ? (s1 - 1) / 16 - first_tile + 1 : 0;
    for (int tt = warp; tt < n_tiles; tt += kDraftWarps) {
        const int base = (first_tile + tt) * 16;
        // ---- K: register-direct B fragments of slots base+qr and base+8+qr
        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        {
            uint32_t w0[SEGW > 0 ? SEGW : 1], w1[SEGW > 0 ? SEGW : 1];
            uint16_t u0[D / 64 > 0 ? D / 64 : 1], u1[D / 64 > 0 ? D / 64 : 1];
            const int sa = base + qr, sb = base + 8 + qr;
            load_k_segment<D, BITS>(kbase + (size_t)min(sa, src.cap - 1) * src.cb_max, qc, w0, u0);
            load_k_segment<D, BITS>(kbase + (size_t)min(sb, src.cap - 1) * src.cb_max, qc, w1, u1);
            if (RAW) {
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    mma16816<true>(sc[0], qa[kk], w0[2 * kk], w0[2 * kk + 1]);
                    mma16816<true>(sc[1], qa[kk], w1[2 * kk], w1[2 * kk + 1]);
                }
            } else {
                float gs[NG][2][4];
#pragma unroll
                for (int g = 0; g < NG; ++g)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) gs[g][nt][0] = gs[g][nt][1] = gs[g][nt][2] = gs[g][nt][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t b00 = codes_to_h2(pair_bits<BITS>(w0, u0, 2 * kk));
                    const uint32_t b01 = codes_to_h2(pair_bits<BITS>(w0, u0, 2 * kk + 1));
                    const uint32_t b10 = codes_to_h2(pair_bits<BITS>(w1, u1, 2 * kk));
                    const uint32_t b11 = codes_to_h2(pair_bits<BITS>(w1, u1, 2 * kk + 1));
                    mma16816<false>(gs[kk / 4][0], qa[kk], b00, b01);
                    mma16816<false>(gs[kk / 4][1], qa[kk], b10, b11);
                }
                // per-slot group scale / lo: this thread's columns are slots
                // base + 8nt + 2qc (+1)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const int sl = base + 8 * nt + 2 * qc;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int slot = min(sl + e, src.cap - 1);
                        float acc = 0.f;
#pragma unroll
                        for (int g = 0; g < NG; ++g) {
                            const float scl = half_bits_to_f32(__ldg(ksl + ((size_t)slot * NG + g) * 2));
                            const float lo = half_bits_to_f32(__ldg(ksl + ((size_t)slot * NG + g) * 2 + 1));
                            acc += scl * gs[g][nt][e] + lo * qsum[g];
                        }
                        sc[nt][e] = acc;
                    }
                }
            }
        }
        // ---- mask (empty slot, outside this CTA's range, future position)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int slot = base + 8 * nt + 2 * qc + e;
                bool ok = slot >= s0 && slot < s1 && qrow;
                if (ok) {
                    const int p = __ldg(cpos + slot);
                    ok = p >= 0 && p <= qpos;
                }
                if (!ok) sc[nt][e] = -INFINITY;
                if (qrow && slot >= s0 && slot < s1 && slot - s0 < da.chunk_cap)
                    sbuf[(size_t)qr * da.chunk_cap + (slot - s0)] = sc[nt][e];
            }
        // ---- online softmax for head qr
        float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float nm = fmaxf(m_run, mx);
        const float alpha = nm == -INFINITY ? 1.f : expf(m_run - nm);
        float p[2][2];
        float psum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                p[nt][e] = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - nm);
                psum += p[nt][e];
            }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l_run = l_run * alpha + psum;
        m_run = nm;
        // rescale O^T columns (heads 2qc, 2qc+1): their alphas live in lanes 8qc and 8qc+4
        const float al0 = __shfl_sync(0xffffffffu, alpha, 8 * qc);
        const float al1 = __shfl_sync(0xffffffffu, alpha, 8 * qc + 4);
#pragma unroll
        for (int md = 0; md < KS; ++md) {
            oacc[md][0] *= al0;
            oacc[md][1] *= al1;
            oacc[md][2] *= al0;
            oacc[md][3] *= al1;
        }
        // ---- V tile (16 slots x D) dequantized into this warp's shared tile
        {
            const int slot_a = base + qr, slot_b = base + 8 + qr;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = qr + 8 * half;
                const int slot = min(half ? slot_b : slot_a, src.cap - 1);
                const uint8_t* vv = vbase + (size_t)slot * src.cb_max;
                constexpr int EPQ = D / 4;            // elements of this quad
#pragma unroll
                for (int c8 = 0; c8 < EPQ / 8; ++c8) {
                    const int e0 = qc * EPQ + c8 * 8;     // first element of this 16-byte chunk
                    uint4 out;
                    if (RAW) {
                        out = __ldg(reinterpret_cast<const uint4*>(vv + e0 * 2));
                    } else {
                        const int g = e0 / 64;
                        const float scl = half_bits_to_f32(__ldg(vsl + ((size_t)slot * NG + g) * 2));
                        const float lo = half_bits_to_f32(__ldg(vsl + ((size_t)slot * NG + g) * 2 + 1));
                        uint32_t wv[2] = {0u, 0u};
                        uint16_t uv[1] = {0};
                        float f[8];
                        if (BITS == 4) {
                            wv[0] = __ldg(reinterpret_cast<const uint32_t*>(vv + e0 / 2));
                        } else if (BITS == 8) {
                            const uint2 t = __ldg(reinterpret_cast<const uint2*>(vv + e0));
                            wv[0] = t.x;
                            wv[1] = t.y;
                        } else if (BITS == 2) {
                            // one word holds 16 codes; elements e0..e0+7 are its pairs (e0%16)/2 .. +3
                            wv[0] = __ldg(reinterpret_cast<const uint32_t*>(vv + (e0 / 16) * 4));
                        } else {  // 3 bit
                            wv[0] = __ldg(reinterpret_cast<const uint32_t*>(vv + (e0 / 16) * 4));
                            uv[0] = __ldg(reinterpret_cast<const uint16_t*>(vv + D / 4 + (e0 / 16) * 2));
                        }
#pragma unroll
                        for (int pi = 0; pi < 4; ++pi) {
                            uint32_t bits;
                            if (BITS == 4) bits = pair_bits<4>(wv, uv, pi);
                            else if (BITS == 8) bits = pair_bits<8>(wv, uv, pi);
                            else if (BITS == 2) bits = pair_bits<2>(wv, uv, ((e0 % 16) / 2) + pi);
                            else bits = pair_bits<3>(wv, uv, ((e0 % 16) / 2) + pi);
                            f[2 * pi] = (float)(bits & 0xFFFFu);
                            f[2 * pi + 1] = (float)(bits >> 16);
                        }
                        out.x = pk_f16(f[0] * scl + lo, f[1] * scl + lo);
                        out.y = pk_f16(f[2] * scl + lo, f[3] * scl + lo);
                        out.z = pk_f16(f[4] * scl + lo, f[5] * scl + lo);
                        out.w = pk_f16(f[6] * scl + lo, f[7] * scl + lo);
                    }
                    const int chunk16 = e0 / 8;
                    *reinterpret_cast<uint4*>(vt + row * D + ((chunk16 ^ (row & 7)) << 3)) = out;
                }
            }
        }
        __syncwarp();
        // ---- O^T += V^T P^T
        uint32_t pb0, pb1;
        if (RAW && src.dtype == DKV_BF16) {
            pb0 = pk_bf16(p[0][0], p[0][1]);
            pb1 = pk_bf16(p[1][0], p[1][1]);
        } else {
            pb0 = pk_f16(p[0][0], p[0][1]);
            pb1 = pk_f16(p[1][0], p[1][1]);
        }
        {
            const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
            for (int md = 0; md < KS; ++md) {
                uint32_t va[4];
                const int row = (mi >> 1) * 8 + ri;
                ldsm4t_(va, vt + row * D + (((2 * md + (mi & 1)) ^ (row & 7)) << 3));
                if (RAW && src.dtype == DKV_BF16)
                    mma16816<true>(oacc[md], va, pb0, pb1);
                else
                    mma16816<false>(oacc[md], va, pb0, pb1);
            }
        }
        __syncwarp();
    }

    // ---- merge the 8 warps (fixed order) into the CTA partial
    __syncthreads();
    float* wo = reinterpret_cast<float*>(vtile);          // [warps][8 heads][D]  (reuses the V tiles)
    __shared__ float wm[kDraftWarps][8], wl[kDraftWarps][8];
    if (qc == 0 && qr < 8) {
        wm[warp][qr] = m_run;
        wl[warp][qr] = l_run;
    }
#pragma unroll
    for (int md = 0; md < KS; ++md) {
        const int d0 = 16 * md + qr;
        wo[((size_t)warp * 8 + 2 * qc) * D + d0] = oacc[md][0];
        wo[((size_t)warp * 8 + 2 * qc + 1) * D + d0] = oacc[md][1];
        wo[((size_t)warp * 8 + 2 * qc) * D + d0 + 8] = oacc[md][2];
        wo[((size_t)warp * 8 + 2 * qc + 1) * D + d0 + 8] = oacc[md][3];
    }
    __syncthreads();
    if (threadIdx.x < 8) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < kDraftWarps; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f;
        for (int w = 0; w < kDraftWarps; ++w)
            if (wm[w][g] != -INFINITY) L += wl[w][g] * expf(wm[w][g] - M);
        cta_m[g] = M;
        cta_l[g] = L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
        const int g = i / D;
        const float M = cta_m[g];
        float acc = 0.f;
        for (int w = 0; w < kDraftWarps; ++w)
            if (wm[w][g] != -INFINITY) acc += wo[((size_t)w * 8 + g) * D + (i % D)] * expf(wm[w][g] - M);
        cta_o[i] = acc;
    }
    cluster.sync();
    // ---- cluster merge through distributed shared memory (rank order)
    if (threadIdx.x < 8) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int r = 0; r < da.cs; ++r) M = fmaxf(M, cluster.map_shared_rank(cta_m, r)[g]);
        float L = 0.f;
        for (int r = 0; r < da.cs; ++r) {
            const float mr = cluster.map_shared_rank(cta_m, r)[g];
            if (mr != -INFINITY) L += cluster.map_shared_rank(cta_l, r)[g] * expf(mr - M);
        }
        glob_m[g] = M;
        glob_l[g] = L;
    }
    __syncthreads();
    {
        const int dper = (D + da.cs - 1) / da.cs;
        const int d0 = rank * dper, d1 = min(D, d0 + dper);
        for (int i = threadIdx.x; i < G * (d1 - d0); i += blockDim.x) {
            const int g = i / (d1 - d0), d = d0 + i % (d1 - d0);
            const float M = glob_m[g];
            float acc = 0.f;
            for (int r = 0; r < da.cs; ++r) {
                const float mr = cluster.map_shared_rank(cta_m, r)[g];
                if (mr != -INFINITY) acc += cluster.map_shared_rank(cta_o, r)[g * D + d] * expf(mr - M);
            }
            const float o = glob_l[g] > 0.f ? acc / glob_l[g] : 0.f;
            store_from_f32(a.out, a.out_dtype, ((size_t)b * HQ + h * G + g) * D + d, o);
        }
    }
    // ---- exact attention mass of this CTA's slots for head h (group sum)
    float* mass_h = a.mass + (bl * a.n_kv + h) * (size_t)src.cap;
    for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
        float mv = 0.f;
        for (int g = 0; g < G; ++g) {
            const float sc = sbuf[(size_t)g * da.chunk_cap + (s - s0)];
            if (sc != -INFINITY && glob_l[g] > 0.f) mv += expf(sc - glob_m[g]) / glob_l[g];
        }
        mass_h[s] = mv;
    }
    cluster.sync();   // remote shared memory stays alive until every CTA has read it
    // ---- fold the heads' masses into the scores of this slot range (head order)
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        uint32_t* tk = da.tickets + bl * 64 + rank;
        const uint32_t prev = atomicAdd(tk, 1u);
        last = prev == (uint32_t)(a.n_kv - 1);
        if (last) *tk = 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    float* sc_row = a.score + bl * src.cap;
    const float* mass_l = a.mass + bl * a.n_kv * (size_t)src.cap;
    for (int s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
        if (__ldcg(cpos + s) < 0) continue;
        float add = 0.f;
        for (int hh = 0; hh < a.n_kv; ++hh) add += __ldcg(mass_l + (size_t)hh * src.cap + s);
        sc_row[s] += add;
    }
}

uint32_t* device_error_word();

template <int D, int BITS>
static cudaError_t launch_draft(const DraftArgs& da, dim3 grid, size_t smem, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = allow_smem_max(attn_draft_tc_kernel<D, BITS>);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(attn_draft_tc_kernel<D, BITS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kDraftThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = da.cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_draft_tc_kernel<D, BITS>, da);
}

int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled,
                 uint32_t* comp_tickets, int raw_dtype);

int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled,
                 uint32_t* comp_tickets, int raw_dtype) {
    (void)work;
    (void)work_bytes;
    *handled = false;
    const int D = dims.d;
    if ((D != 64 && D != 128) || a.group > 8 || comp_tickets == nullptr) return DKV_OK;
    if (a.src.bits == 16 && raw_dtype != DKV_BF16) return DKV_OK;   // fp32 16-bit entries: generic kernel
    DraftArgs da;
    da.a = a;
    int cs = (2 * 148 + dims.batch * dims.n_kv - 1) / (dims.batch * dims.n_kv);
    cs = cs < 1 ? 1 : (cs > 8 ? 8 : cs);
    da.cs = cs;
    da.raw_dtype = raw_dtype;
    da.tickets = comp_tickets;
    da.err = device_error_word();
    da.a.src.dtype = raw_dtype;
    // slots per CTA the shared memory must hold (every CTA sizes for the capacity)
    int per = (a.src.cap + cs - 1) / cs;
    per = (per + 15) / 16 * 16;
    da.chunk_cap = per;
    const size_t fixed = (size_t)kDraftWarps * 16 * D * 2 + (8 + 8 + 8 * D + 16) * sizeof(float);
    const size_t smem = (size_t)a.group * per * sizeof(float) + std::max(fixed, (size_t)kDraftWarps * 8 * D * 4 + 256);
    if (smem > 200 * 1024) return DKV_OK;    // too many slots per CTA: generic kernel
    dim3 grid(cs, dims.n_kv, dims.batch);
    cudaError_t e = cudaSuccess;
    {
        ProfScope ps(DKV_PROF_ATTN_COMP, 0.0, st);
        switch (a.src.bits * 1000 + D) {
            case 2064: e = launch_draft<64, 2>(da, grid, smem, st); break;
            case 3064: e = launch_draft<64, 3>(da, grid, smem, st); break;
            case 4064: e = launch_draft<64, 4>(da, grid, smem, st); break;
            case 8064: e = launch_draft<64, 8>(da, grid, smem, st); break;
            case 16064: e = launch_draft<64, 16>(da, grid, smem, st); break;
            case 2128: e = launch_draft<128, 2>(da, grid, smem, st); break;
            case 3128: e = launch_draft<128, 3>(da, grid, smem, st); break;
            case 4128: e = launch_draft<128, 4>(da, grid, smem, st); break;
            case 8128: e = launch_draft<128, 8>(da, grid, smem, st); break;
            case 16128: e = launch_draft<128, 16>(da, grid, smem, st); break;
            default: return DKV_OK;
        }
    }
    DKV_CUDA(e);
    DKV_LAUNCHED();
    *handled = true;
    return DKV_OK;
}

}  // namespace dkv
