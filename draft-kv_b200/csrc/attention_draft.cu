// Tensor-core drafter attention over the quantized slot cache (T = 1).
//
// Replaces, for a draft step, draftkv/llama.py:202-219 with cache =
// CompressedKVCache (read :135-142) plus note_attention
// (draftkv/compress.py:144-151) summed over the GQA group
// (draftkv/llama.py:213-216).
//
// One thread-block cluster of CS CTAs per (sequence, KV head); CTA r of the
// cluster takes a contiguous 1/CS of the live slot range.  Each of its 8
// warps walks 16-slot tiles through a private ring of NST shared-memory
// stages filled by cp.async (NST-1 tiles in flight while one is consumed).
//
// Codes enter the tensor cores without dequantization.  One LOP3 (or PRMT)
// turns a pair of codes into the f16 pair (1024 + f*c), exact, where f is a
// power of two fixed by the pair's bit position (so no shift is needed to
// align the field).  Then, per 64-group g of a slot:
//   S = K Q^T   A = 16 slots of K in the fragment storage order, B = the
//               group's queries scaled by 1/f (columns = heads, up to 8):
//               sum_d q_d (1024 + f c_d)/f = sum_d q_d c_d + 1024 sum_d q_d/f,
//               so s = scale_g (S_g - off_g) + lo_g sum_d q_d;
//   O^T += X^T P'^T  X = the V codes of slot pairs, byte-permuted straight
//               from the stage into A registers (1024 + F c) with one factor
//               F per bit width, P'_g = p * vscale_g obtained from the S
//               accumulators by movmatrix.trans, and at the end
//               o_d = (acc_d - 1024 sum P'_g) / F + sum p * vlo_g, with
//               sum P'_g from one more product with a row of ones.
// 16-bit entries (raw bf16) take the plain path.  Scores are kept in log2
// units (log2 e folded into the query scale) so the softmax uses exp2.
// Raw scores stay in shared memory, or in the work arena when that lets two
// CTAs share an SM; after the warps' online-softmax states are merged, the
// cluster exchanges (max, sum) through distributed shared memory, each CTA
// writes its share of the output and the exact attention mass of its slots,
// and the last of the n_kv clusters to finish a slot range folds the per-head
// masses into the slot scores in head order (atomic ticket, no wait).
#include <cooperative_groups.h>

#include "attn_common.cuh"

namespace cg = cooperative_groups;

namespace dkv {

namespace {

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

// Transpose of an 8x8 b16 matrix held one row-pair per thread.
DKV_DEV uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}

DKV_DEV void cpa16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
DKV_DEV void cpa8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src));
}
DKV_DEV void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
DKV_DEV void cpa_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

DKV_DEV uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
DKV_DEV __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// Bits of code pair q (consecutive storage positions; the low half holds
// the even position) of a 3-bit segment: plane-A words `w`, plane-B units `u`.
DKV_DEV uint32_t pair_bits3(const uint32_t* w, const uint16_t* u, int q) {
    const uint32_t lo2 = (w[q >> 3] >> (2 * (q & 7))) & 0x00030003u;
    const uint32_t un = u[q >> 3];
    const uint32_t x = (un & 0xFFu) | ((un & 0xFF00u) << 8);
    const uint32_t hb = (x >> (q & 7)) & 0x00010001u;
    return lo2 | (hb << 2);
}

// Power-of-two factor f of code pair q: pair_x() yields 1024 + f*c.
template <int BITS>
DKV_DEV constexpr float pair_factor(int q) {
    return BITS == 4 ? ((q & 1) ? 16.f : 1.f) : BITS == 2 ? (float)(1 << (2 * (q & 3))) : 1.f;
}

// f16 pair (1024 + f*c_even, 1024 + f*c_odd) of code pair q of a packed
// segment held in registers (`w` its 32-bit words; 3 bits: plane-A words and
// plane-B units `u`).  The pair layout puts pair i of a word at bit 2i*bits/2
// of each half, so masking the field in place gives f = 2^(field offset).
template <int BITS>
DKV_DEV uint32_t pair_x(const uint32_t* w, const uint16_t* u, int q) {
    if (BITS == 4) {
        uint32_t x = w[q >> 2];
        if (q & 2) x >>= 8;
        return (x & ((q & 1) ? 0x00F000F0u : 0x000F000Fu)) | 0x64006400u;
    }
    if (BITS == 2) {
        uint32_t x = w[q >> 3];
        if (q & 4) x >>= 8;
        return (x & (0x00030003u << (2 * (q & 3)))) | 0x64006400u;
    }
    if (BITS == 8) return __byte_perm(w[q >> 1], 0x64u, (q & 1) ? 0x4342 : 0x4140);
    return pair_bits3(w, u, q) | 0x64006400u;
}

}  // namespace

constexpr int kDraftWarps = 8;
constexpr int kDraftThreads = kDraftWarps * 32;

// Shared-memory stage of one 16-slot tile: K codes [16][KB], V codes [16][KB]
// (16-bit entries: V rows in the swizzled order ldmatrix reads), K and V
// (scale, lo) [16][NG][2] fp16, positions [16] int32.
template <int D, int BITS>
struct DraftGeo {
    static constexpr bool RAW = BITS == 16;
    static constexpr int KB = RAW ? D * 2 : D * BITS / 8;
    static constexpr int NG = D / 64;
    static constexpr int OFF_V = 16 * KB;
    static constexpr int OFF_KSL = 32 * KB;
    static constexpr int OFF_VSL = OFF_KSL + 16 * NG * 4;
    static constexpr int OFF_POS = OFF_VSL + 16 * NG * 4;
    static constexpr int STAGE = (OFF_POS + 64 + 127) / 128 * 128;
};

struct DraftArgs {
    AttnArgs a;
    int cs;                 // cluster size (CTAs per (sequence, head))
    int chunk_cap;          // slots per CTA the score buffer holds
    int region;             // bytes of the stage rings (or the epilogue's warp partials)
    float* gsc;             // raw scores in global memory [batch][n_kv][group][cap], or null:
                            // in shared memory [group][chunk_cap] after the region
    int raw_dtype;          // dtype of 16-bit entries
    int ch16;               // code rows are 16-byte aligned: 16-byte copies
    int note_mass;          // keep the raw scores and fold the attention mass into the slot scores
    uint32_t* tickets;      // comp->tickets [batch][n_layers][64]
    uint32_t* err;
};

// This thread's K segment (quad c of slot row `row`) from a stage.
template <int D, int BITS>
DKV_DEV void smem_k_segment(const uint8_t* kst, int row, int c, uint32_t* w, uint16_t* u) {
    using Geo = DraftGeo<D, BITS>;
    const uint8_t* vec = kst + row * Geo::KB;
    if (BITS == 16) {
        const uint4* p = reinterpret_cast<const uint4*>(vec + c * (D / 2));
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            const uint4 v = p[i];
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    } else if (BITS == 3) {
        const uint32_t* pa = reinterpret_cast<const uint32_t*>(vec + c * (D / 16));
#pragma unroll
        for (int i = 0; i < D / 64; ++i) w[i] = pa[i];
        const uint16_t* pb = reinterpret_cast<const uint16_t*>(vec + D / 4 + c * (D / 32));
#pragma unroll
        for (int i = 0; i < D / 64; ++i) u[i] = pb[i];
    } else {
        constexpr int SEGB = D * BITS / 32;     // bytes per quad segment
        const uint32_t* p = reinterpret_cast<const uint32_t*>(vec + c * SEGB);
#pragma unroll
        for (int i = 0; i < SEGB / 4; ++i) w[i] = p[i];
    }
}

// V codes of this thread for one 64-group of a slot row (element-order
// storage): elements 64 gg + 8 qr .. +7.  4 bits: one word; 8 bits: two
// words; 2 and 3 bits: the plane-A word of 16 elements (3 bits: and the
// plane-B unit of the same 16 elements).
template <int D, int BITS>
DKV_DEV void load_vwords(const uint8_t* vst, int row, int gg, int qr, uint32_t (&w)[2], uint32_t& u) {
    const uint8_t* rp = vst + row * DraftGeo<D, BITS>::KB;
    if (BITS == 4) {
        w[0] = *reinterpret_cast<const uint32_t*>(rp + 4 * (8 * gg + qr));
    } else if (BITS == 8) {
        const uint2 x = *reinterpret_cast<const uint2*>(rp + 8 * (8 * gg + qr));
        w[0] = x.x;
        w[1] = x.y;
    } else {
        w[0] = *reinterpret_cast<const uint32_t*>(rp + 4 * (4 * gg + (qr >> 1)));
        if (BITS == 3) u = *reinterpret_cast<const uint16_t*>(rp + D / 4 + 2 * (4 * gg + (qr >> 1)));
    }
}

// A operand registers of O^T += X^T P'^T for one 64-group, built from the
// codes of two slots x (low halves) and y (high halves) with no shared-memory
// pass: r[2j + h] = (1024 + F c_x(e), 1024 + F c_y(e)) as exact f16 for
// element offset e = 2j + h of the thread's 8 elements.  The pair layout
// keeps even elements in the low half-word and odd ones in the high half-word
// at the same bit offset, so one byte permutation interleaves the two slots;
// each field is shifted to one fixed position, so every element carries the
// same power-of-two factor F = vfactor<BITS>() and the offset 1024 is
// removed once per tile from the accumulators (1024 x sum P', one more
// product with a row of ones).  F keeps the codes large next to the offset
// (mean F c >= 56), so the fp32 accumulators lose at most a few bits to it.
template <int BITS>
DKV_DEV constexpr float vfactor() {
    return BITS == 8 ? 1.f : BITS == 2 ? 64.f : 16.f;
}

template <int BITS>
DKV_DEV void v_pairs(const uint32_t (&xw)[2], uint32_t xu, const uint32_t (&yw)[2], uint32_t yu, int t,
                     uint32_t (&r)[8]) {
    constexpr uint32_t kOne = 0x64006400u;
    if constexpr (BITS == 4) {
        // nibble j of each half to bits 4-7 (F = 16)
        const uint32_t z[2] = {__byte_perm(xw[0], yw[0], 0x5410), __byte_perm(xw[0], yw[0], 0x7632)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            r[h] = ((z[h] << 4) & 0x00F000F0u) | kOne;
            r[2 + h] = (z[h] & 0x00F000F0u) | kOne;
            r[4 + h] = ((z[h] >> 4) & 0x00F000F0u) | kOne;
            r[6 + h] = ((z[h] >> 8) & 0x00F000F0u) | kOne;
        }
    } else if constexpr (BITS == 8) {
        // bytes as f16 mantissas (F = 1)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t z = __byte_perm(xw[j >> 1], yw[j >> 1], (j & 1) ? 0x7632 : 0x5410);
            r[2 * j] = __byte_perm(z, 0x64u, 0x4240);
            r[2 * j + 1] = __byte_perm(z, 0x64u, 0x4341);
        }
    } else if constexpr (BITS == 2) {
        // field j (bits 2j of the thread's byte) to bits 6-7 (F = 64)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t z = __byte_perm(xw[0], yw[0], h ? 0x7632 : 0x5410);
            if (t) z >>= 8;
            r[h] = ((z << 6) & 0x00C000C0u) | kOne;
            r[2 + h] = ((z << 4) & 0x00C000C0u) | kOne;
            r[4 + h] = ((z << 2) & 0x00C000C0u) | kOne;
            r[6 + h] = (z & 0x00C000C0u) | kOne;
        }
    } else {
        // 3 bits: low two bits (plane A, field j at bits 2j) to bits 4-5 and the
        // high bit (plane B, bit 8h + j) to bit 6 (F = 16)
        uint32_t zb = __byte_perm(xu, yu, 0x5410);
        if (t) zb >>= 4;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t z = __byte_perm(xw[0], yw[0], h ? 0x7632 : 0x5410);
            if (t) z >>= 8;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t lo = (j < 2 ? (z << (4 - 2 * j)) : (z >> (2 * j - 4))) & 0x00300030u;
                const int k = 8 * h + j;
                const uint32_t hb = (k <= 6 ? (zb << (6 - k)) : (zb >> (k - 6))) & 0x00400040u;
                r[2 * j + h] = lo | hb | kOne;
            }
        }
    }
}

// 2^x on the SFU (ex2.approx; -inf gives +0)
DKV_DEV float fast_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

template <int D, int BITS, int NST>
__global__ void __launch_bounds__(kDraftThreads, 2) attn_draft_tc_kernel(DraftArgs da) {
    using Geo = DraftGeo<D, BITS>;
    constexpr bool RAW = Geo::RAW;
    constexpr int KS = D / 16;              // k16 steps over d
    constexpr int NG = Geo::NG;             // quantization groups
    constexpr int KB = Geo::KB;
    constexpr int SEGW = RAW ? D / 8 : (BITS == 3 ? D / 64 : D * BITS / 128);   // words per quad segment
    constexpr float kLog2e = 1.4426950408889634f;
    const AttnArgs& a = da.a;
    pdl_trigger();
    pdl_wait();         // queries and the appended rows come from the previous kernels
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
    const int cc = da.chunk_cap;

    extern __shared__ __align__(128) uint8_t dsm[];
    uint8_t* ring = dsm + (size_t)warp * NST * Geo::STAGE;
    float* tailp = reinterpret_cast<float*>(dsm + da.region);
    // raw scores (log2 units) of this CTA's slots, slot-major:
    // sbuf[(s - s0) * G + g]
    float* sbuf = nullptr;
    if (!da.note_mass) {
    } else if (da.gsc) {
        sbuf = da.gsc + (((size_t)b * a.n_kv + h) * (size_t)src.cap + s0) * G;
    } else {
        sbuf = tailp;
        tailp += (size_t)G * cc;
    }
    float* cta_m = tailp;                                                   // [8]
    float* cta_l = cta_m + 8;                                               // [8]
    float* cta_o = cta_l + 8;                                               // [8][D]
    float* glob_m = cta_o + 8 * D;                                          // [8]
    float* glob_l = glob_m + 8;                                             // [8]

    if (chunk > cc) {       // host sized the launch; never expected
        if (threadIdx.x == 0) atomicOr(da.err, 0x40u);
    }

    const size_t vh = (bl * a.n_kv + h) * (size_t)src.cap;       // first vector of (b, layer, head)
    const uint8_t* kbase = src.k_codes + vh * src.cb_max;
    const uint8_t* vbase = src.v_codes + vh * src.cb_max;
    const uint8_t* kslb = reinterpret_cast<const uint8_t*>(src.k_sl + vh * NG * 2);
    const uint8_t* vslb = reinterpret_cast<const uint8_t*>(src.v_sl + vh * NG * 2);
    const uint8_t* posb = reinterpret_cast<const uint8_t*>(src.cpos + bl * src.cap);

    const int first_tile = s0 / 16;
    const int n_tiles = s1 > s0 ? (s1 - 1) / 16 - first_tile + 1 : 0;
    const int my_n = n_tiles > warp ? (n_tiles - 1 - warp) / kDraftWarps + 1 : 0;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);

    // this lane's copy chunks of a tile: code chunk k is row ck / CPR, column
    // ck % CPR with ck = lane + 32k; one (scale, lo) or position chunk
    constexpr int CW = (KB % 16 == 0) ? 16 : 8;
    const int cw = (CW == 16 && (RAW || da.ch16)) ? 16 : 8;
    const int cpr = KB / cw;
    constexpr int MAXC = (16 * KB / 8 + 31) / 32;
    const int nck = (16 * cpr + 31) / 32;
    constexpr int SLC = NG * 4;      // 16-byte chunks of one (scale, lo) tile
    const uint8_t* aux_src = lane < SLC ? kslb : lane < 2 * SLC ? vslb : posb;
    const int aux_el = lane < 2 * SLC ? NG * 4 : 4;            // bytes per slot of that array
    const int aux_off = (lane < SLC ? lane : lane < 2 * SLC ? lane - SLC : lane - 2 * SLC) * 16;
    const uint32_t aux_dst = (lane < SLC ? Geo::OFF_KSL : lane < 2 * SLC ? Geo::OFF_VSL : Geo::OFF_POS) + aux_off;
    const bool aux_on = lane < 2 * SLC + 4;

    // per chunk: global offset from the tile's first row, K and V stage offsets
    int c_go[MAXC], c_ko[MAXC], c_vo[MAXC];
#pragma unroll
    for (int k = 0; k < MAXC; ++k) {
        const int ck = lane + 32 * k;
        c_go[k] = -1;
        if (k < nck && ck < 16 * cpr) {
            const int row = cw == 16 ? ck / (KB / 16 > 0 ? KB / 16 : 1) : ck / (KB / 8);
            const int col = cw == 16 ? ck % (KB / 16 > 0 ? KB / 16 : 1) : ck % (KB / 8);
            c_go[k] = row * KB + col * cw;
            c_ko[k] = row * KB + col * cw;
            c_vo[k] = Geo::OFF_V + row * KB + (RAW ? ((col ^ (row & 7)) * 16) : col * cw);
        }
    }

    auto issue = [&](int i) {
        if (i < my_n) {
            const int base = (first_tile + warp + i * kDraftWarps) * 16;
            const uint32_t st = ring_s + (uint32_t)((i % NST) * Geo::STAGE);
            const uint8_t* kt = kbase + (size_t)base * KB;          // rows of KB bytes, dense
            const uint8_t* vtile = vbase + (size_t)base * KB;
#pragma unroll
            for (int k = 0; k < MAXC; ++k) {
                if (c_go[k] >= 0) {
                    if (CW == 16 && cw == 16) {
                        cpa16(st + c_ko[k], kt + c_go[k]);
                        cpa16(st + c_vo[k], vtile + c_go[k]);
                    } else {
                        cpa8(st + c_ko[k], kt + c_go[k]);
                        cpa8(st + c_vo[k], vtile + c_go[k]);
                    }
                }
            }
            if (aux_on) cpa16(st + aux_dst, aux_src + (size_t)base * aux_el + aux_off);
        }
        cpa_commit();
    };

#pragma unroll
    for (int i = 0; i < NST - 1; ++i) issue(i);

    // ---- queries as the B operand: column = head qr (heads >= G are zero),
    // scaled by 1/sqrt(d) * log2(e) and, per code pair, by 1/f
    const bool qrow = qr < G;
    const float* qv = a.q + ((size_t)b * HQ + h * G + (qrow ? qr : 0)) * D;
    const float qscale = a.scale * kLog2e;
    uint32_t qb[KS][2];
    float qsum[NG] = {}, qoff[NG] = {};
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        const int d0 = kk * 16 + 2 * qc;
        float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
        if (qrow) {
            x0 = qv[d0] * qscale;
            x1 = qv[d0 + 1] * qscale;
            x2 = qv[d0 + 8] * qscale;
            x3 = qv[d0 + 9] * qscale;
        }
        if constexpr (RAW) {
            qb[kk][0] = pk_bf16(x0, x1);
            qb[kk][1] = pk_bf16(x2, x3);
        } else {
            // the f16-rounded query values q; pair 2kk multiplies d0, d0+1 and
            // pair 2kk+1 multiplies d0+8, d0+9 (exact power-of-two rescale)
            const __half2 h01 = __floats2half2_rn(x0, x1), h23 = __floats2half2_rn(x2, x3);
            const float f0 = pair_factor<BITS>(2 * kk), f1 = pair_factor<BITS>(2 * kk + 1);
            const __half2 s01 = __hmul2(h01, __float2half2_rn(1.f / f0));
            const __half2 s23 = __hmul2(h23, __float2half2_rn(1.f / f1));
            qb[kk][0] = *reinterpret_cast<const uint32_t*>(&s01);
            qb[kk][1] = *reinterpret_cast<const uint32_t*>(&s23);
            qsum[kk / 4] += __low2float(h01) + __high2float(h01) + __low2float(h23) + __high2float(h23);
            qoff[kk / 4] += 1024.f * (__low2float(s01) + __high2float(s01) + __low2float(s23) + __high2float(s23));
        }
    }
    // per head qr, then fetched for this thread's S columns (heads 2qc, 2qc+1)
    float qs0[NG], qs1[NG], qo0[NG], qo1[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
        qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 1);
        qsum[g] += __shfl_xor_sync(0xffffffffu, qsum[g], 2);
        qoff[g] += __shfl_xor_sync(0xffffffffu, qoff[g], 1);
        qoff[g] += __shfl_xor_sync(0xffffffffu, qoff[g], 2);
        qs0[g] = __shfl_sync(0xffffffffu, qsum[g], 8 * qc);
        qs1[g] = __shfl_sync(0xffffffffu, qsum[g], 8 * qc + 4);
        qo0[g] = __shfl_sync(0xffffffffu, qoff[g], 8 * qc);
        qo1[g] = __shfl_sync(0xffffffffu, qoff[g], 8 * qc + 4);
    }

    // online-softmax maxima of heads 2qc (0) and 2qc+1 (1); the sums come
    // from an extra product per tile: C2 = A2 P^T with A2 rows g < NG = vlo_g
    // of the slots and row NG = ones, so C2 row g = sum p * vlo_g and row NG =
    // sum p (16-bit entries: row 0 = sum p)
    constexpr int ROW1 = RAW ? 0 : NG;
    // finite start: a fully masked tile leaves the max at -1e30 and every
    // p = 2^(-inf) = 0 without a special case
    constexpr float kNoMax = -1e30f;
    float m0 = kNoMax, m1 = kNoMax;
    float c2[4] = {0.f, 0.f, 0.f, 0.f};
    // C3 = ones P'^T per 64-group: row 0-7 = sum P'_g (the V offset's weight)
    float c3[NG][4];
#pragma unroll
    for (int g = 0; g < NG; ++g) c3[g][0] = c3[g][1] = c3[g][2] = c3[g][3] = 0.f;
    float oacc[KS][4];                       // O^T: rows d = 16md + qr (+8), cols heads 2qc, 2qc+1
#pragma unroll
    for (int md = 0; md < KS; ++md) oacc[md][0] = oacc[md][1] = oacc[md][2] = oacc[md][3] = 0.f;


    for (int it = 0; it < my_n; ++it) {
        issue(it + NST - 1);
        cpa_wait<NST - 1>();
        __syncwarp();
        const uint8_t* st = ring + (it % NST) * Geo::STAGE;
        const int base = (first_tile + warp + it * kDraftWarps) * 16;

        // ---- S = K Q^T: rows slots qr / qr+8, columns heads 2qc / 2qc+1
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        {
            uint32_t w0[SEGW > 0 ? SEGW : 1], w1[SEGW > 0 ? SEGW : 1];
            uint16_t u0[D / 64 > 0 ? D / 64 : 1], u1[D / 64 > 0 ? D / 64 : 1];
            smem_k_segment<D, BITS>(st, qr, qc, w0, u0);
            smem_k_segment<D, BITS>(st, qr + 8, qc, w1, u1);
            if constexpr (RAW) {
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t af[4] = {w0[2 * kk], w1[2 * kk], w0[2 * kk + 1], w1[2 * kk + 1]};
                    mma16816<true>(sc, af, qb[kk][0], qb[kk][1]);
                }
            } else {
                // accumulators start at -off_g, so they end at S_g - off_g
                float gs[NG][4];
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    gs[g][0] = gs[g][2] = -qo0[g];
                    gs[g][1] = gs[g][3] = -qo1[g];
                }
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t af[4] = {pair_x<BITS>(w0, u0, 2 * kk), pair_x<BITS>(w1, u1, 2 * kk),
                                            pair_x<BITS>(w0, u0, 2 * kk + 1), pair_x<BITS>(w1, u1, 2 * kk + 1)};
                    mma16816<false>(gs[kk / 4], af, qb[kk][0], qb[kk][1]);
                }
                const uint32_t* ksl = reinterpret_cast<const uint32_t*>(st + Geo::OFF_KSL);
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int row = hr ? qr + 8 : qr;
#pragma unroll
                    for (int g = 0; g < NG; ++g) {
                        const uint32_t slw = ksl[row * NG + g];
                        const float2 sl2 = __half22float2(bits_h2(slw));
                        const float scl = sl2.x, lo = sl2.y;
                        sc[2 * hr] = fmaf(scl, gs[g][2 * hr], fmaf(lo, qs0[g], sc[2 * hr]));
                        sc[2 * hr + 1] = fmaf(scl, gs[g][2 * hr + 1], fmaf(lo, qs1[g], sc[2 * hr + 1]));
                    }
                }
            }
        }
        // ---- mask (empty slot, outside this CTA's range, future position)
        const int32_t* ps = reinterpret_cast<const int32_t*>(st + Geo::OFF_POS);
        const int sa = base + qr, sb = base + 8 + qr;
        const bool ina = sa >= s0 && sa < s1, inb = sb >= s0 && sb < s1;
        const int pa = ps[qr], pb = ps[qr + 8];
        if (!(ina && pa >= 0 && pa <= qpos)) sc[0] = sc[1] = -INFINITY;
        if (!(inb && pb >= 0 && pb <= qpos)) sc[2] = sc[3] = -INFINITY;
        {
            const int h0 = 2 * qc;
            auto put = [&](int s, float x, float y) {
                float* p = sbuf + (size_t)(s - s0) * G + h0;
                if ((G & 1) == 0) {
                    *reinterpret_cast<float2*>(p) = make_float2(x, y);    // h0 + 1 < G
                } else {
                    p[0] = x;
                    if (h0 + 1 < G) p[1] = y;
                }
            };
            if (h0 < G && da.note_mass) {
                if (ina && sa - s0 < cc) put(sa, sc[0], sc[1]);
                if (inb && sb - s0 < cc) put(sb, sc[2], sc[3]);
            }
        }
        // ---- online softmax (base 2) of the two heads over the tile's 16 slots
        float t0 = fmaxf(sc[0], sc[2]), t1 = fmaxf(sc[1], sc[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
            t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
        }
        {
            const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
            if (!__all_sync(0xffffffffu, n0 == m0 && n1 == m1)) {
                const float al0 = fast_ex2(m0 - n0), al1 = fast_ex2(m1 - n1);
#pragma unroll
                for (int md = 0; md < KS; ++md) {
                    oacc[md][0] *= al0;
                    oacc[md][1] *= al1;
                    oacc[md][2] *= al0;
                    oacc[md][3] *= al1;
                }
                c2[0] *= al0;
                c2[1] *= al1;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    c3[g][0] *= al0;
                    c3[g][1] *= al1;
                }
                m0 = n0;
                m1 = n1;
            }
        }
        // p (f16): slot qr -> pa2 (heads 2qc, 2qc+1), slot qr+8 -> pb2
        const __half2 pa2 = __floats2half2_rn(fast_ex2(sc[0] - m0), fast_ex2(sc[1] - m1));
        const __half2 pb2 = __floats2half2_rn(fast_ex2(sc[2] - m0), fast_ex2(sc[3] - m1));
        // ---- sums: C2 += A2 P^T
        {
            uint32_t a2[4] = {0u, 0u, 0u, 0u};
            if constexpr (!RAW) {
                if (qr < NG) {
                    const uint32_t* vsl = reinterpret_cast<const uint32_t*>(st + Geo::OFF_VSL);
                    a2[0] = __byte_perm(vsl[(2 * qc) * NG + qr], vsl[(2 * qc + 1) * NG + qr], 0x7632);
                    a2[2] = __byte_perm(vsl[(2 * qc + 8) * NG + qr], vsl[(2 * qc + 9) * NG + qr], 0x7632);
                }
            }
            if (qr == ROW1) a2[0] = a2[2] = 0x3C003C00u;     // f16 ones
            mma16816<false>(c2, a2, movm_t(h2_bits(pa2)), movm_t(h2_bits(pb2)));
        }
        // ---- P'^T fragments (B of O^T += X^T P'^T)
        uint32_t pbf[NG][2];
        if constexpr (RAW) {
            // bf16 entries: P in bf16, V rows by ldmatrix.trans from the stage
            const float2 fa = __half22float2(pa2), fb = __half22float2(pb2);
            pbf[0][0] = movm_t(pk_bf16(fa.x, fa.y));
            pbf[0][1] = movm_t(pk_bf16(fb.x, fb.y));
            const uint16_t* vsrc = reinterpret_cast<const uint16_t*>(st + Geo::OFF_V);
            const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
            for (int md = 0; md < KS; ++md) {
                uint32_t va[4];
                const int row = (mi >> 1) * 8 + ri;
                ldsm4t_(va, vsrc + row * D + (((2 * md + (mi & 1)) ^ (row & 7)) << 3));
                mma16816<true>(oacc[md], va, pbf[0][0], pbf[0][1]);
            }
        } else {
            const uint32_t* vsl = reinterpret_cast<const uint32_t*>(st + Geo::OFF_VSL);
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const __half2 sa2 = bits_h2(__byte_perm(vsl[qr * NG + g], 0u, 0x1010));
                const __half2 sb2 = bits_h2(__byte_perm(vsl[(qr + 8) * NG + g], 0u, 0x1010));
                pbf[g][0] = movm_t(h2_bits(__hmul2(pa2, sa2)));
                pbf[g][1] = movm_t(h2_bits(__hmul2(pb2, sb2)));
            }
            // tile md = 4 gg + j: rows qr / qr + 8 are elements 64 gg + 8 qr + 2j (+1),
            // columns the slots 2qc, 2qc+1 (k 0-7) and 2qc+8, 2qc+9 (k 8-15)
            const uint8_t* vst = st + Geo::OFF_V;
#pragma unroll
            for (int gg = 0; gg < NG; ++gg) {
                uint32_t ra[8], rb[8];
                {
                    uint32_t xw[2] = {0u, 0u}, yw[2] = {0u, 0u}, xu = 0u, yu = 0u;
                    load_vwords<D, BITS>(vst, 2 * qc, gg, qr, xw, xu);
                    load_vwords<D, BITS>(vst, 2 * qc + 1, gg, qr, yw, yu);
                    v_pairs<BITS>(xw, xu, yw, yu, qr & 1, ra);
                }
                {
                    uint32_t xw[2] = {0u, 0u}, yw[2] = {0u, 0u}, xu = 0u, yu = 0u;
                    load_vwords<D, BITS>(vst, 2 * qc + 8, gg, qr, xw, xu);
                    load_vwords<D, BITS>(vst, 2 * qc + 9, gg, qr, yw, yu);
                    v_pairs<BITS>(xw, xu, yw, yu, qr & 1, rb);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t va[4] = {ra[2 * j], ra[2 * j + 1], rb[2 * j], rb[2 * j + 1]};
                    mma16816<false>(oacc[4 * gg + j], va, pbf[gg][0], pbf[gg][1]);
                }
                const uint32_t ones[4] = {0x3C003C00u, 0u, 0x3C003C00u, 0u};
                mma16816<false>(c3[gg], ones, pbf[gg][0], pbf[gg][1]);
            }
        }
        __syncwarp();
    }

    // ---- per-head sums from C2 (row ROW1: sum p; rows g: sum p vlo_g), and
    // o_d = acc_d / f_d + sum p vlo_g
    const float l0 = __shfl_sync(0xffffffffu, c2[0], ROW1 * 4 + qc);
    const float l1 = __shfl_sync(0xffffffffu, c2[1], ROW1 * 4 + qc);
    if constexpr (!RAW) {
        float sl0[NG], sl1[NG];
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            sl0[g] = __shfl_sync(0xffffffffu, c2[0], g * 4 + qc);
            sl1[g] = __shfl_sync(0xffffffffu, c2[1], g * 4 + qc);
        }
        // o = (acc - 1024 sum P'_g) / F + sum p vlo_g
        constexpr float inv_f = 1.f / vfactor<BITS>();
#pragma unroll
        for (int md = 0; md < KS; ++md) {
            const int g = md / 4;
            oacc[md][0] = fmaf(-1024.f, c3[g][0], oacc[md][0]) * inv_f + sl0[g];
            oacc[md][1] = fmaf(-1024.f, c3[g][1], oacc[md][1]) * inv_f + sl1[g];
            oacc[md][2] = fmaf(-1024.f, c3[g][0], oacc[md][2]) * inv_f + sl0[g];
            oacc[md][3] = fmaf(-1024.f, c3[g][1], oacc[md][3]) * inv_f + sl1[g];
        }
    }

    // ---- merge the 8 warps (fixed order) into the CTA partial
    __syncthreads();
    float* wo = reinterpret_cast<float*>(dsm);            // [warps][8 heads][D]  (reuses the rings)
    __shared__ float wm[kDraftWarps][8], wl[kDraftWarps][8];
    if (qr == 0) {
        wm[warp][2 * qc] = m0;
        wm[warp][2 * qc + 1] = m1;
        wl[warp][2 * qc] = l0;
        wl[warp][2 * qc + 1] = l1;
    }
#pragma unroll
    for (int md = 0; md < KS; ++md) {
        // element of rows qr / qr + 8 of tile md
        const int d0 = RAW ? 16 * md + qr : 64 * (md / 4) + 8 * qr + 2 * (md % 4);
        const int d1 = RAW ? d0 + 8 : d0 + 1;
        wo[((size_t)warp * 8 + 2 * qc) * D + d0] = oacc[md][0];
        wo[((size_t)warp * 8 + 2 * qc + 1) * D + d0] = oacc[md][1];
        wo[((size_t)warp * 8 + 2 * qc) * D + d1] = oacc[md][2];
        wo[((size_t)warp * 8 + 2 * qc + 1) * D + d1] = oacc[md][3];
    }
    __syncthreads();
    __shared__ float wf[kDraftWarps][8];       // exp2(m_warp - m_cta) per (warp, head)
    if (threadIdx.x < 8 * kDraftWarps) {
        const int g = threadIdx.x & 7, w = threadIdx.x >> 3;
        float M = -INFINITY;
        for (int ww = 0; ww < kDraftWarps; ++ww) M = fmaxf(M, wm[ww][g]);
        const float f = wm[w][g] == -INFINITY ? 0.f : exp2f(wm[w][g] - M);
        wf[w][g] = f;
        if (w == 0) cta_m[g] = M;
    }
    __syncthreads();
    if (threadIdx.x < 8) {
        const int g = threadIdx.x;
        float L = 0.f;
        for (int w = 0; w < kDraftWarps; ++w) L += wl[w][g] * wf[w][g];
        cta_l[g] = L;
    }
    for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
        const int g = i / D;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kDraftWarps; ++w) acc += wo[((size_t)w * 8 + g) * D + (i % D)] * wf[w][g];
        cta_o[i] = acc;
    }
    cluster.sync();
    // ---- cluster merge through distributed shared memory (rank order)
    __shared__ float rf[8][8];                 // exp2(m_rank - m) / l per (rank, head)
    if (threadIdx.x < 8) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int r = 0; r < da.cs; ++r) M = fmaxf(M, cluster.map_shared_rank(cta_m, r)[g]);
        float L = 0.f;
        for (int r = 0; r < da.cs; ++r) {
            const float mr = cluster.map_shared_rank(cta_m, r)[g];
            const float f = mr == -INFINITY ? 0.f : exp2f(mr - M);
            rf[r][g] = f;
            L += cluster.map_shared_rank(cta_l, r)[g] * f;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int r = 0; r < da.cs; ++r) rf[r][g] *= inv;
        glob_m[g] = M;
        glob_l[g] = inv;                       // holds 1 / l from here on
    }
    __syncthreads();
    {
        const int dper = (D + da.cs - 1) / da.cs;
        const int d0 = rank * dper, d1 = min(D, d0 + dper);
        for (int i = threadIdx.x; i < G * (d1 - d0); i += blockDim.x) {
            const int g = i / (d1 - d0), d = d0 + i % (d1 - d0);
            float v[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) v[r] = r < da.cs ? cluster.map_shared_rank(cta_o, r)[g * D + d] : 0.f;
            float acc = 0.f;
#pragma unroll
            for (int r = 0; r < 8; ++r) acc += r < da.cs ? v[r] * rf[r][g] : 0.f;
            store_from_f32(a.out, a.out_dtype, ((size_t)b * HQ + h * G + g) * D + d, acc);
        }
    }
    // ---- exact attention mass of this CTA's slots for head h (group sum)
    const int32_t* cpos = src.cpos + bl * src.cap;
    float* mass_h = a.mass + (bl * a.n_kv + h) * (size_t)src.cap;
    for (int s = s0 + threadIdx.x; da.note_mass && s < s1; s += blockDim.x) {
        float mv = 0.f;
        if (s - s0 < cc) {
            const float* rp = sbuf + (size_t)(s - s0) * G;
            if ((G & 3) == 0) {
                for (int g = 0; g < G; g += 4) {
                    const float4 r = da.gsc ? __ldcg(reinterpret_cast<const float4*>(rp + g))
                                            : *reinterpret_cast<const float4*>(rp + g);
                    mv += exp2f(r.x - glob_m[g]) * glob_l[g] + exp2f(r.y - glob_m[g + 1]) * glob_l[g + 1] +
                          exp2f(r.z - glob_m[g + 2]) * glob_l[g + 2] + exp2f(r.w - glob_m[g + 3]) * glob_l[g + 3];
                }
            } else {
                for (int g = 0; g < G; ++g) mv += exp2f((da.gsc ? __ldcg(rp + g) : rp[g]) - glob_m[g]) * glob_l[g];
            }
        }
        mass_h[s] = mv;
    }
    if (da.gsc && da.note_mass) {
        // the scores of [s0, s1) are consumed: drop their L2 lines without a
        // write-back (whole 128-byte lines inside the range only; the lines it
        // shares with the neighbouring ranges stay)
        __syncthreads();
        const uintptr_t lo = reinterpret_cast<uintptr_t>(sbuf);
        const uintptr_t hi = reinterpret_cast<uintptr_t>(sbuf + (size_t)(s1 - s0) * G);
        for (uintptr_t q = ((lo + 127) & ~(uintptr_t)127) + 128 * threadIdx.x; q + 128 <= hi; q += 128 * blockDim.x)
            asm volatile("discard.global.L2 [%0], 128;\n" ::"l"(q) : "memory");
    }
    cluster.sync();   // remote shared memory stays alive until every CTA has read it
    if (!da.note_mass) return;
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
    for (int s = s0 + 4 * threadIdx.x; s < s1; s += 4 * blockDim.x) {
        float4 add = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int h0 = 0; h0 < a.n_kv; h0 += 4) {
            float4 mh[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (h0 + u < a.n_kv) mh[u] = __ldcg(reinterpret_cast<const float4*>(mass_l + (size_t)(h0 + u) * src.cap + s));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (h0 + u < a.n_kv) {
                    add.x += mh[u].x;
                    add.y += mh[u].y;
                    add.z += mh[u].z;
                    add.w += mh[u].w;
                }
            }
        }
        const int4 cp = __ldcg(reinterpret_cast<const int4*>(cpos + s));
        if (cp.x >= 0) sc_row[s] += add.x;
        if (s + 1 < s1 && cp.y >= 0) sc_row[s + 1] += add.y;
        if (s + 2 < s1 && cp.z >= 0) sc_row[s + 2] += add.z;
        if (s + 3 < s1 && cp.w >= 0) sc_row[s + 3] += add.w;
    }
}

uint32_t* device_error_word();

namespace {

struct DraftShape {
    int stage;
};

template <int D, int BITS>
DraftShape draft_shape() {
    DraftShape r;
    r.stage = DraftGeo<D, BITS>::STAGE;
    return r;
}

template <int D, int BITS, int NST>
cudaError_t launch_draft(const DraftArgs& da, dim3 grid, size_t smem, cudaStream_t st) {
    static DeviceOnce once;     // attributes are per device
    cudaError_t e = once.run([] {
        cudaError_t r = allow_smem_max(attn_draft_tc_kernel<D, BITS, NST>);
        if (r != cudaSuccess) return r;
        return cudaFuncSetAttribute(attn_draft_tc_kernel<D, BITS, NST>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                                    1);
    });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kDraftThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    // No programmatic dependent launch: clusters placed early, while the
    // previous kernel (the append) still holds a few SMs, can leave a
    // cluster without room in its GPC until a whole first-wave cluster ends
    // (measured on B200 in the decode round: CTAs starting up to 100 us late,
    // the launch running in two waves).  The kernel's own griddepcontrol
    // wait is then a no-op and its trigger still lets the next kernel start.
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = da.cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_draft_tc_kernel<D, BITS, NST>, da);
}

template <int D, int BITS>
cudaError_t launch_draft_nst(int nst, const DraftArgs& da, dim3 grid, size_t smem, cudaStream_t st) {
    if (nst >= 4) return launch_draft<D, BITS, 4>(da, grid, smem, st);
    if (nst == 3) return launch_draft<D, BITS, 3>(da, grid, smem, st);
    return launch_draft<D, BITS, 2>(da, grid, smem, st);
}

}  // namespace

int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled,
                 uint32_t* comp_tickets, int raw_dtype);

int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled,
                 uint32_t* comp_tickets, int raw_dtype) {
    *handled = false;
    const int D = dims.d;
    if ((D != 64 && D != 128) || a.group > 8 || comp_tickets == nullptr) return DKV_OK;
    if (a.src.bits == 16 && raw_dtype != DKV_BF16) return DKV_OK;   // fp32 16-bit entries: generic kernel
    if (a.src.cap % 16 != 0) return DKV_OK;                         // stages copy whole 16-slot tiles
    DraftShape shp{};
    switch (a.src.bits * 1000 + D) {
        case 2064: shp = draft_shape<64, 2>(); break;
        case 3064: shp = draft_shape<64, 3>(); break;
        case 4064: shp = draft_shape<64, 4>(); break;
        case 8064: shp = draft_shape<64, 8>(); break;
        case 16064: shp = draft_shape<64, 16>(); break;
        case 2128: shp = draft_shape<128, 2>(); break;
        case 3128: shp = draft_shape<128, 3>(); break;
        case 4128: shp = draft_shape<128, 4>(); break;
        case 8128: shp = draft_shape<128, 8>(); break;
        case 16128: shp = draft_shape<128, 16>(); break;
        default: return DKV_OK;
    }
    // Cluster size, ring depth and score-buffer place.  Modelled time of a
    // bandwidth-bound launch: waves x (slots streamed by one SM in a wave +
    // a fixed per-CTA cost: query load, ring fill, merges, mass epilogue),
    // with a CTA alone on its SM charged 1.5x (it is latency-bound per warp),
    // a ring of 2 stages (one tile in flight) 1.15x and scores kept in global
    // memory (an L2 round trip per slot and head) 1.05x.
    constexpr size_t kSmemLimit = 220 * 1024, kSmSmem = 228 * 1024;
    constexpr double kFixedSlots = 512.0;
    const int pairs = dims.batch * dims.n_kv;
    const size_t tail = (size_t)(8 + 8 + 8 * D + 16) * sizeof(float);
    // scores in the work arena, past the fixed ticket region that the other
    // attention kernels keep there (counters that must stay zero between calls)
    float* gsc = nullptr;
    if (work) {
        Arena ar(work, work_bytes);
        if (ar.take<unsigned>(16384)) gsc = ar.take<float>((size_t)dims.batch * dims.n_kv * a.group * a.src.cap);
    }
    double best_cost = 0.0;
    int best_cs = 0, best_nst = 0, best_cap = 0;
    bool best_gl = false;
    size_t best_smem = 0, best_region = 0;
    for (int cs = 1; cs <= 8; ++cs) {
        const int chunk_cap = ((a.src.cap + cs - 1) / cs + 15) / 16 * 16;
        const int ctas = pairs * cs;
        for (int nst = 4; nst >= 2; --nst) {
            const size_t region = std::max((size_t)kDraftWarps * nst * shp.stage, (size_t)kDraftWarps * 8 * D * 4);
            // gl = 2: no score buffer (the mass is not folded)
            for (int gl = a.note_mass ? 0 : 2; gl < (a.note_mass ? 2 : 3); ++gl) {
                if (gl == 1 && !gsc) continue;
                const size_t smem = region + tail + (gl ? 0 : (size_t)a.group * chunk_cap * sizeof(float));
                if (smem > kSmemLimit) continue;
                // <= 128 registers a thread (launch bounds): two CTAs per SM
                // when their shared memory fits
                const int per_sm = smem + 1024 <= kSmSmem / 2 ? 2 : 1;
                const int waves = (ctas + 148 * per_sm - 1) / (148 * per_sm);
                const int busy = std::min(per_sm, (ctas + 147) / 148);    // CTAs sharing an SM
                const double cost = (double)waves * ((double)busy * chunk_cap * (nst == 2 ? 1.15 : 1.0) *
                                                         (busy == 1 ? 1.5 : 1.0) * (gl == 1 ? 1.05 : 1.0) +
                                                     kFixedSlots);
                if (best_cs == 0 || cost < best_cost - 1e-9) {
                    best_cost = cost;
                    best_cs = cs;
                    best_nst = nst;
                    best_cap = chunk_cap;
                    best_gl = gl == 1;
                    best_smem = smem;
                    best_region = region;
                }
            }
        }
    }
    if (best_cs == 0) return DKV_OK;       // too many slots per CTA: generic kernel
    DraftArgs da;
    da.a = a;
    da.cs = best_cs;
    da.chunk_cap = best_cap;
    da.region = (int)best_region;
    da.gsc = best_gl ? gsc : nullptr;
    da.raw_dtype = raw_dtype;
    da.ch16 = a.src.cb_max % 16 == 0;
    da.note_mass = a.note_mass;
    da.tickets = comp_tickets;
    da.err = device_error_word();
    da.a.src.dtype = raw_dtype;
    dim3 grid(best_cs, dims.n_kv, dims.batch);
    cudaError_t e = cudaSuccess;
    {
        ProfScope ps(DKV_PROF_ATTN_COMP, 0.0, st);
        const int n = best_nst;
        switch (a.src.bits * 1000 + D) {
            case 2064: e = launch_draft_nst<64, 2>(n, da, grid, best_smem, st); break;
            case 3064: e = launch_draft_nst<64, 3>(n, da, grid, best_smem, st); break;
            case 4064: e = launch_draft_nst<64, 4>(n, da, grid, best_smem, st); break;
            case 8064: e = launch_draft_nst<64, 8>(n, da, grid, best_smem, st); break;
            case 16064: e = launch_draft_nst<64, 16>(n, da, grid, best_smem, st); break;
            case 2128: e = launch_draft_nst<128, 2>(n, da, grid, best_smem, st); break;
            case 3128: e = launch_draft_nst<128, 3>(n, da, grid, best_smem, st); break;
            case 4128: e = launch_draft_nst<128, 4>(n, da, grid, best_smem, st); break;
            case 8128: e = launch_draft_nst<128, 8>(n, da, grid, best_smem, st); break;
            case 16128: e = launch_draft_nst<128, 16>(n, da, grid, best_smem, st); break;
            default: return DKV_OK;
        }
    }
    DKV_CUDA(e);
    DKV_LAUNCHED();
    *handled = true;
    return DKV_OK;
}

}  // namespace dkv
