/*
 * draftkv_b200 -- C ABI of the B200 (sm_100a) self-speculative decode step.
 *
 * The reference (aabhimittal/Draft-KV) is a pure-numpy package with no FFI;
 * each entry point below replaces a named python function of it (file:line in
 * the reference tree), so a binding (ctypes, cffi, cgo ...) can drive the
 * device path with plain pointers.
 *
 * Conventions
 *   - every function returns int status: DKV_OK (0) or a DKV_E* code; the
 *     message of the last failure on the calling thread is dkv_last_error();
 *     no C++ exception crosses this boundary;
 *   - pointers named d_* are device pointers; everything is caller-owned
 *     (the library never allocates device memory and never frees; the one
 *     exception is the fixed DKV_GEMM_NOALLOC_SCRATCH_BYTES array that the
 *     library image itself holds on every GPU that loads it, see
 *     dkv_gemm_noalloc);
 *   - `stream` is a cudaStream_t passed as void*; all work is stream-ordered,
 *     no function synchronizes the host unless documented;
 *   - the library only launches kernels, so a sequence of calls may be
 *     captured into a CUDA graph (after one warm-up call per kernel shape,
 *     which sets kernel attributes).
 *
 * Device memory layouts (all row-major, innermost last)
 *   full (authoritative) KV, paged -- one pool shared by all layers:
 *       k_pool, v_pool  [n_pages][n_kv][page_size][d]      (f32 or bf16)
 *       page_table      [batch][n_layers][max_pages]        int32
 *     position p of (sequence b, layer L) lives in page
 *     page_table[b][L][p / page_size], row p % page_size.
 *   drafter (compressed) KV -- per (sequence, layer) a slot array of `cap`:
 *       k_codes, v_codes [batch][n_layers][n_kv][cap][cb_max]  uint8
 *       k_sl, v_sl       [batch][n_layers][n_kv][cap][d/64][2]   fp16 (scale, lo)
 *       pos              [batch][n_layers][cap]   int32, -1 = empty slot
 *       score            [batch][n_layers][cap]   f32 accumulated attention mass
 *       mass             [batch][n_layers][n_kv][cap] f32 (per-call scratch)
 *       meta             [batch][n_layers][4]     int32 {hwm, count, 0, 0}
 *       seen             [batch]                  int32 logical context length
 *       tickets          [batch][n_layers][64]    uint32, zero at creation
 *     a layer of `bits` uses cb = d*bits/8 bytes per vector (16 bits: the
 *     vector stored unquantized in the model dtype, cb = d*elem).
 *
 * Code order and bit layout of one packed vector (d a multiple of 64; codes
 * are the unsigned q of the quantizer, one fp16 (scale, lo) pair per group of
 * 64 elements in element order):
 *   storage order -- V vectors: element order.  K vectors: the tensor-core
 *     fragment order: for lane quad c = 0..3 and k-step j = 0..d/16-1 the four
 *     elements 16j+2c, 16j+2c+1, 16j+2c+8, 16j+2c+9 follow each other; quad c
 *     owns one contiguous quarter of the vector, k-steps in order;
 *   8 bits: one byte per code, in storage order;
 *   4 bits: each 32-bit little-endian word holds 8 codes of storage positions
 *     8w..8w+7: position 8w+2i at bits [4i, 4i+4), 8w+2i+1 at [16+4i, 20+4i);
 *   2 bits: each word holds 16 codes: 16w+2i at bits [2i, 2i+2), 16w+2i+1 at
 *     [16+2i, 18+2i);
 *   3 bits: two planes: plane A (d/4 bytes) holds every code's low two bits in
 *     the 2-bit layout; plane B (d/8 bytes) follows and holds the high bits,
 *     16 codes per 16-bit unit: position 16u+2i at bit i, 16u+2i+1 at 8+i.
 */
#ifndef DRAFTKV_B200_H
#define DRAFTKV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DKV_API __attribute__((visibility("default")))
#else
#define DKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { DKV_OK = 0, DKV_EINVAL = 1, DKV_ECUDA = 2, DKV_EUNSUPPORTED = 3, DKV_EDEVICE = 4 };
enum { DKV_F32 = 0, DKV_BF16 = 1 };
enum { DKV_ARCH_LLAMA = 0, DKV_ARCH_GPT2 = 1 };

/* ------------------------------------------------------------ plumbing */
DKV_API const char* dkv_last_error(void);
DKV_API int dkv_version(void);
/* Reads and clears the device error word kernels set instead of trapping:
 * 0x10 append rows over the per-call limit, 0x20 drafter slot capacity,
 * 0x100 token id outside the vocabulary, 0x200 position outside the table. */
DKV_API int dkv_device_error(uint32_t* out_code, void* stream);

/* Launch timing by kernel class with CUDA events on the launching stream
 * (no library counterpart in the reference, which has no profiler: it serves
 * the roofline numbers).  start() creates up to max_records event pairs and
 * enables recording; summary() waits for the events and sums one class. */
enum {
    DKV_PROF_GEMM = 0, DKV_PROF_ATTN_FULL = 1, DKV_PROF_ATTN_COMP = 2, DKV_PROF_APPEND = 3,
    DKV_PROF_REBUILD = 4, DKV_PROF_NORM = 5, DKV_PROF_EMBED = 6, DKV_PROF_SAMPLE = 7, DKV_PROF_ACCEPT = 8
};
DKV_API int dkv_prof_start(int max_records);
DKV_API int dkv_prof_stop(void);
DKV_API int dkv_prof_summary(int kind, double* total_ms, int64_t* launches, double* total_bytes);

/* ------------------------------------------------------------ K1 quantize
 * Replaces draftkv/compress.py:21-46 `quantize(x, bits, group=64)`.
 * x [rows][d] f32.  Per group of 64 (zero padded): lo=min, hi=max,
 * scale=max((hi-lo)/(2^bits-1), 1e-8), q=clip(rint((x-lo)/scale)), deq=q*scale+lo,
 * IEEE fp32 arithmetic without contraction, bit-identical to numpy.
 * Outputs (any may be NULL): codes [rows][ceil(d/64)*64] u8, scale/lo
 * [rows][ceil(d/64)] f32, deq [rows][d] f32.  bits in {2,3,4,8}; bits 16 copies x. */
DKV_API int dkv_quantize(const float* d_x, int64_t rows, int d, int bits, uint8_t* d_codes,
                 float* d_scale, float* d_lo, float* d_deq, void* stream);

/* Packs rows into the drafter storage format: codes in the K (fragment) or V
 * (element) order and fp16 (scale, lo).  src [rows][d] in `src_dtype`.
 * The bytes follow the code order and bit layout stated at the top of this
 * file (the tests check them against an independent packing). */
DKV_API int dkv_quantize_pack(const void* d_src, int src_dtype, int64_t rows, int d, int bits,
                      int k_order, uint8_t* d_codes, uint16_t* d_sl, void* stream);

/* ------------------------------------------------------------ caches */
typedef struct {
    void* k_pool;
    void* v_pool;
    const int32_t* page_table;
    int n_pages, page_size, max_pages, dtype;
} dkv_full_cache;

/* Drafter cache (slot arrays).  k_codes / v_codes: batch x n_layers x n_kv
 * regions of cap * cb_max bytes; a layer's vectors are stored densely inside
 * its region at the width of its current configuration (d*bits/8 bytes,
 * 16-bit entries d * element size), slot s at byte s * width.  k_sl / v_sl:
 * per vector and 64-group fp16 (scale, lo).  pos: batch x n_layers x cap
 * (-1 = empty); score (H2O, accumulated only for layers with keep < 1) and
 * mass: batch x n_layers [x n_kv] x cap; meta: {high-water mark, live count,
 * -, -} per (sequence, layer); cap is a multiple of 16. */
typedef struct {
    uint8_t* k_codes;
    uint8_t* v_codes;
    uint16_t* k_sl;
    uint16_t* v_sl;
    int32_t* pos;
    float* score;
    float* mass;
    int32_t* meta;
    int32_t* seen;
    uint32_t* tickets;
    int cap, cb_max;
    /* per layer (host arrays of n_layers): bits, keep_frac, sink, recent */
    const int32_t* bits;
    const double* keep;
    const int32_t* sink;
    const int32_t* recent;
} dkv_comp_cache;

typedef struct {
    int n_layers, n_kv, d, batch;
} dkv_dims;

/* Writes rows into the full cache: for sequence b, row r goes to position
 * pos0[b] + r (r < n_rows[b] when n_rows != NULL, else r < rows).
 * src [batch][rows][n_kv][d] in the cache dtype.  Replaces the append of
 * draftkv/compress.py:59-63 / draftkv/paged.py:120-128. */
DKV_API int dkv_full_write(const dkv_full_cache* full, dkv_dims dims, int layer, const void* d_src,
                   int rows, const int32_t* d_pos0, const int32_t* d_n_rows, void* stream);

/* Gathers positions [0, n) of (b, layer) from the full cache into dst
 * [n][n_kv][d] (cache dtype).  Replaces draftkv/compress.py:65-73 read(). */
DKV_API int dkv_full_read(const dkv_full_cache* full, dkv_dims dims, int b, int layer, int n,
                  void* d_dst, void* stream);

/* Drafter append: replaces draftkv/compress.py:122-133 (append) with
 * :154-179 (budget, eviction) and :181-188 (truncate), fused.
 * For each sequence b and each layer in [layer0, layer0+n_layer_sel):
 *   1. if trunc[b] >= 0: drop entries with pos >= trunc[b];
 *   2. quantize n_rows[b] rows (positions pos0[b] + r) into free slots, score 0;
 *   3. evict: protect the `sink` lowest and `recent` highest positions, drop
 *      the lowest (score, position) others down to the budget
 *      max(rint(keep*max(seen,1)), sink+recent).
 * Rows come from src [batch][rows_stride][n_kv][d] (src_dtype) when src != NULL,
 * else from the full cache at those positions.  `seen` follows the
 * reference: clipped to trunc, advanced to last position+1 when advance_seen.
 * The pending per-head attention mass of each layer is folded into `score`
 * by the attention kernel, so scores are current when this runs. */
DKV_API int dkv_comp_append(const dkv_comp_cache* comp, const dkv_full_cache* full, dkv_dims dims,
                    int layer0, int n_layer_sel, const void* d_src, int src_dtype,
                    int rows_stride, const int32_t* d_pos0, const int32_t* d_n_rows,
                    const int32_t* d_trunc, int advance_seen, void* stream);

/* Rebuild of whole layers from the full cache: replaces
 * draftkv/compress.py:209-230 rebuild_layers() and the first
 * sync_from(full, 0) (:190-207).  Every listed layer of every sequence is
 * cleared and refilled with positions [0, ctx[b]) under eviction with all
 * scores zero, i.e. the sink rows and the newest (budget - sink) rows, which
 * are the only ones quantized.  layers: host array of n_sel layer indices. */
DKV_API int dkv_comp_rebuild(const dkv_comp_cache* comp, const dkv_full_cache* full, dkv_dims dims,
                     const int32_t* layers, int n_sel, const int32_t* d_ctx,
                     int advance_seen, void* stream);

/* Reads layer `layer` of sequence b back, dequantized, in position order:
 * k, v [n][n_kv][d] f32, pos [n] int32; *n_out = number of live entries
 * (host sync).  Replaces draftkv/compress.py:135-142 read() (tests only). */
DKV_API int dkv_comp_read(const dkv_comp_cache* comp, dkv_dims dims, int b, int layer, int max_n,
                  float* d_k, float* d_v, int32_t* d_pos, float* d_score, int* n_out,
                  void* stream);

/* ------------------------------------------------------------ attention
 * Verify / baseline attention over the full cache (draftkv/llama.py:202-219,
 * draftkv/gpt2.py:197-207 with cache = FullKVCache/PagedKVCache): for
 * sequence b, T query tokens at positions pos0[b] .. pos0[b]+T-1, each of the
 * n_kv*group heads attends keys 0 .. its own position (causal).
 * q [batch*T][n_kv*group][d] f32; out [batch*T][n_kv*group*d] (out_dtype).
 * Up to 64 query rows (T * group <= 64: decode, verify) keys are split in
 * fixed chunks of split_keys positions and a row's result does not depend on
 * T (verify row i == decode at that position, bit for bit).  More rows (a
 * prompt chunk) in bf16 take the prompt kernel with splits of at least
 * 16384 keys: within bf16 rounding of the same attention, not bitwise equal
 * to the rows of a decode call. */
DKV_API int dkv_attn_full(const dkv_full_cache* full, dkv_dims dims, int layer, int group, int T,
                  const float* d_q, const int32_t* d_pos0, void* d_out, int out_dtype,
                  int split_keys, void* d_work, size_t work_bytes, void* stream);

/* Draft attention over the drafter cache, T = 1 (same python lines with
 * cache = CompressedKVCache), plus the attention mass of
 * draftkv/compress.py:144-151 note_attention and the GQA group sum of
 * draftkv/llama.py:213-216, folded into `score` in a fixed order. */
DKV_API int dkv_attn_comp(const dkv_comp_cache* comp, dkv_dims dims, int layer, int group,
                  const float* d_q, const int32_t* d_qpos, void* d_out, int out_dtype,
                  void* d_work, size_t work_bytes, void* stream);

/* Scratch bytes the two attention calls need for a given shape. */
DKV_API size_t dkv_attn_work_bytes(dkv_dims dims, int group, int T, int max_ctx, int split_keys,
                           int comp_cap);

/* ------------------------------------------------------------ GEMM
 * Y = X W^T for the projections, MLP and head (draftkv/llama.py:187-225,
 * draftkv/gpt2.py:191-213).  bf16 runs on the tensor cores (tcgen05.mma,
 * accumulators in tensor memory) from weights packed once by
 * dkv_pack_weight; f32 runs on the CUDA cores from row-major weights. */
enum {
    DKV_EPI_STORE = 0,     /* out_f32[n][m] = acc + bias                          */
    DKV_EPI_RESADD = 1,    /* h[n][m] += acc + bias                               */
    DKV_EPI_GELU = 2,      /* act[n][m] = gelu_new(acc + bias)  (act dtype)        */
    DKV_EPI_SWIGLU = 3,    /* rows interleaved 64 gate / 64 up: act = silu(g)*u   */
    DKV_EPI_QKV = 4        /* split q / k / v, RoPE, write K/V (see dkv_epilogue) */
};

typedef struct {
    int kind;
    const float* bias;          /* [M] or NULL */
    float* out_f32;             /* STORE: [N][ld_out]; RESADD: residual h [N][ld_out] */
    void* act;                  /* GELU/SWIGLU output [N][ld_out] */
    int act_dtype, ld_out;
    /* QKV */
    int n_heads, n_kv, d_head, tokens_per_seq;
    const int32_t* pos0;        /* [batch] */
    const float* rope_cos;      /* [max_pos][d/2] or NULL (no rotation) */
    const float* rope_sin;
    float* q_out;               /* [N][n_heads][d] */
    void* kv_stage;             /* [N][n_kv][d] K then V at +N*n_kv*d, or NULL */
    const dkv_full_cache* full; /* write K/V into this cache when kv_stage == NULL */
    int layer, n_layers;
    /* Fused RMSNorm (draftkv/llama.py:93-94), bf16 weights only; all NULL /
     * 0 when unused.  Input side: X holds bf16(h * w) (not yet divided by the
     * rms) and token n's accumulators are multiplied by
     * 1 / sqrt(sum_t norm_in_part[t * norm_ld + n] / norm_dm + norm_eps)
     * (t < norm_n_part, summed in t order) before bias and epilogue.
     * Output side (RESADD only): besides h, writes norm_out_x[n][m] =
     * bf16(h_new[n][m] * norm_out_w[m]) (ld_out columns) and
     * norm_out_part[(m / 128) * norm_ld + n] = sum of h_new^2 over the 128
     * rows m of that row tile, the next GEMM's input side. */
    const float* norm_in_part;
    int norm_n_part, norm_ld, norm_dm;
    float norm_eps;
    float* norm_out_part;
    void* norm_out_x;
    const float* norm_out_w;
} dkv_epilogue;

/* Packed layout of a bf16 weight W [M][K] (M % 128 == 0 after padding,
 * K % 16 == 0): [M/128][Kp/64][128 rows][64 k], Kp = K rounded up to 64
 * (zero columns), each 128 x 64 block (16 KB) in the tensor core's K-major
 * 128-byte-swizzle arrangement: row r at byte (r/8)*1024 + (r%8)*128, its
 * 16-byte chunk c (k = 8c .. 8c+7) at chunk position c ^ (r%8).
 * dkv_pack_weight_bytes(M, K) = M * Kp * 2.  f32 weights are used as-is
 * ([M][K] row-major).  X (bf16) must be 16-byte aligned. */
DKV_API size_t dkv_pack_weight_bytes(int M, int K);
DKV_API int dkv_pack_weight(const uint16_t* d_w, int M, int K, uint16_t* d_packed, void* stream);

/* The work buffer (dkv_gemm_work_bytes; a few bytes for bf16) must be zero
 * when first used: the fp32 kernel's split-K arrival tickets live in it and
 * every call leaves them zero again.  One buffer must not serve calls that
 * may run at the same time (different streams without ordering). */
DKV_API int dkv_gemm(const void* d_x, int x_dtype, const void* d_w, int w_dtype, int M, int N, int K,
             const dkv_epilogue* epi, void* d_work, size_t work_bytes, void* stream);
DKV_API size_t dkv_gemm_work_bytes(int M, int N, int K, int w_dtype);

/* dkv_gemm for callers that cannot allocate device memory: no counterpart in
 * the reference (which has no native code).  Same arguments as dkv_gemm minus
 * the work buffer, and bit-identical results (the same K split, partials
 * summed in the same order).  The bf16 kernel needs no scratch; the f32
 * kernel's split-K scratch is a fixed array of DKV_GEMM_NOALLOC_SCRATCH_BYTES
 * compiled into the library, held on every GPU that loads it until the
 * process exits.  f32 split shapes whose scratch exceeds it return DKV_EINVAL
 * with a message (e.g. 4096 x 4096 at 320 tokens); unsplit shapes use no
 * scratch and have no such limit.  Allocates nothing.  The first f32 call on
 * a device does that device's set-up (the array's device address); make it
 * outside stream capture, and do not call across a cudaDeviceReset() of a
 * device already used.  All calls on a device share the array: calls that
 * overlap on the GPU race. */
#define DKV_GEMM_NOALLOC_SCRATCH_BYTES (16u << 20)
DKV_API int dkv_gemm_noalloc(const void* d_x, int x_dtype, const void* d_w, int w_dtype, int M, int N, int K,
                             const dkv_epilogue* epi, void* stream);

/* ------------------------------------------------------------ small ops */
/* h[n] = emb[tok(n)] (+ pos_emb[pos0[b] + t]); tok(n) = tokens[b*tok_stride + t].
 * Replaces draftkv/gpt2.py:186 and draftkv/llama.py:180.  Ids outside
 * [0, vocab) and positions outside [0, max_pos) are reported in the device
 * error word (dkv_device_error) and read as row 0. */
DKV_API int dkv_embed(const void* d_emb, int emb_dtype, const void* d_pos_emb, const int32_t* d_tokens,
              int tok_stride, int batch, int T, const int32_t* d_pos0, int d_model, int vocab,
              int max_pos, float* d_h, void* stream);
/* x = rmsnorm(h)*w (draftkv/llama.py:93-94) or layernorm(h)*w+b (draftkv/gpt2.py:120-123). */
DKV_API int dkv_norm(const float* d_h, int N, int d_model, int layernorm, const float* d_w,
             const float* d_b, float eps, void* d_x, int x_dtype, void* stream);

/* ------------------------------------------------------------ K5 sampling
 * Replaces draftkv/engine.py:36-42 (_probs), :101-106 (_sample).
 * For each of `rows` logits rows [rows][V]: T <= 0 -> first argmax; else a
 * draw from softmax(logits/T) (fp64) with a Philox4x32-10 uniform keyed by
 * (seed, counter, row).  tokens[r*tok_stride] receives the result. */
DKV_API int dkv_sample(const float* d_logits, int rows, int V, float temperature, uint64_t seed,
               const uint64_t* d_counter, int32_t* d_tokens, int tok_stride, void* d_work,
               size_t work_bytes, void* stream);

/* Acceptance (draftkv/engine.py:188-213) for a batch of sequences:
 *   greedy: k = first i with argmax(verify[i]) != draft[i]; next = argmax(verify[k]);
 *   T > 0: accept draft i if u < min(1, p_i[d]/q_i[d]) (q_i[d] == 0 rejects),
 *          next ~ p_gamma when all accepted, else ~ norm(max(p_k - q_k, 0))
 *          (p_k when that is all zero).
 * verify [batch][gamma+1][V], draft_logits [gamma][batch][V] (T > 0 only),
 * vtok [batch][vstride]: vtok[b][1+i] = draft i.  Writes accepted[b], next[b];
 * then advances the round state on device: vtok[b][0] = next,
 * base_pos[b] += accepted+1, and the resync arguments
 * rs_pos0[b] = old base_pos, rs_rows[b] = accepted+1, rs_trunc[b] = old base_pos. */
DKV_API int dkv_accept(const float* d_verify, const float* d_draft_logits, int batch, int gamma, int V,
               float temperature, uint64_t seed, const uint64_t* d_counter, int32_t* d_vtok,
               int vstride, int32_t* d_base_pos, int32_t* d_accepted, int32_t* d_next,
               int32_t* d_rs_pos0, int32_t* d_rs_rows, int32_t* d_rs_trunc,
               const int32_t* d_active, void* d_work, size_t work_bytes, void* stream);
DKV_API size_t dkv_sample_work_bytes(int rows, int V);

/* ------------------------------------------------------------ forward
 * One forward pass of the whole decoder for `batch` sequences x T tokens
 * (draftkv/llama.py:175-225, draftkv/gpt2.py:182-213): embed, per layer norm /
 * QKV (+RoPE, K/V write) / attention / output projection / norm / MLP, final
 * norm and head.  comp == NULL: attention over the full cache (prefill chunk,
 * verify, baseline decode).  comp != NULL: draft step, T must be 1, K/V are
 * appended to the drafter cache (quantize + evict) instead of the full cache. */
typedef struct {
    const float* n1_w; const float* n1_b;
    const void* w_qkv; const float* b_qkv;
    const void* w_o;   const float* b_o;
    const float* n2_w; const float* n2_b;
    const void* w_up;  const float* b_up;      /* llama: gate/up interleaved by 64 rows */
    const void* w_down; const float* b_down;
} dkv_layer;

typedef struct {
    int arch, dtype;
    int n_layers, d_model, n_heads, n_kv, d_head, d_ff, vocab, vocab_pad, max_pos;
    float eps;
    const void* tok_emb;          /* [vocab][d_model] (model dtype) */
    const void* pos_emb;          /* gpt2 [max_pos][d_model] else NULL */
    const float* rope_cos;        /* llama [max_pos][d_head/2] */
    const float* rope_sin;
    const void* w_head;           /* tiled/row-major [vocab_pad][d_model] */
    const float* nf_w; const float* nf_b;
    const dkv_layer* layers;      /* host array [n_layers] */
    int split_keys;
} dkv_model;

typedef struct {
    int batch, T;
    const int32_t* tokens;        /* token (b,t) = tokens[b*tok_stride + t] */
    int tok_stride;
    const int32_t* pos0;          /* [batch] position of token t=0 */
    float* logits;                /* [batch*T][vocab_pad] f32, or NULL: no final norm and head
                                     (a prefill that only writes the cache; the reference discards
                                     those logits, draftkv/engine.py:133-134).  With NULL each
                                     projection takes the K split that fills the GPU for batch*T
                                     tokens, so the cache rows it writes match a logits forward's
                                     within bf16 rounding, not bit for bit */
    /* scratch (caller allocates dkv_forward_work_bytes) */
    void* work;
    size_t work_bytes;
    int max_ctx;
    int max_T;                    /* workspace layout T (>= T); one buffer serves all T <= max_T */
} dkv_step;

/* Work bytes for `batch` sequences and up to max_T tokens each.  The buffer
 * must be zero when first used (split-K / merge tickets live in it and are
 * left zero by every call) and must not be shared by concurrent streams. */
DKV_API size_t dkv_forward_work_bytes(const dkv_model* m, int batch, int max_T, int max_ctx, int comp_cap);
DKV_API int dkv_forward(const dkv_model* m, const dkv_full_cache* full, const dkv_comp_cache* comp,
                const dkv_step* st, void* stream);

#ifdef __cplusplus
}
#endif
#endif
