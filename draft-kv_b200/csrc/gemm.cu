// K4 weight-streaming GEMM (Y = X W^T): the C-ABI entry points, the split
// choice and the fp32 CUDA-core kernel; the bf16 kernel runs on the tensor
// cores (tcgen05 + TMEM, gemm_tc.cu) and both share the fused epilogues of
// gemm_epilogue.cuh.
//
// Replaces the projections of draftkv/llama.py:187-225 (x @ W.T, SwiGLU :222,
// tied head :224-225, RoPE :197-198 with _rope :164-172) and
// draftkv/gpt2.py:191-213 (Conv1D x @ W + b, gelu_new :126-127, tied head).
//
// Determinism / batch invariance: the split of K across CTAs (S) depends
// only on (M, K) and the device, partial sums are reduced in a fixed order
// (bf16: by the CTAs of a thread-block cluster through distributed shared
// memory; fp32: by the last CTA of each row tile, atomic ticket, no spin),
// and a token's column never depends on the other columns, so a token's
// output is bit-identical whether it is computed with 1 or 64 other tokens.
// This is what makes the verify pass reproduce plain decoding exactly.
#include <algorithm>

#include "gemm_epilogue.cuh"

namespace dkv {

// Split-K tickets of the fp32 kernel occupy a fixed region at the start of
// every GEMM work buffer, so consecutive calls of any shape see them zero
// (each launch resets the tickets it used).
constexpr size_t kGemmTickets = 65536;

uint32_t* device_error_word();
// tensor-core GEMM (gemm_tc.cu)
int choose_split_tc(int M, int K);
int gemm_tc(const void* x, const void* w, int M, int N, int K, int S, const EpiArgs& epi, cudaStream_t st);
int pack_weight_tc(const uint16_t* w, int M, int K, uint16_t* out, cudaStream_t st);
size_t packed_weight_bytes_tc(int M, int K);

// Split-K finish of the fp32 kernel: every CTA of a row tile leaves its
// partial tile; the last to arrive sums them in split order and runs the
// epilogue.
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
    const void* x;      // [N][K] f32
    const void* w;      // [M][K] f32 row-major
    int M, N, K, S;
    float* ws;
    unsigned* tickets;
    EpiArgs epi;
};

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

// K split of the fp32 kernel: S = floor(128 / row tiles) capped at 4 and at
// the number of 256-wide k chunks (one wave of few, long CTAs); depends on
// (M, K) only -- never on the token count.
int choose_split(int M, int K) {
    const int mtiles = M / kTileM > 0 ? M / kTileM : 1;
    const int max_s = K / 256 > 0 ? K / 256 : 1;
    int S = 128 / mtiles;
    S = S < 1 ? 1 : (S > 4 ? 4 : S);
    return S < max_s ? S : max_s;
}

// Columns the epilogue writes: m < min(M, ld_out) (the head is padded to 128
// rows; SwiGLU writes d_ff = ld_out columns from 2 d_ff rows).
int epilogue_columns(const dkv_epilogue* epi, int M, int* M_real, const char* who) {
    *M_real = M;
    if (epi->kind != DKV_EPI_QKV) {
        DKV_REQUIRE(epi->ld_out > 0, "%s: ld_out required", who);
        *M_real = std::min(M, epi->ld_out);
    } else {
        DKV_REQUIRE(epi->q_out && epi->pos0 && epi->d_head > 0 && kTileM % epi->d_head == 0,
                    "%s QKV: q_out/pos0 required and d_head must divide 128", who);
        DKV_REQUIRE(epi->kv_stage || (epi->full && epi->full->k_pool), "%s QKV: no K/V destination", who);
    }
    if (epi->norm_in_part)
        DKV_REQUIRE(epi->norm_n_part > 0 && epi->norm_dm > 0 && epi->norm_ld > 0,
                    "%s: fused norm input needs norm_n_part, norm_dm and norm_ld", who);
    if (epi->norm_out_x || epi->norm_out_part || epi->norm_out_w)
        DKV_REQUIRE(epi->kind == DKV_EPI_RESADD && epi->norm_out_x && epi->norm_out_part && epi->norm_out_w &&
                        epi->norm_ld > 0,
                    "%s: fused norm output needs RESADD and norm_out_x, norm_out_part, norm_out_w, norm_ld", who);
    return DKV_OK;
}

// The fused norm sides live in the tensor-core kernel's epilogue only.
int fused_norm_bf16_only(const dkv_epilogue* epi, int w_dtype, int N, const char* who) {
    const bool fused = epi->norm_in_part || epi->norm_out_x;
    DKV_REQUIRE(!fused || w_dtype == DKV_BF16, "%s: fused RMSNorm needs bf16 weights", who);
    DKV_REQUIRE(!fused || epi->norm_ld >= N, "%s: norm_ld (%d) < N (%d)", who, epi->norm_ld, N);
    return DKV_OK;
}

}  // namespace dkv

using namespace dkv;

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
    a.norm_in_part = e->norm_in_part;
    a.norm_n_part = e->norm_n_part;
    a.norm_ld = e->norm_ld;
    a.norm_dm = e->norm_dm;
    a.norm_eps = e->norm_eps;
    a.norm_out_part = e->norm_out_part;
    a.norm_out_x = e->norm_out_x;
    a.norm_out_w = e->norm_out_w;
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
    if (w_dtype != DKV_F32) return 256;     // bf16: the split-K partials stay in the clusters' shared memory
    const int mtiles = (M + kTileM - 1) / kTileM;
    const int S = choose_split(mtiles * kTileM, K);
    const int nblk = (N + kF32Tok - 1) / kF32Tok;
    const size_t tile = (size_t)kF32Tok * kTileStride * sizeof(float);
    size_t b = kGemmTickets * sizeof(unsigned);
    if (S > 1) b += (size_t)nblk * mtiles * S * tile;
    return b + 256;
}

extern "C" size_t dkv_pack_weight_bytes(int M, int K) {
    if (M <= 0 || K <= 0) return 0;
    return packed_weight_bytes_tc(M, K);
}

extern "C" int dkv_pack_weight(const uint16_t* w, int M, int K, uint16_t* packed, void* stream) {
    DKV_REQUIRE(w && packed && M > 0 && K > 0, "dkv_pack_weight args");
    return pack_weight_tc(w, M, K, packed, (cudaStream_t)stream);
}

namespace {

int launch_f32(const void* x, const void* w, int M, int N, int K, int S, const EpiArgs& epi, float* ws,
               unsigned* tickets, cudaStream_t st) {
    GemmArgs g;
    g.x = x;
    g.w = w;
    g.M = M;
    g.N = N;
    g.K = K;
    g.S = S;
    g.ws = ws;
    g.tickets = tickets;
    g.epi = epi;
    const int mtiles = M / kTileM;
    dim3 grid(mtiles * S, (N + kF32Tok - 1) / kF32Tok);
    const size_t smem = std::max((size_t)kF32Tok * kF32Chunk * 4, (size_t)kF32Tok * kTileStride * 4);
    gemm_f32_kernel<<<grid, 256, smem, st>>>(g);
    DKV_LAUNCHED();
    return DKV_OK;
}

}  // namespace

namespace dkv {
int choose_split_fill(int M, int N, int K);

// dkv_gemm with `fill` set: a bf16 launch takes the K split that fills the
// GPU for this N (choose_split_fill) instead of the one of (M, K) alone, for
// rows that no other launch's rows are compared with (the prompt forward).
int gemm_entry(const void* x, int x_dtype, const void* w, int w_dtype, int M, int N, int K, const dkv_epilogue* epi,
               void* work, size_t work_bytes, void* stream, bool fill) {
    DKV_REQUIRE(x && w && epi && M > 0 && N >= 0 && K > 0, "dkv_gemm: bad arguments");
    DKV_REQUIRE(x_dtype == w_dtype, "dkv_gemm: x and w dtypes must match");
    DKV_REQUIRE(w_dtype == DKV_BF16 || w_dtype == DKV_F32, "dkv_gemm: dtype must be bf16 or f32");
    DKV_REQUIRE(M % kTileM == 0, "dkv_gemm: M (%d) must be padded to a multiple of 128", M);
    DKV_REQUIRE(K % 16 == 0, "dkv_gemm: K (%d) must be a multiple of 16", K);
    if (N == 0) return DKV_OK;
    int M_real = M;
    DKV_TRY(epilogue_columns(epi, M, &M_real, "dkv_gemm"));
    DKV_TRY(fused_norm_bf16_only(epi, w_dtype, N, "dkv_gemm"));
    const EpiArgs ea = make_epi(epi, M_real);
    cudaStream_t st = (cudaStream_t)stream;
    // algorithmic bytes: the weights once, the activations in and out
    const double elem = w_dtype == DKV_F32 ? 4.0 : 2.0;
    ProfScope ps(DKV_PROF_GEMM, (double)M_real * K * elem + (double)N * K * elem + (double)N * M_real * 4.0, st);
    if (w_dtype == DKV_BF16)
        return gemm_tc(x, w, M, N, K, fill ? choose_split_fill(M, N, K) : choose_split_tc(M, K), ea, st);
    const int mtiles = M / kTileM;
    const int S = choose_split(M, K);
    const int nblk = (N + kF32Tok - 1) / kF32Tok;
    DKV_REQUIRE((size_t)nblk * mtiles <= kGemmTickets, "dkv_gemm: too many row tiles x token blocks");
    Arena ar(work, work_bytes);
    unsigned* tickets = ar.take<unsigned>(kGemmTickets);
    float* ws = S > 1 ? ar.take<float>((size_t)nblk * mtiles * S * kF32Tok * kTileStride) : nullptr;
    DKV_REQUIRE(tickets && (S == 1 || ws), "dkv_gemm: work buffer too small (%zu bytes, need %zu)", work_bytes,
                dkv_gemm_work_bytes(M, N, K, w_dtype));
    return launch_f32(x, w, M, N, K, S, ea, ws, tickets, st);
}
}  // namespace dkv

extern "C" int dkv_gemm(const void* x, int x_dtype, const void* w, int w_dtype, int M, int N, int K,
                        const dkv_epilogue* epi, void* work, size_t work_bytes, void* stream) {
    return dkv::gemm_entry(x, x_dtype, w, w_dtype, M, N, K, epi, work, work_bytes, stream, false);
}

// ---------------------------------------------------------------------------
// dkv_gemm_noalloc: the same GEMM for callers that cannot allocate.
//
// Some callers cannot hand the library a work buffer: code that runs where
// device allocation is unavailable or forbidden (inside an allocator hook or
// an out-of-memory handler, a host that preallocated its whole HBM pool up
// front, a plugin whose framework owns every allocation).  For them the
// split-K partial tiles and the arrival tickets of the fp32 kernel live in
// one fixed array compiled into this library, so the call needs nothing but
// its inputs and outputs (the bf16 tensor-core kernel sums its partials in
// shared memory and needs no scratch at all).  The array costs DKV_GEMM_NOALLOC_SCRATCH_BYTES of device memory
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
        g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return DKV_OK;
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
    DKV_TRY(epilogue_columns(epi, M, &M_real, "dkv_gemm_noalloc"));
    DKV_TRY(fused_norm_bf16_only(epi, w_dtype, N, "dkv_gemm_noalloc"));
    if (N == 0) return DKV_OK;
    const EpiArgs ea = make_epi(epi, M_real);
    cudaStream_t st = (cudaStream_t)stream;
    // bf16: the tensor-core kernel keeps its split-K partials in the
    // clusters' shared memory and needs no scratch (same launch as dkv_gemm)
    if (w_dtype == DKV_BF16) return gemm_tc(x, w, M, N, K, choose_split_tc(M, K), ea, st);
    // fp32: the same K split as dkv_gemm, partials summed in the same order
    // by the last CTA of each row tile, in the fixed array
    const int mtiles = M / kTileM;
    const int S = choose_split(M, K);
    const int nblk = (N + kF32Tok - 1) / kF32Tok;
    const size_t tickets = (size_t)nblk * mtiles;
    const size_t partial_bytes = S > 1 ? tickets * S * kF32Tok * kTileStride * sizeof(float) : 0;
    // an unsplit launch touches neither the tickets nor the partials
    DKV_REQUIRE(S == 1 || tickets * sizeof(unsigned) <= kNoAllocTicketBytes,
                "dkv_gemm_noalloc: %zu row tiles x token blocks exceed the %zu tickets of the fixed scratch "
                "(use dkv_gemm with a work buffer)", tickets, kNoAllocTicketBytes / sizeof(unsigned));
    DKV_REQUIRE(partial_bytes <= kNoAllocBytes - kNoAllocTicketBytes,
                "dkv_gemm_noalloc: M=%d N=%d K=%d needs %zu bytes of split-K scratch, the fixed array holds %zu "
                "(use dkv_gemm with a work buffer)", M, N, K, partial_bytes, kNoAllocBytes - kNoAllocTicketBytes);
    unsigned char* scratch = nullptr;
    DKV_TRY(noalloc_scratch(&scratch));
    // The array keeps whatever the previous call left; the tickets must start
    // at zero (a launch that stopped early can leave one raised).
    if (S > 1) DKV_CUDA(cudaMemsetAsync(scratch, 0, tickets * sizeof(unsigned), st));
    return launch_f32(x, w, M, N, K, S, ea, S > 1 ? reinterpret_cast<float*>(scratch + kNoAllocTicketBytes) : nullptr,
                      reinterpret_cast<unsigned*>(scratch), st);
}
