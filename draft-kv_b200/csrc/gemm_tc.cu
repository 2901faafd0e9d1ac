// K4 on the fifth-generation tensor cores: the weight-streaming GEMM
// Y = X W^T with tcgen05.mma, fp32 accumulators in tensor memory (TMEM),
// weights and tokens staged in shared memory by bulk / tensor copies.
//
// Replaces the projections of draftkv/llama.py:187-225 (x @ W.T) and
// draftkv/gpt2.py:191-213 with the fused epilogues of gemm_epilogue.cuh.
//
// Shape of the work.  Decode-time GEMMs stream every weight byte once for a
// few tokens (N = batch x (gamma + 1) <= 64), so weight rows ride on the MMA's
// M (128 rows per CTA) and tokens on its N ("swap-AB"): D[128 x NB] +=
// W[128 x 16] . X[NB x 16]^T, one instruction of N = NB per k-step (NB = the
// token count rounded up to 16), so the weight operand is read from shared
// memory once per k-step.  A token's column is the same dot product in the
// same k order whatever NB is; the tests check that verify rows equal decode
// rows bit for bit.
//
// Data path per CTA (128 threads):
//   warp 0, lane 0 -- producer: per stage one bulk copy of 128 weight rows x
//     128 k (32 KB, contiguous in the packed layout below) and two tensor
//     copies of the tokens' 128 k (SWIZZLE_128B, rows past N and columns past
//     K zero-filled), all completing on the stage's mbarrier; a stage is
//     refilled as soon as the MMAs that read it commit;
//   warp 1, lane 0 -- MMA issuer: waits for a stage, issues its MMAs, commits
//     them to the stage's "empty" mbarrier, and after the last stage commits
//     to the accumulator mbarrier;
//   all four warps -- epilogue: tcgen05.ld of the accumulator (warp w owns
//     TMEM lanes 32w..32w+31 = weight rows), a [token][row] tile in shared
//     memory (the drained ring), then the split-K sum and the fused epilogue.
// The first stages' weight copies are issued before the programmatic
// dependent launch wait (weights never depend on earlier kernels); the token
// copies and every global write come after it.
//
// Split-K: the S CTAs that split one row tile's K range form a thread-block
// cluster and sum their partial tiles in rank order through distributed
// shared memory; S depends on (M, K) and the device only.  Nothing spins on
// another CTA; every mbarrier wait is bounded (error word 0x80).
//
// Packed weight layout (dkv_pack_weight): W [M][K] bf16 becomes
// [M/128][Kp/64][128 rows][64 k] (Kp = K rounded up to 64, zero padded), each
// 128 x 64 block (16 KB) in the canonical K-major SWIZZLE_128B arrangement:
// row r at byte (r/8)*1024 + (r%8)*128, its 16-byte chunk c at chunk
// position c ^ (r%8).  A plain bulk copy into a 1024-byte aligned buffer then
// reproduces exactly what the tensor core reads.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace dkv {

uint32_t* device_error_word();

constexpr int kTcStageKB = 2;                       // k blocks per stage (128 k)
constexpr int kTcThreads = 128;

// Shared-memory budget of the stage ring: 108 KB lets two CTAs share an SM,
// so a launch that follows under programmatic dependent launch places its
// CTAs (and issues its first weight copies) while this one still runs.
// Measured on B200 in the configuration-4 decode round: full-KV decode 582
// tokens/s at 108 KB, 568 at 150 KB and 200 KB (one CTA per SM).
#ifndef DKV_TC_RING_BYTES
#define DKV_TC_RING_BYTES (108 * 1024)
#endif

template <int NB>
struct TcGeo {
    static_assert(NB % 16 == 0 && NB <= 256, "token tile");
    static constexpr int XBLK = NB * 128;                               // one k block of tokens
    // k blocks per stage: 2 (128 k), 1 for the 256-token tile (4 stages of
    // 48 KB keep more copies in flight than 2 of 96 KB)
    static constexpr int SKB = NB >= 256 ? 1 : kTcStageKB;
    static constexpr int STAGE = SKB * (kTcBlockBytes + XBLK);   // multiple of 1024
    // the 256-token tile runs one CTA per SM: 4 stages (192 KB)
    static constexpr int BUDGET = NB >= 256 ? 4 * STAGE : DKV_TC_RING_BYTES;
    static constexpr int NST = STAGE * 5 <= BUDGET ? 5 : (STAGE * 4 <= BUDGET ? 4 : (STAGE * 3 <= BUDGET ? 3 : 2));
    static constexpr int TMEM_COLS = NB <= 32 ? 32 : (NB <= 64 ? 64 : (NB <= 128 ? 128 : 256));
    static constexpr size_t SMEM = (size_t)NST * STAGE + 1024;          // + alignment slack
    static_assert((size_t)NB * kTileStride * 4 <= (size_t)NST * STAGE, "epilogue tile fits the ring");
};

struct TcArgs {
    const uint8_t* w;      // packed weights
    int M, N, K, KB, S;    // KB = k blocks of 64 (K rounded up)
    uint32_t* err;         // device error word (bounded waits)
    EpiArgs epi;
};

template <int NB>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs g) {
    using Geo = TcGeo<NB>;
    constexpr int NST = Geo::NST;
    extern __shared__ uint8_t tc_raw[];
    __shared__ __align__(8) uint64_t full_bar[NST];
    __shared__ __align__(8) uint64_t empty_bar[NST];
    __shared__ __align__(8) uint64_t acc_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ float inv_s[NB];      // fused RMSNorm: 1 / rms of each token row
    uint8_t* ring = tc_raw + ((1024u - (smem_u32(tc_raw) & 1023u)) & 1023u);
    cg::cluster_group cluster = cg::this_cluster();
    const int S = g.S;
    const int s = S > 1 ? (int)cluster.block_rank() : 0;
    // one linear grid: split rank fastest (a cluster is one row tile's split
    // group), then the token block, then the row tile -- the token blocks
    // of a row tile run together and share its weights through L2
    const int nblks = (g.N + NB - 1) / NB;
    const int mtile = (int)(blockIdx.x / S) / nblks;
    const int nblk = (int)(blockIdx.x / S) % nblks, n0 = nblk * NB;
    const int kb0 = (int)((long long)s * g.KB / S), kb1 = (int)((long long)(s + 1) * g.KB / S);
    const int nstages = (kb1 - kb0 + Geo::SKB - 1) / Geo::SKB;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], 1);
        }
        mbar_init(&acc_bar, 1);
        fence_barrier_init();
        fence_async_shared();
    }
    if (warp == 1) tmem_alloc(&tmem_slot, Geo::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_trigger();

    bool ok = true;
    if (warp == 0 && lane == 0) {
        // ---------------- producer
        const uint8_t* wsrc = g.w + ((size_t)mtile * g.KB + kb0) * kTcBlockBytes;
        auto nkb_of = [&](int st) { return min(Geo::SKB, kb1 - kb0 - Geo::SKB * st); };
        auto issue_w = [&](int st) {
            const int slot = st % NST, nkb = nkb_of(st);
            uint8_t* dst = ring + (size_t)slot * Geo::STAGE;
            mbar_expect_tx(&full_bar[slot], (uint32_t)nkb * (kTcBlockBytes + Geo::XBLK));
            bulk_g2s(dst, wsrc + (size_t)st * Geo::SKB * kTcBlockBytes, (uint32_t)nkb * kTcBlockBytes,
                     &full_bar[slot]);
        };
        auto issue_x = [&](int st) {
            const int slot = st % NST, nkb = nkb_of(st);
            uint8_t* dst = ring + (size_t)slot * Geo::STAGE + Geo::SKB * kTcBlockBytes;
            for (int j = 0; j < nkb; ++j)
                tma_load_2d(dst + j * Geo::XBLK, &xmap, (kb0 + Geo::SKB * st + j) * kTcKB, n0, &full_bar[slot]);
        };
        const int pre = min(NST, nstages);
        for (int st = 0; st < pre; ++st) issue_w(st);
        pdl_wait();     // the tokens are written by earlier kernels
        for (int st = 0; st < pre; ++st) issue_x(st);
        for (int st = NST; st < nstages; ++st) {
            const int slot = st % NST;
            // the MMAs of stage st - NST read this slot: wait for their commit
            if (!mbar_wait(&empty_bar[slot], (uint32_t)((st / NST - 1) & 1), g.err)) {
                ok = false;
                break;
            }
            issue_w(st);
            issue_x(st);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        const uint32_t ring_s = smem_u32(ring);
        for (int st = 0; st < nstages; ++st) {
            const int slot = st % NST;
            const int nkb = min(Geo::SKB, kb1 - kb0 - Geo::SKB * st);
            if (!mbar_wait(&full_bar[slot], (uint32_t)((st / NST) & 1), g.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t wbase = ring_s + slot * Geo::STAGE;
            const uint32_t xbase = wbase + Geo::SKB * kTcBlockBytes;
            for (int j = 0; j < nkb; ++j) {
#pragma unroll
                for (int k16 = 0; k16 < kTcKB / 16; ++k16)
                    tc_mma<NB>(tmem, sw128_desc(wbase + j * kTcBlockBytes + k16 * 32),
                               sw128_desc(xbase + j * Geo::XBLK + k16 * 32), (st | j | k16) != 0 ? 1u : 0u);
            }
            tc_commit(&empty_bar[slot]);      // frees the slot once these MMAs have read it
        }
        tc_commit(&acc_bar);                  // the accumulator is final
    }
    __syncwarp();

    // ---------------- epilogue (all warps)
    const bool acc_ok = mbar_wait(&acc_bar, 0u, g.err);
    ok = __syncthreads_and(ok && acc_ok) != 0;      // one verdict for the CTA
    if (!ok && threadIdx.x == 0) {
        // a copy or an MMA never completed: wait (bounded) for everything
        // still in flight before shared and tensor memory are reused or freed
        for (int st = max(0, nstages - NST); st < nstages; ++st)
            mbar_wait(&full_bar[st % NST], (uint32_t)((st / NST) & 1), nullptr);
        mbar_wait(&acc_bar, 0u, nullptr);
    }
    __syncthreads();
    tc_fence_after();
    pdl_wait();      // outputs and residuals belong to earlier kernels
    float* tile = reinterpret_cast<float*>(ring);   // the drained ring holds the tile [n][m]
    if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < NB; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[(c0 + j) * kTileStride + warp * 32 + lane] = __uint_as_float(r[j]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Geo::TMEM_COLS);
    }
    const int nb = min(NB, g.N - n0);
    const int j0 = s * nb / S, j1 = (s + 1) * nb / S;
    if (S > 1) {
        cluster.sync();
        if (ok) {
            // this CTA's token rows [j0, j1): the S partial tiles summed in
            // rank order; the S loads of an element (two elements a pass) are
            // issued before the sum
            const float* rt[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) rt[q] = q < S ? cluster.map_shared_rank(tile, q) : tile;
            const int cnt = (j1 - j0) * kTileM;
            for (int e0 = threadIdx.x; e0 < cnt; e0 += 2 * kTcThreads) {
                float v[2][8];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int e = e0 + k * kTcThreads;
                    const int o = (j0 + e / kTileM) * kTileStride + e % kTileM;
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[k][q] = (q < S && e < cnt) ? rt[q][o] : 0.f;
                }
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int e = e0 + k * kTcThreads;
                    if (e >= cnt) continue;
                    float acc = v[k][0];
#pragma unroll
                    for (int q = 1; q < 8; ++q)
                        if (q < S) acc += v[k][q];
                    tile[(j0 + e / kTileM) * kTileStride + e % kTileM] = acc;
                }
            }
        }
        // done reading the other CTAs' tiles: they may leave once every CTA
        // has arrived (waited for below, after this CTA's epilogue)
        cluster_arrive();
        __syncthreads();
    }
    if (ok) {
        const bool norm_in = g.epi.norm_in_part != nullptr;
        if (norm_in) {
            epi_token_inv(g.epi, n0, j0, j1, inv_s);
            __syncthreads();
        }
        run_epilogue(g.epi, tile, mtile, n0, nb, j0, j1, norm_in ? inv_s : nullptr);
        if (g.epi.norm_out_x) {
            __syncthreads();
            epi_norm_partials(g.epi, tile, mtile, n0, j0, j1);
        }
    }
    if (S > 1) cluster_wait();    // no CTA leaves while another reads its tile
}

// Packs W [M][K] bf16 into the layout above (2-byte elements).
__global__ void pack_weight_tc_kernel(const uint16_t* __restrict__ w, int M, int K, int KB,
                                      uint16_t* __restrict__ out) {
    const size_t total = (size_t)M * KB * kTcKB;
    for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int e = (int)(o & 7);                 // element within a 16-byte chunk
        const int pc = (int)((o >> 3) & 7);         // stored chunk position
        const int r8 = (int)((o >> 6) & 7);         // row within an 8-row group
        const int g16 = (int)((o >> 9) & 15);       // 8-row group within the block
        const size_t blk = o >> 13;                 // (row tile, k block)
        const int kb = (int)(blk % KB);
        const int mt = (int)(blk / KB);
        const int c = pc ^ r8;                      // logical chunk
        const int row = mt * kTileM + g16 * 8 + r8;
        const int col = kb * kTcKB + c * 8 + e;
        out[o] = col < K ? w[(size_t)row * K + col] : (uint16_t)0;
    }
}

// ---------------------------------------------------------------- host
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode(PFN_cuTensorMapEncodeTiled_v12000* fn) {
    std::call_once(g_encode_once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    DKV_REQUIRE(g_encode, "cuTensorMapEncodeTiled is unavailable");
    *fn = g_encode;
    return DKV_OK;
}

}  // namespace

// A bf16 tensor map with 128-byte swizzle, no interleave, zero fill (shared
// by the attention kernels).
int encode_bf16_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    DKV_TRY(get_encode(&enc));
    DKV_REQUIRE(((uintptr_t)base & 15) == 0, "tensor map base not 16-byte aligned");
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides[i];
    }
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx,
                           es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    DKV_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DKV_OK;
}

// Tensor maps of the token matrices, keyed by (address, N, K, box rows): the
// activation buffers of a forward sit at fixed addresses, so a map is encoded
// once and reused.
namespace {
struct MapEntry {
    const void* x;
    int N, K, NB;
    CUtensorMap map;
};
std::mutex g_map_mu;
MapEntry g_maps[256];
int g_map_n = 0, g_map_next = 0;

}  // namespace

int token_map(const void* x, int N, int K, int NB, CUtensorMap* out) {
    std::lock_guard<std::mutex> lock(g_map_mu);
    for (int i = 0; i < g_map_n; ++i)
        if (g_maps[i].x == x && g_maps[i].N == N && g_maps[i].K == K && g_maps[i].NB == NB) {
            *out = g_maps[i].map;
            return DKV_OK;
        }
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    DKV_TRY(get_encode(&enc));
    DKV_REQUIRE(((uintptr_t)x & 15) == 0, "dkv_gemm: activations must be 16-byte aligned");
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcKB, (cuuint32_t)NB};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    DKV_REQUIRE(r == CUDA_SUCCESS, "dkv_gemm: cuTensorMapEncodeTiled failed (%d) for N=%d K=%d", (int)r, N, K);
    MapEntry& e = g_maps[g_map_next];
    e.x = x;
    e.N = N;
    e.K = K;
    e.NB = NB;
    e.map = m;
    g_map_next = (g_map_next + 1) % 256;
    g_map_n = std::min(g_map_n + 1, 256);
    *out = m;
    return DKV_OK;
}

namespace {

template <int NB>
cudaError_t tc_attrs() {
    static DeviceOnce once;
    return once.run([] {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)TcGeo<NB>::SMEM);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(gemm_tc_kernel<NB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    });
}

// Clusters of S CTAs of the kernel that can be resident at once on the
// current device (a cluster stays inside one GPC).
int tc_active(int S) {
    static int cache[64][9] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || S < 1 || S > 8) return 0;
    if (cache[dev][S] == 0) {
        if (tc_attrs<16>() != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S * 148);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = TcGeo<16>::SMEM;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<16>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return 0;
        }
        // the query counts one CTA of the kernel per SM, while two of its
        // ~110 KB CTAs run on an SM at once (measured on B200: 256 CTAs of a
        // 4096 x 4096 launch start within 2 us on 142 SMs)
        cache[dev][S] = 2 * n;
    }
    return cache[dev][S];
}

template <int NB>
cudaError_t tc_launch(const CUtensorMap& map, const TcArgs& g, int mtiles, int nblk, cudaStream_t st) {
    cudaError_t e = tc_attrs<NB>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mtiles * nblk * g.S);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = TcGeo<NB>::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = g.S;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = g.S > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<NB>, map, g);
}

}  // namespace

// K split of the tensor-core GEMM for an (M, K) weight: the S in {1, 2, 4, 8}
// (at most the number of 128-wide k stages) that minimises the modelled time
// of one CTA in k16 steps, rounds x (ceil(KB / S) x 4 + 32), where rounds =
// row tiles per cluster with as many clusters as fit at once and 32 k16
// steps charge a CTA's fixed costs (launch, first copies landing, epilogue),
// plus 8 per extra partial summed; 1 when the row tiles alone outnumber the
// CTAs that fit at once.  Depends on (M, K) and the device only.  Measured on
// B200 (decode chains of QKV, O, gate/up, down under programmatic dependent
// launch, N = 4 and 8): splits 4, 4, 1, 4 of the Llama-3-8B layer within 2 %
// of the best of the sweep.
int choose_split_tc(int M, int K) {
    const int mtiles = M / kTileM > 0 ? M / kTileM : 1;
    const int KB = (K + kTcKB - 1) / kTcKB;
    const int max_s = std::max(1, std::min(8, KB / kTcStageKB));
    // more row tiles than CTAs fit at once: the weight stream already fills
    // the GPU, a split only adds partial sums
    if (mtiles >= tc_active(1)) return 1;
    int best = 1;
    double best_cost = 0.0;
    for (int S = 1; S <= max_s; S *= 2) {
        const int act = tc_active(S);
        if (act <= 0) continue;
        const int ncl = std::min(mtiles, act);
        const int rounds = (mtiles + ncl - 1) / ncl;
        const double cost = (double)rounds * (((KB + S - 1) / S) * 4 + 32) + 8.0 * (S - 1);
        if (S == 1 || cost < best_cost - 1e-9) {
            best = S;
            best_cost = cost;
        }
    }
    return best;
}

// Token tile of a launch: N rounded up to 16 up to 64, 128 up to 512, 256
// beyond (a prompt chunk: an MMA of N = 256 reads 12 KB of operands per
// 128 x 256 x 16 product, 94 bytes a clock at the tensor rate, where N = 128
// needs the full 128 bytes a clock of shared memory).
int tc_token_tile(int N) { return N <= 64 ? (N + 15) / 16 * 16 : (N <= 512 ? 128 : 256); }

// K split for a launch whose rows need not match any other launch's (the
// prompt forward, whose rows feed only the cache): the least power of two
// that gives row tiles x token blocks x S two waves of the CTAs resident at
// once, at most choose_split_tc(M, K).  A prompt chunk of 4 x 512 tokens runs
// every Llama-3-8B projection unsplit (measured on B200, N = 2048: the QKV
// and O projections at split 4 reach 297 and 292 TF/s).
int choose_split_fill(int M, int N, int K) {
    const int cap = choose_split_tc(M, K);
    const int mtiles = M / kTileM > 0 ? M / kTileM : 1;
    const int NB = tc_token_tile(N);
    const long long ctas = (long long)mtiles * ((N + NB - 1) / NB);
    // CTAs resident at once (the 256-token tile runs one per SM); at least
    // two waves, so that no SM idles through a long last wave
    const int act = NB >= 256 ? tc_active(1) / 2 : tc_active(1);
    int S = 1;
    while (S < cap && ctas * S < 2 * act) S *= 2;
    return S;
}

size_t packed_weight_bytes_tc(int M, int K) { return (size_t)M * ((K + kTcKB - 1) / kTcKB) * kTcKB * 2; }

int pack_weight_tc(const uint16_t* w, int M, int K, uint16_t* out, cudaStream_t st) {
    DKV_REQUIRE(M % kTileM == 0 && K % 16 == 0, "dkv_pack_weight: M %% 128 and K %% 16 must be 0 (M=%d K=%d)", M, K);
    const int KB = (K + kTcKB - 1) / kTcKB;
    pack_weight_tc_kernel<<<1184, 256, 0, st>>>(w, M, K, KB, out);
    DKV_LAUNCHED();
    return DKV_OK;
}

// Launches Y = X W^T on the tensor cores with split S.
int gemm_tc(const void* x, const void* w, int M, int N, int K, int S, const EpiArgs& epi, cudaStream_t st) {
    DKV_REQUIRE(M % kTileM == 0 && K % 16 == 0, "dkv_gemm: M %% 128 and K %% 16 must be 0 (M=%d K=%d)", M, K);
    DKV_REQUIRE(((uintptr_t)w & 15) == 0, "dkv_gemm: packed weights must be 16-byte aligned");
    const int NB = tc_token_tile(N);
    const int nblk = (N + NB - 1) / NB;
    TcArgs g;
    g.w = reinterpret_cast<const uint8_t*>(w);
    g.M = M;
    g.N = N;
    g.K = K;
    g.KB = (K + kTcKB - 1) / kTcKB;
    g.S = S;
    g.err = device_error_word();
    g.epi = epi;
    DKV_REQUIRE(S >= 1 && S <= g.KB, "dkv_gemm: split %d outside 1..%d", S, g.KB);
    DKV_REQUIRE(g.err, "dkv_gemm: device error word unavailable");
    CUtensorMap map;
    DKV_TRY(token_map(x, N, K, NB, &map));
    const int mtiles = M / kTileM;
    cudaError_t e;
    switch (NB) {
        case 16: e = tc_launch<16>(map, g, mtiles, nblk, st); break;
        case 32: e = tc_launch<32>(map, g, mtiles, nblk, st); break;
        case 48: e = tc_launch<48>(map, g, mtiles, nblk, st); break;
        case 64: e = tc_launch<64>(map, g, mtiles, nblk, st); break;
        case 128: e = tc_launch<128>(map, g, mtiles, nblk, st); break;
        default: e = tc_launch<256>(map, g, mtiles, nblk, st); break;
    }
    DKV_CUDA(e);
    DKV_LAUNCHED();
    return DKV_OK;
}

}  // namespace dkv

