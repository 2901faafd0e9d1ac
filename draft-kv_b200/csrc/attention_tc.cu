// Tensor-core attention kernels (bf16 caches): verify / baseline over the
// paged full cache, and the drafter over quantized slots.  Shapes they do not
// cover report handled = false and the generic kernel runs instead.
#include "common.cuh"

namespace dkv {
struct AttnArgs;
struct dkv_dims_fwd;

int attn_full_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, int max_keys, cudaStream_t st,
                 bool* handled) {
    (void)a;
    (void)dims;
    (void)work;
    (void)work_bytes;
    (void)max_keys;
    (void)st;
    *handled = false;
    return DKV_OK;
}

int attn_comp_tc(AttnArgs& a, dkv_dims dims, void* work, size_t work_bytes, cudaStream_t st, bool* handled) {
    (void)a;
    (void)dims;
    (void)work;
    (void)work_bytes;
    (void)st;
    *handled = false;
    return DKV_OK;
}
}  // namespace dkv
