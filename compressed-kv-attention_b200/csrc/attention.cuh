// attention.cuh -- declarations shared by the attention kernels and the host plan code.
#pragma once

#include "common.cuh"

namespace kvx {

// One flat block of a batched step: the K and V index entries of the same token range.
// `tok0` is the block's first token (used by the BF16 kernel, whose "blocks" are tiles of
// block_tokens rows of a plain [seq, dim] array).
struct FlatBlock {
    uint32_t k_off;   // XKV: header offset in the K blob.  BF16: first token.
    uint32_t v_off;   // XKV: header offset in the V blob.  BF16: first token.
    uint16_t k_nesc;  // escape words
    uint16_t v_nesc;
    uint8_t k_mode;   // 0 raw, 2, 4
    uint8_t v_mode;
    uint8_t n_tok;    // tokens in the encoded block (layout)
    uint8_t valid;    // tokens attended (< n_tok only for the last block of a unit)
};
static_assert(sizeof(FlatBlock) == 16, "FlatBlock is 16 bytes");

// Device copy of one unit.
struct UnitDev {
    const uint8_t *k;
    const uint8_t *v;
    const uint16_t *q;
    float *out;
    int64_t block_begin;  // flat index of the unit's first block
    int32_t n_blocks;
    int32_t n_q;          // <= 8 (larger query groups are split into several units)
    int32_t q_stride;     // elements between query rows of q / out
    int32_t pad0;
    float *lse;           // optional [n_q]: log-sum-exp of the scores per query
};
static_assert(sizeof(UnitDev) == 64, "UnitDev is 64 bytes");

struct AttnArgs {
    const UnitDev *units;
    const FlatBlock *flat;      // [n_blocks]
    const int32_t *flat_unit;   // [n_blocks] unit of each flat block
    const int64_t *range_begin; // [n_workers + 1] flat-block range of each worker warp
    float *partials;            // [n_workers][2][8 + 8 + 8 * dim]
    int *status;                // [2] first error (code, detail)
    int n_workers;
};

struct CombineArgs {
    const UnitDev *units;
    const int32_t *split_units;   // units whose blocks span several workers
    const int64_t *range_begin;    // [n_workers + 1]
    const float *partials;
    int n_workers;
};

// Partial-state stride (floats) for one (worker, slot): m[8], l[8], acc[8][dim].
__host__ __device__ inline int partial_stride(int dim) { return 16 + 8 * dim; }

// Worker that owns flat block b: the last worker whose range starts at or before b.
__host__ __device__ inline int worker_of_block(const int64_t *range_begin, int n_workers, int64_t b) {
    int lo = 0, hi = n_workers - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (range_begin[mid] <= b) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Launchers (attention.cu).  Return cudaError_t of the launch.
cudaError_t launch_attention(int dim, bool bf16_input, const AttnArgs &a, int grid, cudaStream_t s);
cudaError_t launch_combine(int dim, const CombineArgs &a, int n_split, cudaStream_t s);
// Cost-balanced worker ranges over the flat block list: range_begin[0..n_workers].
cudaError_t launch_split(const FlatBlock *flat, int64_t n_blocks, int n_workers, int64_t *range_begin,
                         cudaStream_t s);
int attention_workers_per_cta(int dim);
size_t attention_smem_bytes(int dim);
bool attention_dim_supported(int dim);

}  // namespace kvx
