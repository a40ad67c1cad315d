// codec.cuh -- device XKV codec: header walk (block index), plan flattening, decode and encode.
#pragma once

#include "attention.cuh"

namespace kvx {

// Encoder per-block analysis (phase 1 output).
struct EncBlock {
    uint32_t bytes;   // container bytes of the block
    uint16_t n_esc;
    uint8_t mode;
    uint8_t n_tok;
};

// Index walk of one device blob (single thread; validates like parse_block).
// Exponent statistics per (block, dim): best[w][block][dim] for code widths 3, 7, 15 and
// entropy[block][dim] (see exp_stats_kernel).
cudaError_t launch_exp_stats(const uint16_t *kv, int seq, int dim, int bt, int *best, float *entropy,
                             cudaStream_t s);
cudaError_t launch_index_walk(const uint8_t *blob, uint64_t bytes, int dim, kvx_block *index,
                              uint32_t *tok_start, int cap, int *counts /*[2] blocks, tokens lo*/,
                              long long *n_tokens, int *status, cudaStream_t s);

// Flatten units into FlatBlock entries (validates entries against blob sizes and seq).  Unit u's
// blocks start at flat index block_begin[u]; src_begin[u] (NULL: block_begin) is the flat index
// of the first block of the unit whose K/V blocks -- and escape records -- they are.
cudaError_t launch_build_flat(const kvx_unit *units, const int64_t *block_begin,
                              const int64_t *src_begin, int n_units, int dim, int block_tokens,
                              bool bf16, FlatBlock *flat, int *status, cudaStream_t s);

// Decode blocks [0, n_blocks) of a blob into [seq, dim] BF16 (out rows beyond seq untouched).
cudaError_t launch_decode(const uint8_t *blob, const kvx_block *index, const uint32_t *tok_start,
                          int n_blocks, int dim, int seq, uint16_t *out, int *status,
                          cudaStream_t s);

// Encoder phase 1: one CTA per block of n_tensors tensors of [seq, dim] (device pointer table).
// code_bits: the residual widths a block may take (bit b: b-bit codes; KVX_CODE_BITS_*).
cudaError_t launch_encode_analyze(const uint16_t *const *tensors, int n_tensors, int seq, int dim,
                                  int block_tokens, int code_bits, EncBlock *blocks, uint8_t *bases,
                                  cudaStream_t s);
// Encoder phase 3: emit blocks at byte offsets (per block, relative to `arena`).
cudaError_t launch_encode_emit(const uint16_t *const *tensors, int n_tensors, int seq, int dim,
                               int block_tokens, const EncBlock *blocks, const uint8_t *bases,
                               const uint64_t *block_off, uint8_t *arena, kvx_block *index,
                               const uint64_t *blob_off, int *status, cudaStream_t s);

// [rows, dim] BF16 -> [rows, dp] BF16 with zero columns past dim.
cudaError_t launch_pad_rows(const uint16_t *in, int64_t rows, int dim, int dp, uint16_t *out,
                            cudaStream_t s);

cudaError_t launch_synth(uint16_t *out, int seq, int dim, uint64_t seed, uint64_t stream_id,
                         int profile, uint32_t rate, cudaStream_t s);
cudaError_t launch_read_probe(const uint4 *buf, size_t n16, uint32_t *sink, int grid,
                              cudaStream_t s);

}  // namespace kvx
