// attention.cuh -- declarations shared by the attention kernels and the host plan code.
#pragma once

#include <cstddef>

#include "common.cuh"

namespace kvx {

// One flat block of a batched step: the K and V index entries of the same token range.
// For the BF16 kernel, whose "blocks" are tiles of block_tokens rows of a plain [seq, dim] array,
// k_off / v_off hold the tile's first token.
struct FlatBlock {
    uint32_t k_off;   // XKV: header offset in the K blob.  BF16: first token.
    uint32_t v_off;   // XKV: header offset in the V blob.  BF16: first token.
    uint32_t k_rec;   // escape record of the K block in the step's record array (u32 units)
    uint32_t v_rec;
    uint16_t k_nesc;  // escape words
    uint16_t v_nesc;
    uint8_t k_mode;   // 0 raw, 2, 3 (extension), 4
    uint8_t v_mode;
    uint8_t n_tok;    // tokens in the encoded block (layout)
    uint8_t valid;    // tokens attended (< n_tok only for the last block of a unit)
    int32_t unit;     // device unit the block belongs to
    int32_t src;      // flat block whose escape records this one shares (itself unless it is the
                      // same K/V block seen by another query group of the same unit)
};
static_assert(sizeof(FlatBlock) == 32, "FlatBlock is 32 bytes");

// Escape record of one coded block with escape words (u32 array):
//   [0, 16)           e[i - 1] = escape words of tokens [0, 16 i), i = 1..16 (clamped to the
//                     block), so the escapes of tokens [16 a, 16 b) are [e(a), e(b)), e(0) = 0;
//   [16, 16 + n_esc)  for every escape, in the container's scan order: the byte of the element it
//                     replaces in the attention kernel's BF16 tile (esc_scratch_slot of its token
//                     within the kernel's stage and its channel) in bits 0-15, the escape word
//                     (the element's BF16 value) in bits 16-31.
// Built once per plan from the blob's residual codes and escape words; raw blocks and blocks
// without escapes have none.
constexpr int kEscRecHead = 16;

// Tokens of one MMA tile of the attention kernel: each consumer warp decodes 16-token tiles of
// K and V into its BF16 tile and runs them through the tensor cores.
constexpr int kTileTokens = 16;

// Byte of element (token r of a 16-token tile, channel c) in the attention kernel's BF16 tile:
// rows of 2 dim bytes, 16-byte chunks XOR-swizzled by the row (chunk c / 8 of row r sits at chunk
// position (c / 8) ^ (r & 7), or ^ ((r / 2) & 3) for dim 32).  The same for K and V.
__host__ __device__ inline uint32_t esc_scratch_slot(int dim, int T, int r, int c) {
    (void)T;
    const int c8 = c >> 3;
    const int sw = dim == 32 ? (r >> 1) & 3 : r & 7;
    return uint32_t(r * 2 * dim + ((c8 ^ sw) << 4) + 2 * (c & 7));
}

// Consumer warps per CTA of the attention kernel (one CTA per SM; one more warp issues the
// copies): a CTA of 16 warps at 128 registers a thread for dim <= 64, 12 at 168 for dim 128, 8 at
// 255 for dim 256.  A stage of 128 tokens (64 at dim 128, 32 at dim 256) is 8 (4, 2) tiles, dealt
// round robin.
__host__ __device__ constexpr int attention_consumer_warps(int dim) {
    return dim >= 256 ? 7 : (dim >= 128 ? 11 : 15);
}

// Tokens per ring stage of the attention kernel: 8 KiB of BF16 per tensor (128 tokens at dim <= 64).
__host__ __device__ constexpr int attention_stage_tokens(int dim) {
    return 8192 / dim < 128 ? 8192 / dim : 128;
}

__device__ __forceinline__ FlatBlock load_flat(const FlatBlock *f, int64_t i) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(f + i));
    const uint4 b = __ldg(reinterpret_cast<const uint4 *>(f + i) + 1);
    FlatBlock r;
    r.k_off = a.x;
    r.v_off = a.y;
    r.k_rec = a.z;
    r.v_rec = a.w;
    r.k_nesc = uint16_t(b.x & 0xFFFF);
    r.v_nesc = uint16_t(b.x >> 16);
    r.k_mode = uint8_t(b.y & 0xFF);
    r.v_mode = uint8_t((b.y >> 8) & 0xFF);
    r.n_tok = uint8_t((b.y >> 16) & 0xFF);
    r.valid = uint8_t(b.y >> 24);
    r.unit = int32_t(b.z);
    r.src = int32_t(b.w);
    return r;
}

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

// Everything the attention kernel needs to stream one flat block, built once per plan (after
// the escape records) and fetched by one 128-byte bulk copy, two blocks ahead of its use.
struct BlockDesc {
    uint64_t k, v;          // XKV: address of the K / V block header.  BF16: of the block's first row.
    uint32_t k_rec, v_rec;  // FlatBlock::k_rec / v_rec
    uint16_t k_nesc, v_nesc;
    uint8_t k_mode, v_mode, n_tok, valid;
    int32_t unit;
    uint8_t align[4];       // K rows, K codes, V rows, V codes: offset of the section's first byte
                            // in its 16-byte line (codes 0 for a raw block)
    uint8_t flags;          // kDescFirst | kDescLast
    uint8_t pad0[3];
    int32_t b7_block;       // flat block whose merge words (AttnArgs::b7) this block uses
    uint8_t pad1[16];
    uint16_t em[2][16];     // K / V escape count headers, e(i) at [i - 1] (zeros without a record)
};
static_assert(sizeof(BlockDesc) == 128 && offsetof(BlockDesc, align) == 36 &&
                  offsetof(BlockDesc, b7_block) == 44 && offsetof(BlockDesc, em) == 64,
              "BlockDesc layout");
constexpr uint8_t kDescFirst = 1, kDescLast = 2;  // the first / last block of its unit

// Copy list of one ring stage of the attention kernel, built once per plan (launch_stage_table)
// so that a producer warp only loads it and issues: kStageRecWords 16-byte words, word i read by
// producer lane i.  Words 0-7 are the stage's pieces {source address (low, high), bytes copied
// (a multiple of 16; 0: none), destination offset in the ring slot}: 0 the block descriptor, 1 the
// merge words, 2 + 3 T / 3 + 3 T / 4 + 3 T tensor T's rows (with the codes when the stage is the
// whole block), residual codes and escape-record entries.  Word 8: {K escape entries, V escape
// entries (int32 offsets in the slot from which entry i is read at + 4 i), the stage's total
// bytes, bit 0 / 1: the K / V entries are staged (else they stay in HBM)}.
constexpr int kStageRecWords = 9;

struct AttnArgs {
    const UnitDev *units;
    const FlatBlock *flat;      // [n_blocks]
    const BlockDesc *desc;      // [n_blocks]
    const uint4 *stages;        // [n_blocks][stages_per_block][kStageRecWords] copy lists, or null
                                // (the producer then works the pieces out from the descriptors)
    const uint32_t *esc;        // escape records (FlatBlock::k_rec / v_rec index it)
    const uint32_t *b7;         // [n_blocks][dim] merge words of each coded block: K, then V
    const int64_t *range_begin; // [n_ranges + 1] flat-block range of each CTA
    const int32_t *seg_base;    // [n_ranges] first partial-state row of each CTA
    float *partials;            // [rows][consumer warps][partial_stride(dim)]
    int *status;                // [2] first error (code, detail)
    int n_ranges;
    int stages_per_block;       // > 0: every block takes this many ring stages (empty ones past
                                //      its tokens); 0: each block takes as many as its tokens need
};

// A unit as the combine pass sees it (host-built, so the kernel's first load is all it needs):
// where its outputs go and the contiguous run of partial states [first_state, first_state +
// n_states) that its blocks left (one per consumer warp of every CTA that held some of them).
struct SplitUnit {
    float *out;
    float *lse;
    int32_t first_state, n_states, n_q, q_stride, pad0, pad1;
};
static_assert(sizeof(SplitUnit) == 40, "SplitUnit is 40 bytes");

struct CombineArgs {
    const SplitUnit *split;
    const float *partials;
};

// Partial-state stride (floats) of one consumer warp's segment: m[8], l[8], acc[8][dim].
__host__ __device__ inline int partial_stride(int dim) { return 16 + 8 * dim; }

// Partial-state rows of a step: every CTA writes one row (all its consumer warps) per unit segment
// in its block range, rows numbered CTA by CTA; a unit's rows are therefore contiguous.  From the
// CTA ranges and the units' flat block ranges (in flat order): seg_base[c] = first row of CTA c,
// and per unit its first row and row count.  Returns the number of rows.
inline int64_t segment_rows(const int64_t *range_begin, int n_ranges, const int64_t *unit_begin,
                            const int32_t *unit_blocks, int n_units, int32_t *seg_base,
                            int32_t *unit_first_row, int32_t *unit_rows) {
    int64_t row = 0;
    int u = 0;
    for (int i = 0; i < n_units; ++i) unit_rows[i] = 0;
    for (int c = 0; c < n_ranges; ++c) {
        seg_base[c] = int32_t(row);
        int64_t b = range_begin[c];
        const int64_t e = range_begin[c + 1];
        while (b < e) {
            while (u < n_units && unit_begin[u] + unit_blocks[u] <= b) ++u;
            if (unit_rows[u]++ == 0) unit_first_row[u] = int32_t(row);
            ++row;
            b = unit_begin[u] + unit_blocks[u] < e ? unit_begin[u] + unit_blocks[u] : e;
        }
    }
    return row;
}

// Launchers (attention.cu).  Return cudaError_t of the launch.
// compact: every block of the step is coded (the 6-slot ring sized for coded stages; raw rows do
// not fit its slots).
cudaError_t launch_attention(int dim, bool bf16_input, bool compact, const AttnArgs &a, int grid,
                             cudaStream_t s);
cudaError_t launch_combine(int dim, const CombineArgs &a, int n_split, cudaStream_t s);
// Merge words of a step's coded blocks (blocks that share another block's K/V blocks -- a later
// query group of the same unit -- use that block's): for block f and tensor T, word w of
// b7 + f dim + T dim / 2 holds the base exponents of head dims 2w and 2w + 1 moved to where the
// decode adds the residual codes (base[2w] << 7 | base[2w + 1] << 23).
cudaError_t launch_b7(const UnitDev *units, const FlatBlock *flat, int64_t n_blocks, int dim,
                      uint32_t *b7, cudaStream_t s);
// Block descriptors of a step from its flat blocks, units and escape records.
cudaError_t launch_block_desc(const UnitDev *units, const FlatBlock *flat, const uint32_t *esc, int64_t n,
                              int dim, bool bf16, BlockDesc *desc, cudaStream_t s);
// Stage copy lists of a step (stages_per_block stages of every flat block) from its block
// descriptors, merge words and escape records.
cudaError_t launch_stage_table(int dim, bool bf16, bool compact, const BlockDesc *desc, const uint32_t *b7,
                               const uint32_t *esc, int64_t n_blocks, int stages_per_block,
                               uint4 *table, cudaStream_t s);
cudaError_t launch_fold(const float *parts, int n_parts, int n_rows, int dim, float *out,
                        float *lse_out, cudaStream_t s);
// m = -inf, l = 0 in n_states partial states (so that states no warp writes add nothing).
cudaError_t launch_init_partials(float *partials, int64_t n_states, int dim, cudaStream_t s);
// out[0] = the largest number of attended tokens of any flat block; out[1] != 0 when some block
// has a raw K or V.
cudaError_t launch_max_valid(const FlatBlock *flat, int64_t n_blocks, int *out, cudaStream_t s);
// Escape records: sizes and offsets (single CTA; *total receives the record array length in u16,
// blocks whose src is another block take that block's offsets, and a record that would end past
// `cap` entries reports DERR_ESC_CAP), then the records themselves (the fill reports
// DERR_ESC_OVERRUN for a block with more sentinels than escape words).
cudaError_t launch_esc_layout(FlatBlock *flat, int64_t n_blocks, unsigned long long *total,
                              unsigned long long cap, int *status, cudaStream_t s);
cudaError_t launch_esc_fill(const UnitDev *units, const FlatBlock *flat, int64_t n_blocks, int dim,
                            uint32_t *esc, unsigned long long cap, int *status, cudaStream_t s);
// Cost-balanced CTA ranges over the flat block list: range_begin[0..n_ranges].  by_tokens: every
// attended token costs the same whatever the block's encoding (the split then depends only on
// the token counts, so an XKV step and a BF16 step over the same tokens get the same ranges).
cudaError_t launch_split(const FlatBlock *flat, int64_t n_blocks, int n_ranges, bool by_tokens, int dim,
                         int64_t *range_begin, cudaStream_t s);
bool attention_dim_supported(int dim);

}  // namespace kvx
