/*
 * xkv_oracle.h -- CPU restatement of kvexp's XKV codec and scalar decode attention.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or calls this
 * code; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, and
 * only as the checker.  It restates, in plain C, the algorithms of the reference project
 * cvs0/compressed-kv-attention (library `kvexp`):
 *
 *   ox_encode_bf16     src/codec.cpp:39-164 (best_base :18-35)
 *   ox_decode_bf16     src/codec.cpp:166-174 over XkvReader include/kvexp/scan.hpp:79-165
 *   ox_parse_block     include/kvexp/scan.hpp:28-66
 *   ox_block_walk      include/kvexp/scan.hpp:94-123 / :192-218 (linear header walk)
 *   ox_attention_decode  src/dispatch.cpp:27-104 with detail::range_scalar
 *                      src/attention_scalar.cpp:46-85, apply_token :19-42, hsum8 :13-17,
 *                      softmax_coeff / merge_state / finalize_state src/softmax.hpp:8-41
 *
 * Build flags must be -ffp-contract=off -fno-fast-math (the reference's own flags,
 * CMakeLists.txt:48), so fmaf/expf/+/* round exactly as the reference's scalar kernel.
 * Errors are returned as codes instead of C++ exceptions; ox_last_error() holds the
 * reference's exception message for the failure.
 */
#ifndef XKV_ORACLE_H
#define XKV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes: which C++ exception type the reference throws for the same failure. */
enum {
    OX_OK = 0,
    OX_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    OX_RUNTIME = 2,          /* std::runtime_error    */
    OX_LOGIC = 3             /* std::logic_error      */
};

const char *ox_last_error(void);

/* Container size model, include/kvexp/bf16.hpp:39-49. */
int ox_exp_payload_bytes(int n_tokens, int dim, int bits);
int ox_coded_block_bytes(int n_tokens, int dim, int bits, int n_escape);
int ox_raw_block_bytes(int n_tokens, int dim);

/* Upper bound on the container bytes encode can produce for [seq, dim]. */
size_t ox_encode_bound(int seq, int dim, int block_tokens);

/* Encode [seq, dim] BF16 bits into `out` (capacity out_cap). *out_bytes = container size.
 * Per-block mode choice is written to modes[] (one byte per block) when modes != NULL. */
int ox_encode_bf16(const uint16_t *kv, int seq, int dim, int block_tokens, uint8_t *out,
                   size_t out_cap, size_t *out_bytes, uint8_t *modes);

/* Decode an XKV container into [seq, dim] BF16 bits. */
/* The same with a mask of allowed code widths (bit b: b-bit residuals): OX_MODES_REFERENCE is the
 * reference encoder's {2, 4}; OX_MODES_ALL adds this library's 3-bit extension. */
#define OX_MODES_REFERENCE ((1 << 2) | (1 << 4))
#define OX_MODES_ALL ((1 << 2) | (1 << 3) | (1 << 4))
int ox_encode_bf16_modes(const uint16_t *kv, int seq, int dim, int block_tokens, int mode_mask,
                         uint8_t *out, size_t out_cap, size_t *out_bytes, uint8_t *modes);

int ox_decode_bf16(const uint8_t *blob, size_t bytes, int seq, int dim, uint16_t *out);

/* One parsed block header (include/kvexp/scan.hpp:12-22 BlockView, as offsets). */
typedef struct {
    int mode, n_tokens, n_escape;
    size_t offset;   /* header offset inside the blob */
    size_t next;     /* offset of the byte after this block */
} ox_block;

/* Parse the block at `offset`; returns an error code (scan.hpp:28-66 rules). */
int ox_parse_block(const uint8_t *blob, size_t bytes, size_t offset, int dim, ox_block *b);

/* Walk every header of a blob. Fills up to cap entries, *n_blocks = count.
 * Also checks that the blocks cover exactly `seq` tokens when seq > 0. */
int ox_block_walk(const uint8_t *blob, size_t bytes, int dim, int seq, ox_block *blocks,
                  int cap, int *n_blocks);

/* kvexp::attention_decode restated for the Scalar backend (also bit-identical to Avx2,
 * tests/test_main.cpp:146-148).  n_threads ranges run one after another and fold in thread
 * order exactly like the OpenMP region of src/dispatch.cpp:79-102. */
int ox_attention_decode(const uint16_t *q, const uint16_t *k_raw, const uint16_t *v_raw,
                        const uint8_t *k_xkv, size_t k_bytes, const uint8_t *v_xkv,
                        size_t v_bytes, float *out, int n_q, int dim, int seq, int n_threads,
                        int split_tokens);

/* Bench-style model_heads loop (src/bench.cpp:711-728): units one after another, each a
 * single-thread attention_decode over XKV blobs.  Used for the timed CPU baseline. */
int ox_model_heads(int n_units, const uint16_t *const *q, const uint8_t *const *k_xkv,
                   const size_t *k_bytes, const uint8_t *const *v_xkv, const size_t *v_bytes,
                   float *const *out, int n_q, int dim, int seq);

#ifdef __cplusplus
}
#endif

#endif
