/*
 * kvexp_b200.h -- C ABI of the B200 (sm_100a) implementation of kvexp's compressed-KV decode
 * attention and XKV codec.
 *
 * The first block of entry points replaces the reference library's public C++ API one for one
 * (same argument order and meaning; a C++ exception becomes a status code whose kind says which
 * exception type the reference throws, and kvx_last_error() holds its message).  Pointers in
 * those calls may be host or device memory; the library detects which.  The second block is the
 * GPU-native batched interface for device-resident caches (no reference counterpart except the
 * per-head loop it replaces).
 *
 * Every entry point returns KVX_OK (0) or a kvx_status.  Calls are synchronous unless they take a
 * stream.  Device pointers given to the batched interface must be 16-byte aligned, and the
 * allocation behind an XKV blob must stay readable up to the next 16-byte boundary after its
 * last byte (cudaMalloc and the PyTorch caching allocator both guarantee this).
 */
#ifndef KVEXP_B200_H
#define KVEXP_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KVX_API __attribute__((visibility("default")))
#else
#define KVX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1..3 name the C++ exception type the reference throws for the same failure. */
typedef enum kvx_status {
    KVX_OK = 0,
    KVX_ERR_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    KVX_ERR_RUNTIME = 2,          /* std::runtime_error: malformed blob, backend, ... */
    KVX_ERR_LOGIC = 3,            /* std::logic_error: encoder size-model drift */
    KVX_ERR_CUDA = 4,             /* a CUDA runtime call failed */
    KVX_ERR_TIMEOUT = 5,          /* a bounded device-side wait expired */
    KVX_ERR_UNSUPPORTED = 6       /* shape outside this library's kernels */
} kvx_status;

/* Backend selector of the reference (include/kvexp/attention.hpp:10-14).  All three run the same
 * GPU kernels here; the value only selects which shape rule and error text the reference applies
 * (dim % 8 for Scalar/Avx2, dim % 32 for Avx512Bf16). */
enum { KVX_BACKEND_SCALAR = 0, KVX_BACKEND_AVX2 = 1, KVX_BACKEND_AVX512BF16 = 2 };

/* Message of the last failure on the calling thread ("" after success). */
KVX_API const char *kvx_last_error(void);

/* Library version string. */
KVX_API const char *kvx_version(void);

/* ---- drop-in replacements of the reference API ------------------------------------------- */

/* Replaces kvexp::detect_cpu (include/kvexp/attention.hpp:21, src/cpu.cpp:35-61): instead of
 * CPUID it reports the current CUDA device.  Returns KVX_ERR_RUNTIME when no sm_100 device. */
KVX_API int kvx_device_info(int *sm_major, int *sm_minor, int *sm_count, size_t *hbm_bytes);

/* Replaces kvexp::attention_decode (include/kvexp/attention.hpp:58-61, src/dispatch.cpp:27-104).
 * One decode step for n_q queries sharing one KV head: out[n_q, dim] (FP32) =
 * softmax(q K^T) V with the online-softmax semantics of src/softmax.hpp.  Exactly one of
 * (k_raw, k_xkv) and of (v_raw, v_xkv) is non-NULL.  n_threads and split_tokens keep their
 * reference meaning for validation (a thread split that falls inside an encoded block is an
 * error, as in the reference); the GPU chooses its own parallel split.  For XKV input the GPU
 * result is bit-identical to the same call with raw K/V of the decoded values. */
KVX_API int kvx_attention_decode(int backend, const uint16_t *q, const uint16_t *k_raw,
                         const uint16_t *v_raw, const uint8_t *k_xkv, size_t k_bytes,
                         const uint8_t *v_xkv, size_t v_bytes, float *out, int n_q, int dim,
                         int seq, int n_threads, int split_tokens);

/* Batched form of the reference's per-head loop (src/bench.cpp:711-728 `model_heads`): n_units
 * independent attention_decode calls over XKV blobs, all with the same n_q, dim, seq, run as one
 * GPU job.  Pointer arrays live in host memory; the pointers they hold may be host or device.
 * With host buffers the blobs go to the GPU on a library-owned non-blocking stream while the host
 * walks their headers and builds the step's plan; the call returns when the outputs are back.
 * Its device buffers come from the device's default CUDA memory pool, whose release threshold
 * the library raises to 1 GiB (the pool then keeps up to 1 GiB between calls).  Outputs in host
 * memory come back through a pinned host buffer the library keeps per device (the size of the
 * largest call's outputs). */
KVX_API int kvx_attention_decode_units(int backend, int n_units, const uint16_t *const *q,
                               const uint8_t *const *k_xkv, const size_t *k_bytes,
                               const uint8_t *const *v_xkv, const size_t *v_bytes,
                               float *const *out, int n_q, int dim, int seq, int split_tokens);

/* Replaces kvexp::encode_bf16 (include/kvexp/codec.hpp:45-46, src/codec.cpp:39-164): encodes
 * [seq_len, head_dim] BF16 bits into the XKV container, byte-identical to the reference.
 * `out` must hold kvx_encode_bound() bytes; *out_bytes receives the container size. */
KVX_API size_t kvx_encode_bound(int seq_len, int head_dim, int block_tokens);
KVX_API int kvx_encode_bf16(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                    uint8_t *out, size_t out_capacity, size_t *out_bytes);

/* Residual code widths the encoder may choose per block, as a bit mask (bit b: b-bit codes).
 * KVX_CODE_BITS_REFERENCE is the reference encoder's {2, 4} (what kvx_encode_bf16,
 * kvx_encode_batch and kvx_cache_append use); KVX_CODE_BITS_ALL adds the 3-bit mode, this
 * library's extension of the container, which the reference measured (README.md:35) and does not
 * implement: mode byte 3, base window of 7 exponents with code 7 the escape sentinel, element i's
 * code in bits [3 i, 3 i + 3) of the little-endian code bytes, the code section padded with a zero
 * byte to an even length.  Blobs holding mode-3 blocks are read by every entry point of this
 * library and rejected by the reference ("unknown xkv block mode").  The mode choice extends the
 * reference's tie rules: smaller block, then raw, then fewer escapes, then the narrower code. */
#define KVX_CODE_BITS_REFERENCE 0x14
#define KVX_CODE_BITS_ALL 0x1C

/* kvx_encode_bf16 with a code-width mask (KVX_CODE_BITS_REFERENCE gives the same bytes).  No
 * counterpart in the reference (3-bit blocks are this library's extension). */
KVX_API int kvx_encode_bf16_bits(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                         int code_bits, uint8_t *out, size_t out_capacity, size_t *out_bytes);

/* The statistics behind the reference's exponent analyser (python/analyze_exponents.py:57-72
 * `block_conditional_entropy`, :117-156 `policy_size`), on the GPU.  For every block of
 * block_tokens tokens of a [seq_len, head_dim] BF16 tensor (the last block may be shorter) and
 * every head dim: best[w][block][dim] = the largest number of the block's exponents that fall in
 * any window of 3, 7 or 15 consecutive exponents (w = 0, 1, 2: 2-, 3- and 4-bit residual codes),
 * entropy[block][dim] = Shannon entropy (bits) of the block's exponents.  kv, best and entropy
 * may be host or device memory; best holds 3 * n_blocks * head_dim ints, entropy
 * n_blocks * head_dim floats. */
KVX_API int kvx_exponent_stats(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                               int *best, float *entropy);

/* Replaces kvexp::decode_bf16 (include/kvexp/codec.hpp:48, src/codec.cpp:166-174). */
KVX_API int kvx_decode_bf16(const uint8_t *blob, size_t bytes, int seq_len, int head_dim,
                    uint16_t *out);

/* ---- GPU-native batched interface (device-resident caches) -------------------------------- */

/* One entry per encoded block: the block-offset index that the reference recomputes by walking
 * headers (include/kvexp/scan.hpp:94-123, :192-218).  Written by the GPU encoder or built once
 * by kvx_xkv_index. */
typedef struct kvx_block {
    uint32_t offset;   /* byte offset of the block header inside its blob */
    uint16_t n_escape; /* escape words (0 for raw blocks) */
    uint8_t mode;      /* 0 raw, 2 or 4 bits */
    uint8_t n_tokens;  /* tokens in the block */
} kvx_block;

/* Walk the headers of a device-resident blob and write its index (device memory, capacity
 * max_blocks).  Validates every header like parse_block (include/kvexp/scan.hpp:28-66).
 * *n_blocks and *n_tokens receive the counts (host).  Synchronous. */
KVX_API int kvx_xkv_index(const uint8_t *blob, size_t bytes, int head_dim, kvx_block *index,
                  int max_blocks, int *n_blocks, long long *n_tokens);

/* One (layer, KV head[, sequence]) unit of a batched decode step.  All pointers are device
 * pointers.  For XKV caches k_index/v_index are the blobs' block indexes; for the uncompressed
 * BF16 kernel they are NULL and k/v point at [seq, dim] BF16 arrays. */
typedef struct kvx_unit {
    const void *k;
    const void *v;
    const kvx_block *k_index;
    const kvx_block *v_index;
    const uint16_t *q; /* [n_q, dim] BF16 */
    float *out;        /* [n_q, dim] FP32 */
    uint64_t k_bytes;  /* blob sizes (XKV) */
    uint64_t v_bytes;
    int32_t n_blocks;  /* XKV blocks covering the first `seq` tokens */
    int32_t seq;       /* tokens attended */
    float *lse;        /* optional [n_q] FP32: m + ln(l) of each query's softmax (the log of its
                        * normaliser), for folding outputs of sequence shards; NULL = not written */
} kvx_unit;

typedef struct kvx_plan_s *kvx_plan;

/* Build a reusable launch plan for a fixed set of units (host array of n_units descriptors).
 * block_tokens is the encode block size (the tile split of the BF16 kernel).  The plan uploads
 * the descriptors, cuts the step's blocks into one range of about equal decode cost per SM, and
 * owns the scratch for the partial softmax states.  Its device memory per (unit, block): a 32 B
 * flat entry, a 128 B descriptor, 4 dim B of merge words, the escape records (4 B per escape word
 * plus 64 B per coded block with escapes) and 144 B of stage copy lists per ring stage (one stage
 * per 128-token block at dim <= 64, two at 128, four at 256). */
KVX_API int kvx_plan_create(const kvx_unit *units, int n_units, int n_q, int dim, int block_tokens,
                    kvx_plan *plan);
/* Launch one decode step for every unit on `stream` (a cudaStream_t; NULL = default stream).
 * A plan's steps run one after another on a stream: a step that overlaps the plan's previous
 * one (another stream) races on the plan's scratch. */
KVX_API int kvx_plan_run(kvx_plan plan, void *stream);
/* Launch one part of a step: 0 = the fused decode-attention kernel, 1 = the combine kernel that
 * folds every unit's partial softmax states (one per consumer warp of every CTA that held some of
 * its blocks) into its outputs.  kvx_plan_run = part 0 then 1. */
KVX_API int kvx_plan_run_part(kvx_plan plan, int part, void *stream);
/* Synchronise the plan's last run and report device-side errors (malformed blocks, timeouts). */
KVX_API int kvx_plan_check(kvx_plan plan);
/* Number of kernel launches one kvx_plan_run makes. */
KVX_API int kvx_plan_launches(kvx_plan plan);
/* Number of the plan's units (query groups of <= 8) that the combine kernel folds: all of them
 * (each unit's tiles are spread over several consumer warps). */
KVX_API int kvx_plan_split_units(kvx_plan plan);
KVX_API void kvx_plan_destroy(kvx_plan plan);

/* GPU encoder for caches built on the device: encodes n_tensors [seq, head_dim] BF16 tensors
 * (device pointers in a host array) into one device arena.  Blob t starts at arena +
 * blob_offset[t] (16-byte aligned), its index at index + index_offset[t].  Capacities from
 * kvx_encode_batch_bounds.  Byte-identical to kvexp::encode_bf16 per tensor.  Synchronous. */
KVX_API int kvx_encode_batch_bounds(int n_tensors, int seq, int head_dim, int block_tokens,
                            size_t *arena_bytes, size_t *index_entries);
KVX_API int kvx_encode_batch(int n_tensors, const uint16_t *const *kv, int seq, int head_dim,
                     int block_tokens, uint8_t *arena, size_t arena_capacity,
                     kvx_block *index, uint64_t *blob_offset, uint64_t *blob_bytes,
                     void *stream);
/* kvx_encode_batch with a code-width mask (KVX_CODE_BITS_*). */
KVX_API int kvx_encode_batch_bits(int n_tensors, const uint16_t *const *kv, int seq, int head_dim,
                          int block_tokens, int code_bits, uint8_t *arena,
                          size_t arena_capacity, kvx_block *index, uint64_t *blob_offset,
                          uint64_t *blob_bytes, void *stream);

/* Append tokens to a device-resident cache: encode [n_new, head_dim] BF16 (device) as whole
 * blocks starting at byte `at` of `blob` (capacity `capacity`), writing the new blocks' index
 * entries at `index`.  *bytes_written / *blocks_written receive the growth.  Synchronous. */
KVX_API int kvx_cache_append(const uint16_t *kv_new, int n_new, int head_dim, int block_tokens,
                     uint8_t *blob, size_t at, size_t capacity, kvx_block *index,
                     size_t *bytes_written, int *blocks_written, void *stream);
/* kvx_cache_append with a code-width mask (KVX_CODE_BITS_*). */
KVX_API int kvx_cache_append_bits(const uint16_t *kv_new, int n_new, int head_dim, int block_tokens,
                          int code_bits, uint8_t *blob, size_t at, size_t capacity,
                          kvx_block *index, size_t *bytes_written, int *blocks_written,
                          void *stream);

/* Fold the results of a sequence split (one shard per rank, in rank order) into the result over
 * the whole sequence.  Per row (unit, query): M = max_r lse_r, w_r = exp(lse_r - M),
 * out = (sum_r w_r o_r) * (1 / sum_r w_r), summed in rank order -- the reference's fold of its
 * thread ranges (src/dispatch.cpp:98-103: merge_state, src/softmax.hpp:16-30, then
 * finalize_state, :32-41) applied to normalised shard outputs.  parts: device memory, n_parts
 * consecutive parts of n_rows * dim + n_rows FP32 each: the shard's outputs [n_rows, dim] (the
 * kvx_unit.out rows of its units, back to back) followed by their lse [n_rows] (kvx_unit.lse),
 * which is what an all-gather of one such buffer per rank yields.  A part whose lse is -inf (an
 * empty shard) contributes nothing.  out [n_rows, dim] FP32; lse_out [n_rows] (optional) gets the
 * lse of the whole sequence.  Asynchronous on `stream`. */
KVX_API int kvx_fold_shards(const float *parts, int n_parts, int n_rows, int dim, float *out,
                            float *lse_out, void *stream);

/* Decode attention that allocates no GPU memory.  No counterpart in the reference: it exists for
 * callers that cannot allocate while they run, such as serving engines that reserve the
 * device's memory for their KV-cache pool at start-up and treat a later cudaMalloc as a failure,
 * or decode loops that cannot take the device-wide stall of cudaFree.  Same result as
 * kvx_attention_decode for one KV head (within FP32 rounding), with every buffer in device
 * memory: q [n_q, dim] BF16, the K/V XKV blobs (16-byte aligned) with their block indexes
 * (n_blocks entries each, from kvx_xkv_index or the GPU encoder), out [n_q, dim] FP32.  Its
 * scratch is one fixed 40 MiB array in the library's device image, held by every device that
 * loads the library until the process exits; limits: n_blocks <= 8192, n_q <= 64, and the
 * blobs' escape words plus 16 per coded block that has any at most 3 Mi (about 1 in 6 elements
 * of 8192 blocks of 128 x 128) -- larger calls fail with KVX_ERR_INVALID_ARGUMENT (the escape
 * limit is found on the device: such a call launches its kernels, which then do no work).  The
 * first call on a device looks up the array's device
 * address (and loads the module there); make that first call before any stream capture.  All
 * calls share the array, so calls whose GPU work overlaps (other streams, other host threads)
 * race; run them one after another.  Launches on `stream`, then synchronises it to report
 * device-side errors. */
KVX_API int kvx_attention_decode_noalloc(const uint16_t *q, const uint8_t *k_xkv, size_t k_bytes,
                                 const kvx_block *k_index, const uint8_t *v_xkv, size_t v_bytes,
                                 const kvx_block *v_index, int n_blocks, float *out, int n_q,
                                 int dim, int seq, void *stream);

/* ---- benchmark support -------------------------------------------------------------------- */

/* Fill [seq, dim] BF16 on the device with the seeded synthetic distribution `profile`
 * (bit-identical to the numpy generator in synth.py). */
KVX_API int kvx_synth_bf16(uint16_t *out, int seq, int dim, uint64_t seed, uint64_t stream_id,
                   int profile, uint32_t rate, void *stream);

/* Device HBM read probe: streams `bytes` of `buf` with 16-byte loads, returns GB/s (1e9). */
KVX_API int kvx_hbm_read_probe(const void *buf, size_t bytes, int reps, double *gbps);

#ifdef __cplusplus
}
#endif

#endif /* KVEXP_B200_H */
