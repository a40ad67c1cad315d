// kvexp_gpu_shim.cpp -- the reference library's public C++ API (namespace kvexp) on top of the
// C ABI of libkvexp_b200.so.
//
// A maintainer builds this one translation unit into the reference's build instead of
// src/dispatch.cpp, src/codec.cpp and src/cpu.cpp (compiled against the reference's own
// include/kvexp headers, linked against libkvexp_b200.so); kvexp_tests and kvexp_bench then relink
// unchanged.  Every call forwards to the GPU; a failure status becomes the C++ exception type the
// reference throws for the same failure (include/kvexp/attention.hpp:58-61,
// include/kvexp/codec.hpp:45-48; KVX_ERR_INVALID_ARGUMENT -> std::invalid_argument,
// KVX_ERR_LOGIC -> std::logic_error, everything else -> std::runtime_error) with the library's
// message, which keeps the reference's wording.
#include "kvexp/attention.hpp"
#include "kvexp/codec.hpp"
#include "kvexp_b200.h"

#include <stdexcept>

namespace {

void check(int rc) {
    if (rc == KVX_OK) return;
    const char *msg = kvx_last_error();
    if (rc == KVX_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    if (rc == KVX_ERR_LOGIC) throw std::logic_error(msg);
    throw std::runtime_error(msg);
}

}  // namespace

namespace kvexp {

// Replaces the CPUID probe (src/cpu.cpp:35-61): with an sm_100 device every backend value is
// served (each runs the same GPU kernels and differs only in its shape rule); without one, none
// is, and attention_decode reports the missing device for any backend.
CpuFeatures detect_cpu() {
    CpuFeatures f;
    int major = 0, minor = 0, sms = 0;
    size_t mem = 0;
    const bool gpu = kvx_device_info(&major, &minor, &sms, &mem) == KVX_OK;
    f.avx2 = gpu;
    f.avx512_bf16 = gpu;
    return f;
}

void attention_decode(Backend backend, const uint16_t *q, const uint16_t *k_raw,
                      const uint16_t *v_raw, const uint8_t *k_xkv, size_t k_bytes,
                      const uint8_t *v_xkv, size_t v_bytes, float *out, int n_q, int dim, int seq,
                      int n_threads, int split_tokens) {
    check(kvx_attention_decode(static_cast<int>(backend), q, k_raw, v_raw, k_xkv, k_bytes, v_xkv,
                               v_bytes, out, n_q, dim, seq, n_threads, split_tokens));
}

EncodedTensor encode_bf16(const uint16_t *kv, int seq_len, int head_dim, int block_tokens) {
    EncodedTensor t;
    t.bytes.resize(kvx_encode_bound(seq_len, head_dim, block_tokens));
    size_t n = 0;
    check(kvx_encode_bf16(kv, seq_len, head_dim, block_tokens, t.bytes.data(), t.bytes.size(), &n));
    t.bytes.resize(n);
    t.seq_len = seq_len;
    t.head_dim = head_dim;
    t.block_tokens = block_tokens;
    return t;
}

void decode_bf16(const uint8_t *blob, size_t bytes, int seq_len, int head_dim, uint16_t *out) {
    check(kvx_decode_bf16(blob, bytes, seq_len, head_dim, out));
}

}  // namespace kvexp
