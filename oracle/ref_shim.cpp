// ref_shim.cpp -- extern "C" entry points over the UNMODIFIED reference library `kvexp`.
//
// TEST / BASELINE INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own sources (src/codec.cpp, src/cpu.cpp, src/attention_*.cpp,
// src/dispatch.cpp, read in place from the reference checkout) into oracle/_ref/.  It is
// used to pin the C restatement (xkv_oracle.c), to generate the golden fixtures under
// tests/golden/, and as the timed CPU reference arm of bench.py.  It calls only the
// reference's public API (include/kvexp/attention.hpp:58-61, include/kvexp/codec.hpp:45-48)
// and, for the timed loop, repeats the OpenMP `model_heads` pattern of src/bench.cpp:711-728.
#include "kvexp/attention.hpp"
#include "kvexp/codec.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <omp.h>
#include <stdexcept>

namespace {

thread_local char g_err[256];

int record(int code, const char *what) {
    std::snprintf(g_err, sizeof g_err, "%s", what);
    return code;
}

// Same code numbering as the C restatement: which exception type the reference threw.
template <class F> int guarded(F &&fn) {
    try {
        fn();
        return 0;
    } catch (const std::invalid_argument &e) {
        return record(1, e.what());
    } catch (const std::logic_error &e) {
        return record(3, e.what());
    } catch (const std::runtime_error &e) {
        return record(2, e.what());
    } catch (const std::exception &e) {
        return record(2, e.what());
    }
}

kvexp::Backend backend_of(int b) {
    switch (b) {
    case 1:
        return kvexp::Backend::Avx2;
    case 2:
        return kvexp::Backend::Avx512Bf16;
    default:
        return kvexp::Backend::Scalar;
    }
}

} // namespace

extern "C" {

const char *ref_last_error() { return g_err; }

void ref_detect(int *avx2, int *avx512_bf16) {
    const kvexp::CpuFeatures f = kvexp::detect_cpu();
    *avx2 = f.avx2 ? 1 : 0;
    *avx512_bf16 = f.avx512_bf16 ? 1 : 0;
}

// Encode; the container is malloc'd and handed to the caller (free with ref_free).
int ref_encode(const uint16_t *kv, int seq, int dim, int block, uint8_t **out, size_t *bytes) {
    *out = nullptr;
    *bytes = 0;
    return guarded([&] {
        kvexp::EncodedTensor enc = kvexp::encode_bf16(kv, seq, dim, block);
        uint8_t *p = static_cast<uint8_t *>(std::malloc(enc.bytes.size() ? enc.bytes.size() : 1));
        if (!p) throw std::runtime_error("ref_encode: out of memory");
        std::memcpy(p, enc.bytes.data(), enc.bytes.size());
        *out = p;
        *bytes = enc.bytes.size();
    });
}

void ref_free(void *p) { std::free(p); }

int ref_decode(const uint8_t *blob, size_t bytes, int seq, int dim, uint16_t *out) {
    return guarded([&] { kvexp::decode_bf16(blob, bytes, seq, dim, out); });
}

int ref_attention(int backend, const uint16_t *q, const uint16_t *k_raw, const uint16_t *v_raw,
                  const uint8_t *k_xkv, size_t k_bytes, const uint8_t *v_xkv, size_t v_bytes,
                  float *out, int n_q, int dim, int seq, int n_threads, int split_tokens) {
    return guarded([&] {
        kvexp::attention_decode(backend_of(backend), q, k_raw, v_raw, k_xkv, k_bytes, v_xkv,
                                v_bytes, out, n_q, dim, seq, n_threads, split_tokens);
    });
}

// One `model_heads` pass: OpenMP over units, one thread per unit, each unit a single-thread
// attention_decode over its XKV blobs (src/bench.cpp:711-728).
int ref_model_heads(int backend, int n_units, const uint16_t *const *q,
                    const uint8_t *const *k_xkv, const size_t *k_bytes,
                    const uint8_t *const *v_xkv, const size_t *v_bytes, float *const *out,
                    int n_q, int dim, int seq, int threads, int block) {
    int rc = 0;
    omp_set_dynamic(0);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int u = 0; u < n_units; ++u) {
        const int r = guarded([&] {
            kvexp::attention_decode(backend_of(backend), q[u], nullptr, nullptr, k_xkv[u],
                                    k_bytes[u], v_xkv[u], v_bytes[u], out[u], n_q, dim, seq, 1,
                                    block);
        });
        if (r != 0) {
#pragma omp critical
            rc = r;
        }
    }
    return rc;
}

} // extern "C"
