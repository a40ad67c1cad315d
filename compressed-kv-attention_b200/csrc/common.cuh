// common.cuh -- shared device-side definitions: XKV format constants, device error reporting and
// thin wrappers over the sm_90+/sm_100 PTX used by the kernels (mbarrier, bulk async copy,
// ldmatrix, movmatrix, mma.sync bf16).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/kvexp_b200.h"

namespace kvx {

// XKV container constants (include/kvexp/bf16.hpp:12-13, include/kvexp/codec.hpp:18-31 of the
// reference): 8-byte block header {u8 mode, u8 n_tokens, u16 n_escape, u16 head_dim, u16 0}.
constexpr int kHeaderBytes = 8;
constexpr int kMaxHeadDim = 256;
constexpr int kDefaultBlock = 128;

// Device-side error detail codes (status word [1]); the host maps them to the reference's
// exception messages.
enum DeviceError : int {
    DERR_NONE = 0,
    DERR_TRUNC_HEADER = 1,  // "truncated xkv block header"
    DERR_DIM_LEN = 2,       // "xkv block dimension or length mismatch"
    DERR_TRUNC_RAW = 3,     // "truncated raw xkv block"
    DERR_MODE = 4,          // "unknown xkv block mode"
    DERR_TRUNC_CODED = 5,   // "truncated coded xkv block"
    DERR_OUT_OF_TOKENS = 6, // blob has fewer tokens than seq
    DERR_ESC_OVERRUN = 7,   // more sentinels than n_escape
    DERR_KV_MISMATCH = 8,   // K and V blocks cover different token counts
    DERR_TIMEOUT = 9,       // bounded mbarrier wait expired
    DERR_INDEX_CAP = 10,    // more blocks than the index capacity
    DERR_RANGE = 11,        // an index entry points outside its blob
    DERR_ESC_CAP = 12,      // escape records do not fit the fixed scratch
};

// Residual code bytes of a coded block: the reference's formula for 2 and 4 bits
// (include/kvexp/bf16.hpp:39-41); the 3-bit extension rounds 3 n dim / 8 up to an even count so
// that the escape words that follow stay 2-byte aligned.
__host__ __device__ inline int exp_payload_bytes(int n_tokens, int dim, int bits) {
    if (bits == 3) return (n_tokens * dim * 3 + 15) / 16 * 2;
    return (n_tokens * dim * bits + 7) / 8;
}
__host__ __device__ inline int coded_block_bytes(int n_tokens, int dim, int bits, int n_escape) {
    return kHeaderBytes + dim + n_tokens * dim + exp_payload_bytes(n_tokens, dim, bits) + 2 * n_escape;
}
__host__ __device__ inline int raw_block_bytes(int n_tokens, int dim) {
    return kHeaderBytes + 2 * n_tokens * dim;
}
// Bytes of one block as described by its index entry.
__host__ __device__ inline uint32_t block_bytes(const kvx_block &b, int dim) {
    return b.mode == 0 ? (uint32_t)raw_block_bytes(b.n_tokens, dim)
                       : (uint32_t)coded_block_bytes(b.n_tokens, dim, b.mode, b.n_escape);
}

// First error wins; detail says which check failed.
__device__ inline void report(int *status, int code, int detail) {
    if (status != nullptr && atomicCAS(status, 0, code) == 0) status[1] = detail;
}

// ---- PTX wrappers --------------------------------------------------------------------------

__device__ inline uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ inline void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ inline void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ inline void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ inline bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ inline uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: gives up once `limit_us` microseconds of wall time have passed.
__device__ inline bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint32_t limit_us) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    const uint64_t lim = uint64_t(limit_us) * 1000ull;
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > lim) return false;
    return true;
}

// 1-D bulk copy global -> shared (TMA engine), completing on an mbarrier.  dst, src and bytes
// must all be multiples of 16.
__device__ inline void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ inline void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                               uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ inline void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                 uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ inline uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C (f32)
__device__ inline void mma_bf16(float &d0, float &d1, float &d2, float &d3, uint32_t a0,
                                uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ inline uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ inline uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ inline void lds_v4(uint32_t a, uint32_t &x, uint32_t &y, uint32_t &z, uint32_t &w) {
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a));
}
__device__ inline void sts_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}
__device__ inline void sts_u16(uint32_t a, uint32_t x) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)x) : "memory");
}
__device__ inline void sts_u32(uint32_t a, uint32_t x) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(x) : "memory");
}

__device__ inline uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

}  // namespace kvx
