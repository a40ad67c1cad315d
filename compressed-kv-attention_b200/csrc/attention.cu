// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened; each team of two warps owns a contiguous range.
//  * Warp 0 lane 0 streams the team's compressed tiles (16 tokens of K and V: sign/mantissa rows,
//    packed exponent residuals, or raw rows) from HBM into a shared-memory byte ring with 1-D bulk
//    async copies (TMA engine) completing on mbarriers; block bases and escape words go to two
//    per-block meta slots.  Only the compressed bytes cross HBM.
//  * Warp 0 rebuilds the K tile and warp 1 the V tile as BF16 in registers (exponent = base +
//    residual, escapes patched in scan order via warp ballots) and stores them to a swizzled tile.
//  * Both warps compute S^T = K Q^T on the tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate,
//    tokens as rows, the GQA group's queries as columns), the online softmax in fp32, and P V with P
//    split into bf16 hi + mid parts (so P enters with 16 significant bits), each warp for half of the
//    head dimension.
//  * Unit segments that span several teams leave (m, l, acc) partial states that combine_kernel folds
//    in team order with merge_state semantics (src/softmax.hpp:16-30), then finalizes like
//    finalize_state (src/softmax.hpp:32-41: reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template with a loader that reads [seq, dim] BF16
// rows; for the same blocks it produces bit-identical outputs to the XKV variant, because both
// rebuild identical BF16 tiles and run identical arithmetic afterwards.
#include "attention.cuh"

#include <cfloat>

namespace kvx {
namespace {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int TT = 16;  // tokens per tile (one m16 row block of the QK MMA)

__host__ __device__ constexpr int round16(int x) { return (x + 15) & ~15; }

template <int D> struct Cfg {
    static constexpr int CH = D / 8;         // 16-byte chunks per BF16 row
    static constexpr int STEPS = D / 16;     // 256-element warp steps per 16-row tile
    static constexpr int ESC_CAP = 2048;     // escape bytes staged per block and tensor
    static constexpr int INFO = 64;
    static constexpr int BASE_SLOT = round16(D + 32);
    static constexpr int ESC_SLOT = ESC_CAP + 32;
    static constexpr int META = INFO + 2 * BASE_SLOT + 2 * ESC_SLOT;
    static constexpr int TILE = TT * D * 2;  // bytes of one BF16 tile
    static constexpr int RING = D == 32 ? 16384 : D == 64 ? 24576 : D == 128 ? 32768 : 40960;
    static constexpr int NB = 8;             // tiles in flight at most
    static constexpr int OFF_META = RING;
    static constexpr int OFF_KT = RING + 2 * META;
    static constexpr int OFF_VT = OFF_KT + TILE;
    static constexpr int OFF_BAR = OFF_VT + TILE;
    static constexpr int OFF_FLAG = OFF_BAR + (NB + 2) * 8;
    static constexpr int TEAM = (OFF_FLAG + 16 + 127) & ~127;
    static constexpr int TEAMS = (232448 / TEAM) > 6 ? 6 : (232448 / TEAM);
    static_assert(TEAMS >= 1, "team does not fit in shared memory");
    static_assert(RING >= 2 * (2 * TT * D * 2 + 64), "ring holds at least two raw tiles");
};

// Swizzle of 16-byte chunks inside a BF16 tile row, so that ldmatrix row reads and the decoder's
// 16-byte stores hit distinct bank groups.
template <int D> __device__ __forceinline__ int swz(int row) {
    return D >= 64 ? (row & 7) : ((row >> 1) & 3);
}

// ---- tile geometry ----------------------------------------------------------------------------

struct Piece {
    const uint8_t *src;  // 16-byte aligned source
    uint32_t alloc;      // bytes copied (multiple of 16)
    uint32_t data;       // offset of the first wanted byte inside the copy
};

__device__ __forceinline__ Piece make_piece(const uint8_t *p, uint32_t len) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t lo = a & ~uintptr_t(15);
    const uintptr_t hi = (a + len + 15) & ~uintptr_t(15);
    return Piece{reinterpret_cast<const uint8_t *>(lo), uint32_t(hi - lo), uint32_t(a - lo)};
}

// Pieces of one tensor's tile: [0] sm rows or raw rows, [1] residual rows (coded only).
template <int D, bool BF16IN>
__device__ __forceinline__ int tile_pieces(const uint8_t *blob, uint32_t off, int mode, int n_tok,
                                           int tile, Piece (&pc)[2]) {
    const int t0 = tile * TT;
    const int rows = min(TT, n_tok - t0);
    if (BF16IN) {
        pc[0] = make_piece(blob + (size_t(off) + t0) * (2 * D), uint32_t(rows * 2 * D));
        return 1;
    }
    const uint8_t *b = blob + off + kHeaderBytes;
    if (mode == 0) {
        pc[0] = make_piece(b + size_t(t0) * 2 * D, uint32_t(rows * 2 * D));
        return 1;
    }
    pc[0] = make_piece(b + D + size_t(t0) * D, uint32_t(rows * D));
    pc[1] = make_piece(b + D + size_t(n_tok) * D + size_t(t0) * D * mode / 8,
                       uint32_t(rows * D * mode / 8));
    return 2;
}

__device__ __forceinline__ FlatBlock load_flat(const FlatBlock *f, int64_t i) {
    const uint4 r = __ldg(reinterpret_cast<const uint4 *>(f) + i);
    FlatBlock b;
    b.k_off = r.x;
    b.v_off = r.y;
    b.k_nesc = uint16_t(r.z & 0xFFFF);
    b.v_nesc = uint16_t(r.z >> 16);
    b.k_mode = uint8_t(r.w & 0xFF);
    b.v_mode = uint8_t((r.w >> 8) & 0xFF);
    b.n_tok = uint8_t((r.w >> 16) & 0xFF);
    b.valid = uint8_t(r.w >> 24);
    return b;
}

// ---- shared-memory readers ---------------------------------------------------------------------

// 32-bit word at a 2-byte aligned shared address (MIS: address is 2 mod 4).
template <bool MIS> __device__ __forceinline__ uint32_t ldw(const uint8_t *p) {
    if (!MIS) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - 2);
    return prmt(q[0], q[1], 0x5432);
}

// ---- decode of one tensor tile into a swizzled BF16 tile ---------------------------------------

struct Esc {
    uint32_t run;          // escapes consumed so far in this block
    uint32_t n;            // escape words in this block
    const uint8_t *sm;     // staged escape words in shared memory (nullptr: read global)
    const uint8_t *gm;     // escape words in global memory
};

__device__ __forceinline__ uint32_t esc_word(const Esc &e, uint32_t r, int *status) {
    if (r >= e.n) {
        report(status, KVX_ERR_RUNTIME, DERR_ESC_OVERRUN);
        return 0;
    }
    if (e.sm != nullptr) return *reinterpret_cast<const uint16_t *>(e.sm + 2 * r);
    return __ldg(reinterpret_cast<const unsigned short *>(e.gm) + r);
}

__device__ __forceinline__ uint32_t set_half(uint32_t x, uint32_t v, int hi) {
    return hi ? prmt(x, v, 0x5410) : prmt(x, v, 0x3254);
}

// Exponent/sign merge per 16-bit half: sign and mantissa from the sign-replicated sm byte pair,
// exponent bits from (code + base) << 7.  The bit-select drops the carry out of bit 14, so the
// exponent wraps modulo 256 exactly like bf16_from_delta's uint8 sum (include/kvexp/bf16.hpp:35-37).
__device__ __forceinline__ uint32_t merge(uint32_t sg, uint32_t code_pair, uint32_t b7) {
    const uint32_t e = code_pair * 128u + b7;
    return (sg & 0x807F807Fu) | (e & 0x7F807F80u);
}

// Sign-replicating byte pairs of element i (from S0) and i + 4 (from S1).
__device__ __forceinline__ uint32_t sm_pair(uint32_t s0, uint32_t s1, int i) {
    // byte0 = s0.b[i], byte1 = signrep(s0.b[i]), byte2 = s1.b[i], byte3 = signrep(s1.b[i])
    const uint32_t sel = uint32_t(i) | (uint32_t(i | 8) << 4) | (uint32_t(4 + i) << 8) |
                         (uint32_t((4 + i) | 8) << 12);
    return prmt(s0, s1, sel);
}

// Patch sentinel elements (mask bit SH*k for element k) with escape words, in scan order.
template <int SH>
__device__ __forceinline__ void patch_escapes(uint32_t (&bf)[4], uint32_t m, Esc &es,
                                              int *status) {
    const uint32_t cnt = __popc(m);
    const uint32_t lt = lanemask_lt();
    const uint32_t c0 = __ballot_sync(FULL, cnt & 1), c1 = __ballot_sync(FULL, cnt & 2);
    const uint32_t c2 = __ballot_sync(FULL, cnt & 4), c3 = __ballot_sync(FULL, cnt & 8);
    uint32_t r = es.run + __popc(c0 & lt) + 2 * __popc(c1 & lt) + 4 * __popc(c2 & lt) +
                 8 * __popc(c3 & lt);
    es.run += __popc(c0) + 2 * __popc(c1) + 4 * __popc(c2) + 8 * __popc(c3);
    if (m != 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (m & (1u << (SH * k))) {
                bf[k & 3] = set_half(bf[k & 3], esc_word(es, r, status), k >> 2);
                ++r;
            }
        }
    }
}

template <int D, bool MIS>
__device__ __forceinline__ void decode_tile_impl(uint8_t *tile, int mode, int rows,
                                                 const uint8_t *p0, const uint8_t *p1,
                                                 const uint32_t (&b7)[4], Esc &es, int *status,
                                                 int lane) {
    constexpr int CH = Cfg<D>::CH;
    const int ch = lane % CH;
#pragma unroll 2
    for (int c = 0; c < Cfg<D>::STEPS; ++c) {
        const int e0 = 256 * c + 8 * lane;
        const int row = e0 / D;
        const bool valid = row < rows;
        uint32_t bf[4] = {0, 0, 0, 0};
        uint32_t m = 0;
        if (mode == 4) {
            uint32_t C = 0, S0 = 0, S1 = 0;
            if (valid) {
                C = ldw<MIS>(p1 + e0 / 2);
                S0 = ldw<MIS>(p0 + e0);
                S1 = ldw<MIS>(p0 + e0 + 4);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
                bf[i] = merge(sm_pair(S0, S1, i), (C >> (4 * i)) & 0x000F000Fu, b7[i]);
            uint32_t t = C & (C >> 1);
            t &= t >> 2;
            m = valid ? (t & 0x11111111u) : 0u;
            if (__any_sync(FULL, m != 0)) patch_escapes<4>(bf, m, es, status);
        } else if (mode == 2) {
            uint32_t C = 0, S0 = 0, S1 = 0;
            if (valid) {
                C = *reinterpret_cast<const uint16_t *>(p1 + e0 / 4);
                S0 = ldw<MIS>(p0 + e0);
                S1 = ldw<MIS>(p0 + e0 + 4);
            }
            // element k's code at bits 2k; move elements 4..7 up to bits 16..23
            const uint32_t X = prmt(C, 0, 0x0110);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                bf[i] = merge(sm_pair(S0, S1, i), (X >> (2 * i)) & 0x00030003u, b7[i]);
            m = valid ? (C & (C >> 1) & 0x5555u) : 0u;
            if (__any_sync(FULL, m != 0)) patch_escapes<2>(bf, m, es, status);
        } else {
            if (valid) {
                const uint32_t w0 = ldw<MIS>(p0 + 2 * e0), w1 = ldw<MIS>(p0 + 2 * e0 + 4);
                const uint32_t w2 = ldw<MIS>(p0 + 2 * e0 + 8), w3 = ldw<MIS>(p0 + 2 * e0 + 12);
                bf[0] = prmt(w0, w2, 0x5410);
                bf[1] = prmt(w0, w2, 0x7632);
                bf[2] = prmt(w1, w3, 0x5410);
                bf[3] = prmt(w1, w3, 0x7632);
            }
        }
        if (!valid) bf[0] = bf[1] = bf[2] = bf[3] = 0u;
        uint8_t *dst = tile + row * (2 * D) + 16 * (ch ^ swz<D>(row));
        *reinterpret_cast<uint4 *>(dst) = make_uint4(bf[0], bf[1], bf[2], bf[3]);
    }
}

template <int D>
__device__ __forceinline__ void decode_tile(uint8_t *tile, int mode, int rows, const uint8_t *p0,
                                            const uint8_t *p1, const uint32_t (&b7)[4], Esc &es,
                                            int *status, int lane) {
    if ((reinterpret_cast<uintptr_t>(p0) & 3u) != 0u)
        decode_tile_impl<D, true>(tile, mode, rows, p0, p1, b7, es, status, lane);
    else
        decode_tile_impl<D, false>(tile, mode, rows, p0, p1, b7, es, status, lane);
}

// b7[i] = (base[d0+i] << 7) | (base[d0+i+4] << 23)
__device__ __forceinline__ void load_base(const uint8_t *p, uint32_t (&b7)[4]) {
    uint32_t B0, B1;
    if ((reinterpret_cast<uintptr_t>(p) & 3u) != 0u) {
        B0 = ldw<true>(p);
        B1 = ldw<true>(p + 4);
    } else {
        B0 = ldw<false>(p);
        B1 = ldw<false>(p + 4);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
        b7[i] = (prmt(B0, B1, uint32_t(i) | (uint32_t(4 + i) << 8)) & 0x00FF00FFu) << 7;
}

// ---- tensor-core part of one tile ----------------------------------------------------------------

template <int D> struct State {
    float acc[Cfg<D>::CH / 2][4];  // this warp's half of the head dim: n-tiles x (hi0, hi1, mid0, mid1)
    float m0, m1, l0, l1;          // queries 2*tig, 2*tig+1: running max and lane-partial sum
};

template <int D>
__device__ __forceinline__ void attend_tile(const uint8_t *kt, const uint8_t *vt, int rows,
                                            const uint32_t (&qb)[D / 16][2], State<D> &st, int w,
                                            int lane) {
    constexpr int CH = Cfg<D>::CH;
    const int gi = lane >> 2;
    const int mat = lane >> 3;
    const int r = (lane & 7) + 8 * (mat & 1);
    const int cadd = mat >> 1;
    const int sw = swz<D>(r);

    // S^T[16 tokens x 8 queries] = K[16 x D] * Q^T[D x 8]
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    const uint32_t krow = smem_u32(kt) + uint32_t(r * 2 * D);
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(krow + 16u * uint32_t((2 * s + cadd) ^ sw), a0, a1, a2, a3);
        mma_bf16(s0, s1, s2, s3, a0, a1, a2, a3, qb[s][0], qb[s][1]);
    }
    if (gi >= rows) s0 = s1 = -INFINITY;
    if (gi + 8 >= rows) s2 = s3 = -INFINITY;

    // online softmax over this tile (per query 2*tig, 2*tig+1)
    float t0 = fmaxf(s0, s2), t1 = fmaxf(s1, s3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(FULL, t0, o));
        t1 = fmaxf(t1, __shfl_xor_sync(FULL, t1, o));
    }
    const float mn0 = fmaxf(st.m0, t0), mn1 = fmaxf(st.m1, t1);
    const float al0 = expf(st.m0 - mn0), al1 = expf(st.m1 - mn1);
    const float p0 = expf(s0 - mn0), p1 = expf(s1 - mn1);
    const float p2 = expf(s2 - mn0), p3 = expf(s3 - mn1);
    st.l0 = __fmaf_rn(st.l0, al0, __fadd_rn(p0, p2));
    st.l1 = __fmaf_rn(st.l1, al1, __fadd_rn(p1, p3));
    st.m0 = mn0;
    st.m1 = mn1;

    // rescale the accumulators of query gi when its max moved (alpha == 1 leaves acc unchanged)
    const float x0 = __shfl_sync(FULL, al0, gi >> 1), x1 = __shfl_sync(FULL, al1, gi >> 1);
    const float al = (gi & 1) ? x1 : x0;
    if (__any_sync(FULL, al != 1.0f)) {
#pragma unroll
        for (int j = 0; j < CH / 2; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) st.acc[j][e] = __fmul_rn(st.acc[j][e], al);
    }

    // P^T tiles -> P A-fragments: rows 0-7 carry bf16(p), rows 8-15 bf16(p - bf16(p))
    const uint32_t h01 = pack_bf16x2(p1, p0), h23 = pack_bf16x2(p3, p2);
    const float r0 = __fsub_rn(p0, bf16lo_to_f32(h01)), r1 = __fsub_rn(p1, bf16hi_to_f32(h01));
    const float r2 = __fsub_rn(p2, bf16lo_to_f32(h23)), r3 = __fsub_rn(p3, bf16hi_to_f32(h23));
    const uint32_t m01 = pack_bf16x2(r1, r0), m23 = pack_bf16x2(r3, r2);
    const uint32_t A0 = movm_t(h01), A1 = movm_t(m01), A2 = movm_t(h23), A3 = movm_t(m23);

    // O[16 x 8 per n-tile] += P[16 x 16 tokens] * V[16 tokens x 8 dims]
    const uint32_t vrow = smem_u32(vt) + uint32_t(r * 2 * D);
#pragma unroll
    for (int j = 0; j < CH / 2; j += 2) {
        const int c = w * (CH / 2) + j + cadd;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vrow + 16u * uint32_t(c ^ sw), v0, v1, v2, v3);
        mma_bf16(st.acc[j][0], st.acc[j][1], st.acc[j][2], st.acc[j][3], A0, A1, A2, A3, v0, v1);
        mma_bf16(st.acc[j + 1][0], st.acc[j + 1][1], st.acc[j + 1][2], st.acc[j + 1][3], A0, A1,
                 A2, A3, v2, v3);
    }
}

// Q B-fragments for the unit: qb[s][0] = (Q[gi][16s+tig], Q[gi][16s+4+tig]),
// qb[s][1] = (Q[gi][16s+8+tig], Q[gi][16s+12+tig]) -- the column order of the BF16 tiles.
template <int D>
__device__ __forceinline__ void load_q(const uint16_t *q, int n_q, int stride, uint32_t (&qb)[D / 16][2],
                                       int lane) {
    const int gi = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v = 0;
            if (gi < n_q) {
                const uint16_t *row = q + size_t(gi) * stride + 16 * s + 8 * h + tig;
                v = uint32_t(__ldg(reinterpret_cast<const unsigned short *>(row))) |
                    (uint32_t(__ldg(reinterpret_cast<const unsigned short *>(row + 4))) << 16);
            }
            qb[s][h] = v;
        }
    }
}

template <int D>
__device__ __forceinline__ void reset_state(State<D> &st) {
#pragma unroll
    for (int j = 0; j < Cfg<D>::CH / 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st.acc[j][e] = 0.f;
    st.m0 = st.m1 = -INFINITY;
    st.l0 = st.l1 = 0.f;
}

// Write the segment: final output (whole unit) or partial state (m, l, unnormalised acc).
template <int D>
__device__ __forceinline__ void finish_segment(const State<D> &st, const UnitDev &u, bool whole,
                                               float *partial, int w, int lane) {
    constexpr int CH = Cfg<D>::CH;
    const int gi = lane >> 2, tig = lane & 3;
    float l0 = st.l0, l1 = st.l1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        l0 = __fadd_rn(l0, __shfl_xor_sync(FULL, l0, o));
        l1 = __fadd_rn(l1, __shfl_xor_sync(FULL, l1, o));
    }
    const float y0 = __shfl_sync(FULL, l0, gi >> 1), y1 = __shfl_sync(FULL, l1, gi >> 1);
    const float lq = (gi & 1) ? y1 : y0;
    if (whole) {
        if (gi < u.n_q) {
            const float inv = __frcp_rn(lq);
            float *o = u.out + size_t(gi) * u.q_stride;
#pragma unroll
            for (int j = 0; j < CH / 2; ++j) {
                const int c = w * (CH / 2) + j;
                o[8 * c + tig] = __fmul_rn(__fadd_rn(st.acc[j][0], st.acc[j][2]), inv);
                o[8 * c + 4 + tig] = __fmul_rn(__fadd_rn(st.acc[j][1], st.acc[j][3]), inv);
            }
        }
        return;
    }
    if (w == 0 && gi == 0) {
        partial[2 * tig] = st.m0;
        partial[2 * tig + 1] = st.m1;
        partial[8 + 2 * tig] = l0;
        partial[8 + 2 * tig + 1] = l1;
    }
    float *acc = partial + 16 + gi * D;
#pragma unroll
    for (int j = 0; j < CH / 2; ++j) {
        const int c = w * (CH / 2) + j;
        acc[8 * c + tig] = __fadd_rn(st.acc[j][0], st.acc[j][2]);
        acc[8 * c + 4 + tig] = __fadd_rn(st.acc[j][1], st.acc[j][3]);
    }
}

// ---- the kernel -------------------------------------------------------------------------------

template <int D, bool BF16IN>
__global__ void __launch_bounds__(64 * Cfg<D>::TEAMS, 1) attn_kernel(const AttnArgs a) {
    using C = Cfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tl = warp >> 1, w = warp & 1;
    const int team = blockIdx.x * C::TEAMS + tl;
    if (team >= a.n_teams) return;
    const int64_t fb0 = a.team_begin[team], fb1 = a.team_begin[team + 1];
    if (fb0 >= fb1) return;

    uint8_t *T = smem + tl * C::TEAM;
    uint8_t *ring = T;
    uint8_t *kt = T + C::OFF_KT, *vt = T + C::OFF_VT;
    const uint32_t bar0 = smem_u32(T + C::OFF_BAR);  // NB tile barriers, then 2 meta barriers
    volatile int *flag = reinterpret_cast<volatile int *>(T + C::OFF_FLAG);
    const int bar_id = tl + 1;
    const bool issuer = (w == 0 && lane == 0);

    if (issuer) {
        for (int i = 0; i < C::NB + 2; ++i) mbar_init(bar0 + 8 * i, 1);
        fence_mbar_init();
    }
    named_bar(bar_id, 64);

    // ---- producer state (warp 0) ----
    int64_t p_fb = fb0;
    int p_tile = 0, p_i = 0, p_jb = 0;
    bool p_meta = false;
    int64_t p_pos = 0;
    FlatBlock p_blk{}, nx_blk{};
    int p_unit = -1, nx_unit = -1;
    const uint8_t *pk = nullptr, *pv = nullptr;
    if (w == 0) {
        p_blk = load_flat(a.flat, p_fb);
        p_unit = __ldg(a.flat_unit + p_fb);
        pk = a.units[p_unit].k;
        pv = a.units[p_unit].v;
        if (p_fb + 1 < fb1) {
            nx_blk = load_flat(a.flat, p_fb + 1);
            nx_unit = __ldg(a.flat_unit + p_fb + 1);
        }
    }

    // ---- consumer state ----
    int64_t c_fb = fb0;
    int c_tile = 0, c_i = 0, c_jb = 0;
    int64_t c_run = 0;
    FlatBlock cb{};
    int c_unit = -1;
    UnitDev cu{};
    int64_t seg_begin = fb0;
    uint32_t qb[D / 16][2];
    State<D> st;
    reset_state(st);
    uint32_t b7[4] = {0, 0, 0, 0};
    Esc es{0, 0, nullptr, nullptr};
    const uint8_t *c_blob = nullptr;
    bool ok = true;

    while (c_fb < fb1) {
        // -------- producer: issue tiles ahead --------
        if (w == 0) {
            while (p_fb < fb1 && p_i - c_i < C::NB) {
                const int p_ntiles = (p_blk.valid + TT - 1) / TT;
                if (!p_meta) {
                    if (p_jb - c_jb >= 2) break;
                    uint8_t *M = T + C::OFF_META + (p_jb & 1) * C::META;
                    const uint32_t mbar = bar0 + 8 * (C::NB + (p_jb & 1));
                    uint32_t tx = 0;
                    Piece mp[4];
                    bool stage[4] = {false, false, false, false};
                    if (!BF16IN) {
                        const uint8_t *blobs[2] = {pk, pv};
                        const uint32_t offs[2] = {p_blk.k_off, p_blk.v_off};
                        const int modes[2] = {p_blk.k_mode, p_blk.v_mode};
                        const int nesc[2] = {p_blk.k_nesc, p_blk.v_nesc};
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            if (modes[t] == 0) continue;
                            const uint8_t *b = blobs[t] + offs[t] + kHeaderBytes;
                            mp[2 * t] = make_piece(b, D);
                            stage[2 * t] = true;
                            const uint8_t *e = b + D + size_t(p_blk.n_tok) * D +
                                               size_t(p_blk.n_tok) * D * modes[t] / 8;
                            mp[2 * t + 1] = make_piece(e, uint32_t(2 * nesc[t]));
                            stage[2 * t + 1] = nesc[t] > 0 && mp[2 * t + 1].alloc <= C::ESC_SLOT;
                        }
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            if (stage[t]) tx += mp[t].alloc;
                    }
                    if (issuer) {
                        uint32_t *info = reinterpret_cast<uint32_t *>(M);
                        info[0] = p_blk.k_off;
                        info[1] = p_blk.v_off;
                        info[2] = uint32_t(p_blk.k_nesc) | (uint32_t(p_blk.v_nesc) << 16);
                        info[3] = uint32_t(p_blk.k_mode) | (uint32_t(p_blk.v_mode) << 8) |
                                  (uint32_t(p_blk.n_tok) << 16) | (uint32_t(p_blk.valid) << 24);
                        info[4] = uint32_t(p_unit);
                        info[5] = (stage[1] ? 1u : 0u) | (stage[3] ? 2u : 0u);
                        fence_proxy_async();
                        if (tx == 0) {
                            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(mbar)
                                         : "memory");
                        } else {
                            mbar_arrive_expect_tx(mbar, tx);
                            const uint32_t dst[4] = {
                                smem_u32(M + C::INFO), smem_u32(M + C::INFO + C::BASE_SLOT),
                                smem_u32(M + C::INFO + 2 * C::BASE_SLOT),
                                smem_u32(M + C::INFO + 2 * C::BASE_SLOT + C::ESC_SLOT)};
                            // order: K base, V base, K esc, V esc
                            const int pi[4] = {0, 2, 1, 3};
#pragma unroll
                            for (int t = 0; t < 4; ++t)
                                if (stage[pi[t]]) bulk_g2s(dst[t], mp[pi[t]].src, mp[pi[t]].alloc, mbar);
                        }
                    }
                    p_meta = true;
                    ++p_jb;
                }
                // tile pieces
                Piece kp[2], vp[2];
                const int nk = tile_pieces<D, BF16IN>(pk, p_blk.k_off, p_blk.k_mode, p_blk.n_tok, p_tile, kp);
                const int nv = tile_pieces<D, BF16IN>(pv, p_blk.v_off, p_blk.v_mode, p_blk.n_tok, p_tile, vp);
                uint32_t size = 0;
                for (int t = 0; t < nk; ++t) size += kp[t].alloc;
                for (int t = 0; t < nv; ++t) size += vp[t].alloc;
                int64_t pos = p_pos;
                if ((pos % C::RING) + size > uint32_t(C::RING)) pos = (pos / C::RING + 1) * C::RING;
                if (pos + size - c_run > C::RING) break;
                if (issuer) {
                    const uint32_t bar = bar0 + 8 * (p_i % C::NB);
                    fence_proxy_async();
                    mbar_arrive_expect_tx(bar, size);
                    uint32_t dst = smem_u32(ring + (pos % C::RING));
                    for (int t = 0; t < nk; ++t) {
                        bulk_g2s(dst, kp[t].src, kp[t].alloc, bar);
                        dst += kp[t].alloc;
                    }
                    for (int t = 0; t < nv; ++t) {
                        bulk_g2s(dst, vp[t].src, vp[t].alloc, bar);
                        dst += vp[t].alloc;
                    }
                }
                p_pos = pos + size;
                ++p_i;
                if (++p_tile == p_ntiles) {
                    p_tile = 0;
                    p_meta = false;
                    ++p_fb;
                    if (p_fb < fb1) {
                        p_blk = nx_blk;
                        if (nx_unit != p_unit) {
                            p_unit = nx_unit;
                            pk = a.units[p_unit].k;
                            pv = a.units[p_unit].v;
                        }
                        if (p_fb + 1 < fb1) {
                            nx_blk = load_flat(a.flat, p_fb + 1);
                            nx_unit = __ldg(a.flat_unit + p_fb + 1);
                        }
                    }
                }
            }
        }

        // -------- consumer: wait for tile c_i (and the block's meta) --------
        const bool first = (c_tile == 0);
        if (w == 0) {
            bool got = true;
            if (first)
                got = mbar_wait_bounded(bar0 + 8 * (C::NB + (c_jb & 1)), (c_jb >> 1) & 1, a.wait_limit);
            if (got)
                got = mbar_wait_bounded(bar0 + 8 * (c_i % C::NB), (c_i / C::NB) & 1, a.wait_limit);
            if (lane == 0) *flag = got ? 1 : 0;
        }
        named_bar(bar_id, 64);  // (A) tile data visible; previous tile fully consumed
        if (*flag == 0) {
            ok = false;
            break;
        }
        const uint8_t *M = T + C::OFF_META + (c_jb & 1) * C::META;
        if (first) {
            const uint32_t *info = reinterpret_cast<const uint32_t *>(M);
            cb.k_off = info[0];
            cb.v_off = info[1];
            cb.k_nesc = uint16_t(info[2] & 0xFFFF);
            cb.v_nesc = uint16_t(info[2] >> 16);
            cb.k_mode = uint8_t(info[3] & 0xFF);
            cb.v_mode = uint8_t((info[3] >> 8) & 0xFF);
            cb.n_tok = uint8_t((info[3] >> 16) & 0xFF);
            cb.valid = uint8_t(info[3] >> 24);
            const int unit = int(info[4]);
            const uint32_t staged = info[5];
            if (unit != c_unit) {
                c_unit = unit;
                cu = a.units[unit];
            }
            if (c_fb == seg_begin) {
                load_q<D>(cu.q, cu.n_q, cu.q_stride, qb, lane);
                reset_state(st);
            }
            // this warp's tensor: base registers and escape source
            if (!BF16IN) {
                const int mode = w == 0 ? cb.k_mode : cb.v_mode;
                c_blob = w == 0 ? cu.k : cu.v;
                const uint32_t off = w == 0 ? cb.k_off : cb.v_off;
                if (mode != 0) {
                    const uint8_t *b = c_blob + off + kHeaderBytes;
                    const uintptr_t mis = reinterpret_cast<uintptr_t>(b) & 15u;
                    load_base(M + C::INFO + w * C::BASE_SLOT + mis + 8 * (lane % C::CH), b7);
                    const uint8_t *e = b + D + size_t(cb.n_tok) * D + size_t(cb.n_tok) * D * mode / 8;
                    es.run = 0;
                    es.n = w == 0 ? cb.k_nesc : cb.v_nesc;
                    es.gm = e;
                    es.sm = (staged & (1u << w))
                                ? M + C::INFO + 2 * C::BASE_SLOT + w * C::ESC_SLOT +
                                      (reinterpret_cast<uintptr_t>(e) & 15u)
                                : nullptr;
                }
            } else {
                c_blob = w == 0 ? cu.k : cu.v;
            }
        }
        const int rows = min(TT, int(cb.valid) - c_tile * TT);

        // replay the ring allocation of tile c_i
        Piece kp[2], vp[2];
        const int nk = tile_pieces<D, BF16IN>(cu.k, cb.k_off, cb.k_mode, cb.n_tok, c_tile, kp);
        const int nv = tile_pieces<D, BF16IN>(cu.v, cb.v_off, cb.v_mode, cb.n_tok, c_tile, vp);
        uint32_t size = 0;
        for (int t = 0; t < nk; ++t) size += kp[t].alloc;
        for (int t = 0; t < nv; ++t) size += vp[t].alloc;
        int64_t pos = c_run;
        if ((pos % C::RING) + size > uint32_t(C::RING)) pos = (pos / C::RING + 1) * C::RING;
        const uint8_t *base = ring + (pos % C::RING);

        // -------- decode: warp 0 -> K tile, warp 1 -> V tile --------
        {
            const uint8_t *q0, *q1 = nullptr;
            int mode;
            if (w == 0) {
                q0 = base + kp[0].data;
                if (nk == 2) q1 = base + kp[0].alloc + kp[1].data;
                mode = BF16IN ? 0 : cb.k_mode;
            } else {
                uint32_t vo = 0;
                for (int t = 0; t < nk; ++t) vo += kp[t].alloc;
                q0 = base + vo + vp[0].data;
                if (nv == 2) q1 = base + vo + vp[0].alloc + vp[1].data;
                mode = BF16IN ? 0 : cb.v_mode;
            }
            decode_tile<D>(w == 0 ? kt : vt, mode, rows, q0, q1, b7, es, a.status, lane);
        }
        named_bar(bar_id, 64);  // (B) both BF16 tiles written

        attend_tile<D>(kt, vt, rows, qb, st, w, lane);

        c_run = pos + size;
        ++c_i;
        if (++c_tile * TT >= int(cb.valid)) {
            // block done
            c_tile = 0;
            ++c_jb;
            const int64_t ub = cu.block_begin + cu.n_blocks;
            const bool seg_end = (c_fb + 1 == fb1) || (c_fb + 1 == ub);
            if (seg_end) {
                const bool whole = (seg_begin == cu.block_begin) && (c_fb + 1 == ub);
                const int slot = (seg_begin == fb0) ? 0 : 1;
                float *part = a.partials + (size_t(team) * 2 + slot) * partial_stride(D);
                finish_segment<D>(st, cu, whole, part, w, lane);
                seg_begin = c_fb + 1;
            }
            ++c_fb;
        }
    }

    if (!ok) {
        // bounded drain of the copies still in flight, then leave
        if (issuer) {
            report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
            for (int i = c_i; i < p_i; ++i)
                mbar_wait_bounded(bar0 + 8 * (i % C::NB), (i / C::NB) & 1, a.wait_limit);
            for (int j = c_jb; j < p_jb; ++j)
                mbar_wait_bounded(bar0 + 8 * (C::NB + (j & 1)), (j >> 1) & 1, a.wait_limit);
        }
    }
}

// ---- combine ------------------------------------------------------------------------------------

// Fold the partial states of a unit in team order (merge_state, src/softmax.hpp:16-30) and
// finalize (finalize_state, src/softmax.hpp:32-41).
template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const CombineArgs a) {
    const int u = a.split_units[blockIdx.x];
    const UnitDev unit = a.units[u];
    const int t0 = team_of_block(a.team_begin, a.n_teams, unit.block_begin);
    const int t1 = team_of_block(a.team_begin, a.n_teams, unit.block_begin + unit.n_blocks - 1);
    const int ps = partial_stride(D);
    for (int idx = threadIdx.x; idx < unit.n_q * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float m = 0.f, l = 0.f, acc = 0.f;
        for (int t = t0; t <= t1; ++t) {
            const int slot = (a.team_begin[t] >= unit.block_begin) ? 0 : 1;
            const float *p = a.partials + (size_t(t) * 2 + slot) * ps;
            const float mb = p[g], lb = p[8 + g], ab = p[16 + g * D + d];
            if (t == t0) {
                m = mb;
                l = lb;
                acc = ab;
                continue;
            }
            const float mm = (m < mb) ? mb : m;
            const float e1 = expf(m - mm), e2 = expf(mb - mm);
            l = __fmaf_rn(l, e1, __fmul_rn(lb, e2));
            acc = __fmaf_rn(acc, e1, __fmul_rn(ab, e2));
            m = mm;
        }
        const float inv = __frcp_rn(l);
        unit.out[size_t(g) * unit.q_stride + d] = __fmul_rn(acc, inv);
    }
}

template <int D> void configure(bool bf16) {
    static bool done[2] = {false, false};
    if (done[bf16]) return;
    if (bf16)
        cudaFuncSetAttribute(attn_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::TEAM * Cfg<D>::TEAMS);
    else
        cudaFuncSetAttribute(attn_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::TEAM * Cfg<D>::TEAMS);
    done[bf16] = true;
}

template <int D>
cudaError_t launch_d(bool bf16, const AttnArgs &a, int grid, cudaStream_t s) {
    configure<D>(bf16);
    const int threads = 64 * Cfg<D>::TEAMS;
    const size_t sm = size_t(Cfg<D>::TEAM) * Cfg<D>::TEAMS;
    if (bf16)
        attn_kernel<D, true><<<grid, threads, sm, s>>>(a);
    else
        attn_kernel<D, false><<<grid, threads, sm, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

bool attention_dim_supported(int dim) {
    return dim == 32 || dim == 64 || dim == 128 || dim == 256;
}

int attention_teams_per_cta(int dim) {
    switch (dim) {
    case 32: return Cfg<32>::TEAMS;
    case 64: return Cfg<64>::TEAMS;
    case 128: return Cfg<128>::TEAMS;
    case 256: return Cfg<256>::TEAMS;
    default: return 0;
    }
}

size_t attention_smem_bytes(int dim) {
    switch (dim) {
    case 32: return size_t(Cfg<32>::TEAM) * Cfg<32>::TEAMS;
    case 64: return size_t(Cfg<64>::TEAM) * Cfg<64>::TEAMS;
    case 128: return size_t(Cfg<128>::TEAM) * Cfg<128>::TEAMS;
    case 256: return size_t(Cfg<256>::TEAM) * Cfg<256>::TEAMS;
    default: return 0;
    }
}

cudaError_t launch_attention(int dim, bool bf16_input, const AttnArgs &a, int grid, int /*teams*/,
                             cudaStream_t s) {
    switch (dim) {
    case 32: return launch_d<32>(bf16_input, a, grid, s);
    case 64: return launch_d<64>(bf16_input, a, grid, s);
    case 128: return launch_d<128>(bf16_input, a, grid, s);
    case 256: return launch_d<256>(bf16_input, a, grid, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_combine(int dim, const CombineArgs &a, int n_split, cudaStream_t s) {
    if (n_split <= 0) return cudaSuccess;
    switch (dim) {
    case 32: combine_kernel<32><<<n_split, 256, 0, s>>>(a); break;
    case 64: combine_kernel<64><<<n_split, 256, 0, s>>>(a); break;
    case 128: combine_kernel<128><<<n_split, 256, 0, s>>>(a); break;
    case 256: combine_kernel<256><<<n_split, 256, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace kvx
