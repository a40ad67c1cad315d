// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened; each team of two warps owns a contiguous range.
//  * K-warp lane 0 streams the team's compressed tiles (16 tokens of K and V: sign/mantissa rows and
//    packed exponent residuals, or raw rows) from HBM into a shared-memory byte ring with 1-D bulk
//    async copies (TMA engine) completing on mbarriers; block bases and escape words go to two
//    per-block meta slots.  Only the compressed bytes cross HBM.
//  * The K-warp rebuilds the K tile as BF16 (exponent = base + residual, escapes patched in scan
//    order), computes S^T = K Q^T on the tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate,
//    tokens as rows, the GQA group's queries as columns) and the online softmax, and hands P to the
//    V-warp as ready MMA A-fragments (bf16 hi + mid parts, so P enters with 16 significant bits)
//    together with the per-query rescale factors.
//  * The V-warp rebuilds the V tile and accumulates O += P V for the whole head dimension.
//  * The two warps synchronise only through mbarriers with bounded waits: a stuck wait ends the
//    kernel with an error status instead of hanging.
//  * Unit segments that span several teams leave (m, l, acc) partial states that combine_kernel
//    folds in team order with merge_state semantics (src/softmax.hpp:16-30), then finalizes like
//    finalize_state (src/softmax.hpp:32-41: reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template with a loader that reads [seq, dim] BF16
// rows; for the same blocks it produces bit-identical outputs to the XKV variant, because both
// rebuild identical BF16 tiles and run identical arithmetic afterwards.
#include "attention.cuh"

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
    static constexpr int TILE = TT * D * 2;                 // bytes of one BF16 tile
    static constexpr int MAXTILE = 2 * (TT * D * 2 + 32);   // largest K+V allocation (raw)
    static constexpr int RING = D == 32 ? 8192 : D == 64 ? 16384 : D == 128 ? 20480 : 36864;
    static constexpr int NB = 8;                            // tile barriers
    static constexpr int PSLOT = 640;                       // P fragments + alpha + m + l
    static constexpr int OFF_META = RING;
    static constexpr int OFF_KT = RING + 2 * META;
    static constexpr int OFF_VT = OFF_KT + TILE;
    static constexpr int OFF_PS = OFF_VT + TILE;
    static constexpr int OFF_BAR = OFF_PS + 2 * PSLOT;
    static constexpr int NBARS = NB + 6;                    // tiles, meta x2, full x2, empty x2
    static constexpr int OFF_FLAG = OFF_BAR + NBARS * 8;
    static constexpr int TEAM = (OFF_FLAG + 16 + 127) & ~127;
    static constexpr int BY_SMEM = 232448 / TEAM;
    static constexpr int BY_REGS = D <= 64 ? 6 : (D == 128 ? 6 : 4);
    static constexpr int TEAMS = BY_SMEM < BY_REGS ? BY_SMEM : BY_REGS;
    static_assert(TEAMS >= 1, "team does not fit in shared memory");
    static_assert(RING >= 2 * MAXTILE, "ring must hold two of the largest tiles");
};

// Swizzle of 16-byte chunks inside a BF16 tile row, so that ldmatrix row reads and the decoder's
// 16-byte stores hit distinct bank groups.
template <int D> __device__ __forceinline__ int swz(int row) {
    return D >= 64 ? (row & 7) : ((row >> 1) & 3);
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

// One tensor of one block: where its sections start.
struct Geo {
    const uint8_t *s0;  // sign/mantissa rows (coded) or BF16 rows (raw)
    const uint8_t *s1;  // packed residual rows (coded)
    int mode;           // 0 raw, 2, 4
};

template <int D, bool BF16IN>
__device__ __forceinline__ Geo make_geo(const uint8_t *blob, uint32_t off, int mode, int n_tok) {
    Geo g;
    if (BF16IN) {
        g.s0 = blob + size_t(off) * (2 * D);
        g.s1 = nullptr;
        g.mode = 0;
        return g;
    }
    const uint8_t *b = blob + off + kHeaderBytes;
    g.mode = mode;
    if (mode == 0) {
        g.s0 = b;
        g.s1 = nullptr;
    } else {
        g.s0 = b + D;
        g.s1 = b + D + size_t(n_tok) * D;
    }
    return g;
}

// Pieces of one tensor's tile `tile` (rows rows): [0] sm or raw rows, [1] residual rows.
template <int D>
__device__ __forceinline__ int geo_pieces(const Geo &g, int tile, int rows, Piece (&pc)[2]) {
    const int t0 = tile * TT;
    if (g.mode == 0) {
        pc[0] = make_piece(g.s0 + t0 * (2 * D), uint32_t(rows * 2 * D));
        return 1;
    }
    pc[0] = make_piece(g.s0 + t0 * D, uint32_t(rows * D));
    pc[1] = make_piece(g.s1 + t0 * D * g.mode / 8, uint32_t(rows * D * g.mode / 8));
    return 2;
}

// Ring placement: a tile never wraps; it starts at 0 when it does not fit before the end.
template <int RING> __device__ __forceinline__ uint32_t place(uint32_t pos, uint32_t size) {
    return (pos % RING) + size > uint32_t(RING) ? pos + (RING - pos % RING) : pos;
}

// ---- decode of one tensor tile into a swizzled BF16 tile ---------------------------------------

// 32-bit word at a 2-byte aligned shared address; sel = 0x3210 (aligned) or 0x5432 (2 mod 4).
__device__ __forceinline__ uint32_t ldw(const uint8_t *p, uint32_t mis, uint32_t sel) {
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - mis);
    return prmt(q[0], q[1], sel);
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
    const uint32_t sel = uint32_t(i) | (uint32_t(i | 8) << 4) | (uint32_t(4 + i) << 8) |
                         (uint32_t((4 + i) | 8) << 12);
    return prmt(s0, s1, sel);
}

struct Esc {
    uint32_t run;        // escapes consumed so far in this block
    uint32_t n;          // escape words in this block
    const uint8_t *sm;   // staged escape words in shared memory (nullptr: read global)
    const uint8_t *gm;   // escape words in global memory
};

// Sentinel elements of this lane (mask bit SH*k for element k of its 8) take the next escape words
// in scan order: lane order inside the 256-element step, element order inside the lane.  The
// BF16 value is written straight into the tile slot of that element: element k sits at half
// (k >> 2) of 32-bit word (k & 3) of the lane's 16-byte chunk.
template <int SH>
__device__ __noinline__ void patch_escapes(uint8_t *chunk, uint32_t m, Esc &es, int *status) {
    const uint32_t cnt = __popc(m);
    const uint32_t lt = lanemask_lt();
    const uint32_t c0 = __ballot_sync(FULL, cnt & 1u);
    const uint32_t big = __ballot_sync(FULL, cnt > 1u);
    uint32_t pre, tot;
    if (big == 0u) {
        pre = __popc(c0 & lt);
        tot = __popc(c0);
    } else {
        const uint32_t c1 = __ballot_sync(FULL, cnt & 2u), c2 = __ballot_sync(FULL, cnt & 4u);
        const uint32_t c3 = __ballot_sync(FULL, cnt & 8u);
        pre = __popc(c0 & lt) + 2 * __popc(c1 & lt) + 4 * __popc(c2 & lt) + 8 * __popc(c3 & lt);
        tot = __popc(c0) + 2 * __popc(c1) + 4 * __popc(c2) + 8 * __popc(c3);
    }
    uint32_t r = es.run + pre;
    es.run += tot;
    while (m != 0u) {
        const int k = (__ffs(m) - 1) / SH;
        m &= m - 1u;
        uint32_t v = 0;
        if (r < es.n) {
            v = es.sm != nullptr ? *reinterpret_cast<const uint16_t *>(es.sm + 2 * r)
                                 : __ldg(reinterpret_cast<const unsigned short *>(es.gm) + r);
        } else {
            report(status, KVX_ERR_RUNTIME, DERR_ESC_OVERRUN);
        }
        ++r;
        *reinterpret_cast<uint16_t *>(chunk + 4 * (k & 3) + 2 * (k >> 2)) = uint16_t(v);
    }
}

template <int D>
__device__ __forceinline__ void decode_tile(uint8_t *tile, int mode, int rows, const uint8_t *p0,
                                            const uint8_t *p1, const uint32_t (&b7)[4], Esc &es,
                                            int *status, int lane) {
    constexpr int CH = Cfg<D>::CH;
    const int ch = lane % CH;
    const uint32_t mis = uint32_t(reinterpret_cast<uintptr_t>(p0) & 2u);
    const uint32_t sel = mis ? 0x5432u : 0x3210u;
#pragma unroll 1
    for (int c = 0; c < Cfg<D>::STEPS; ++c) {
        const int e0 = 256 * c + 8 * lane;
        const int row = e0 / D;
        uint32_t bf0 = 0, bf1 = 0, bf2 = 0, bf3 = 0;
        uint32_t m = 0;
        if (row < rows) {
            if (mode == 0) {
                const uint8_t *p = p0 + 2 * e0;
                const uint32_t w0 = ldw(p, mis, sel), w1 = ldw(p + 4, mis, sel);
                const uint32_t w2 = ldw(p + 8, mis, sel), w3 = ldw(p + 12, mis, sel);
                bf0 = prmt(w0, w2, 0x5410);
                bf1 = prmt(w0, w2, 0x7632);
                bf2 = prmt(w1, w3, 0x5410);
                bf3 = prmt(w1, w3, 0x7632);
            } else {
                const uint32_t S0 = ldw(p0 + e0, mis, sel), S1 = ldw(p0 + e0 + 4, mis, sel);
                uint32_t X, sh, mask;
                if (mode == 4) {
                    X = ldw(p1 + e0 / 2, mis, sel);  // element k at bits 4k
                    uint32_t t = X & (X >> 1);
                    t &= t >> 2;
                    m = t & 0x11111111u;
                    sh = 4;
                    mask = 0x000F000Fu;
                } else {
                    const uint32_t C = *reinterpret_cast<const uint16_t *>(p1 + e0 / 4);
                    m = C & (C >> 1) & 0x5555u;       // element k at bits 2k
                    X = prmt(C, 0, 0x0110);           // elements 4..7 up to bits 16..23
                    sh = 2;
                    mask = 0x00030003u;
                }
                bf0 = merge(sm_pair(S0, S1, 0), X & mask, b7[0]);
                bf1 = merge(sm_pair(S0, S1, 1), (X >> sh) & mask, b7[1]);
                bf2 = merge(sm_pair(S0, S1, 2), (X >> (2 * sh)) & mask, b7[2]);
                bf3 = merge(sm_pair(S0, S1, 3), (X >> (3 * sh)) & mask, b7[3]);
            }
        }
        uint8_t *dst = tile + row * (2 * D) + 16 * (ch ^ swz<D>(row));
        *reinterpret_cast<uint4 *>(dst) = make_uint4(bf0, bf1, bf2, bf3);
        if (mode != 0 && __any_sync(FULL, m != 0u)) {
            if (mode == 4) patch_escapes<4>(dst, m, es, status);
            else patch_escapes<2>(dst, m, es, status);
        }
    }
}

// b7[i] = (base[d0+i] << 7) | (base[d0+i+4] << 23)
__device__ __forceinline__ void load_base(const uint8_t *p, uint32_t (&b7)[4]) {
    const uint32_t mis = uint32_t(reinterpret_cast<uintptr_t>(p) & 2u);
    const uint32_t sel = mis ? 0x5432u : 0x3210u;
    const uint32_t B0 = ldw(p, mis, sel), B1 = ldw(p + 4, mis, sel);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        b7[i] = (prmt(B0, B1, uint32_t(i) | (uint32_t(4 + i) << 8)) & 0x00FF00FFu) << 7;
}

// Q B-fragments of the QK MMA: qb[s][0] = (Q[gi][16s+tig], Q[gi][16s+4+tig]),
// qb[s][1] = (Q[gi][16s+8+tig], Q[gi][16s+12+tig]) -- the column order the decoder stores:
// 16-byte chunk c of a BF16 tile row holds dims 8c + {0,4,1,5,2,6,3,7}.
template <int D>
__device__ __forceinline__ void load_q_frags(const uint16_t *q, int n_q, int stride,
                                             uint32_t (&qb)[D / 16][2], int lane) {
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

// ---- the kernel -------------------------------------------------------------------------------

struct Team {
    uint8_t *T;
    uint32_t bar0;
    volatile int *abort;
};

template <int NB> __device__ __forceinline__ uint32_t tile_bar(uint32_t bar0, int i) {
    return bar0 + 8u * uint32_t(i % NB);
}

// Bounded wait that also gives up when the partner warp aborted.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const Team &t,
                                         const AttnArgs &a) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    const uint64_t lim = uint64_t(a.wait_limit) * 1000ull;
    while (!mbar_try_wait(bar, parity)) {
        if (*t.abort) return false;
        if (global_ns() - t0 > lim) {
            *t.abort = 1;
            report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

struct BlockInfo {
    FlatBlock fb;
    int unit;
    uint32_t staged;  // bit0: K escapes staged, bit1: V escapes staged
};

__device__ __forceinline__ BlockInfo read_info(const uint8_t *M) {
    const uint4 w = *reinterpret_cast<const uint4 *>(M);
    const uint2 x = *reinterpret_cast<const uint2 *>(M + 16);
    BlockInfo b;
    b.fb.k_off = w.x;
    b.fb.v_off = w.y;
    b.fb.k_nesc = uint16_t(w.z & 0xFFFF);
    b.fb.v_nesc = uint16_t(w.z >> 16);
    b.fb.k_mode = uint8_t(w.w & 0xFF);
    b.fb.v_mode = uint8_t((w.w >> 8) & 0xFF);
    b.fb.n_tok = uint8_t((w.w >> 16) & 0xFF);
    b.fb.valid = uint8_t(w.w >> 24);
    b.unit = int(x.x);
    b.staged = x.y;
    return b;
}

// Consumer-side position in the team's tile stream; both warps keep an identical copy.
template <int D, bool BF16IN> struct Stream {
    int64_t fb0, fb1, fb, seg_begin;
    int tile = 0, i = 0, jb = 0;
    uint32_t pos = 0;
    BlockInfo bi{};
    int unit = -1;
    UnitDev cu{};
    Geo gk{}, gv{};
    // the current tile
    Piece kp[2], vp[2];
    int nk = 0, nv = 0, rows = 0;
    uint32_t ksz = 0, size = 0, at = 0;
    bool first = true, last_tile = false, seg_end = false;

    __device__ Stream(int64_t b0, int64_t b1) : fb0(b0), fb1(b1), fb(b0), seg_begin(b0) {}

    // Block start: wait for the block's meta, read its info, set up this warp's tensor.
    __device__ bool begin_block(const Team &tm, const AttnArgs &a, int w, int lane,
                                uint32_t (&b7)[4], Esc &es) {
        using C = Cfg<D>;
        const uint8_t *M = tm.T + C::OFF_META + (jb & 1) * C::META;
        const uint32_t meta_bar = tm.bar0 + 8u * C::NB + 8u * uint32_t(jb & 1);
        if (!wait_bar(meta_bar, (jb >> 1) & 1, tm, a)) return false;
        bi = read_info(M);
        if (bi.unit != unit) {
            unit = bi.unit;
            cu = a.units[unit];
        }
        gk = make_geo<D, BF16IN>(cu.k, bi.fb.k_off, bi.fb.k_mode, bi.fb.n_tok);
        gv = make_geo<D, BF16IN>(cu.v, bi.fb.v_off, bi.fb.v_mode, bi.fb.n_tok);
        const Geo &mine = w == 0 ? gk : gv;
        if (!BF16IN && mine.mode != 0) {
            const uint8_t *b = mine.s0 - D;  // the block's base array
            load_base(M + C::INFO + w * C::BASE_SLOT + (reinterpret_cast<uintptr_t>(b) & 15u) +
                          8 * (lane % C::CH),
                      b7);
            const uint8_t *e = mine.s1 + size_t(bi.fb.n_tok) * D * mine.mode / 8;
            es.run = 0;
            es.n = w == 0 ? bi.fb.k_nesc : bi.fb.v_nesc;
            es.gm = e;
            es.sm = (bi.staged & (1u << w)) ? M + C::INFO + 2 * C::BASE_SLOT + w * C::ESC_SLOT +
                                                  (reinterpret_cast<uintptr_t>(e) & 15u)
                                            : nullptr;
        }
        return true;
    }

    // Geometry of tile `tile` of the current block and where the producer put it in the ring.
    __device__ void locate() {
        using C = Cfg<D>;
        first = tile == 0;
        const int rows_layout = min(TT, int(bi.fb.n_tok) - tile * TT);
        rows = min(TT, int(bi.fb.valid) - tile * TT);
        nk = geo_pieces<D>(gk, tile, rows_layout, kp);
        nv = geo_pieces<D>(gv, tile, rows_layout, vp);
        ksz = kp[0].alloc + (nk == 2 ? kp[1].alloc : 0u);
        size = ksz + vp[0].alloc + (nv == 2 ? vp[1].alloc : 0u);
        at = place<C::RING>(pos, size);
        last_tile = (tile + 1) * TT >= int(bi.fb.valid);
        const int64_t ub = cu.block_begin + cu.n_blocks;
        seg_end = last_tile && ((fb + 1 == fb1) || (fb + 1 == ub));
    }

    __device__ bool whole_unit() const {
        return seg_begin == cu.block_begin && fb + 1 == cu.block_begin + cu.n_blocks;
    }

    __device__ void advance() {
        pos = at + size;
        ++i;
        if (last_tile) {
            tile = 0;
            ++jb;
            if (seg_end) seg_begin = fb + 1;
            ++fb;
        } else {
            ++tile;
        }
    }
};

// K-warp: issues the TMA copies, rebuilds K, runs QK and the online softmax, hands P over.
template <int D, bool BF16IN>
__device__ __forceinline__ void k_warp(const AttnArgs &a, const Team &tm, int team, int64_t fb0,
                                       int64_t fb1, int lane) {
    using C = Cfg<D>;
    uint8_t *ring = tm.T;
    uint8_t *kt = tm.T + C::OFF_KT;
    const uint32_t meta_bar = tm.bar0 + 8u * C::NB;
    const uint32_t full_bar = meta_bar + 16u;
    const uint32_t empty_bar = full_bar + 16u;
    const int gi = lane >> 2, tig = lane & 3;
    Stream<D, BF16IN> st(fb0, fb1);
    uint32_t b7[4] = {0, 0, 0, 0};
    Esc es{0, 0, nullptr, nullptr};
    bool ok = true;

    // producer state
    int64_t p_fb = fb0;
    int p_tile = 0, p_i = 0, p_jb = 0;
    bool p_meta = false;
    uint32_t p_pos = 0;
    FlatBlock p_blk = load_flat(a.flat, p_fb), nx_blk{};
    int p_unit = __ldg(a.flat_unit + p_fb), nx_unit = -1;
    const uint8_t *pk = a.units[p_unit].k, *pv = a.units[p_unit].v;
    int p_ntiles = (p_blk.valid + TT - 1) / TT;
    if (p_fb + 1 < fb1) {
        nx_blk = load_flat(a.flat, p_fb + 1);
        nx_unit = __ldg(a.flat_unit + p_fb + 1);
    }
    uint32_t tail = 0;                // ring bytes before this position are free
    uint32_t end_m1 = 0, end_m2 = 0;  // ring end of tiles i-1, i-2
    int last_m1 = 0, last_m2 = 0;     // were they the last tile of their block
    int rel_jb = 0;                   // blocks whose meta both warps are done with

    uint32_t qb[D / 16][2];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int mat = lane >> 3;
    const int r = (lane & 7) + 8 * (mat & 1);
    const int cadd = mat >> 1;
    const int sw = swz<D>(r);
    const uint32_t krow = smem_u32(kt) + uint32_t(r * 2 * D);

    while (st.fb < fb1) {
        const int slot = st.i & 1;
        // The V-warp is done with tile i - 2: its ring bytes, its P slot and (for a block's last
        // tile) its meta slot are free.  With that, tile i can always be issued: at most tiles
        // i - 1 and i are live and the ring holds two of the largest tiles.
        if (st.i >= 2) {
            if (!wait_bar(empty_bar + 8u * uint32_t(slot), ((st.i - 2) >> 1) & 1, tm, a)) {
                ok = false;
                break;
            }
            tail = end_m2;
            if (last_m2) ++rel_jb;
        }
        // ---- producer: issue tiles ahead ----
        while (p_fb < fb1 && p_i - st.i < C::NB - 2) {
            if (!p_meta) {
                if (p_jb - rel_jb >= 2) break;
                uint8_t *M = tm.T + C::OFF_META + (p_jb & 1) * C::META;
                const uint32_t mbar = meta_bar + 8u * uint32_t(p_jb & 1);
                uint32_t tx = 0;
                Piece mp[4];
                bool stage[4] = {false, false, false, false};
                if (!BF16IN) {
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int mode = t == 0 ? p_blk.k_mode : p_blk.v_mode;
                        if (mode == 0) continue;
                        const uint8_t *b =
                            (t == 0 ? pk + p_blk.k_off : pv + p_blk.v_off) + kHeaderBytes;
                        const int nesc = t == 0 ? p_blk.k_nesc : p_blk.v_nesc;
                        mp[2 * t] = make_piece(b, D);
                        stage[2 * t] = true;
                        const uint8_t *e = b + D + size_t(p_blk.n_tok) * D +
                                           size_t(p_blk.n_tok) * D * mode / 8;
                        mp[2 * t + 1] = make_piece(e, uint32_t(2 * nesc));
                        stage[2 * t + 1] = nesc > 0 && mp[2 * t + 1].alloc <= uint32_t(C::ESC_SLOT);
                    }
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        if (stage[t]) tx += mp[t].alloc;
                }
                if (lane == 0) {
                    *reinterpret_cast<uint4 *>(M) = make_uint4(
                        p_blk.k_off, p_blk.v_off,
                        uint32_t(p_blk.k_nesc) | (uint32_t(p_blk.v_nesc) << 16),
                        uint32_t(p_blk.k_mode) | (uint32_t(p_blk.v_mode) << 8) |
                            (uint32_t(p_blk.n_tok) << 16) | (uint32_t(p_blk.valid) << 24));
                    *reinterpret_cast<uint2 *>(M + 16) =
                        make_uint2(uint32_t(p_unit), (stage[1] ? 1u : 0u) | (stage[3] ? 2u : 0u));
                    fence_proxy_async();
                    if (tx == 0) {
                        mbar_arrive(mbar);
                    } else {
                        mbar_arrive_expect_tx(mbar, tx);
                        // mp order: K base, K escapes, V base, V escapes
                        const uint32_t dst[4] = {
                            smem_u32(M + C::INFO), smem_u32(M + C::INFO + 2 * C::BASE_SLOT),
                            smem_u32(M + C::INFO + C::BASE_SLOT),
                            smem_u32(M + C::INFO + 2 * C::BASE_SLOT + C::ESC_SLOT)};
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            if (stage[t]) bulk_g2s(dst[t], mp[t].src, mp[t].alloc, mbar);
                    }
                }
                p_meta = true;
                ++p_jb;
            }
            const Geo g0 = make_geo<D, BF16IN>(pk, p_blk.k_off, p_blk.k_mode, p_blk.n_tok);
            const Geo g1 = make_geo<D, BF16IN>(pv, p_blk.v_off, p_blk.v_mode, p_blk.n_tok);
            const int prow = min(TT, int(p_blk.n_tok) - p_tile * TT);
            Piece kp[2], vp[2];
            const int nk = geo_pieces<D>(g0, p_tile, prow, kp);
            const int nv = geo_pieces<D>(g1, p_tile, prow, vp);
            const uint32_t size = kp[0].alloc + (nk == 2 ? kp[1].alloc : 0u) + vp[0].alloc +
                                  (nv == 2 ? vp[1].alloc : 0u);
            const uint32_t pos = place<C::RING>(p_pos, size);
            if (pos + size - tail > uint32_t(C::RING)) break;
            if (lane == 0) {
                const uint32_t bar = tile_bar<C::NB>(tm.bar0, p_i);
                fence_proxy_async();
                mbar_arrive_expect_tx(bar, size);
                uint32_t dst = smem_u32(ring + pos % C::RING);
                bulk_g2s(dst, kp[0].src, kp[0].alloc, bar);
                dst += kp[0].alloc;
                if (nk == 2) {
                    bulk_g2s(dst, kp[1].src, kp[1].alloc, bar);
                    dst += kp[1].alloc;
                }
                bulk_g2s(dst, vp[0].src, vp[0].alloc, bar);
                dst += vp[0].alloc;
                if (nv == 2) bulk_g2s(dst, vp[1].src, vp[1].alloc, bar);
            }
            p_pos = pos + size;
            ++p_i;
            if (++p_tile == p_ntiles) {
                p_tile = 0;
                p_meta = false;
                ++p_fb;
                if (p_fb < fb1) {
                    p_blk = nx_blk;
                    p_ntiles = (p_blk.valid + TT - 1) / TT;
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

        // ---- consume tile i ----
        if (st.tile == 0) {
            if (!st.begin_block(tm, a, 0, lane, b7, es)) {
                ok = false;
                break;
            }
            if (st.fb == st.seg_begin) {
                load_q_frags<D>(st.cu.q, st.cu.n_q, st.cu.q_stride, qb, lane);
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
            }
        }
        if (!wait_bar(tile_bar<C::NB>(tm.bar0, st.i), (st.i / C::NB) & 1, tm, a)) {
            ok = false;
            break;
        }
        st.locate();
        const uint8_t *base = ring + st.at % C::RING;
        const int rows = st.rows;
        decode_tile<D>(kt, st.gk.mode, rows, base + st.kp[0].data,
                       st.nk == 2 ? base + st.kp[0].alloc + st.kp[1].data : nullptr, b7, es,
                       a.status, lane);
        __syncwarp();
        // S^T[16 tokens x 8 queries] = K[16 x D] * Q^T[D x 8]
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(krow + 16u * uint32_t((2 * s + cadd) ^ sw), a0, a1, a2, a3);
            mma_bf16(s0, s1, s2, s3, a0, a1, a2, a3, qb[s][0], qb[s][1]);
        }
        if (gi >= rows) s0 = s1 = -INFINITY;
        if (gi + 8 >= rows) s2 = s3 = -INFINITY;
        float t0 = fmaxf(s0, s2), t1 = fmaxf(s1, s3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            t0 = fmaxf(t0, __shfl_xor_sync(FULL, t0, o));
            t1 = fmaxf(t1, __shfl_xor_sync(FULL, t1, o));
        }
        const float mn0 = fmaxf(m0, t0), mn1 = fmaxf(m1, t1);
        const float al0 = expf(m0 - mn0), al1 = expf(m1 - mn1);
        const float p0 = expf(s0 - mn0), p1 = expf(s1 - mn1);
        const float p2 = expf(s2 - mn0), p3 = expf(s3 - mn1);
        l0 = __fmaf_rn(l0, al0, __fadd_rn(p0, p2));
        l1 = __fmaf_rn(l1, al1, __fadd_rn(p1, p3));
        m0 = mn0;
        m1 = mn1;
        // P^T tiles -> P A-fragments: rows 0-7 carry bf16(p), rows 8-15 bf16(p - bf16(p))
        const uint32_t h01 = pack_bf16x2(p1, p0), h23 = pack_bf16x2(p3, p2);
        const float r0 = __fsub_rn(p0, bf16lo_to_f32(h01));
        const float r1 = __fsub_rn(p1, bf16hi_to_f32(h01));
        const float r2 = __fsub_rn(p2, bf16lo_to_f32(h23));
        const float r3 = __fsub_rn(p3, bf16hi_to_f32(h23));
        const uint32_t mm01 = pack_bf16x2(r1, r0), mm23 = pack_bf16x2(r3, r2);
        uint8_t *P = tm.T + C::OFF_PS + slot * C::PSLOT;
        reinterpret_cast<uint4 *>(P)[lane] =
            make_uint4(movm_t(h01), movm_t(mm01), movm_t(h23), movm_t(mm23));
        float *pf = reinterpret_cast<float *>(P + 512);
        if (st.seg_end) {
            float lt0 = l0, lt1 = l1;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                lt0 = __fadd_rn(lt0, __shfl_xor_sync(FULL, lt0, o));
                lt1 = __fadd_rn(lt1, __shfl_xor_sync(FULL, lt1, o));
            }
            if (gi == 0) {
                pf[8 + 2 * tig] = m0;
                pf[8 + 2 * tig + 1] = m1;
                pf[16 + 2 * tig] = lt0;
                pf[16 + 2 * tig + 1] = lt1;
            }
        }
        if (gi == 0) {
            pf[2 * tig] = al0;
            pf[2 * tig + 1] = al1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(full_bar + 8u * uint32_t(slot));
        end_m2 = end_m1;
        last_m2 = last_m1;
        end_m1 = st.at + st.size;
        last_m1 = st.last_tile ? 1 : 0;
        st.advance();
    }

    if (!ok && lane == 0) {
        // bounded drain of the copies still in flight, then leave
        for (int i = st.i; i < p_i; ++i)
            mbar_wait_bounded(tile_bar<C::NB>(tm.bar0, i), (i / C::NB) & 1, a.wait_limit);
        for (int j = st.jb; j < p_jb; ++j)
            mbar_wait_bounded(meta_bar + 8u * uint32_t(j & 1), (j >> 1) & 1, a.wait_limit);
    }
}

// V-warp: rebuilds V, accumulates O += P V over the whole head dim, writes outputs or partials.
template <int D, bool BF16IN>
__device__ __forceinline__ void v_warp(const AttnArgs &a, const Team &tm, int team, int64_t fb0,
                                       int64_t fb1, int lane) {
    using C = Cfg<D>;
    uint8_t *ring = tm.T;
    uint8_t *vt = tm.T + C::OFF_VT;
    const uint32_t full_bar = tm.bar0 + 8u * C::NB + 16u;
    const uint32_t empty_bar = full_bar + 16u;
    const int gi = lane >> 2, tig = lane & 3;
    Stream<D, BF16IN> st(fb0, fb1);
    uint32_t b7[4] = {0, 0, 0, 0};
    Esc es{0, 0, nullptr, nullptr};
    float acc[C::CH][4];  // rows gi: hi part, rows gi + 8: mid part of query gi
    const int mat = lane >> 3;
    const int r = (lane & 7) + 8 * (mat & 1);
    const int cadd = mat >> 1;
    const int sw = swz<D>(r);
    const uint32_t vrow = smem_u32(vt) + uint32_t(r * 2 * D);

    while (st.fb < fb1) {
        const int slot = st.i & 1;
        if (st.tile == 0) {
            if (!st.begin_block(tm, a, 1, lane, b7, es)) break;
            if (st.fb == st.seg_begin) {
#pragma unroll
                for (int j = 0; j < C::CH; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
            }
        }
        if (!wait_bar(tile_bar<C::NB>(tm.bar0, st.i), (st.i / C::NB) & 1, tm, a)) break;
        st.locate();
        const uint8_t *base = ring + st.at % C::RING + st.ksz;
        decode_tile<D>(vt, st.gv.mode, st.rows, base + st.vp[0].data,
                       st.nv == 2 ? base + st.vp[0].alloc + st.vp[1].data : nullptr, b7, es,
                       a.status, lane);
        __syncwarp();
        if (!wait_bar(full_bar + 8u * uint32_t(slot), (st.i >> 1) & 1, tm, a)) break;
        const uint8_t *P = tm.T + C::OFF_PS + slot * C::PSLOT;
        const uint4 A = reinterpret_cast<const uint4 *>(P)[lane];
        const float *pf = reinterpret_cast<const float *>(P + 512);
        const float al = pf[gi];
        if (__any_sync(FULL, al != 1.0f)) {
#pragma unroll
            for (int j = 0; j < C::CH; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[j][e] = __fmul_rn(acc[j][e], al);
        }
#pragma unroll
        for (int j = 0; j < C::CH; j += 2) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(vrow + 16u * uint32_t((j + cadd) ^ sw), v0, v1, v2, v3);
            mma_bf16(acc[j][0], acc[j][1], acc[j][2], acc[j][3], A.x, A.y, A.z, A.w, v0, v1);
            mma_bf16(acc[j + 1][0], acc[j + 1][1], acc[j + 1][2], acc[j + 1][3], A.x, A.y, A.z,
                     A.w, v2, v3);
        }
        if (st.seg_end) {
            const UnitDev &cu = st.cu;
            if (st.whole_unit()) {
                if (gi < cu.n_q) {
                    const float inv = __frcp_rn(pf[16 + gi]);
                    float *o = cu.out + size_t(gi) * cu.q_stride;
#pragma unroll
                    for (int j = 0; j < C::CH; ++j) {
                        o[8 * j + tig] = __fmul_rn(__fadd_rn(acc[j][0], acc[j][2]), inv);
                        o[8 * j + 4 + tig] = __fmul_rn(__fadd_rn(acc[j][1], acc[j][3]), inv);
                    }
                }
            } else {
                const int ps = (st.seg_begin == fb0) ? 0 : 1;
                float *part = a.partials + (size_t(team) * 2 + ps) * partial_stride(D);
                if (lane < 16) part[lane] = pf[8 + lane];  // m[8], l[8]
                float *ac = part + 16 + gi * D;
#pragma unroll
                for (int j = 0; j < C::CH; ++j) {
                    ac[8 * j + tig] = __fadd_rn(acc[j][0], acc[j][2]);
                    ac[8 * j + 4 + tig] = __fadd_rn(acc[j][1], acc[j][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar + 8u * uint32_t(slot));
        st.advance();
    }
}

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

    Team tm;
    tm.T = smem + tl * C::TEAM;
    tm.bar0 = smem_u32(tm.T + C::OFF_BAR);
    tm.abort = reinterpret_cast<volatile int *>(tm.T + C::OFF_FLAG);
    if (w == 0 && lane == 0) {
        for (int i = 0; i < C::NBARS; ++i) mbar_init(tm.bar0 + 8 * i, 1);
        *tm.abort = 0;
        fence_mbar_init();
    }
    named_bar(tl + 1, 64);

    if (w == 0)
        k_warp<D, BF16IN>(a, tm, team, fb0, fb1, lane);
    else
        v_warp<D, BF16IN>(a, tm, team, fb0, fb1, lane);
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
