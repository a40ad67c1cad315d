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
constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the SFU (ex2.approx.f32, subnormal results kept).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__host__ __device__ constexpr int round16(int x) { return (x + 15) & ~15; }

template <int D> struct Cfg {
    static constexpr int CH = D / 8;          // 16-byte chunks per BF16 row
    static constexpr int STEPS = D / 16;      // 256-element warp steps per 16-row tile
    static constexpr int ESC_CAP = 1536;      // escape bytes staged per block and tensor
    static constexpr int SLOT = 32 * D + 32;  // one tensor tile: raw rows, or sm + residual rows
    static constexpr int NSTAGE = D <= 64 ? 4 : 3;
    static constexpr int BASE_SLOT = round16(D + 32);
    static constexpr int MSLOT = BASE_SLOT + ESC_CAP + 32;  // base + escapes of one block
    static constexpr int TILE = TT * D * 2;                  // bytes of one BF16 tile
    static constexpr int PSLOT = 640;                        // p values + alpha + m + l
    // per-warp region: ring | meta x2 | BF16 tile | stage barriers
    static constexpr int W_META = NSTAGE * SLOT;
    static constexpr int W_TILE = W_META + 2 * MSLOT;
    static constexpr int W_BAR = W_TILE + TILE;
    static constexpr int WARP_BYTES = (W_BAR + NSTAGE * 8 + 127) & ~127;
    // team: K-warp region | V-warp region | P slots x2 | full x2, empty x2 | abort flag
    static constexpr int OFF_PS = 2 * WARP_BYTES;
    static constexpr int OFF_BAR = OFF_PS + 2 * PSLOT;
    static constexpr int OFF_FLAG = OFF_BAR + 4 * 8;
    static constexpr int TEAM = (OFF_FLAG + 16 + 127) & ~127;
    static constexpr int BY_SMEM = 232448 / TEAM;
    static constexpr int TEAMS = BY_SMEM < 8 ? BY_SMEM : 8;
    static_assert(TEAMS >= 1, "team does not fit in shared memory");
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

__device__ __forceinline__ uint32_t esc_word(uint32_t r, uint32_t n, const uint8_t *sm,
                                             const uint8_t *gm, int *status) {
    if (r >= n) {
        report(status, KVX_ERR_RUNTIME, DERR_ESC_OVERRUN);
        return 0;
    }
    return sm != nullptr ? *reinterpret_cast<const uint16_t *>(sm + 2 * r)
                         : __ldg(reinterpret_cast<const unsigned short *>(gm) + r);
}

// General case of escape patching (some lane holds two or more sentinels).  Sentinel elements
// take the next escape words in scan order: lane order inside the 256-element step, element
// order inside the lane.  Element k of a lane sits at half (k >> 2) of 32-bit word (k & 3) of the
// lane's 16-byte tile chunk.  Returns the new running escape count.
template <int SH>
__device__ __noinline__ uint32_t patch_general(uint8_t *chunk, uint32_t m, uint32_t run, uint32_t n,
                                               const uint8_t *sm, const uint8_t *gm, int *status) {
    const uint32_t cnt = __popc(m);
    const uint32_t lt = lanemask_lt();
    const uint32_t c0 = __ballot_sync(FULL, cnt & 1u), c1 = __ballot_sync(FULL, cnt & 2u);
    const uint32_t c2 = __ballot_sync(FULL, cnt & 4u), c3 = __ballot_sync(FULL, cnt & 8u);
    uint32_t r = run + __popc(c0 & lt) + 2 * __popc(c1 & lt) + 4 * __popc(c2 & lt) +
                 8 * __popc(c3 & lt);
    const uint32_t tot = __popc(c0) + 2 * __popc(c1) + 4 * __popc(c2) + 8 * __popc(c3);
    while (m != 0u) {
        const int k = (__ffs(m) - 1) / SH;
        m &= m - 1u;
        *reinterpret_cast<uint16_t *>(chunk + 4 * (k & 3) + 2 * (k >> 2)) =
            uint16_t(esc_word(r, n, sm, gm, status));
        ++r;
    }
    return run + tot;
}

// Escape patching for one 256-element step: fast path when every lane holds at most one sentinel.
template <int SH>
__device__ __forceinline__ void patch(uint8_t *chunk, uint32_t m, Esc &es, int *status) {
    const uint32_t has = __ballot_sync(FULL, m != 0u);
    if (has == 0u) return;
    if (__ballot_sync(FULL, (m & (m - 1u)) != 0u) == 0u) {
        if (m != 0u) {
            const uint32_t r = es.run + __popc(has & lanemask_lt());
            const int k = (__ffs(m) - 1) / SH;
            *reinterpret_cast<uint16_t *>(chunk + 4 * (k & 3) + 2 * (k >> 2)) =
                uint16_t(esc_word(r, es.n, es.sm, es.gm, status));
        }
        es.run += __popc(has);
    } else {
        es.run = patch_general<SH>(chunk, m, es.run, es.n, es.sm, es.gm, status);
    }
}

template <bool MIS> __device__ __forceinline__ uint32_t ldw2(const uint8_t *p) {
    if (!MIS) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - 2);
    return prmt(q[0], q[1], 0x5432);
}

template <int D, bool MIS>
__device__ __forceinline__ void decode_tile_t(uint8_t *tile, int mode, int rows, const uint8_t *p0,
                                              const uint8_t *p1, const uint32_t (&b7)[4], Esc &es,
                                              int *status, int lane) {
    constexpr int CH = Cfg<D>::CH;
    const int ch = lane % CH;
#pragma unroll 1
    for (int c = 0; c < Cfg<D>::STEPS; ++c) {
        const int e0 = 256 * c + 8 * lane;
        const int row = e0 / D;
        uint32_t bf0 = 0, bf1 = 0, bf2 = 0, bf3 = 0;
        uint32_t m = 0;
        if (row < rows) {
            if (mode == 0) {
                const uint8_t *p = p0 + 2 * e0;
                const uint32_t w0 = ldw2<MIS>(p), w1 = ldw2<MIS>(p + 4);
                const uint32_t w2 = ldw2<MIS>(p + 8), w3 = ldw2<MIS>(p + 12);
                bf0 = prmt(w0, w2, 0x5410);
                bf1 = prmt(w0, w2, 0x7632);
                bf2 = prmt(w1, w3, 0x5410);
                bf3 = prmt(w1, w3, 0x7632);
            } else {
                const uint32_t S0 = ldw2<MIS>(p0 + e0), S1 = ldw2<MIS>(p0 + e0 + 4);
                uint32_t X, sh, mask;
                if (mode == 4) {
                    X = ldw2<MIS>(p1 + e0 / 2);  // element k at bits 4k
                    uint32_t t = X & (X >> 1);
                    t &= t >> 2;
                    m = t & 0x11111111u;
                    sh = 4;
                    mask = 0x000F000Fu;
                } else {
                    const uint32_t C = *reinterpret_cast<const uint16_t *>(p1 + e0 / 4);
                    m = C & (C >> 1) & 0x5555u;   // element k at bits 2k
                    X = prmt(C, 0, 0x0110);       // elements 4..7 up to bits 16..23
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
        if (mode == 4) patch<4>(dst, m, es, status);
        else if (mode == 2) patch<2>(dst, m, es, status);
    }
}

template <int D>
__device__ __forceinline__ void decode_tile(uint8_t *tile, int mode, int rows, const uint8_t *p0,
                                            const uint8_t *p1, const uint32_t (&b7)[4], Esc &es,
                                            int *status, int lane) {
    if (reinterpret_cast<uintptr_t>(p0) & 2u)
        decode_tile_t<D, true>(tile, mode, rows, p0, p1, b7, es, status, lane);
    else
        decode_tile_t<D, false>(tile, mode, rows, p0, p1, b7, es, status, lane);
}

// b7[i] = (base[d0+i] << 7) | (base[d0+i+4] << 23)
__device__ __forceinline__ void load_base(const uint8_t *p, uint32_t (&b7)[4]) {
    const bool mis = (reinterpret_cast<uintptr_t>(p) & 2u) != 0u;
    const uint32_t B0 = mis ? ldw2<true>(p) : ldw2<false>(p);
    const uint32_t B1 = mis ? ldw2<true>(p + 4) : ldw2<false>(p + 4);
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// The warp copies one piece: lane l moves 16-byte chunks l, l + 32, ...
__device__ __forceinline__ void copy_piece(uint32_t dst, const Piece &p, int lane) {
    const uint32_t n = p.alloc >> 4;
    for (uint32_t j = lane; j < n; j += 32) cp_async16(dst + 16 * j, p.src + 16 * j);
}

struct Team {
    uint8_t *T;
    uint32_t bar0;  // full x2, empty x2
    volatile int *abort;
};

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

// Walks the team's flat blocks with one block of prefetch.
struct Walker {
    int64_t fb, fb1;
    FlatBlock cur, nxt;
    int unit, nunit;
    __device__ void init(const AttnArgs &a, int64_t b0, int64_t b1) {
        fb = b0;
        fb1 = b1;
        cur = load_flat(a.flat, fb);
        unit = __ldg(a.flat_unit + fb);
        nunit = unit;
        if (fb + 1 < fb1) {
            nxt = load_flat(a.flat, fb + 1);
            nunit = __ldg(a.flat_unit + fb + 1);
        }
    }
    __device__ void next(const AttnArgs &a) {
        ++fb;
        if (fb < fb1) {
            cur = nxt;
            unit = nunit;
            if (fb + 1 < fb1) {
                nxt = load_flat(a.flat, fb + 1);
                nunit = __ldg(a.flat_unit + fb + 1);
            }
        }
    }
};

// One warp's own copy pipeline for its tensor (t = 0: K, 1: V): cp.async tiles into a ring of
// NSTAGE slots, each completing on its own mbarrier; a block's first tile also brings the block's
// base array and (when they fit) its escape words into a meta slot.
template <int D, bool BF16IN> struct Pipe {
    using C = Cfg<D>;
    uint8_t *R;       // this warp's region
    uint32_t sbar;    // stage barriers
    int t;            // tensor
    Walker pw;        // producer position
    int p_tile = 0, p_stage = 0, p_bseq = 0;
    int p_unit = -1;
    const uint8_t *p_blob = nullptr;

    __device__ static int mode_of(const FlatBlock &f, int t) { return t == 0 ? f.k_mode : f.v_mode; }
    __device__ static uint32_t off_of(const FlatBlock &f, int t) { return t == 0 ? f.k_off : f.v_off; }
    __device__ static int nesc_of(const FlatBlock &f, int t) { return t == 0 ? f.k_nesc : f.v_nesc; }

    // Escape words of a block and whether they are staged in the meta slot.
    __device__ static Piece esc_piece(const Geo &g, int n_tok, int nesc, bool &staged) {
        const Piece e = make_piece(g.s1 + size_t(n_tok) * D * g.mode / 8, uint32_t(2 * nesc));
        staged = nesc > 0 && e.alloc <= uint32_t(C::ESC_CAP + 32);
        return e;
    }

    // Issue tiles while a ring slot is free; block starts wait until the consumer is at most one
    // block behind, so a meta slot is never overwritten while in use.
    __device__ void produce(const AttnArgs &a, int c_stage, int64_t c_fb, int lane) {
        while (pw.fb < pw.fb1 && p_stage - c_stage < C::NSTAGE) {
            if (p_tile == 0 && pw.fb - c_fb >= 2) break;
            const FlatBlock &f = pw.cur;
            if (pw.unit != p_unit) {
                p_unit = pw.unit;
                p_blob = t == 0 ? a.units[p_unit].k : a.units[p_unit].v;
            }
            const Geo g = make_geo<D, BF16IN>(p_blob, off_of(f, t), mode_of(f, t), f.n_tok);
            const int rows = min(TT, int(f.n_tok) - p_tile * TT);
            Piece pc[2];
            const int np = geo_pieces<D>(g, p_tile, rows, pc);
            const uint32_t slot = smem_u32(R + (p_stage % C::NSTAGE) * C::SLOT);
            copy_piece(slot, pc[0], lane);
            if (np == 2) copy_piece(slot + pc[0].alloc, pc[1], lane);
            if (!BF16IN && p_tile == 0 && g.mode != 0) {
                const uint32_t ms = smem_u32(R + C::W_META + (p_bseq & 1) * C::MSLOT);
                copy_piece(ms, make_piece(g.s0 - D, D), lane);
                bool staged;
                const Piece e = esc_piece(g, f.n_tok, nesc_of(f, t), staged);
                if (staged) copy_piece(ms + C::BASE_SLOT, e, lane);
            }
            cp_async_arrive(sbar + 8u * uint32_t(p_stage % C::NSTAGE));
            ++p_stage;
            if (++p_tile * TT >= int(f.valid)) {
                p_tile = 0;
                ++p_bseq;
                pw.next(a);
            }
        }
    }
};

// Consumer-side position (both warps keep their own copy).
template <int D, bool BF16IN> struct Cursor {
    using C = Cfg<D>;
    Walker cw;
    int64_t fb0, seg_begin;
    int tile = 0, stage = 0, bseq = 0, unit = -1;
    UnitDev cu{};
    Geo g{};          // this warp's tensor in the current block
    int rows = 0;
    bool first = true, last_tile = false, seg_end = false;

    __device__ void init(const AttnArgs &a, int64_t b0, int64_t b1) {
        cw.init(a, b0, b1);
        fb0 = b0;
        seg_begin = b0;
    }
    // Set up the current tile; at a block start also the base registers and escape source
    // (the meta slot was filled by the block's first stage, which the caller has waited for).
    __device__ void setup(const AttnArgs &a, const uint8_t *R, int t, int lane, uint32_t (&b7)[4],
                          Esc &es) {
        const FlatBlock &f = cw.cur;
        first = tile == 0;
        if (first) {
            if (cw.unit != unit) {
                unit = cw.unit;
                cu = a.units[unit];
            }
            g = make_geo<D, BF16IN>(t == 0 ? cu.k : cu.v, Pipe<D, BF16IN>::off_of(f, t),
                                    Pipe<D, BF16IN>::mode_of(f, t), f.n_tok);
            if (!BF16IN && g.mode != 0) {
                const uint8_t *ms = R + C::W_META + (bseq & 1) * C::MSLOT;
                const uint8_t *b = g.s0 - D;
                load_base(ms + (reinterpret_cast<uintptr_t>(b) & 15u) + 8 * (lane % C::CH), b7);
                bool staged;
                const Piece e = Pipe<D, BF16IN>::esc_piece(g, f.n_tok, Pipe<D, BF16IN>::nesc_of(f, t),
                                                           staged);
                es.run = 0;
                es.n = Pipe<D, BF16IN>::nesc_of(f, t);
                es.gm = e.src + e.data;
                es.sm = staged ? ms + C::BASE_SLOT + e.data : nullptr;
            }
        }
        rows = min(TT, int(f.valid) - tile * TT);
        last_tile = (tile + 1) * TT >= int(f.valid);
        const int64_t ub = cu.block_begin + cu.n_blocks;
        seg_end = last_tile && ((cw.fb + 1 == cw.fb1) || (cw.fb + 1 == ub));
    }
    __device__ bool whole_unit() const {
        return seg_begin == cu.block_begin && cw.fb + 1 == cu.block_begin + cu.n_blocks;
    }
    // Where this tile's data starts in the slot.
    __device__ void data(const uint8_t *R, const uint8_t *&p0, const uint8_t *&p1) const {
        const FlatBlock &f = cw.cur;
        const int rl = min(TT, int(f.n_tok) - tile * TT);
        Piece pc[2];
        const int np = geo_pieces<D>(g, tile, rl, pc);
        const uint8_t *slot = R + (stage % C::NSTAGE) * C::SLOT;
        p0 = slot + pc[0].data;
        p1 = np == 2 ? slot + pc[0].alloc + pc[1].data : nullptr;
    }
    __device__ void advance(const AttnArgs &a) {
        ++stage;
        if (last_tile) {
            tile = 0;
            ++bseq;
            if (seg_end) seg_begin = cw.fb + 1;
            cw.next(a);
        } else {
            ++tile;
        }
    }
};

// K-warp: streams and rebuilds K, runs QK and the online softmax, hands p over to the V-warp.
template <int D, bool BF16IN>
__device__ __forceinline__ void k_warp(const AttnArgs &a, const Team &tm, uint8_t *R, int64_t fb0,
                                       int64_t fb1, int lane) {
    using C = Cfg<D>;
    const uint32_t full_bar = tm.bar0, empty_bar = tm.bar0 + 16u;
    const int gi = lane >> 2, tig = lane & 3;
    Pipe<D, BF16IN> pp;
    pp.R = R;
    pp.sbar = smem_u32(R + C::W_BAR);
    pp.t = 0;
    pp.pw.init(a, fb0, fb1);
    Cursor<D, BF16IN> cs;
    cs.init(a, fb0, fb1);
    uint32_t b7[4] = {0, 0, 0, 0};
    Esc es{0, 0, nullptr, nullptr};
    uint8_t *kt = R + C::W_TILE;
    uint32_t qb[D / 16][2];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int mat = lane >> 3;
    const int r = (lane & 7) + 8 * (mat & 1);
    const int cadd = mat >> 1;
    const int sw = swz<D>(r);
    const uint32_t krow = smem_u32(kt) + uint32_t(r * 2 * D);
    bool ok = true;

    while (cs.cw.fb < fb1) {
        pp.produce(a, cs.stage, cs.cw.fb, lane);
        if (!wait_bar(pp.sbar + 8u * uint32_t(cs.stage % C::NSTAGE), (cs.stage / C::NSTAGE) & 1, tm,
                      a)) {
            ok = false;
            break;
        }
        cs.setup(a, R, 0, lane, b7, es);
        if (cs.first && cs.cw.fb == cs.seg_begin) {
            load_q_frags<D>(cs.cu.q, cs.cu.n_q, cs.cu.q_stride, qb, lane);
            m0 = m1 = -INFINITY;
            l0 = l1 = 0.f;
        }
        const uint8_t *p0, *p1;
        cs.data(R, p0, p1);
        const int rows = cs.rows;
        decode_tile<D>(kt, cs.g.mode, rows, p0, p1, b7, es, a.status, lane);
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
        // p = 2^(s log2e - m log2e): one FMA and one ex2 per score
        const float mn0 = fmaxf(m0, t0), mn1 = fmaxf(m1, t1);
        const float ml0 = __fmul_rn(mn0, kLog2e), ml1 = __fmul_rn(mn1, kLog2e);
        const float al0 = ex2(__fmaf_rn(m0, kLog2e, -ml0)), al1 = ex2(__fmaf_rn(m1, kLog2e, -ml1));
        const float p0v = ex2(__fmaf_rn(s0, kLog2e, -ml0)), p1v = ex2(__fmaf_rn(s1, kLog2e, -ml1));
        const float p2v = ex2(__fmaf_rn(s2, kLog2e, -ml0)), p3v = ex2(__fmaf_rn(s3, kLog2e, -ml1));
        l0 = __fmaf_rn(l0, al0, __fadd_rn(p0v, p2v));
        l1 = __fmaf_rn(l1, al1, __fadd_rn(p1v, p3v));
        m0 = mn0;
        m1 = mn1;
        float lt0 = l0, lt1 = l1;
        if (cs.seg_end) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                lt0 = __fadd_rn(lt0, __shfl_xor_sync(FULL, lt0, o));
                lt1 = __fadd_rn(lt1, __shfl_xor_sync(FULL, lt1, o));
            }
        }
        // hand p over; slot reuse waits until the V-warp is done with tile stage - 2
        const int slot = cs.stage & 1;
        if (cs.stage >= 2 &&
            !wait_bar(empty_bar + 8u * uint32_t(slot), ((cs.stage - 2) >> 1) & 1, tm, a)) {
            ok = false;
            break;
        }
        uint8_t *P = tm.T + C::OFF_PS + slot * C::PSLOT;
        reinterpret_cast<float4 *>(P)[lane] = make_float4(p0v, p1v, p2v, p3v);
        float *pf = reinterpret_cast<float *>(P + 512);
        if (gi == 0) {
            pf[2 * tig] = al0;
            pf[2 * tig + 1] = al1;
            if (cs.seg_end) {
                pf[8 + 2 * tig] = m0;
                pf[8 + 2 * tig + 1] = m1;
                pf[16 + 2 * tig] = lt0;
                pf[16 + 2 * tig + 1] = lt1;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(full_bar + 8u * uint32_t(slot));
        cs.advance(a);
    }
    if (!ok) {
        // bounded drain of this warp's copies still in flight
        for (int i = cs.stage; i < pp.p_stage; ++i)
            mbar_wait_bounded(pp.sbar + 8u * uint32_t(i % C::NSTAGE), (i / C::NSTAGE) & 1,
                              a.wait_limit);
    }
}

// V-warp: streams and rebuilds V, accumulates O += P V over the whole head dim, writes outputs
// or partial states.
template <int D, bool BF16IN>
__device__ __forceinline__ void v_warp(const AttnArgs &a, const Team &tm, uint8_t *R, int team,
                                       int64_t fb0, int64_t fb1, int lane) {
    using C = Cfg<D>;
    const uint32_t full_bar = tm.bar0, empty_bar = tm.bar0 + 16u;
    const int gi = lane >> 2, tig = lane & 3;
    Pipe<D, BF16IN> pp;
    pp.R = R;
    pp.sbar = smem_u32(R + C::W_BAR);
    pp.t = 1;
    pp.pw.init(a, fb0, fb1);
    Cursor<D, BF16IN> cs;
    cs.init(a, fb0, fb1);
    uint32_t b7[4] = {0, 0, 0, 0};
    Esc es{0, 0, nullptr, nullptr};
    uint8_t *vt = R + C::W_TILE;
    float acc[C::CH][4];  // rows gi: hi part, rows gi + 8: mid part of query gi
    const int mat = lane >> 3;
    const int r = (lane & 7) + 8 * (mat & 1);
    const int cadd = mat >> 1;
    const int sw = swz<D>(r);
    const uint32_t vrow = smem_u32(vt) + uint32_t(r * 2 * D);
    bool ok = true;

    while (cs.cw.fb < fb1) {
        pp.produce(a, cs.stage, cs.cw.fb, lane);
        if (!wait_bar(pp.sbar + 8u * uint32_t(cs.stage % C::NSTAGE), (cs.stage / C::NSTAGE) & 1, tm,
                      a)) {
            ok = false;
            break;
        }
        cs.setup(a, R, 1, lane, b7, es);
        if (cs.first && cs.cw.fb == cs.seg_begin) {
#pragma unroll
            for (int j = 0; j < C::CH; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        }
        const uint8_t *p0, *p1;
        cs.data(R, p0, p1);
        decode_tile<D>(vt, cs.g.mode, cs.rows, p0, p1, b7, es, a.status, lane);
        __syncwarp();
        const int slot = cs.stage & 1;
        if (!wait_bar(full_bar + 8u * uint32_t(slot), (cs.stage >> 1) & 1, tm, a)) {
            ok = false;
            break;
        }
        const uint8_t *P = tm.T + C::OFF_PS + slot * C::PSLOT;
        const float4 pv4 = reinterpret_cast<const float4 *>(P)[lane];
        const float *pf = reinterpret_cast<const float *>(P + 512);
        // P^T tile (lane: tokens gi, gi+8 x queries 2tig, 2tig+1) -> P A-fragments: rows 0-7
        // carry bf16(p), rows 8-15 bf16(p - bf16(p)), so P enters the MMA with 16 bits
        uint4 A;
        {
            const uint32_t h01 = pack_bf16x2(pv4.y, pv4.x), h23 = pack_bf16x2(pv4.w, pv4.z);
            const float r0 = __fsub_rn(pv4.x, bf16lo_to_f32(h01));
            const float r1 = __fsub_rn(pv4.y, bf16hi_to_f32(h01));
            const float r2 = __fsub_rn(pv4.z, bf16lo_to_f32(h23));
            const float r3 = __fsub_rn(pv4.w, bf16hi_to_f32(h23));
            const uint32_t mm01 = pack_bf16x2(r1, r0), mm23 = pack_bf16x2(r3, r2);
            A = make_uint4(movm_t(h01), movm_t(mm01), movm_t(h23), movm_t(mm23));
        }
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
        if (cs.seg_end) {
            const UnitDev &cu = cs.cu;
            if (cs.whole_unit()) {
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
                const int ps = (cs.seg_begin == fb0) ? 0 : 1;
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
        cs.advance(a);
    }
    if (!ok) {
        for (int i = cs.stage; i < pp.p_stage; ++i)
            mbar_wait_bounded(pp.sbar + 8u * uint32_t(i % C::NSTAGE), (i / C::NSTAGE) & 1,
                              a.wait_limit);
    }
}

template <int D, bool BF16IN>
__global__ void __launch_bounds__(64 * Cfg<D>::TEAMS, 1) attn_kernel(const AttnArgs a) {
    using C = Cfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tl = warp >> 1;
    // K-warp of team tl is warp 2*tl + ((tl >> 1) & 1): spreads the roles over all four SM
    // sub-partitions (warp % 4).
    const int w = (warp & 1) ^ ((tl >> 1) & 1);
    const int team = blockIdx.x * C::TEAMS + tl;
    if (team >= a.n_teams) return;
    const int64_t fb0 = a.team_begin[team], fb1 = a.team_begin[team + 1];
    if (fb0 >= fb1) return;

    Team tm;
    tm.T = smem + tl * C::TEAM;
    tm.bar0 = smem_u32(tm.T + C::OFF_BAR);
    tm.abort = reinterpret_cast<volatile int *>(tm.T + C::OFF_FLAG);
    uint8_t *R = tm.T + w * C::WARP_BYTES;
    if (lane == 0) {
        // each warp initialises its own stage barriers (one arrival per lane); the K-warp the
        // shared full / empty barriers
        const uint32_t sbar = smem_u32(R + C::W_BAR);
        for (int i = 0; i < C::NSTAGE; ++i) mbar_init(sbar + 8 * i, 32);
        if (w == 0) {
            for (int i = 0; i < 4; ++i) mbar_init(tm.bar0 + 8 * i, 1);
            *tm.abort = 0;
        }
        fence_mbar_init();
    }
    named_bar(tl + 1, 64);
    if (w == 0)
        k_warp<D, BF16IN>(a, tm, R, fb0, fb1, lane);
    else
        v_warp<D, BF16IN>(a, tm, R, team, fb0, fb1, lane);
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
