// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened; each worker warp owns a contiguous range and
//    streams the compressed 16-token tiles of K and V (sign/mantissa rows and packed exponent
//    residuals, or raw BF16 rows) through its own shared-memory ring with cp.async, one cp.async
//    group per tile.  A block's base exponents and escape words ride along with its first tile.
//    Only the compressed bytes cross HBM, and no warp ever waits on another warp.
//  * K rows are rebuilt straight into mma.sync A fragments: lane (g, t) rebuilds tokens g and g+8,
//    head dims [t D/4, (t+1) D/4).  The MMA's k index runs over the head dims in that permuted
//    order and the query B fragments use the same order, so S = K Q^T (tokens x queries, fp32
//    accumulate) needs no shared-memory staging of a BF16 tile.
//  * The online softmax runs on the S fragments: lane (g, t) holds queries 2t and 2t+1, which are
//    also the output columns it accumulates, so the rescale factors never leave the lane.
//  * V rows are rebuilt into A fragments of V^T: lane (g, t) rebuilds tokens 2t, 2t+1, 2t+8, 2t+9,
//    head dims [g D/8, (g+1) D/8).  O^T += V^T P^T with P^T split into a bf16 part and a bf16
//    residual part (two MMAs), so P enters with 16 significant bits.
//  * Exponent escapes are patched in the staged words before the rebuild, in the container's scan
//    order (token-major); the lane order of both fragment layouts gives each sentinel its rank with
//    a few warp ballots.
//  * Unit segments that span several workers leave (m, l, acc) partial states that combine_kernel
//    folds in worker order with merge_state semantics (src/softmax.hpp:16-30), then finalizes like
//    finalize_state (src/softmax.hpp:32-41: reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template reading [seq, dim] BF16 rows; for the same
// blocks and worker ranges it produces bit-identical outputs to the XKV variant, because both
// rebuild identical BF16 fragments and run identical arithmetic afterwards.  (Ranges are one block
// per worker whenever the step has no more blocks than workers; beyond that they are balanced by
// cost, and escape words count towards an XKV block's cost.)
#include "attention.cuh"

namespace kvx {
namespace {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int TT = 16;  // tokens per tile (one m16 block of the QK MMA)
constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the SFU (ex2.approx.f32, subnormal results kept).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__host__ __device__ constexpr int round16(int x) { return (x + 15) & ~15; }
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

#ifndef KVX_NSTAGE64
#define KVX_NSTAGE64 2
#endif
#ifndef KVX_MAXWARPS
#define KVX_MAXWARPS 12
#endif

template <int D> struct Cfg {
    static constexpr int DK = D / 4;        // head dims per lane in a K row
    static constexpr int NK = D / 8;        // K fragment registers per row (dim pairs)
    static constexpr int DV = D / 8;        // head dims per lane in a V token (= V registers)
    static constexpr int KS = D / 16;       // k-steps of QK = M-tiles of PV
    static constexpr bool SPLIT = D > 128;  // rebuild row halves one at a time (register budget)
    static constexpr bool B7REG = D <= 128; // keep the block's base exponents in registers
    static constexpr int ESC_CAP = 1536;    // escape bytes staged per block and tensor
    // A ring stage holds TSC tokens of a coded block or TT tokens of a raw one (raw rows take
    // two bytes per element, coded ones 1.25-1.5), for K and V.
    static constexpr int TSC = D <= 128 ? 2 * TT : TT;
    static constexpr int SUBS = TSC / TT;         // 16-token sub-tiles per stage at most
    static constexpr int TR = round16(cmax(TSC * D * 3 / 2 + 48, TT * 2 * D + 32));  // one tensor
    static constexpr int CODE_OFF = TSC * D + 16;  // residual-code rows inside a coded tensor stage
    static constexpr int SLOT = 2 * TR;            // K stage | V stage
    static constexpr int NSTAGE = D <= 32 ? 3 : D == 64 ? KVX_NSTAGE64 : 2;
    static_assert(NSTAGE >= 2 && NSTAGE <= 4, "stage waits cover at most 3 younger groups");
    static constexpr int BASE = round16(D + 32);  // one block's base exponents (+ alignment slack)
    static constexpr int ESCB = ESC_CAP + 32;
    static constexpr int M_K = 0, M_V = BASE, M_EK = 2 * BASE, M_EV = 2 * BASE + ESCB;
    static constexpr int MSLOT = 2 * BASE + 2 * ESCB;
    // Escape scratch: the consumed sm rows of the sub-tile, except when the row halves are rebuilt
    // one at a time (then the second half's rows are still unread): a region of its own.
    static constexpr int SCR = SPLIT ? TT * D : 0;
    static constexpr int W_META = NSTAGE * SLOT;  // per-warp region: ring | meta x2 | scratch
    static constexpr int W_SCR = W_META + 2 * MSLOT;
    static constexpr int WARP_BYTES = (W_SCR + SCR + 127) & ~127;
    static constexpr int WARPS = cmin(KVX_MAXWARPS, 232448 / WARP_BYTES);
    static_assert(WARPS >= 1, "worker does not fit in shared memory");
};

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

// ---- copies ------------------------------------------------------------------------------------

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

// No "memory" clobber: a clobber would pin every address-taken local in memory around each copy.
// Ordering against this warp's own shared-memory reads comes from __syncwarp() before a slot is
// refilled and from the clobber on cp_async_wait() before it is read.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
// One cp.async group per ring stage; a consumer waits until at most `younger` groups issued after
// the stage it needs are still in flight.  These waits end by themselves: they wait for this
// thread's own copies only.
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait(int younger) {
    switch (younger) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}
// The warp copies one piece of at most MAXB bytes: lane l moves 16-byte chunks l, l + 32, ...
template <int MAXB>
__device__ __forceinline__ void copy_piece(uint8_t *dst, const Piece p, int lane) {
    constexpr int MAXC = (MAXB / 16 + 31) / 32;
    const uint32_t n = p.alloc >> 4;
    const uint32_t d = smem_u32(dst) + 16u * uint32_t(lane);
    const uint8_t *src = p.src + 16 * lane;
#pragma unroll
    for (int k = 0; k < MAXC; ++k)
        if (uint32_t(lane + 32 * k) < n) cp_async16(d + 512u * k, src + 512 * k);
}

// Section pointers of one tensor of one block.
struct Sections {
    const uint8_t *rows;   // coded: sign/mantissa rows; raw / BF16: BF16 rows
    const uint8_t *codes;  // coded: packed residual codes
    const uint8_t *esc;    // coded: escape words
};

template <int D, bool BF16IN>
__device__ __forceinline__ Sections sections(const uint8_t *blob, uint32_t off, int mode, int n_tok) {
    Sections s;
    if (BF16IN) {
        s.rows = blob + size_t(off) * (2 * D);
        s.codes = s.esc = nullptr;
    } else if (mode == 0) {
        s.rows = blob + off + kHeaderBytes;
        s.codes = s.esc = nullptr;
    } else {
        s.rows = blob + off + kHeaderBytes + D;
        s.codes = s.rows + size_t(n_tok) * D;
        s.esc = s.codes + size_t(n_tok) * D * mode / 8;
    }
    return s;
}

// Whether a block's escape words fit its meta slot (producer and consumer agree on this).
template <int D> __device__ __forceinline__ bool esc_staged(const Piece &e, int nesc) {
    return nesc > 0 && e.alloc <= uint32_t(Cfg<D>::ESCB);
}

// ---- decode helpers ----------------------------------------------------------------------------

// NW 32-bit words of shared memory starting at any byte address (byte 0 in bits 0-7 of w[0]).
// The aligned pointer is derived from p by pointer arithmetic (not through an integer), so the
// compiler keeps these as 32-bit shared-memory loads.
template <int NW> __device__ __forceinline__ void lds_words(const uint8_t *p, uint32_t (&w)[NW]) {
    const uint32_t mis = uint32_t(reinterpret_cast<uintptr_t>(p)) & 3u;
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - mis);
    const uint32_t sh = mis * 8u;
    uint32_t x[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) x[i] = q[i];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(x[i], x[i + 1], sh);
}

__host__ __device__ constexpr uint32_t sel_pair(int j) {  // bytes j, j+1 of A with sign bytes
    return uint32_t(j) | (uint32_t(j | 8) << 4) | (uint32_t(j + 1) << 8) | (uint32_t((j + 1) | 8) << 12);
}
__host__ __device__ constexpr uint32_t sel_cross(int b) {  // byte b of A and of B with sign bytes
    return uint32_t(b) | (uint32_t(b | 8) << 4) | (uint32_t(4 + b) << 8) | (uint32_t((4 + b) | 8) << 12);
}
__host__ __device__ constexpr uint32_t sel_code(int j) {  // byte j of A -> bits 0-7, of B -> 16-23
    return uint32_t(j) | (uint32_t(j) << 4) | (uint32_t(4 + j) << 8) | (uint32_t(4 + j) << 12);
}
__host__ __device__ constexpr uint32_t low_bytes(int nb) {
    return nb >= 4 ? 0xFFFFFFFFu : (1u << (8 * nb)) - 1u;
}

// Two BF16 values from a sign-replicated sm pair and a code pair: exponent offsets in bytes 0 and
// 2 of cw (bytes 1 and 3 hold other offsets and are masked off).  Offsets are 8-bit wide because
// an escaped element carries its full offset (exponent - base) mod 256 there.  Exponent = base +
// offset modulo 256 like bf16_from_delta's uint8 sum (include/kvexp/bf16.hpp:35-37 of the
// reference): the carry out of bit 14 is masked away.
__device__ __forceinline__ uint32_t merge(uint32_t sg, uint32_t cw, uint32_t b7) {
    const uint32_t e = (cw & 0x00FF00FFu) * 128u + b7;
    return (sg & 0x807F807Fu) | (e & 0x7F807F80u);
}

__device__ __forceinline__ uint32_t sent4(uint32_t x) {  // nibble == 15 -> bit 4k
    uint32_t t = x & (x >> 1);
    t &= t >> 2;
    return t & 0x11111111u;
}
__device__ __forceinline__ uint32_t sent2(uint32_t x) {  // 2-bit code == 3 -> bit 2k
    return x & (x >> 1) & 0x55555555u;
}

// b7 of a K register (dims d, d+1): base[d] << 7 | base[d+1] << 23; of a V register (one dim,
// two tokens): base[d] << 7 | base[d] << 23.
template <int D>
__device__ __forceinline__ void load_b7k(const uint8_t *base, uint32_t (&b7)[Cfg<D>::NK]) {
    uint32_t B[Cfg<D>::DK / 4];
    lds_words<Cfg<D>::DK / 4>(base, B);
#pragma unroll
    for (int p = 0; p < Cfg<D>::NK; ++p) {
        const int j = 2 * (p & 1);
        b7[p] = prmt(B[p >> 1], 0u, uint32_t(j) | (4u << 4) | (uint32_t(j + 1) << 8) | (4u << 12)) << 7;
    }
}
template <int D>
__device__ __forceinline__ void load_b7v(const uint8_t *base, uint32_t (&b7)[Cfg<D>::DV]) {
    uint32_t B[Cfg<D>::DV / 4];
    lds_words<Cfg<D>::DV / 4>(base, B);
#pragma unroll
    for (int e = 0; e < Cfg<D>::DV; ++e) {
        const int j = e & 3;
        b7[e] = prmt(B[e >> 2], 0u, uint32_t(j) | (4u << 4) | (uint32_t(j) << 8) | (4u << 12)) << 7;
    }
}

// ---- escapes -----------------------------------------------------------------------------------
//
// A sentinel element takes the next escape word of its block in scan order (token-major).  The
// rows are rebuilt first (a sentinel comes out with a wrong exponent).  When a row half holds a
// sentinel, every lane writes its fragment registers to scratch in shared memory (the half's
// sign/mantissa rows, already consumed), lanes write their escape words over the sentinel
// elements in place, and every lane reads its registers back.  Ranks come from warp ballots.

struct Esc {
    uint32_t run;               // escapes consumed so far in this block
    uint32_t n;                 // escape words in this block
    const uint8_t *sm;          // staged escape words (shared memory), or nullptr
    const unsigned short *gm;   // escape words in global memory
};

__device__ __forceinline__ uint32_t esc_word(uint32_t r, const Esc &es, int *status) {
    if (r >= es.n) {
        report(status, KVX_ERR_RUNTIME, DERR_ESC_OVERRUN);
        return 0u;
    }
    return es.sm != nullptr ? uint32_t(*reinterpret_cast<const uint16_t *>(es.sm + 2 * r))
                            : uint32_t(__ldg(es.gm + r));
}

// First escape rank of this lane when the scan order is the lane order (K rows): exclusive
// prefix of the per-lane sentinel counts, bit by bit (one step when no lane holds two).
__device__ __forceinline__ uint32_t rank_lanes(uint32_t cnt, Esc &es) {
    const uint32_t lt = lanemask_lt();
    const int bits = 32 - __clz(__reduce_max_sync(FULL, cnt));
    uint32_t pre = 0, tot = 0;
#pragma unroll 1
    for (int b = 0; b < bits; ++b) {
        const uint32_t B = __ballot_sync(FULL, (cnt >> b) & 1u);
        pre += uint32_t(__popc(B & lt)) << b;
        tot += uint32_t(__popc(B)) << b;
    }
    const uint32_t r = es.run + pre;
    es.run += tot;
    return r;
}

// First escape ranks of tokens A and B of a V token half.  Lane 4g + t holds tokens 2t (A) and
// 2t+1 (B) of the half, dims [g D/8, (g+1) D/8); the scan order inside the half is
// (t, A/B, g, element).
__device__ __forceinline__ void rank_tokens(uint32_t ca, uint32_t cb, Esc &es, int lane,
                                            uint32_t &ra, uint32_t &rb) {
    const uint32_t lt = lanemask_lt();
    const int tig = lane & 3;
    const uint32_t G = 0x11111111u << tig;                // lanes with this t
    const uint32_t L = 0x11111111u * ((1u << tig) - 1u);  // lanes with a smaller t
    const int bits = 32 - __clz(__reduce_max_sync(FULL, ca > cb ? ca : cb));
    uint32_t sl = 0, sag = 0, saglt = 0, sbglt = 0, tot = 0;
#pragma unroll 1
    for (int b = 0; b < bits; ++b) {
        const uint32_t BA = __ballot_sync(FULL, (ca >> b) & 1u);
        const uint32_t BB = __ballot_sync(FULL, (cb >> b) & 1u);
        sl += uint32_t(__popc(BA & L) + __popc(BB & L)) << b;
        sag += uint32_t(__popc(BA & G)) << b;
        saglt += uint32_t(__popc(BA & G & lt)) << b;
        sbglt += uint32_t(__popc(BB & G & lt)) << b;
        tot += uint32_t(__popc(BA) + __popc(BB)) << b;
    }
    ra = es.run + sl + saglt;
    rb = es.run + sl + sag + sbglt;
    es.run += tot;
}

template <int N>
__device__ __forceinline__ void regs_to(uint32_t *p, const uint32_t (&o)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
        *reinterpret_cast<uint4 *>(p + i) = make_uint4(o[i], o[i + 1], o[i + 2], o[i + 3]);
}
template <int N> __device__ __forceinline__ void regs_from(const uint32_t *p, uint32_t (&o)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        const uint4 v = *reinterpret_cast<const uint4 *>(p + i);
        o[i] = v.x;
        o[i + 1] = v.y;
        o[i + 2] = v.z;
        o[i + 3] = v.w;
    }
}

// ---- decode ------------------------------------------------------------------------------------
//
// A K row (one token, this lane's DK dims) or a V token pair (two tokens, this lane's DV dims) is
// loaded into staged words (sign/mantissa bytes, one exponent code byte per element) and merged
// into BF16 pairs; the sentinel masks are kept for the escape walk.

// One K row of this lane (dims c0 .. c0 + DK - 1 of one token).
template <int D, int MODE> struct KRow {
    using C = Cfg<D>;
    static constexpr int NS = C::DK / 4;                                    // sm words
    static constexpr int NW = MODE == 2 ? cmax(1, C::DK / 16) : C::DK / 8;  // code words
    uint32_t S[NS], L[NW], H[NW], Cd[4][NW], mk[NW];
    uint32_t cnt;

    __device__ __forceinline__ void load(const uint8_t *rp, const uint8_t *cp, bool valid) {
        lds_words<NS>(rp, S);
        uint32_t N[NW];
        lds_words<NW>(cp, N);
        cnt = 0;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            if (MODE == 4) {
                L[i] = N[i] & 0x0F0F0F0Fu;
                H[i] = (N[i] >> 4) & 0x0F0F0F0Fu;
                mk[i] = valid ? sent4(N[i]) : 0u;
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) Cd[k][i] = (N[i] >> (2 * k)) & 0x03030303u;
                mk[i] = valid ? (sent2(N[i]) & low_bytes(C::DK / 4)) : 0u;
            }
            cnt += __popc(mk[i]);
        }
    }
    // element index of mask bit b of word i
    __device__ __forceinline__ static int elem(int i, int b) {
        return MODE == 4 ? 8 * i + (b >> 2) : 16 * i + (b >> 1);
    }
    __device__ __forceinline__ void merge_into(const uint32_t (&b7)[C::NK], uint32_t (&o)[C::NK]) const {
#pragma unroll
        for (int p = 0; p < C::NK; ++p) {
            const uint32_t sg = prmt(S[p >> 1], 0u, sel_pair(2 * (p & 1)));
            uint32_t cw;
            if (MODE == 4) {
                cw = prmt(L[p >> 2], H[p >> 2], sel_code(p & 3));
            } else {
                const int e = 2 * p, i = e >> 4, j = (e & 15) >> 2, k = e & 3;
                cw = prmt(Cd[k][i], Cd[k + 1][i], sel_code(j));
            }
            o[p] = merge(sg, cw, b7[p]);
        }
    }
};

// Escapes of one K row half (rows 0-7 or 8-15; scan order (row, dim) = (lane, element)), through
// scratch: o holds dims c0 + 2p (low half) and c0 + 2p + 1 (high half), so element e sits at
// 16-bit position e of the lane's words.  Called by the whole warp when some lane's row has one.
template <int D, int MODE>
__device__ __forceinline__ void esc_k_half(uint32_t (&o)[Cfg<D>::NK], const KRow<D, MODE> &w,
                                           uint8_t *scr, Esc &es, int *status, int lane) {
    uint32_t *mine = reinterpret_cast<uint32_t *>(scr) + lane * Cfg<D>::NK;
    __syncwarp();  // every lane has read the rows this scratch overlays
    regs_to(mine, o);
    uint32_t r = rank_lanes(w.cnt, es);
    uint16_t *h16 = reinterpret_cast<uint16_t *>(mine);
#pragma unroll
    for (int i = 0; i < KRow<D, MODE>::NW; ++i) {
        uint32_t mm = w.mk[i];
#pragma unroll 1
        while (mm != 0u) {
            const int e = KRow<D, MODE>::elem(i, __ffs(mm) - 1);
            mm &= mm - 1u;
            h16[e] = uint16_t(esc_word(r++, es, status));
        }
    }
    regs_from(mine, o);
}

// Two V tokens (A -> low halves, B -> high halves; dims v0 .. v0 + DV - 1).
template <int D, int MODE> struct VPair {
    using C = Cfg<D>;
    static constexpr int NS = C::DV / 4;
    static constexpr int NB = MODE == 2 ? C::DV / 4 : C::DV / 2;  // code bytes per token
    static constexpr int NW = (NB + 3) / 4;
    uint32_t SA[NS], SB[NS], LA[NW], HA[NW], LB[NW], HB[NW], CA[4][NW], CB[4][NW], ma[NW], mb[NW];
    uint32_t ca, cb;

    __device__ __forceinline__ void load(const uint8_t *ra, const uint8_t *rb, const uint8_t *pa,
                                         const uint8_t *pb, bool va, bool vb) {
        lds_words<NS>(ra, SA);
        lds_words<NS>(rb, SB);
        uint32_t WA[NW], WB[NW];
        lds_words<NW>(pa, WA);
        lds_words<NW>(pb, WB);
        ca = cb = 0;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            if (MODE == 4) {
                LA[i] = WA[i] & 0x0F0F0F0Fu;
                HA[i] = (WA[i] >> 4) & 0x0F0F0F0Fu;
                LB[i] = WB[i] & 0x0F0F0F0Fu;
                HB[i] = (WB[i] >> 4) & 0x0F0F0F0Fu;
                ma[i] = va ? (sent4(WA[i]) & low_bytes(NB)) : 0u;
                mb[i] = vb ? (sent4(WB[i]) & low_bytes(NB)) : 0u;
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    CA[k][i] = (WA[i] >> (2 * k)) & 0x03030303u;
                    CB[k][i] = (WB[i] >> (2 * k)) & 0x03030303u;
                }
                ma[i] = va ? (sent2(WA[i]) & low_bytes(NB)) : 0u;
                mb[i] = vb ? (sent2(WB[i]) & low_bytes(NB)) : 0u;
            }
            ca += __popc(ma[i]);
            cb += __popc(mb[i]);
        }
    }
    __device__ __forceinline__ static int elem(int i, int b) {
        return MODE == 4 ? 8 * i + (b >> 2) : 16 * i + (b >> 1);
    }
    __device__ __forceinline__ void merge_into(const uint32_t (&b7)[C::DV], uint32_t (&o)[C::DV]) const {
#pragma unroll
        for (int e = 0; e < C::DV; ++e) {
            const uint32_t sg = prmt(SA[e >> 2], SB[e >> 2], sel_cross(e & 3));
            uint32_t cw;
            if (MODE == 4) {
                const int i = e >> 3, j = (e & 7) >> 1;
                cw = (e & 1) ? prmt(HA[i], HB[i], sel_code(j)) : prmt(LA[i], LB[i], sel_code(j));
            } else {
                const int i = e >> 4, j = (e & 15) >> 2, k = e & 3;
                cw = prmt(CA[k][i], CB[k][i], sel_code(j));
            }
            o[e] = merge(sg, cw, b7[e]);
        }
    }
};

// Escapes of one V token half, through scratch: o[e] holds dim v0 + e of token A (low half) and
// token B (high half), so element e of token A (B) sits at 16-bit position 2e (2e + 1).
template <int D, int MODE>
__device__ __forceinline__ void esc_v_half(uint32_t (&o)[Cfg<D>::DV], const VPair<D, MODE> &p,
                                           uint8_t *scr, Esc &es, int *status, int lane) {
    uint32_t *mine = reinterpret_cast<uint32_t *>(scr) + lane * Cfg<D>::DV;
    __syncwarp();
    regs_to(mine, o);
    uint32_t ra, rb;
    rank_tokens(p.ca, p.cb, es, lane, ra, rb);
    uint16_t *h16 = reinterpret_cast<uint16_t *>(mine);
#pragma unroll
    for (int i = 0; i < VPair<D, MODE>::NW; ++i) {
        uint32_t mm = p.ma[i];
#pragma unroll 1
        while (mm != 0u) {
            const int e = VPair<D, MODE>::elem(i, __ffs(mm) - 1);
            mm &= mm - 1u;
            h16[2 * e] = uint16_t(esc_word(ra++, es, status));
        }
        mm = p.mb[i];
#pragma unroll 1
        while (mm != 0u) {
            const int e = VPair<D, MODE>::elem(i, __ffs(mm) - 1);
            mm &= mm - 1u;
            h16[2 * e + 1] = uint16_t(esc_word(rb++, es, status));
        }
    }
    regs_from(mine, o);
}

// ---- per-tile stages ----------------------------------------------------------------------------

// Where the current sub-tile's tensors sit in the ring slot (with the block's source alignment
// already applied), and the block's base exponents in its meta slot.
struct TileView {
    const uint8_t *k_rows, *k_codes, *v_rows, *v_codes;
    const uint8_t *k_base, *v_base;  // this lane's first base byte
    uint8_t *k_scr, *v_scr;          // 16 D bytes of consumed sm rows (16-byte aligned), scratch
    int rows;                        // valid tokens in the sub-tile
};

// S^T fragment of the tile: s0/s1 token g (queries 2t, 2t+1), s2/s3 token g + 8.
template <int D, int MODE>
__device__ __forceinline__ void qk_tile(const TileView &tv, const uint32_t (&b7r)[Cfg<D>::NK],
                                        const uint32_t (&qb)[Cfg<D>::KS][2], Esc &es, int *status,
                                        int lane, float (&s)[4]) {
    using C = Cfg<D>;
    const int gi = lane >> 2, tig = lane & 3;
    constexpr int RS = MODE == 0 ? 2 * D : D;  // row stride of the row section
    constexpr int CS = D * MODE / 8;           // row stride of the code section
    const int c0 = tig * C::DK;
    const uint8_t *r0 = tv.k_rows + gi * RS + (MODE == 0 ? 2 * c0 : c0);
    const uint8_t *q0 = tv.k_codes + gi * CS + c0 * MODE / 8;
    s[0] = s[1] = s[2] = s[3] = 0.f;
    if (MODE == 0) {
        uint32_t ka0[C::NK], ka1[C::NK];
        lds_words<C::NK>(r0, ka0);
        lds_words<C::NK>(r0 + 8 * RS, ka1);
#pragma unroll
        for (int k = 0; k < C::KS; ++k)
            mma_bf16(s[0], s[1], s[2], s[3], ka0[2 * k], ka1[2 * k], ka0[2 * k + 1], ka1[2 * k + 1],
                     qb[k][0], qb[k][1]);
        return;
    }
    uint32_t b7[C::NK];
#pragma unroll
    for (int p = 0; p < C::NK; ++p) b7[p] = b7r[p];
    if (!C::B7REG) load_b7k<D>(tv.k_base, b7);
    if (!C::SPLIT) {
        uint32_t ka0[C::NK], ka1[C::NK];
        KRow<D, MODE> w0, w1;
        w0.load(r0, q0, gi < tv.rows);
        w1.load(r0 + 8 * RS, q0 + 8 * CS, gi + 8 < tv.rows);
        w0.merge_into(b7, ka0);
        w1.merge_into(b7, ka1);
        if (__ballot_sync(FULL, w0.cnt != 0u) != 0u) esc_k_half<D, MODE>(ka0, w0, tv.k_scr, es, status, lane);
        if (__ballot_sync(FULL, w1.cnt != 0u) != 0u) esc_k_half<D, MODE>(ka1, w1, tv.k_scr, es, status, lane);
#pragma unroll
        for (int k = 0; k < C::KS; ++k)
            mma_bf16(s[0], s[1], s[2], s[3], ka0[2 * k], ka1[2 * k], ka0[2 * k + 1], ka1[2 * k + 1],
                     qb[k][0], qb[k][1]);
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t ka[C::NK];
            KRow<D, MODE> w;
            w.load(r0 + 8 * h * RS, q0 + 8 * h * CS, gi + 8 * h < tv.rows);
            w.merge_into(b7, ka);
            if (__ballot_sync(FULL, w.cnt != 0u) != 0u) esc_k_half<D, MODE>(ka, w, tv.k_scr, es, status, lane);
#pragma unroll
            for (int k = 0; k < C::KS; ++k) {
                if (h == 0)
                    mma_bf16(s[0], s[1], s[2], s[3], ka[2 * k], 0u, ka[2 * k + 1], 0u, qb[k][0], qb[k][1]);
                else
                    mma_bf16(s[0], s[1], s[2], s[3], 0u, ka[2 * k], 0u, ka[2 * k + 1], qb[k][0], qb[k][1]);
            }
        }
    }
}

// Raw V token pair (tokens 2t + 8h, 2t + 8h + 1) of this lane.
template <int D>
__device__ __forceinline__ void v_raw(const uint8_t *r0, int RS, uint32_t (&o)[Cfg<D>::DV]) {
    uint32_t RA[Cfg<D>::DV / 2], RB[Cfg<D>::DV / 2];
    lds_words<Cfg<D>::DV / 2>(r0, RA);
    lds_words<Cfg<D>::DV / 2>(r0 + RS, RB);
#pragma unroll
    for (int e = 0; e < Cfg<D>::DV; ++e) o[e] = prmt(RA[e >> 1], RB[e >> 1], (e & 1) ? 0x7632u : 0x5410u);
}

// Zero the halves of tokens past the sub-tile's valid rows (P is 0 there, V must be finite).
template <int D>
__device__ __forceinline__ void v_tail(int t, int rows, uint32_t (&va)[Cfg<D>::DV]) {
    const uint32_t keep = (t < rows ? 0x0000FFFFu : 0u) | (t + 1 < rows ? 0xFFFF0000u : 0u);
#pragma unroll
    for (int e = 0; e < Cfg<D>::DV; ++e) va[e] &= keep;
}

// O^T += V^T P^T for the tile (P^T as B fragments: bh = bf16 part, bm = residual part).
template <int D, int MODE>
__device__ __forceinline__ void pv_tile(const TileView &tv, const uint32_t (&b7r)[Cfg<D>::DV],
                                        const uint32_t (&bh)[2], const uint32_t (&bm)[2], Esc &es,
                                        int *status, int lane, float (&acc)[Cfg<D>::KS][4]) {
    using C = Cfg<D>;
    const int gi = lane >> 2, tig = lane & 3;
    constexpr int RS = MODE == 0 ? 2 * D : D;
    constexpr int CS = D * MODE / 8;
    const int v0 = gi * C::DV;
    const int t = 2 * tig;
    const uint8_t *r0 = tv.v_rows + t * RS + (MODE == 0 ? 2 * v0 : v0);
    const uint8_t *q0 = tv.v_codes + t * CS + v0 * MODE / 8;
    uint32_t b7[C::DV];
#pragma unroll
    for (int e = 0; e < C::DV; ++e) b7[e] = b7r[e];
    if (!C::B7REG && MODE != 0) load_b7v<D>(tv.v_base, b7);
    if (!C::SPLIT) {
        uint32_t va0[C::DV], va1[C::DV];
        if (MODE == 0) {
            v_raw<D>(r0, RS, va0);
            v_raw<D>(r0 + 8 * RS, RS, va1);
        } else {
            VPair<D, MODE> p0, p1;
            p0.load(r0, r0 + RS, q0, q0 + CS, t < tv.rows, t + 1 < tv.rows);
            p1.load(r0 + 8 * RS, r0 + 9 * RS, q0 + 8 * CS, q0 + 9 * CS, t + 8 < tv.rows,
                    t + 9 < tv.rows);
            p0.merge_into(b7, va0);
            p1.merge_into(b7, va1);
            if (__ballot_sync(FULL, (p0.ca | p0.cb) != 0u) != 0u)
                esc_v_half<D, MODE>(va0, p0, tv.v_scr, es, status, lane);
            if (__ballot_sync(FULL, (p1.ca | p1.cb) != 0u) != 0u)
                esc_v_half<D, MODE>(va1, p1, tv.v_scr, es, status, lane);
        }
        if (tv.rows < TT) {
            v_tail<D>(t, tv.rows, va0);
            v_tail<D>(t + 8, tv.rows, va1);
        }
#pragma unroll
        for (int m = 0; m < C::KS; ++m) {
            mma_bf16(acc[m][0], acc[m][1], acc[m][2], acc[m][3], va0[2 * m], va0[2 * m + 1],
                     va1[2 * m], va1[2 * m + 1], bh[0], bh[1]);
            mma_bf16(acc[m][0], acc[m][1], acc[m][2], acc[m][3], va0[2 * m], va0[2 * m + 1],
                     va1[2 * m], va1[2 * m + 1], bm[0], bm[1]);
        }
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t va[C::DV];
            if (MODE == 0) {
                v_raw<D>(r0 + 8 * h * RS, RS, va);
            } else {
                VPair<D, MODE> p;
                p.load(r0 + 8 * h * RS, r0 + (8 * h + 1) * RS, q0 + 8 * h * CS, q0 + (8 * h + 1) * CS,
                       t + 8 * h < tv.rows, t + 8 * h + 1 < tv.rows);
                p.merge_into(b7, va);
                if (__ballot_sync(FULL, (p.ca | p.cb) != 0u) != 0u)
                    esc_v_half<D, MODE>(va, p, tv.v_scr, es, status, lane);
            }
            if (tv.rows < TT) v_tail<D>(t + 8 * h, tv.rows, va);
#pragma unroll
            for (int m = 0; m < C::KS; ++m) {
                const uint32_t x0 = h == 0 ? va[2 * m] : 0u, x1 = h == 0 ? va[2 * m + 1] : 0u;
                const uint32_t x2 = h == 0 ? 0u : va[2 * m], x3 = h == 0 ? 0u : va[2 * m + 1];
                mma_bf16(acc[m][0], acc[m][1], acc[m][2], acc[m][3], x0, x1, x2, x3, bh[0], bh[1]);
                mma_bf16(acc[m][0], acc[m][1], acc[m][2], acc[m][3], x0, x1, x2, x3, bm[0], bm[1]);
            }
        }
    }
}

// Q B fragments: qb[k][0] = Q[g][t D/4 + 4k + {0,1}], qb[k][1] = Q[g][t D/4 + 4k + {2,3}] -- the
// head-dim order of the K fragments.
template <int D>
__device__ __forceinline__ void load_q(const uint16_t *q, int n_q, int stride,
                                       uint32_t (&qb)[Cfg<D>::KS][2], int lane) {
    const int gi = lane >> 2, tig = lane & 3;
    const uint32_t *row =
        reinterpret_cast<const uint32_t *>(q + size_t(gi < n_q ? gi : 0) * stride + tig * Cfg<D>::DK);
#pragma unroll
    for (int k = 0; k < Cfg<D>::KS; ++k) {
        qb[k][0] = gi < n_q ? __ldg(row + 2 * k) : 0u;
        qb[k][1] = gi < n_q ? __ldg(row + 2 * k + 1) : 0u;
    }
}

// ---- the worker -------------------------------------------------------------------------------

// Walks the worker's flat blocks with one block of prefetch (flat indices fit 32 bits: the plan
// refuses larger steps).
struct Walker {
    int fb, fb1;
    FlatBlock cur, nxt;
    int unit, nunit;
    __device__ __forceinline__ void init(const AttnArgs &a, int b0, int b1) {
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
    __device__ __forceinline__ void next(const AttnArgs &a) {
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

// Tokens per ring stage for a block: TSC when both tensors are coded, TT when either is raw.
template <int D, bool BF16IN>
__device__ __forceinline__ int stage_tokens(int km, int vm) {
    return (BF16IN || km == 0 || vm == 0) ? TT : Cfg<D>::TSC;
}

// Copy side of the worker's ring.
template <int D, bool BF16IN> struct Producer {
    using C = Cfg<D>;
    Walker w;
    int tile = 0, stage = 0, bseq = 0;
    const uint8_t *kr = nullptr, *vr = nullptr;  // row sections of the current block
    int km = 0, vm = 0, st = TT;

    __device__ __forceinline__ static void tensor(uint8_t *dst, const uint8_t *rows, int mode,
                                                  int n_tok, int t0, int n, int lane) {
        if (BF16IN || mode == 0) {
            copy_piece<TT * 2 * D + 16>(
                dst, make_piece(rows + size_t(t0) * (2 * D), uint32_t(n * 2 * D)), lane);
        } else {
            copy_piece<C::TSC * D + 16>(dst, make_piece(rows + size_t(t0) * D, uint32_t(n * D)), lane);
            const uint8_t *codes = rows + size_t(n_tok) * D;
            copy_piece<C::TSC * D / 2 + 16>(
                dst + C::CODE_OFF,
                make_piece(codes + size_t(t0) * D * mode / 8, uint32_t(n * D * mode / 8)), lane);
        }
    }
    __device__ __forceinline__ static void meta(uint8_t *base, uint8_t *escs, const Sections &s,
                                                int nesc, int lane) {
        copy_piece<D + 32>(base, make_piece(s.rows - D, D), lane);
        const Piece e = make_piece(s.esc, uint32_t(2 * nesc));
        if (esc_staged<D>(e, nesc)) copy_piece<C::ESCB>(escs, e, lane);
    }

    // Issue stages while a ring slot is free; a block start waits until the consumer is at most
    // one block behind, so a meta slot is never overwritten while in use.
    __device__ __forceinline__ void produce(const AttnArgs &a, uint8_t *ring, uint8_t *metas,
                                            int c_stage, int c_fb, int lane) {
        while (w.fb < w.fb1 && stage - c_stage < C::NSTAGE) {
            if (tile == 0 && w.fb - c_fb >= 2) break;
            const FlatBlock &f = w.cur;
            if (tile == 0) {
                km = BF16IN ? 0 : f.k_mode;
                vm = BF16IN ? 0 : f.v_mode;
                st = stage_tokens<D, BF16IN>(km, vm);
                const Sections sk = sections<D, BF16IN>(a.units[w.unit].k, f.k_off, km, f.n_tok);
                const Sections sv = sections<D, BF16IN>(a.units[w.unit].v, f.v_off, vm, f.n_tok);
                kr = sk.rows;
                vr = sv.rows;
                if (!BF16IN) {
                    uint8_t *ms = metas + (bseq & 1) * C::MSLOT;
                    if (km != 0) meta(ms + C::M_K, ms + C::M_EK, sk, f.k_nesc, lane);
                    if (vm != 0) meta(ms + C::M_V, ms + C::M_EV, sv, f.v_nesc, lane);
                }
            }
            const int t0 = tile * st;
            const int n = min(st, int(f.valid) - t0);
            uint8_t *slot = ring + (stage % C::NSTAGE) * C::SLOT;
            tensor(slot, kr, km, f.n_tok, t0, n, lane);
            tensor(slot + C::TR, vr, vm, f.n_tok, t0, n, lane);
            cp_async_commit();
            ++stage;
            if (t0 + st >= int(f.valid)) {
                tile = 0;
                ++bseq;
                w.next(a);
            } else {
                ++tile;
            }
        }
    }
};

template <int D, bool BF16IN>
__device__ __forceinline__ void worker(const AttnArgs &a, uint8_t *R, int wk, int fb0, int fb1,
                                       int lane) {
    using C = Cfg<D>;
    const int gi = lane >> 2, tig = lane & 3;
    uint8_t *ring = R;
    uint8_t *metas = R + C::W_META;
    Producer<D, BF16IN> pp;
    pp.w.init(a, fb0, fb1);
    Walker cw;
    cw.init(a, fb0, fb1);
    int tile = 0, stage = 0, bseq = 0;
    int ubeg = 0, uend = 0, seg_begin = fb0;  // the current unit's flat block range
    int kmode = 0, vmode = 0, st = TT;
    uint32_t kd = 0, vd = 0;  // source alignment of the block's row sections
    Esc ek{0, 0, nullptr, nullptr}, ev{0, 0, nullptr, nullptr};
    uint32_t b7k[C::NK], b7v[C::DV];
#pragma unroll
    for (int p = 0; p < C::NK; ++p) b7k[p] = 0u;
#pragma unroll
    for (int e = 0; e < C::DV; ++e) b7v[e] = 0u;
    uint32_t qb[C::KS][2];
    float acc[C::KS][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    while (cw.fb < fb1) {
        pp.produce(a, ring, metas, stage, cw.fb, lane);
        cp_async_wait(pp.stage - stage - 1);
        __syncwarp();
        const FlatBlock f = cw.cur;
        const uint8_t *ms = metas + (bseq & 1) * C::MSLOT;
        if (tile == 0) {
            const UnitDev *U = a.units + cw.unit;
            ubeg = int(U->block_begin);
            uend = ubeg + U->n_blocks;
            kmode = BF16IN ? 0 : f.k_mode;
            vmode = BF16IN ? 0 : f.v_mode;
            st = stage_tokens<D, BF16IN>(kmode, vmode);
            const Sections sk = sections<D, BF16IN>(U->k, f.k_off, kmode, f.n_tok);
            const Sections sv = sections<D, BF16IN>(U->v, f.v_off, vmode, f.n_tok);
            kd = uint32_t(reinterpret_cast<uintptr_t>(sk.rows) & 15u);
            vd = uint32_t(reinterpret_cast<uintptr_t>(sv.rows) & 15u);
            if (kmode != 0) {
                if (C::B7REG) load_b7k<D>(ms + C::M_K + kd + tig * C::DK, b7k);
                const Piece e = make_piece(sk.esc, uint32_t(2 * f.k_nesc));
                ek.run = 0;
                ek.n = f.k_nesc;
                ek.gm = reinterpret_cast<const unsigned short *>(sk.esc);
                ek.sm = esc_staged<D>(e, f.k_nesc) ? ms + C::M_EK + e.data : nullptr;
            }
            if (vmode != 0) {
                if (C::B7REG) load_b7v<D>(ms + C::M_V + vd + gi * C::DV, b7v);
                const Piece e = make_piece(sv.esc, uint32_t(2 * f.v_nesc));
                ev.run = 0;
                ev.n = f.v_nesc;
                ev.gm = reinterpret_cast<const unsigned short *>(sv.esc);
                ev.sm = esc_staged<D>(e, f.v_nesc) ? ms + C::M_EV + e.data : nullptr;
            }
            if (cw.fb == seg_begin) {
                load_q<D>(U->q, U->n_q, U->q_stride, qb, lane);
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
#pragma unroll
                for (int m = 0; m < C::KS; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
            }
        }
        const uint8_t *slot = ring + (stage % C::NSTAGE) * C::SLOT;
        const int t0 = tile * st;
        const int rows_stage = min(st, int(f.valid) - t0);
        const bool last_tile = t0 + st >= int(f.valid);
        const bool seg_end = last_tile && (cw.fb + 1 == fb1 || cw.fb + 1 == uend);

#pragma unroll 1
        for (int sub = 0; sub < C::SUBS; ++sub) {
            if (sub * TT >= rows_stage) break;
            TileView tv;
            tv.rows = min(TT, rows_stage - sub * TT);
            tv.k_rows = slot + kd + sub * TT * (kmode == 0 ? 2 * D : D);
            tv.k_codes = slot + C::CODE_OFF + kd + sub * TT * (D * kmode / 8);
            tv.v_rows = slot + C::TR + vd + sub * TT * (vmode == 0 ? 2 * D : D);
            tv.v_codes = slot + C::TR + C::CODE_OFF + vd + sub * TT * (D * vmode / 8);
            tv.k_base = ms + C::M_K + kd + tig * C::DK;
            tv.v_base = ms + C::M_V + vd + gi * C::DV;
            tv.k_scr = C::SPLIT ? R + C::W_SCR : const_cast<uint8_t *>(slot) + sub * TT * D;
            tv.v_scr = C::SPLIT ? R + C::W_SCR : const_cast<uint8_t *>(slot) + C::TR + sub * TT * D;

            // S^T = K Q^T
            float s[4];
            if (kmode == 4) qk_tile<D, 4>(tv, b7k, qb, ek, a.status, lane, s);
            else if (kmode == 2) qk_tile<D, 2>(tv, b7k, qb, ek, a.status, lane, s);
            else qk_tile<D, 0>(tv, b7k, qb, ek, a.status, lane, s);
            if (gi >= tv.rows) s[0] = s[1] = -INFINITY;
            if (gi + 8 >= tv.rows) s[2] = s[3] = -INFINITY;

            // online softmax over the sub-tile's tokens; p = 2^(s log2e - m log2e)
            float t0m = fmaxf(s[0], s[2]), t1m = fmaxf(s[1], s[3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                t0m = fmaxf(t0m, __shfl_xor_sync(FULL, t0m, o));
                t1m = fmaxf(t1m, __shfl_xor_sync(FULL, t1m, o));
            }
            const float mn0 = fmaxf(m0, t0m), mn1 = fmaxf(m1, t1m);
            const float ml0 = __fmul_rn(mn0, kLog2e), ml1 = __fmul_rn(mn1, kLog2e);
            const float al0 = ex2(__fmaf_rn(m0, kLog2e, -ml0)), al1 = ex2(__fmaf_rn(m1, kLog2e, -ml1));
            const float p0 = ex2(__fmaf_rn(s[0], kLog2e, -ml0)), p1 = ex2(__fmaf_rn(s[1], kLog2e, -ml1));
            const float p2 = ex2(__fmaf_rn(s[2], kLog2e, -ml0)), p3 = ex2(__fmaf_rn(s[3], kLog2e, -ml1));
            l0 = __fmaf_rn(l0, al0, __fadd_rn(p0, p2));
            l1 = __fmaf_rn(l1, al1, __fadd_rn(p1, p3));
            m0 = mn0;
            m1 = mn1;

            // P^T B fragments: bf16(p) and bf16(p - bf16(p))
            uint32_t bh[2], bm[2];
            {
                const uint32_t h01 = pack_bf16x2(p1, p0), h23 = pack_bf16x2(p3, p2);
                const float r0 = __fsub_rn(p0, bf16lo_to_f32(h01)), r1 = __fsub_rn(p1, bf16hi_to_f32(h01));
                const float r2 = __fsub_rn(p2, bf16lo_to_f32(h23)), r3 = __fsub_rn(p3, bf16hi_to_f32(h23));
                bh[0] = movm_t(h01);
                bh[1] = movm_t(h23);
                bm[0] = movm_t(pack_bf16x2(r1, r0));
                bm[1] = movm_t(pack_bf16x2(r3, r2));
            }
            if (__any_sync(FULL, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
                for (int m = 0; m < C::KS; ++m) {
                    acc[m][0] = __fmul_rn(acc[m][0], al0);
                    acc[m][1] = __fmul_rn(acc[m][1], al1);
                    acc[m][2] = __fmul_rn(acc[m][2], al0);
                    acc[m][3] = __fmul_rn(acc[m][3], al1);
                }
            }
            // O^T += V^T P^T
            if (vmode == 4) pv_tile<D, 4>(tv, b7v, bh, bm, ev, a.status, lane, acc);
            else if (vmode == 2) pv_tile<D, 2>(tv, b7v, bh, bm, ev, a.status, lane, acc);
            else pv_tile<D, 0>(tv, b7v, bh, bm, ev, a.status, lane, acc);
        }

        if (seg_end) {
            float lt0 = l0, lt1 = l1;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                lt0 = __fadd_rn(lt0, __shfl_xor_sync(FULL, lt0, o));
                lt1 = __fadd_rn(lt1, __shfl_xor_sync(FULL, lt1, o));
            }
            const int qa = 2 * tig, qc = 2 * tig + 1;
            const int d0 = gi * C::DV;
            if (seg_begin == ubeg && cw.fb + 1 == uend) {
                const UnitDev *U = a.units + cw.unit;
                const int n_q = U->n_q, stride = U->q_stride;
                float *out = U->out;
                float *lse = U->lse;
                const float inv0 = __frcp_rn(lt0), inv1 = __frcp_rn(lt1);
                if (lse != nullptr && gi == 0) {
                    if (qa < n_q) lse[qa] = m0 + logf(lt0);
                    if (qc < n_q) lse[qc] = m1 + logf(lt1);
                }
                if (qa < n_q) {
                    float *o = out + size_t(qa) * stride + d0;
#pragma unroll
                    for (int m = 0; m < C::KS; ++m)
                        *reinterpret_cast<float2 *>(o + 2 * m) =
                            make_float2(__fmul_rn(acc[m][0], inv0), __fmul_rn(acc[m][2], inv0));
                }
                if (qc < n_q) {
                    float *o = out + size_t(qc) * stride + d0;
#pragma unroll
                    for (int m = 0; m < C::KS; ++m)
                        *reinterpret_cast<float2 *>(o + 2 * m) =
                            make_float2(__fmul_rn(acc[m][1], inv1), __fmul_rn(acc[m][3], inv1));
                }
            } else {
                const int ps = (seg_begin == fb0) ? 0 : 1;
                float *part = a.partials + (size_t(wk) * 2 + ps) * partial_stride(D);
                if (gi == 0) {
                    part[qa] = m0;
                    part[qc] = m1;
                    part[8 + qa] = lt0;
                    part[8 + qc] = lt1;
                }
                float *oa = part + 16 + qa * D + d0;
                float *oc = part + 16 + qc * D + d0;
#pragma unroll
                for (int m = 0; m < C::KS; ++m) {
                    *reinterpret_cast<float2 *>(oa + 2 * m) = make_float2(acc[m][0], acc[m][2]);
                    *reinterpret_cast<float2 *>(oc + 2 * m) = make_float2(acc[m][1], acc[m][3]);
                }
            }
        }
        __syncwarp();  // every lane is done with this ring slot before it is refilled
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
}

template <int D, bool BF16IN>
__global__ void __launch_bounds__(32 * Cfg<D>::WARPS, 1) attn_kernel(const AttnArgs a) {
    using C = Cfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // consecutive workers on different SMs: neighbouring ranges often share a cost profile
    const int wk = warp * gridDim.x + blockIdx.x;
    if (wk >= a.n_workers) return;
    const int fb0 = int(a.range_begin[wk]), fb1 = int(a.range_begin[wk + 1]);
    if (fb0 >= fb1) return;
    worker<D, BF16IN>(a, smem + warp * C::WARP_BYTES, wk, fb0, fb1, lane);
}

// ---- combine ------------------------------------------------------------------------------------

// Combine the partial states of one query of a split unit: with M = max m_t over the unit's
// segments, l = sum l_t e^(m_t - M) and acc = sum acc_t e^(m_t - M) (merge_state's arithmetic,
// src/softmax.hpp:16-30, applied to all segments at once instead of a left fold), then
// out = acc * (1 / l) like finalize_state (src/softmax.hpp:32-41).  One CTA per (unit, query);
// the sums run over fixed slices of the segments, so the result is deterministic.
constexpr int kCombineThreads = 256;
constexpr int kMaxSegments = 4096;

template <int D>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const CombineArgs a) {
    constexpr int S = kCombineThreads / D;  // segment slices summed in parallel
    __shared__ float e[kMaxSegments];
    __shared__ float red[kCombineThreads];
    const int u = a.split_units[blockIdx.x];
    const int g = blockIdx.y;
    const UnitDev unit = a.units[u];
    if (g >= unit.n_q) return;
    const int t0 = worker_of_block(a.range_begin, a.n_workers, unit.block_begin);
    const int t1 = worker_of_block(a.range_begin, a.n_workers, unit.block_begin + unit.n_blocks - 1);
    const int nt = min(t1 - t0 + 1, kMaxSegments);
    const int ps = partial_stride(D);
    auto part = [&](int i) {
        const int t = t0 + i;
        const int slot = (a.range_begin[t] >= unit.block_begin) ? 0 : 1;
        return a.partials + (size_t(t) * 2 + slot) * ps;
    };
    const int tid = threadIdx.x;
    float mx = -INFINITY;
    for (int i = tid; i < nt; i += kCombineThreads) {
        const float m = part(i)[g];
        e[i] = m;
        mx = fmaxf(mx, m);
    }
    red[tid] = mx;
    __syncthreads();
    for (int o = kCombineThreads / 2; o > 0; o >>= 1) {
        if (tid < o) red[tid] = fmaxf(red[tid], red[tid + o]);
        __syncthreads();
    }
    const float M = red[0];
    __syncthreads();
    float ls = 0.f;
    for (int i = tid; i < nt; i += kCombineThreads) {
        const float w = expf(e[i] - M);
        e[i] = w;
        ls = __fmaf_rn(part(i)[8 + g], w, ls);
    }
    red[tid] = ls;
    __syncthreads();
    for (int o = kCombineThreads / 2; o > 0; o >>= 1) {
        if (tid < o) red[tid] = __fadd_rn(red[tid], red[tid + o]);
        __syncthreads();
    }
    const float lsum = red[0];
    const float inv = __frcp_rn(lsum);
    __syncthreads();
    const int d = tid % D, sl = tid / D;
    float acc = 0.f;
    if (sl < S)
        for (int i = sl; i < nt; i += S) acc = __fmaf_rn(part(i)[16 + g * D + d], e[i], acc);
    red[tid] = acc;
    __syncthreads();
    if (sl == 0) {
        float v = red[d];
        for (int j = 1; j < S; ++j) v = __fadd_rn(v, red[j * D + d]);
        unit.out[size_t(g) * unit.q_stride + d] = __fmul_rn(v, inv);
    }
    if (tid == 0 && unit.lse != nullptr) unit.lse[g] = M + logf(lsum);
}

// ---- worker ranges -----------------------------------------------------------------------------

// Cost of one flat block for the worker split: 8 per attended token plus kEscCost per escape word
// (a worker's time grows with its tokens and, on escape-dense blocks, with its escape words).
#ifndef KVX_ESC_COST
#define KVX_ESC_COST 4
#endif
constexpr uint32_t kEscCost = KVX_ESC_COST;
__device__ __forceinline__ uint64_t block_cost(const FlatBlock &b) {
    return 8ull * b.valid + kEscCost * (uint64_t(b.k_nesc) + b.v_nesc);
}

// One CTA: range_begin[w] = first block whose cost prefix reaches w * total / n_workers.
__global__ void __launch_bounds__(1024) split_kernel(const FlatBlock *flat, int64_t n, int nw,
                                                     int64_t *range_begin) {
    __shared__ unsigned long long part[1024];
    const int t = threadIdx.x, T = blockDim.x;
    const int64_t chunk = (n + T - 1) / T;
    const int64_t lo = min(n, t * chunk), hi = min(n, lo + chunk);
    unsigned long long sum = 0;
    for (int64_t b = lo; b < hi; ++b) sum += block_cost(load_flat(flat, b));
    part[t] = sum;
    __syncthreads();
    for (int o = 1; o < T; o <<= 1) {  // inclusive scan
        const unsigned long long v = t >= o ? part[t - o] : 0ull;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    const unsigned long long total = part[T - 1];
    unsigned long long c = part[t] - sum;  // cost before block lo
    if (t == 0) {
        range_begin[0] = 0;
        range_begin[nw] = n;
        for (int w0 = 1; w0 < nw && uint64_t(w0) * total / nw == 0; ++w0) range_begin[w0] = 0;
    }
    // worker w starts after the block whose cost interval (c, c + cost] holds w * total / nw
    int w = int(c * uint64_t(nw) / (total ? total : 1));
    for (int64_t b = lo; b < hi; ++b) {
        const unsigned long long cn = c + block_cost(load_flat(flat, b));
        while (w < nw && uint64_t(w) * total / nw <= c) ++w;
        while (w < nw && uint64_t(w) * total / nw <= cn) range_begin[w++] = b + 1;
        c = cn;
    }
    if (t == 0 && total == 0)
        for (int w2 = 1; w2 < nw; ++w2) range_begin[w2] = n;
}

template <int D> void configure(bool bf16) {
    static bool done[2] = {false, false};
    if (done[bf16]) return;
    if (bf16)
        cudaFuncSetAttribute(attn_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::WARP_BYTES * Cfg<D>::WARPS);
    else
        cudaFuncSetAttribute(attn_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::WARP_BYTES * Cfg<D>::WARPS);
    done[bf16] = true;
}

template <int D>
cudaError_t launch_d(bool bf16, const AttnArgs &a, int grid, cudaStream_t s) {
    configure<D>(bf16);
    const int threads = 32 * Cfg<D>::WARPS;
    const size_t sm = size_t(Cfg<D>::WARP_BYTES) * Cfg<D>::WARPS;
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

int attention_workers_per_cta(int dim) {
    switch (dim) {
    case 32: return Cfg<32>::WARPS;
    case 64: return Cfg<64>::WARPS;
    case 128: return Cfg<128>::WARPS;
    case 256: return Cfg<256>::WARPS;
    default: return 0;
    }
}

size_t attention_smem_bytes(int dim) {
    switch (dim) {
    case 32: return size_t(Cfg<32>::WARP_BYTES) * Cfg<32>::WARPS;
    case 64: return size_t(Cfg<64>::WARP_BYTES) * Cfg<64>::WARPS;
    case 128: return size_t(Cfg<128>::WARP_BYTES) * Cfg<128>::WARPS;
    case 256: return size_t(Cfg<256>::WARP_BYTES) * Cfg<256>::WARPS;
    default: return 0;
    }
}

cudaError_t launch_attention(int dim, bool bf16_input, const AttnArgs &a, int grid, cudaStream_t s) {
    switch (dim) {
    case 32: return launch_d<32>(bf16_input, a, grid, s);
    case 64: return launch_d<64>(bf16_input, a, grid, s);
    case 128: return launch_d<128>(bf16_input, a, grid, s);
    case 256: return launch_d<256>(bf16_input, a, grid, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_split(const FlatBlock *flat, int64_t n_blocks, int n_workers, int64_t *range_begin,
                         cudaStream_t s) {
    split_kernel<<<1, 1024, 0, s>>>(flat, n_blocks, n_workers, range_begin);
    return cudaGetLastError();
}

cudaError_t launch_combine(int dim, const CombineArgs &a, int n_split, cudaStream_t s) {
    if (n_split <= 0) return cudaSuccess;
    const dim3 grid(n_split, 8);  // (split unit, query); units hold at most 8 queries
    switch (dim) {
    case 32: combine_kernel<32><<<grid, kCombineThreads, 0, s>>>(a); break;
    case 64: combine_kernel<64><<<grid, kCombineThreads, 0, s>>>(a); break;
    case 128: combine_kernel<128><<<grid, kCombineThreads, 0, s>>>(a); break;
    case 256: combine_kernel<256><<<grid, kCombineThreads, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace kvx
