// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened and cut into one cost-balanced range per CTA
//    (one CTA per SM).  A CTA streams its blocks through a shared-memory ring of stages; a stage
//    is up to TSB tokens of one block: the block's descriptor, and per tensor its base exponents,
//    sign/mantissa rows, packed residual codes and the escape-record entries of those tokens (or
//    raw BF16 rows).  One producer warp issues each stage from its copy list (built once per plan
//    by stage_table_kernel): lanes 0-7 each issue one 1-D bulk copy of the TMA engine, completing
//    on the slot's "full" mbarrier.  Only the compressed bytes cross HBM (plus, for a coded block
//    with escapes, its escape record: 4 bytes per escape word and a 64-byte count header, built
//    once per plan).  Steps whose blocks are all coded use a 6-slot ring sized for coded stages,
//    others a 4-slot ring that also takes raw rows.
//  * The consumer warps (15 at D <= 64, 11 at D = 128, 7 at D = 256) share every stage: the
//    stage's 16-token tiles go to them in groups, round-robin (group j of the CTA to warp j mod
//    NW), each warp keeping its own online-softmax state.  A warp rebuilds its tiles' K rows into
//    BF16 words in its private tiles (16 rows of D BF16 values, 16-byte chunks swizzled so that
//    neither the decode stores nor the ldmatrix reads conflict on banks): per pair of elements two
//    byte permutes, one multiply-add that adds the residual to the base exponent, and one
//    bit-select.  Escape words are stored over their elements, one 16-bit store each, at the tile
//    byte the escape record gives.
//  * S = K Q^T on the tensor cores (mma.sync m16n8k16, tokens x queries, fp32 accumulate), the
//    online softmax on the S fragment (lane (g, t) holds queries 2t and 2t+1, which are also the
//    output columns it accumulates), then the tile's V rows replace K in the tile and
//    O^T += V^T P^T reads V^T with ldmatrix.trans; P^T enters as three bf16 terms (all 24 bits of
//    the fp32 weight).  Each warp arrives on the slot's "empty" mbarrier once it has read the
//    stage, which frees the slot for the producer when every consumer warp has.
//  * At the end of each unit segment of the CTA's range every consumer warp writes its (m, l,
//    acc) state; combine_kernel folds a unit's states with merge_state semantics
//    (src/softmax.hpp:16-30) and finalizes like finalize_state (src/softmax.hpp:32-41:
//    reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template reading [seq, dim] BF16 rows into the same
// tile; for the same blocks and CTA ranges it produces bit-identical outputs to the XKV variant,
// because the tensor cores see identical BF16 tiles and everything after them is the same code.
// (The drop-in single-head entry point cuts both inputs into CTA ranges by token counts alone, so
// the ranges always agree there.)

#include "attention.cuh"

namespace kvx {
namespace {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int TT = kTileTokens;  // tokens per MMA tile (one m16 block of the QK MMA)
constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the SFU (ex2.approx.ftz.f32: one instruction; results below 2^-126, softmax weights
// under 1e-38 of the largest, flush to zero).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__host__ __device__ constexpr int round16(int x) { return (x + 15) & ~15; }

// One verdict for the whole warp on a condition its lanes may see differently (a bounded wait that
// times out in some lanes just as the phase completes for others).
__device__ __forceinline__ bool uni(bool c) { return __all_sync(0xFFFFFFFFu, c); }


// Kernel geometry of head dim D.  CP: the compact ring, for steps whose blocks are all coded (6 slots
// sized for a coded stage: D bytes of sign/mantissa and at most D / 2 bytes of residual codes per
// token); otherwise 4 slots that also take raw BF16 rows (2 D bytes per token).  Only the ring's
// layout differs: the tiles, their order and the arithmetic are the same in both.
template <int D, bool CP = false> struct Cfg {
    static constexpr int KS = D / 16;             // k-steps of QK = M-tiles of PV
    static constexpr int C8 = D / 8;              // 8-element chunks per row
    static constexpr int NIT = TT * C8 / 32;      // chunk steps of a lane per tile and tensor
    static constexpr int TSB = attention_stage_tokens(D);  // tokens per ring stage
    static constexpr int TPS = TSB / TT;          // tiles per stage
    // Tiles a consumer warp takes together (one visit of a stage): two at D <= 64, where the
    // per-visit work (waits, descriptor fields, layout selectors, escape bounds, the softmax's
    // vote) is then shared by 32 tokens and the two tiles' chains interleave; one above, where the
    // registers are taken by the wider tiles.
    static constexpr int NT = D <= 64 ? 2 : 1;
    static constexpr int TPP = TPS / NT;          // tile groups (visits) per stage
    static constexpr int NW = attention_consumer_warps(D);  // consumer warps
    static constexpr int NSLOT = CP ? 6 : 4;      // ring slots
    // Escape-record entries of one tensor that a stage stages (12.5 % of its elements, or 256 in
    // the compact ring); a stage with more leaves them in HBM, where the consumers read them.
    static constexpr int ESC_CAP = CP ? 256 : TSB * D / 8;
    // One tensor's region of a slot: rows at 0 (raw: 2 D bytes per token; coded: D bytes, then the
    // residual codes at CODE_OFF), escape entries at E_OFF.  Every piece lands 0-15 bytes past its
    // 16-byte aligned start.
    static constexpr int R_BYTES = (CP ? TSB * D + TSB * D / 2 : 2 * TSB * D) + 32;
    static constexpr int CODE_OFF = TSB * D + 16;
    static constexpr int E_OFF = R_BYTES;
    static constexpr int T_BYTES = round16(E_OFF + 4 * ESC_CAP + 32);
    // A slot: the block descriptor (128 bytes), the block's merge words (K then V, 2 D bytes each),
    // the stage's escape words, then the K and V regions.
    static constexpr int S_B7 = 128;
    // Two words the producer writes for the stage: per tensor, the shared address (bit 0 set) from
    // which the stage's staged escape-record entry i is read at + 4 i, or 0 when they stay in HBM.
    static constexpr int S_INFO = S_B7 + 4 * D;
    static constexpr int S_T = S_INFO + 16;
    static constexpr int SLOT = S_T + 2 * T_BYTES;
    static constexpr int TILE1 = TT * 2 * D;      // one 16-token BF16 tile
    static constexpr int TILE = NT * TILE1;       // one consumer warp's NT tiles (K, then V)
    static constexpr int O_TILE = NSLOT * SLOT;
    static constexpr int O_BAR = O_TILE + NW * TILE;  // full[NSLOT], then empty[NSLOT]
    static constexpr int SMEM = O_BAR + 16 * NSLOT;
    static constexpr int NP = 1;                  // producer warps (stages go round-robin over them)
    static constexpr int THREADS = 32 * (NW + NP);
    static_assert(SMEM + 16 <= 232448, "stage ring and tiles exceed shared memory");
    static_assert(NW >= TPP, "a consumer warp takes at most one tile group of a stage");
    static_assert(TPS % NT == 0, "a stage holds whole tile groups");
    // Every use of a slot comes from the same producer warp (stage gs goes to warp gs mod NP), so
    // that warp has waited for the slot's previous use to be released before it waits for the
    // current one: with slots shared between the producers, a producer could test the slot's empty
    // barrier for a phase two uses back and pass one phase early.
    static_assert(NSLOT % NP == 0, "each ring slot is served by one producer warp");
    // A consumer warp's tile groups are NW groups apart, so its stages at most ceil(NW / TPP) apart.
    // Its wait for stage gs tests the slot's empty barrier for the release of stage gs - NSLOT by
    // parity, which is only sound while the barrier is at most one phase behind: stage gs - 2 NSLOT
    // must be released already.  It is when the warp's previous stage (issued, so every stage
    // before it was issued, each after its slot's previous release) is at least gs - NSLOT.
    static_assert((NW + TPP - 1) / TPP <= NSLOT, "a consumer warp's stages are at most NSLOT apart");
    static_assert(32 % C8 == 0 && NIT >= 1, "a warp step covers whole rows");
    static_assert((TSB * D) % 4096 == 0, "stage offsets keep every section's 16-byte alignment");
};

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

// Stages arrive through the TMA engine: one 1-D bulk copy per piece (16-byte aligned source,
// destination and size), each completing its byte count on the ring slot's mbarrier; the
// consumer waits on the barrier's phase for that use of the slot.

// Longest a warp waits for one stage before it reports DERR_TIMEOUT and stops (microseconds).
constexpr uint32_t kStageWaitUs = 1000000;


// ---- escape records ----------------------------------------------------------------------------


// e(i) of tensor T from a block descriptor's headers.
__device__ __forceinline__ int esc_ms(const BlockDesc &bd, int T, int i) {
    return i == 0 ? 0 : int(bd.em[T][i - 1]);
}

// Byte offset inside a 16-byte line of entry i of the escape record at `rec` (the record array is
// 16-byte aligned).
__device__ __forceinline__ uint32_t esc_rec_line(uint32_t rec, int i) {
    return (4u * (rec + uint32_t(kEscRecHead) + uint32_t(i))) & 15u;
}

// e(i) of tensor T from a block descriptor in global memory (the producer's copy).
__device__ __forceinline__ int esc_gd(const BlockDesc *gd, int T, int i) {
    return i == 0 ? 0 : int(__ldg(&gd->em[T][i - 1]));
}

// ---- decode helpers ----------------------------------------------------------------------------

__host__ __device__ constexpr uint32_t rep2(uint32_t b) {  // bytes b, b, b+1, b+1
    return b | (b << 4) | ((b + 1) << 8) | ((b + 1) << 12);
}
__host__ __device__ constexpr uint32_t shift4(uint32_t o) {  // bytes o .. o+3
    return o | ((o + 1) << 4) | ((o + 2) << 8) | ((o + 3) << 12);
}
__host__ __device__ constexpr uint32_t sel_code(int j) {  // byte j of A -> bytes 0, 1; of B -> 2, 3
    return uint32_t(j) | (uint32_t(j) << 4) | (uint32_t(4 + j) << 8) | (uint32_t(4 + j) << 12);
}

// Two BF16 values from sign/mantissa bytes (bytes 0 and 1 of each half hold the element's byte:
// bits 0-6 give the mantissa, bit 15 the sign) and exponent residuals in bytes 0 and 2 of cw.
// Exponent = base + residual modulo 256 like bf16_from_delta's uint8 sum (reference
// include/kvexp/bf16.hpp:35-37).  Bytes 1 and 3 of cw may hold other residuals (< 16): times 128
// they land in bits 15-18 of each half, which the select drops, and no carry reaches bit 23.
// The select is written as one LOP3 (mask 0x807F807F picks sg, its complement the sum).
__device__ __forceinline__ uint32_t merge(uint32_t sg, uint32_t cw, uint32_t b7) {
    uint32_t t, w;
    asm("mad.lo.u32 %0, %1, 128, %2;" : "=r"(t) : "r"(cw), "r"(b7));
    asm("lop3.b32 %0, %1, %2, 0x807F807F, 0xE4;" : "=r"(w) : "r"(sg), "r"(t));
    return w;
}

// How this lane reads one tensor of the current block from a ring stage: the 8-element chunk c8
// (head dims 8 c8 .. 8 c8 + 7) of rows t0 + RPI k.  The residual codes start in the 16-byte line at
// code_base (the codes' own copy, or right behind the rows when rows and codes came as one).  Row
// sections start m = 0 or 2 bytes past a 4-byte boundary of the ring; the chunk adds a multiple of
// 4 to the sign/mantissa and raw rows, and 4 (4-bit), 3 (3-bit) or 2 (2-bit) bytes per chunk to
// the residual rows.
struct Lay {
    uint32_t p0, p1;  // sign/mantissa bytes of element pairs 2q and 2q+1 from words q, q+1
    uint32_t w;       // one realigned word from two loaded ones (raw rows)
    uint32_t cs;      // one realigned word of residual codes
    uint32_t rows;    // byte offset of the lane's row window in the stage (4-aligned)
    uint32_t codes;   // byte offset of the lane's residual window in the stage (4-aligned)
};
// rd / cd: data offsets of the block's row and code pieces.
template <int D>
__device__ __forceinline__ Lay make_lay(uint32_t rd, uint32_t cd, int mode, int c8, bool bf16,
                                       uint32_t code_base) {
    // Every offset in a blob is even, so a section starts 0 or 2 bytes past a 4-byte boundary and
    // each selector is one of two constants.
    Lay l;
    const bool m2 = (rd & 2u) != 0u;
    l.p0 = m2 ? rep2(2) : rep2(0);
    l.p1 = m2 ? rep2(4) : rep2(2);
    l.w = m2 ? shift4(2) : shift4(0);
    l.rows = (rd & ~3u) + uint32_t((bf16 || mode == 0) ? 16 * c8 : 8 * c8);
    const uint32_t cb = (cd & 3u) + uint32_t(c8 * (mode == 0 ? 0 : mode));
    l.cs = shift4(0) + (cb & 3u) * 0x1111u;  // bytes o .. o + 3, o = cb mod 4 (odd only for 3-bit)
    l.codes = code_base + (cd & ~3u) + (cb & ~3u);
    return l;
}

// Byte offset of 16-byte chunk c8 of tile row t: rows of 2 D bytes, chunks XOR-swizzled by the
// row so that eight rows read at one chunk position (ldmatrix) and eight chunks of a row written
// by eight lanes (decode) fall on distinct banks.
template <int D> __device__ __forceinline__ uint32_t xb_off(int t, int c8) {
    return uint32_t(t * (2 * D)) + (uint32_t(c8 ^ (D == 32 ? (t >> 1) & 3 : t & 7)) << 4);
}

// ---- stage decode ------------------------------------------------------------------------------

// Tile addresses of this lane's chunks: chunk j of a stage (row r0 + RPI j, head dims 8 c8 ..
// 8 c8 + 7) is stored at st[j % NB] + j RPI 2 D.  The swizzle of row t depends on t mod 8 (D 32:
// on t / 2 mod 4), so NB bases cover every chunk; for D 256 (NB 8) the base is computed per chunk.
template <int D> struct StoreMap {
    static constexpr int RPI = 32 / Cfg<D>::C8;
    static constexpr int NB = D == 32 ? 1 : 8 / RPI;
    static constexpr int NR = NB <= 4 ? NB : 1;  // bases held in registers
    uint32_t st[NR];
    uint32_t row, c16;  // D 256: xb + r0 2 D and c8 << 4
    __device__ __forceinline__ void init(uint32_t xb, int lane) {
        const int c8 = lane % Cfg<D>::C8, r0 = lane / Cfg<D>::C8;
        row = xb + uint32_t(r0 * (2 * D));
        c16 = uint32_t(c8) << 4;
#pragma unroll
        for (int k = 0; k < NR; ++k) st[k] = xb + xb_off<D>(r0 + RPI * k, c8);
    }
    // j is a constant after unrolling
    __device__ __forceinline__ uint32_t at(int j) const {
        if constexpr (NB <= 4) return st[j % NB] + uint32_t((j / NB) * NB * RPI * 2 * D);
        else return row + uint32_t(j * RPI * 2 * D) + (c16 ^ uint32_t((j & 7) << 4));
    }
};

// Loads of chunk steps [K0, K0 + G) of one tensor's stage: row words W, residual code words X.
template <int D, int MODE, int G, int K0>
__device__ __forceinline__ void load_chunks(uint32_t qr, uint32_t qc, uint32_t (&W)[G][MODE == 0 ? 5 : 3],
                                            uint32_t (&X)[G][2]) {
    constexpr int RPI = 32 / Cfg<D>::C8;
    constexpr int RB = MODE == 0 ? 2 * D : D;  // row bytes
    constexpr int CB = D * MODE / 8;           // residual bytes per row
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const uint32_t q = qr + uint32_t((K0 + g) * RPI * RB);
#pragma unroll
        for (int i = 0; i < (MODE == 0 ? 5 : 3); ++i) W[g][i] = lds_u32(q + 4u * i);
        if constexpr (MODE != 0) {
            const uint32_t c = qc + uint32_t((K0 + g) * RPI * CB);
            X[g][0] = lds_u32(c);
            if constexpr (MODE >= 3) X[g][1] = lds_u32(c + 4u);
        }
    }
}

// The four BF16 pair words of one chunk from its loaded words.
template <int MODE>
__device__ __forceinline__ void build_chunk(const Lay &ly, const uint32_t (&b7)[4],
                                            const uint32_t (&W)[MODE == 0 ? 5 : 3], const uint32_t (&X)[2],
                                            uint32_t (&w)[4]) {
    if constexpr (MODE == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = prmt(W[i], W[i + 1], ly.w);
    } else {
        uint32_t c0, c1, c2, c3;
        if constexpr (MODE == 4) {
            const uint32_t x = prmt(X[0], X[1], ly.cs);
            const uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
            c0 = prmt(lo, hi, sel_code(0));
            c1 = prmt(lo, hi, sel_code(1));
            c2 = prmt(lo, hi, sel_code(2));
            c3 = prmt(lo, hi, sel_code(3));
        } else if constexpr (MODE == 3) {
            // 8 residuals of 3 bits in bits 0-23 of x (the library's 3-bit extension): pair j is
            // the 6 bits at 6 j; times 0x2001 puts its first residual at bit 0 and its second at
            // bit 16, and the mask keeps those
            const uint32_t x = prmt(X[0], X[1], ly.cs);
            c0 = ((x & 0x3Fu) * 0x2001u) & 0x70007u;
            c1 = (((x >> 6) & 0x3Fu) * 0x2001u) & 0x70007u;
            c2 = (((x >> 12) & 0x3Fu) * 0x2001u) & 0x70007u;
            c3 = (((x >> 18) & 0x3Fu) * 0x2001u) & 0x70007u;
        } else {  // 8 residuals of 2 bits in the low 16 bits of x
            const uint32_t x = prmt(X[0], 0u, ly.cs);
            const uint32_t ev = x & 0x3333u, od = (x >> 2) & 0x3333u;
            const uint32_t el = ev & 0x0F0Fu, eh = (ev >> 4) & 0x0F0Fu;
            const uint32_t ol = od & 0x0F0Fu, oh = (od >> 4) & 0x0F0Fu;
            c0 = prmt(el, ol, sel_code(0));
            c1 = prmt(eh, oh, sel_code(0));
            c2 = prmt(el, ol, sel_code(1));
            c3 = prmt(eh, oh, sel_code(1));
        }
        w[0] = merge(prmt(W[0], W[1], ly.p0), c0, b7[0]);
        w[1] = merge(prmt(W[0], W[1], ly.p1), c1, b7[1]);
        w[2] = merge(prmt(W[1], W[2], ly.p0), c2, b7[2]);
        w[3] = merge(prmt(W[1], W[2], ly.p1), c3, b7[3]);
    }
}

// Chunk steps [K0, NT NIT) in groups of G (the NT tiles' rows follow one another in the stage and
// in the warp's tile buffer, so step k of tile t is step t NIT + k): the loads of the next group
// are issued before the current group's arithmetic and stores (the shared-memory accesses keep
// their written order).
template <int D, int MODE, int G, int K0, int TO>
__device__ __forceinline__ void decode_groups(uint32_t qr, uint32_t qc, const Lay &ly, const uint32_t (&b7)[4],
                                              const StoreMap<D> &sm, uint32_t (&W)[G][MODE == 0 ? 5 : 3],
                                              uint32_t (&X)[G][2]) {
    constexpr int NIT = Cfg<D>::NT * Cfg<D>::NIT;
    uint32_t Wn[G][MODE == 0 ? 5 : 3], Xn[G][2];
    if constexpr (K0 + G < NIT) load_chunks<D, MODE, G, K0 + G>(qr, qc, Wn, Xn);
    uint32_t w[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) build_chunk<MODE>(ly, b7, W[g], X[g], w[g]);
#pragma unroll
    for (int g = 0; g < G; ++g) sts_v4(sm.at(K0 + g) + uint32_t(TO), w[g][0], w[g][1], w[g][2], w[g][3]);
    if constexpr (K0 + G < NIT) decode_groups<D, MODE, G, K0 + G, TO>(qr, qc, ly, b7, sm, Wn, Xn);
}

// Rebuild this lane's chunks of one tensor's NT 16-token tiles into the warp's BF16 tiles (MODE
// 4 / 3 / 2 coded, 0 raw BF16).  rb / cb: the first tile's rows / residual codes are at rb + ly.rows
// and cb + ly.codes (plus the lane's row).
template <int D, int MODE, int TO>
__device__ __forceinline__ void decode_tile(uint32_t rb, uint32_t cb, const Lay &ly, const uint32_t (&b7)[4],
                                            const StoreMap<D> &sm, int lane) {
    using C = Cfg<D>;
    // chunk steps per group (two groups' loads are live at a time)
    constexpr int G = C::NIT < 4 ? C::NIT : 4;
    const int r0 = lane / C::C8;
    const uint32_t qr = rb + ly.rows + uint32_t(r0 * (MODE == 0 ? 2 * D : D));
    const uint32_t qc = cb + ly.codes + uint32_t(r0 * (D * MODE / 8));
    uint32_t W[G][MODE == 0 ? 5 : 3], X[G][2];
    load_chunks<D, MODE, G, 0>(qr, qc, W, X);
    decode_groups<D, MODE, G, 0, TO>(qr, qc, ly, b7, sm, W, X);
}

// Zero this lane's chunks of tile rows at or past `from` (V rows past the block's valid tokens:
// P is 0 there and V must be finite).
template <int D, int TO, int J = 0>
__device__ __forceinline__ void zero_rows(const StoreMap<D> &sm, int from, int lane) {
    if constexpr (J < Cfg<D>::NT * Cfg<D>::NIT) {
        if (lane / Cfg<D>::C8 + J * StoreMap<D>::RPI >= from) sts_v4(sm.at(J) + uint32_t(TO), 0u, 0u, 0u, 0u);
        zero_rows<D, TO, J + 1>(sm, from, lane);
    }
}

// The escape-record entries where the second, third, ... of a warp's NT tiles begin: entry i belongs
// to tile tile(i).
template <int NT> struct EscBounds {
    int b[NT > 1 ? NT - 1 : 1];
    __device__ __forceinline__ int tile(int i) const {
        int k = 0;
#pragma unroll
        for (int j = 0; j + 1 < NT; ++j) k += i >= b[j] ? 1 : 0;
        return k;
    }
};

// Store escapes [e0, e1) of a block over their elements in the warp's NT tiles: record entry i
// (byte of the element in its 16-token tile | escape word << 16) is the u32 at ents + 4 i -- a
// shared address of the staged copy, or (HBM variant) the record in global memory; it belongs to
// tile k.  Elements in rows at or past `rows` (counted from the first tile's first row) are
// skipped; bytes are even.
__device__ __forceinline__ void esc_store(uint32_t xb, uint32_t e, int k, int rows, int tile_bytes,
                                          int row_bytes) {
    const int rt = rows - k * kTileTokens;
    if ((e & 0xFFFFu) < uint32_t(max(rt, 0)) * uint32_t(row_bytes))
        sts_u16(xb + uint32_t(k * tile_bytes) + (e & 0xFFFEu), e >> 16);
}
template <int D>
__device__ __forceinline__ void esc_patch(uint32_t xb, uint32_t ents, int e0, int e1,
                                          const EscBounds<Cfg<D>::NT> &eb, int rows, int lane) {
    for (int i = e0 + lane; i < e1; i += 32)
        esc_store(xb, lds_u32(ents + 4u * uint32_t(i)), eb.tile(i), rows, Cfg<D>::TILE1, 2 * D);
}
template <int D>
__device__ __noinline__ void esc_patch_hbm(uint32_t xb, const uint32_t *ents, int e0, int e1,
                                           const EscBounds<Cfg<D>::NT> eb, int rows, int lane) {
    for (int i = e0 + lane; i < e1; i += 32)
        esc_store(xb, __ldg(ents + i), eb.tile(i), rows, Cfg<D>::TILE1, 2 * D);
}

// ---- tiles on the tensor cores ------------------------------------------------------------------

// S^T fragment of the 16-token tile at tile row r0: s0/s1 token g (queries 2t, 2t+1), s2/s3
// token g + 8.  K A fragments by ldmatrix: lanes 8 i .. 8 i + 7 address matrix i (rows 0-7 / 8-15,
// head dims 0-7 / 8-15 of the k-step).
template <int D, int NT>
__device__ __forceinline__ void qk_tiles(uint32_t xb, const uint32_t (&qb)[Cfg<D>::KS][2], int lane,
                                         float (&s)[NT][4]) {
    // the NT tiles' MMA chains interleave (independent accumulators); ldmatrix runs ahead
    constexpr int KS = Cfg<D>::KS, G = KS < 2 ? KS : 2;
    const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
    const uint32_t base = xb + uint32_t(row * (2 * D));
    const int y = (lane >> 4) ^ (D == 32 ? (row >> 1) & 3 : row & 7);
#pragma unroll
    for (int t = 0; t < NT; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < KS; k0 += G) {
        uint32_t a[G][NT][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int t = 0; t < NT; ++t)
                ldsm_x4(base + uint32_t(t * TT * 2 * D) + (uint32_t((2 * (k0 + g)) ^ y) << 4),
                        a[g][t][0], a[g][t][1], a[g][t][2], a[g][t][3]);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int t = 0; t < NT; ++t)
                mma_bf16(s[t][0], s[t][1], s[t][2], s[t][3], a[g][t][0], a[g][t][1], a[g][t][2],
                         a[g][t][3], qb[k0 + g][0], qb[k0 + g][1]);
    }
}

// O^T += V^T P^T for the 16-token tile at tile row r0 (P^T as B fragments: three bf16 terms
// bh + bm + bl = p that carry p's 24 significant bits, so the tensor cores see the fp32 softmax
// weight exactly).  V^T A fragments by ldmatrix.trans: matrix i
// covers tokens 0-7 / 8-15 (i / 2) and head dims 0-7 / 8-15 (i % 2) of the m-tile.  The three
// MMAs accumulate the smallest term first.
template <int D>
__device__ __forceinline__ void pv_tile(uint32_t xb, int r0, const uint32_t (&bh)[2],
                                        const uint32_t (&bm)[2], const uint32_t (&bl)[2], int lane,
                                        float (&acc)[Cfg<D>::KS][4]) {
    constexpr int KS = Cfg<D>::KS, G = KS < 4 ? KS : 4;
    const int row = r0 + (lane & 7) + (lane >> 4) * 8;
    const uint32_t base = xb + uint32_t(row * (2 * D));
    const int y = ((lane >> 3) & 1) ^ (D == 32 ? (row >> 1) & 3 : row & 7);
#pragma unroll
    for (int m0 = 0; m0 < KS; m0 += G) {
        uint32_t a[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
            ldsm_x4_t(base + (uint32_t((2 * (m0 + g)) ^ y) << 4), a[g][0], a[g][1], a[g][2], a[g][3]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float (&c)[4] = acc[m0 + g];
            mma_bf16(c[0], c[1], c[2], c[3], a[g][0], a[g][1], a[g][2], a[g][3], bl[0], bl[1]);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float (&c)[4] = acc[m0 + g];
            mma_bf16(c[0], c[1], c[2], c[3], a[g][0], a[g][1], a[g][2], a[g][3], bm[0], bm[1]);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float (&c)[4] = acc[m0 + g];
            mma_bf16(c[0], c[1], c[2], c[3], a[g][0], a[g][1], a[g][2], a[g][3], bh[0], bh[1]);
        }
    }
}

// Q B fragments: qb[k][0] = Q[g][16k + 2t + {0,1}], qb[k][1] = Q[g][16k + 8 + 2t + {0,1}].
template <int D>
__device__ __forceinline__ void load_q(const uint16_t *q, int n_q, int stride,
                                       uint32_t (&qb)[Cfg<D>::KS][2], int lane) {
    const int gi = lane >> 2, tig = lane & 3;
    const uint32_t *row =
        reinterpret_cast<const uint32_t *>(q + size_t(gi < n_q ? gi : 0) * stride + 2 * tig);
#pragma unroll
    for (int k = 0; k < Cfg<D>::KS; ++k) {
        qb[k][0] = gi < n_q ? __ldg(row + 8 * k) : 0u;
        qb[k][1] = gi < n_q ? __ldg(row + 8 * k + 4) : 0u;
    }
}

// ---- the CTA: one producer warp, NW consumer warps -------------------------------------------

__device__ __forceinline__ const uint8_t *gptr(uint64_t a) { return reinterpret_cast<const uint8_t *>(a); }

// Shared-memory address of ring barrier `i` (full: i < NSLOT; empty: NSLOT + i).
template <int D, bool CP> __device__ __forceinline__ uint32_t ring_bar(uint32_t sb, int i) {
    return sb + uint32_t(Cfg<D, CP>::O_BAR + 8 * i);
}

// One bulk copy of [src, src + len) into the shared region at `dst`: the 16-byte aligned superset
// lands at dst (the wanted bytes start (src & 15) bytes in).  Returns the bytes copied.
__device__ __forceinline__ uint32_t stage_piece(uint32_t dst, const uint8_t *src, uint32_t len,
                                                uint32_t bar) {
    if (len == 0u) return 0u;
    const Piece p = make_piece(src, len);
    bulk_g2s(dst, p.src, p.alloc, bar);
    return p.alloc;
}

// The descriptor words the producer needs of one block: bytes 0-47 (K / V addresses, escape
// record offsets and counts, modes, tokens, the block of its merge words) and, when a block takes
// several stages, the escape count headers (bytes 64-127).
template <bool MULTI> struct PDesc {
    uint4 w0, w1, w2;
    uint4 e[MULTI ? 4 : 1];
};

template <bool MULTI>
__device__ __forceinline__ void pdesc_load(const BlockDesc *gd, PDesc<MULTI> &d) {
    const uint4 *p = reinterpret_cast<const uint4 *>(gd);
    d.w0 = __ldg(p);
    d.w1 = __ldg(p + 1);
    d.w2 = __ldg(p + 2);
    if constexpr (MULTI) {
#pragma unroll
        for (int i = 0; i < 4; ++i) d.e[i] = __ldg(p + 4 + i);
    }
}

// Escape count e(i), i = 1..16, of tensor T from a prefetched descriptor (em[T][i - 1]).
__device__ __forceinline__ int pdesc_esc(const uint4 (&e)[4], int T, int i) {
    const int w = (i - 1) >> 1;  // u32 word of em[T] holding entry i - 1
    const uint4 a = T ? e[2] : e[0], b = T ? e[3] : e[1];
    uint32_t r = a.x;
    r = w == 1 ? a.y : r;
    r = w == 2 ? a.z : r;
    r = w == 3 ? a.w : r;
    r = w == 4 ? b.x : r;
    r = w == 5 ? b.y : r;
    r = w == 6 ? b.z : r;
    r = w == 7 ? b.w : r;
    return int((r >> (16 * ((i - 1) & 1))) & 0xFFFFu);
}

// A producer warp (one of NP; producer pw takes the stages gs with gs mod NP == pw): for each of
// its stages of the CTA's blocks, wait until the slot is free, issue the stage's copies and
// announce their byte count on the slot's full barrier (lane 0).  Lane l holds
// the descriptor of block base + l; the next 32 are loaded while the current 32 are issued, so
// the issuing lane never waits on a global load.  On a timeout it reports DERR_TIMEOUT and waits
// (bounded) for the copies it issued before it returns.
template <int D, bool CP, bool BF16IN>
__device__ void producer(const AttnArgs &a, uint8_t *smem, int fb0, int fb1, int pw, int lane) {
    using C = Cfg<D, CP>;
    constexpr bool MULTI = C::TSB < 128;  // a 128-token block takes several stages
    const uint32_t sb = smem_u32(smem);
    int gs = 0;  // stages issued
    bool ok = true;
    PDesc<MULTI> cur, nxt;
    if (fb0 + lane < fb1) pdesc_load<MULTI>(a.desc + fb0 + lane, cur);
    for (int base = fb0; base < fb1 && ok; base += 32) {
        if (base + 32 + lane < fb1) pdesc_load<MULTI>(a.desc + base + 32 + lane, nxt);
        const int nb = min(32, fb1 - base);
        for (int j = 0; j < nb && ok; ++j) {
            const BlockDesc *gd = a.desc + base + j;
            const uint64_t kp = (uint64_t(__shfl_sync(FULL, cur.w0.y, j)) << 32) | __shfl_sync(FULL, cur.w0.x, j);
            const uint64_t vp = (uint64_t(__shfl_sync(FULL, cur.w0.w, j)) << 32) | __shfl_sync(FULL, cur.w0.z, j);
            const uint32_t krec = __shfl_sync(FULL, cur.w1.x, j), vrec = __shfl_sync(FULL, cur.w1.y, j);
            const uint32_t nesc = __shfl_sync(FULL, cur.w1.z, j), mw = __shfl_sync(FULL, cur.w1.w, j);
            const int b7_block = int(__shfl_sync(FULL, cur.w2.w, j));
            const int km = BF16IN ? 0 : int(mw & 0xFFu), vm = BF16IN ? 0 : int((mw >> 8) & 0xFFu);
            const int n_tok = int((mw >> 16) & 0xFFu), valid = int(mw >> 24);
            // e(i) of tensor T of this block (uniform i)
            auto esc_count = [&](int T, int i) -> int {
                if (i == 0) return 0;
                if constexpr (MULTI) {
                    return __shfl_sync(FULL, pdesc_esc(cur.e, T, i), j);
                } else {
                    if (16 * i >= n_tok) return int(T ? nesc >> 16 : nesc & 0xFFFFu);
                    return esc_gd(gd, T, i);  // blocks over 128 tokens: not prefetched
                }
            };
            // every block takes a.stages_per_block stages when that is set (the ones past its
            // tokens carry only the descriptor)
            const int t_end = a.stages_per_block > 0 ? a.stages_per_block * C::TSB : valid;
            for (int t0 = 0; t0 < t_end; t0 += C::TSB) {
                if (gs % C::NP != pw) {  // the other producer warp's stage
                    ++gs;
                    continue;
                }
                const int slot = gs % C::NSLOT;
                const uint32_t full = ring_bar<D, CP>(sb, slot), empty = ring_bar<D, CP>(sb, C::NSLOT + slot);
                if (gs >= C::NSLOT &&
                    !uni(mbar_wait_bounded(empty, uint32_t((gs / C::NSLOT - 1) & 1), kStageWaitUs))) {
                    if (lane == 0) report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
                    ok = false;
                    break;
                }
                const int n = min(C::TSB, valid - t0);
                int ea[2] = {0, 0}, eb[2] = {0, 0};
                if (!BF16IN && n > 0) {
#pragma unroll
                    for (int T = 0; T < 2; ++T) {
                        ea[T] = esc_count(T, t0 >> 4);
                        eb[T] = esc_count(T, min(16, (t0 + C::TSB) >> 4));
                    }
                }
                // The stage's pieces go out in parallel, one per lane: 0 the descriptor, 1 the merge
                // words, 2 + 3 T the rows of tensor T (with its residual codes when the stage is the
                // whole block: they follow the rows in the blob), 3 + 3 T its codes otherwise, 4 + 3 T
                // its escape-record entries.  Lane 0 then tells the slot's barrier the byte count; the
                // barrier's tx-count may run below zero until then, and the phase cannot complete
                // before that arrive.
                const bool whole = t0 == 0 && n == n_tok;
                const uint32_t dslot = sb + uint32_t(slot * C::SLOT);
                const uint8_t *src = nullptr;
                uint32_t len = 0u, dst = 0u;
                if (lane == 0) {
                    src = reinterpret_cast<const uint8_t *>(gd), len = uint32_t(sizeof(BlockDesc)), dst = dslot;
                } else if (lane == 1) {
                    if (!BF16IN && (km | vm) != 0 && n > 0) {
                        src = reinterpret_cast<const uint8_t *>(a.b7 + size_t(b7_block) * D);
                        len = uint32_t(4 * D), dst = dslot + C::S_B7;
                    }
                } else if (lane < 8 && n > 0) {
                    const int T = (lane - 2) / 3, part = (lane - 2) % 3;
                    const uint8_t *blk = gptr(T ? vp : kp);
                    const int mode = T ? vm : km;
                    const uint32_t reg = dslot + uint32_t(C::S_T + T * C::T_BYTES);
                    if (part == 0) {
                        dst = reg;
                        if (BF16IN) {
                            src = blk + size_t(t0) * 2 * D, len = uint32_t(n * 2 * D);
                        } else if (mode == 0) {
                            src = blk + kHeaderBytes + size_t(t0) * 2 * D, len = uint32_t(n * 2 * D);
                        } else {
                            src = blk + kHeaderBytes + D + size_t(t0) * D;
                            len = uint32_t(n * D + (whole ? n * D * mode / 8 : 0));
                        }
                    } else if (!BF16IN && mode != 0) {
                        if (part == 1) {
                            if (!whole) {
                                src = blk + kHeaderBytes + D + size_t(n_tok) * D + size_t(t0) * D * mode / 8;
                                len = uint32_t(n * D * mode / 8), dst = reg + C::CODE_OFF;
                            }
                        } else {
                            const int e0 = T ? ea[1] : ea[0], e1 = T ? eb[1] : eb[0];
                            if (e1 > e0 && e1 - e0 <= C::ESC_CAP) {
                                src = reinterpret_cast<const uint8_t *>(a.esc + (T ? vrec : krec) + kEscRecHead + e0);
                                len = uint32_t(4 * (e1 - e0)), dst = reg + C::E_OFF;
                            }
                        }
                    }
                }
                const uint32_t total = __reduce_add_sync(FULL, stage_piece(dst, src, len, full));
                if (lane == 0) {
                    if (!BF16IN) {
#pragma unroll
                        for (int T = 0; T < 2; ++T) {
                            const int e0 = T ? ea[1] : ea[0], e1 = T ? eb[1] : eb[0];
                            const uint32_t rec = T ? vrec : krec;
                            const uint32_t ents = dslot + uint32_t(C::S_T + T * C::T_BYTES + C::E_OFF) +
                                                  esc_rec_line(rec, e0) - 4u * uint32_t(e0);
                            sts_u32(dslot + uint32_t(C::S_INFO + 4 * T),
                                    e1 > e0 && e1 - e0 <= C::ESC_CAP ? (ents | 1u) : 0u);
                        }
                    }
                    // (the stores above are ordered before the arrive, which releases them)
                    mbar_arrive_expect_tx(full, total);
                }
                __syncwarp();
                ++gs;
            }
        }
        cur = nxt;
    }
    if (!ok && lane == 0) {
        // let the copies already issued land before this CTA's shared memory goes away
        for (int s = max(0, gs - C::NSLOT); s < gs; ++s)
            if (s % C::NP == pw)
                mbar_wait_bounded(ring_bar<D, CP>(sb, s % C::NSLOT), uint32_t((s / C::NSLOT) & 1), kStageWaitUs);
    }
}

// A producer warp with the plan's stage copy lists (AttnArgs::stages): for each of its stages
// (gs mod NP == pw), wait until the slot is free, then lanes 0-7 issue the stage's pieces as the
// list gives them and lane 8 writes the stage's escape-entry words and announces the
// stage's bytes on the slot's full barrier.  Each lane keeps its word of the lists of its next PF
// stages in registers, loaded PF stages ahead.  On a timeout it reports DERR_TIMEOUT and waits
// (bounded) for the copies it issued before it returns.
template <int D, bool CP, bool BF16IN>
__device__ void producer_listed(const AttnArgs &a, uint8_t *smem, int fb0, int fb1, int pw, int lane) {
    using C = Cfg<D, CP>;
    constexpr int PF = 3;
    const uint32_t sb = smem_u32(smem);
    const int n_st = (fb1 - fb0) * a.stages_per_block;
    const uint4 *rec = a.stages + size_t(fb0) * size_t(a.stages_per_block) * kStageRecWords + lane;
    auto fetch = [&](int g) -> uint4 {
        return lane < kStageRecWords && g < n_st ? __ldg(rec + size_t(g) * kStageRecWords) : make_uint4(0u, 0u, 0u, 0u);
    };
    uint4 r[PF];
#pragma unroll
    for (int k = 0; k < PF; ++k) r[k] = fetch(pw + k * C::NP);
    int gs = pw;
    bool ok = true;
    for (; gs < n_st; gs += C::NP) {
        const uint4 w = r[0];
#pragma unroll
        for (int k = 0; k + 1 < PF; ++k) r[k] = r[k + 1];
        r[PF - 1] = fetch(gs + PF * C::NP);
        const int slot = gs % C::NSLOT;
        const uint32_t full = ring_bar<D, CP>(sb, slot), empty = ring_bar<D, CP>(sb, C::NSLOT + slot);
        if (gs >= C::NSLOT &&
            !uni(mbar_wait_bounded(empty, uint32_t((gs / C::NSLOT - 1) & 1), kStageWaitUs))) {
            if (lane == 0) report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
            ok = false;
            break;
        }
        const uint32_t dslot = sb + uint32_t(slot * C::SLOT);
        if (lane < 8 && w.z != 0u)
            bulk_g2s(dslot + w.w, reinterpret_cast<const void *>((uint64_t(w.y) << 32) | w.x), w.z, full);
        if (lane == 8) {
            if (!BF16IN) {
                sts_u32(dslot + uint32_t(C::S_INFO), (w.w & 1u) ? ((dslot + w.x) | 1u) : 0u);
                sts_u32(dslot + uint32_t(C::S_INFO + 4), (w.w & 2u) ? ((dslot + w.y) | 1u) : 0u);
            }
            // (the stores above are ordered before the arrive, which releases them; copies that
            // complete before it only run the barrier's tx-count below zero meanwhile)
            mbar_arrive_expect_tx(full, w.z);
        }
        __syncwarp();
    }
    if (!ok && lane < 8) {
        // let the copies already issued land before this CTA's shared memory goes away
        for (int s = max(0, gs - C::NSLOT); s < gs; ++s)
            if (s % C::NP == pw)
                mbar_wait_bounded(ring_bar<D, CP>(sb, s % C::NSLOT), uint32_t((s / C::NSLOT) & 1), kStageWaitUs);
    }
}

// The descriptor fields a consumer warp uses during one visit of a stage, read from the slot's
// copy of the block descriptor by two 16-byte loads (bytes 16-47 of BlockDesc).
struct VisitDesc {
    uint32_t k_rec, v_rec, nesc;
    uint32_t mw;      // k_mode | v_mode << 8 | n_tok << 16 | valid << 24
    int32_t unit;
    uint32_t align;   // BlockDesc::align as one word
    uint32_t flags, b7_block;
    __device__ __forceinline__ int k_mode() const { return int(mw & 0xFFu); }
    __device__ __forceinline__ int v_mode() const { return int((mw >> 8) & 0xFFu); }
    __device__ __forceinline__ int n_tok() const { return int((mw >> 16) & 0xFFu); }
    __device__ __forceinline__ int valid() const { return int(mw >> 24); }
};
static_assert(offsetof(BlockDesc, k_rec) == 16 && offsetof(BlockDesc, k_mode) == 28 &&
                  offsetof(BlockDesc, valid) == 31 && offsetof(BlockDesc, unit) == 32,
              "VisitDesc mirrors bytes 16-47 of BlockDesc");
__device__ __forceinline__ VisitDesc load_visit(uint32_t slot_addr) {
    VisitDesc v;
    uint32_t u;
    lds_v4(slot_addr + 16u, v.k_rec, v.v_rec, v.nesc, v.mw);
    lds_v4(slot_addr + 32u, u, v.align, v.flags, v.b7_block);
    v.unit = int32_t(u);
    return v;
}

// One tensor of the warp's NT tiles (tiles tw .. tw + NT - 1 of the stage) into its BF16 tiles,
// escapes included.  reg: the tensor's region of the slot; b7s: the tensor's merge words in the
// slot; info: the producer's escape word of the tensor for this stage; g16: the first tile's
// 16-token group in the block; t0: the stage's first token in the block; rows: valid rows from the
// first tile's first row on; zero_from: rows at or past it are zeroed.
template <int D, bool CP, int T>
__device__ __forceinline__ void tile_tensor(const AttnArgs &a, const BlockDesc &bd, const VisitDesc &vd,
                                            int mode, uint32_t al, uint32_t reg, uint32_t b7s, uint32_t info,
                                            int tw, uint32_t xb,
                                            const StoreMap<D> &sm, int g16, int t0, int rows,
                                            int zero_from, bool bf16, int lane) {
    using C = Cfg<D, CP>;
    const int c8 = lane % C::C8;
    const uint32_t rd = al & 15u, cd = (al >> 8) & 15u;
    // a whole block in one stage came as one copy: the codes follow its n rows
    const int n = min(C::TSB, vd.valid() - t0);
    const bool whole = t0 == 0 && n == vd.n_tok();
    const uint32_t code_base = whole ? ((rd + uint32_t(n * D)) & ~15u) : uint32_t(C::CODE_OFF);
    const Lay ly = make_lay<D>(rd, cd, mode, c8, bf16, code_base);
    const uint32_t rb = reg + uint32_t(TT * tw * (mode == 0 ? 2 * D : D));
    const uint32_t cb = reg + uint32_t(TT * tw * (D * mode / 8));
    // The tiles' escapes [e0, e1) are fetched before the decode, one entry per lane (more than 32
    // occur only in escape-dense blocks; those lanes take the rest after the first 32), so that only
    // their stores follow the decode.  EscBounds says which tile each entry is in.
    constexpr int NT = C::NT;
    const int e0 = esc_ms(bd, T, g16), e1 = esc_ms(bd, T, g16 + NT);
    EscBounds<NT> eb;
#pragma unroll
    for (int j = 0; j + 1 < NT; ++j) eb.b[j] = esc_ms(bd, T, g16 + 1 + j);
    uint32_t ents = 0u, ent = 0u;
    if (e1 > e0) {
        ents = lds_u32(info);  // the producer's word for this stage and tensor
        if (e0 + lane < e1)
            ent = (ents & 1u) ? lds_u32((ents & ~1u) + 4u * uint32_t(e0 + lane))
                              : __ldg(a.esc + (T ? vd.v_rec : vd.k_rec) + kEscRecHead + e0 + lane);
    }
    if (mode != 0) {
        uint32_t b7[4];
        lds_v4(b7s + 16u * uint32_t(c8), b7[0], b7[1], b7[2], b7[3]);
        if (mode == 4) decode_tile<D, 4, 0>(rb, cb, ly, b7, sm, lane);
        else if (mode == 2) decode_tile<D, 2, 0>(rb, cb, ly, b7, sm, lane);
        else decode_tile<D, 3, 0>(rb, cb, ly, b7, sm, lane);
    } else {
        const uint32_t b7[4] = {0u, 0u, 0u, 0u};
        decode_tile<D, 0, 0>(rb, cb, ly, b7, sm, lane);
    }
    if (zero_from < NT * TT) zero_rows<D, 0>(sm, zero_from, lane);
    if (e1 > e0) {
        // entry: the element's byte in its tile (bits 0-15, even) | its BF16 word << 16; elements
        // in rows at or past `rows` are skipped
        __syncwarp();  // the decoded words are in place before escapes overwrite some
        if (e0 + lane < e1) esc_store(xb, ent, eb.tile(e0 + lane), rows, C::TILE1, 2 * D);
        if (e1 - e0 > 32) {
            if (ents & 1u)
                esc_patch<D>(xb, ents & ~1u, e0 + 32, e1, eb, rows, lane);
            else
                esc_patch_hbm<D>(xb, a.esc + (T ? vd.v_rec : vd.k_rec) + kEscRecHead, e0 + 32, e1, eb,
                                 rows, lane);
        }
    }
    __syncwarp();
}

// Per-warp online-softmax state: lane (g, t) holds queries 2t (m0, l0, acc[m][0 / 2]) and 2t + 1
// (m1, l1, acc[m][1 / 3]); acc[m][0 / 1] is head dim 16 m + g, acc[m][2 / 3] head dim 16 m + g + 8.
template <int D> struct SoftState {
    float acc[Cfg<D>::KS][4];
    float m0, m1, l0, l1;
    __device__ __forceinline__ void reset() {
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
#pragma unroll
        for (int m = 0; m < Cfg<D>::KS; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    }
};

// The warp's NT 16-token tiles of K and V (tiles tw .. tw + NT - 1 of the stage): decode K into
// the warp's tiles, S = K Q^T on the tensor cores, decode V into the same tiles (the MMAs have their
// K fragments and run meanwhile), free the slot, online softmax, O += P V.  rows: valid rows from
// the first tile's first row (1 .. NT 16).
template <int D, bool CP, bool BF16IN>
__device__ __forceinline__ void tile_step(const AttnArgs &a, const BlockDesc &bd, const VisitDesc &vd,
                                          uint32_t slot_addr,
                                          uint32_t empty, uint32_t xb, const StoreMap<D> &sm, int tw,
                                          int t0, int rows, const uint32_t (&qb)[Cfg<D>::KS][2],
                                          SoftState<D> &st, int lane) {
    using C = Cfg<D, CP>;
    constexpr int NT = C::NT;
    const int gi = lane >> 2;
    const uint32_t al = vd.align;
    const int km = BF16IN ? 0 : vd.k_mode(), vm = BF16IN ? 0 : vd.v_mode();
    const int g16 = (t0 >> 4) + tw;
    const uint32_t kreg = slot_addr + uint32_t(C::S_T), vreg = kreg + uint32_t(C::T_BYTES);

    // S^T = K Q^T (rows past `rows` hold stale words: their scores are dropped)
    tile_tensor<D, CP, 0>(a, bd, vd, km, al & 0xFFFFu, kreg, slot_addr + uint32_t(C::S_B7),
                      slot_addr + uint32_t(C::S_INFO), tw, xb, sm, g16, t0, rows, NT * TT, BF16IN, lane);
    float s[NT][4];
    qk_tiles<D, NT>(xb, qb, lane, s);
    // V replaces K in the tiles once every lane's K fragments are loaded (the MMAs above need only
    // those registers); rows past `rows` are zeroed (P is 0 there and V must be finite)
    __syncwarp();
    tile_tensor<D, CP, 1>(a, bd, vd, vm, al >> 16, vreg, slot_addr + uint32_t(C::S_B7 + 2 * D),
                      slot_addr + uint32_t(C::S_INFO + 4), tw, xb, sm, g16, t0, rows, rows, BF16IN, lane);
    if (lane == 0) mbar_arrive(empty);  // this warp has read everything it needs from the slot
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (rows < TT * (t + 1)) {
            if (gi >= rows - TT * t) s[t][0] = s[t][1] = -INFINITY;
            if (gi + 8 >= rows - TT * t) s[t][2] = s[t][3] = -INFINITY;
        }
    }

    // online softmax (src/softmax.hpp:8-14): p = 2^((s - m) log2e); the warp-wide maximum and the
    // rescale of the accumulators only when some score exceeds the running maximum.  s - m is
    // formed first, like the reference's expf(s - m), so that huge scores keep the largest weight
    // at exactly 1.
    float t0m = fmaxf(s[0][0], s[0][2]), t1m = fmaxf(s[0][1], s[0][3]);
#pragma unroll
    for (int t = 1; t < NT; ++t) {
        t0m = fmaxf(t0m, fmaxf(s[t][0], s[t][2]));
        t1m = fmaxf(t1m, fmaxf(s[t][1], s[t][3]));
    }
    const bool grow = __any_sync(FULL, t0m > st.m0 || t1m > st.m1);
    float mn0 = st.m0, mn1 = st.m1, al0 = 1.0f, al1 = 1.0f;
    if (grow) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            t0m = fmaxf(t0m, __shfl_xor_sync(FULL, t0m, o));
            t1m = fmaxf(t1m, __shfl_xor_sync(FULL, t1m, o));
        }
        mn0 = fmaxf(st.m0, t0m);
        mn1 = fmaxf(st.m1, t1m);
        al0 = ex2(__fmul_rn(__fsub_rn(st.m0, mn0), kLog2e));
        al1 = ex2(__fmul_rn(__fsub_rn(st.m1, mn1), kLog2e));
    }
    // P^T B fragments per tile: p = h + m + l exactly, each term the upper 16 bits of what remains
    // (h = p truncated to bf16, m = (p - h) truncated, l = p - h - m); the differences are exact in
    // fp32 and l has at most 8 significant bits, so the three bf16 terms carry all 24 bits of p.
    // Two weights pack into one B register with one byte permute.
    uint32_t bh[NT][2], bm[NT][2], bl[NT][2];
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        constexpr uint32_t HI = 0xFFFF0000u, PK = 0x7632u;  // PK: the upper halves of a and b
        const float p0 = ex2(__fmul_rn(__fsub_rn(s[t][0], mn0), kLog2e));
        const float p1 = ex2(__fmul_rn(__fsub_rn(s[t][1], mn1), kLog2e));
        const float p2 = ex2(__fmul_rn(__fsub_rn(s[t][2], mn0), kLog2e));
        const float p3 = ex2(__fmul_rn(__fsub_rn(s[t][3], mn1), kLog2e));
        const uint32_t P0 = __float_as_uint(p0), P1 = __float_as_uint(p1);
        const uint32_t P2 = __float_as_uint(p2), P3 = __float_as_uint(p3);
        const float r0 = __fsub_rn(p0, __uint_as_float(P0 & HI)), r1 = __fsub_rn(p1, __uint_as_float(P1 & HI));
        const float r2 = __fsub_rn(p2, __uint_as_float(P2 & HI)), r3 = __fsub_rn(p3, __uint_as_float(P3 & HI));
        const uint32_t R0 = __float_as_uint(r0), R1 = __float_as_uint(r1);
        const uint32_t R2 = __float_as_uint(r2), R3 = __float_as_uint(r3);
        const float u0 = __fsub_rn(r0, __uint_as_float(R0 & HI)), u1 = __fsub_rn(r1, __uint_as_float(R1 & HI));
        const float u2 = __fsub_rn(r2, __uint_as_float(R2 & HI)), u3 = __fsub_rn(r3, __uint_as_float(R3 & HI));
        bh[t][0] = movm_t(prmt(P0, P1, PK));
        bh[t][1] = movm_t(prmt(P2, P3, PK));
        bm[t][0] = movm_t(prmt(R0, R1, PK));
        bm[t][1] = movm_t(prmt(R2, R3, PK));
        bl[t][0] = movm_t(prmt(__float_as_uint(u0), __float_as_uint(u1), PK));
        bl[t][1] = movm_t(prmt(__float_as_uint(u2), __float_as_uint(u3), PK));
        ps0 = __fadd_rn(ps0, __fadd_rn(p0, p2));
        ps1 = __fadd_rn(ps1, __fadd_rn(p1, p3));
    }
    st.l0 = __fmaf_rn(st.l0, al0, ps0);
    st.l1 = __fmaf_rn(st.l1, al1, ps1);
    st.m0 = mn0;
    st.m1 = mn1;
    if (grow) {
#pragma unroll
        for (int m = 0; m < C::KS; ++m) {
            st.acc[m][0] = __fmul_rn(st.acc[m][0], al0);
            st.acc[m][1] = __fmul_rn(st.acc[m][1], al1);
            st.acc[m][2] = __fmul_rn(st.acc[m][2], al0);
            st.acc[m][3] = __fmul_rn(st.acc[m][3], al1);
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) pv_tile<D>(xb, TT * t, bh[t], bm[t], bl[t], lane, st.acc);
    __syncwarp();  // every lane is done with the tiles before the next decode writes them
}

// The warp's state for one unit segment goes to partial state `idx` (m, l summed over the lanes
// of each query, acc).
template <int D>
__device__ __forceinline__ void flush_state(const AttnArgs &a, size_t idx, const SoftState<D> &st, int lane) {
    const int gi = lane >> 2, tig = lane & 3;
    float lt0 = st.l0, lt1 = st.l1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        lt0 = __fadd_rn(lt0, __shfl_xor_sync(FULL, lt0, o));
        lt1 = __fadd_rn(lt1, __shfl_xor_sync(FULL, lt1, o));
    }
    float *part = a.partials + idx * size_t(partial_stride(D));
    const int qa = 2 * tig, qc = 2 * tig + 1;
    if (gi == 0) {
        part[qa] = st.m0;
        part[qc] = st.m1;
        part[8 + qa] = lt0;
        part[8 + qc] = lt1;
    }
    float *oa = part + 16 + qa * D + gi;
    float *oc = part + 16 + qc * D + gi;
#pragma unroll
    for (int m = 0; m < Cfg<D>::KS; ++m) {
        oa[16 * m] = st.acc[m][0];
        oa[16 * m + 8] = st.acc[m][2];
        oc[16 * m] = st.acc[m][1];
        oc[16 * m + 8] = st.acc[m][3];
    }
}

// A consumer warp: visits every stage of the CTA's range in order, takes the tile groups dealt to it,
// arrives once per stage on the slot's empty barrier, and writes its state at every segment end
// (the unit's last block, or the end of the range).  It has seen stage gs - 1 (and so gs - NSLOT)
// land before it waits on stage gs, so the parity of the slot's full barrier identifies the stage.
template <int D, bool CP, bool BF16IN>
__device__ void consumer(const AttnArgs &a, uint8_t *smem, int w, int lane, int fb0, int fb1, int row0) {
    using C = Cfg<D, CP>;
    const uint32_t sb = smem_u32(smem);
    const uint32_t xb = sb + uint32_t(C::O_TILE + w * C::TILE);
    StoreMap<D> sm;
    sm.init(xb, lane);
    uint32_t qb[C::KS][2];
    SoftState<D> st;
    st.reset();
    int row = row0;
    int gs = 0;   // stages consumed
    int tp = w;   // this warp's tile group in stage gs: (w - gs TPP) mod NW (none when >= TPP)
    for (int b = fb0; b < fb1; ++b) {
        for (int t0 = 0;; t0 += C::TSB) {
            const int slot = gs % C::NSLOT;
            const uint32_t full = ring_bar<D, CP>(sb, slot), empty = ring_bar<D, CP>(sb, C::NSLOT + slot);
            if (!uni(mbar_wait_bounded(full, uint32_t((gs / C::NSLOT) & 1), kStageWaitUs))) {
                if (lane == 0) report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
                return;
            }
            const uint8_t *sp = smem + slot * C::SLOT;
            const BlockDesc &bd = *reinterpret_cast<const BlockDesc *>(sp);
            const VisitDesc vd = load_visit(smem_u32(sp));
            const int valid = vd.valid();
            const uint32_t flags = vd.flags;
            if (t0 == 0 && (b == fb0 || (flags & kDescFirst) != 0u)) {
                const UnitDev *U = a.units + vd.unit;
                load_q<D>(U->q, U->n_q, U->q_stride, qb, lane);
                st.reset();
            }
            const bool last = t0 + C::TSB >= valid;
            const bool seg_end = last && ((flags & kDescLast) != 0u || b + 1 == fb1);
            const int rows = valid - t0 - TT * C::NT * tp;
            if (tp < C::TPP && rows > 0) {
                tile_step<D, CP, BF16IN>(a, bd, vd, smem_u32(sp), empty, xb, sm, C::NT * tp, t0,
                                     min(rows, C::NT * TT), qb, st, lane);
            } else {
                __syncwarp();  // every lane has read the descriptor
                if (lane == 0) mbar_arrive(empty);
            }
            if (seg_end) {
                flush_state<D>(a, size_t(row) * C::NW + size_t(w), st, lane);
                ++row;
            }
            ++gs;
            tp -= C::TPP;
            if (tp < 0) tp += C::NW;
            if (last) break;
        }
    }
}

// Wait until stage gs of the CTA has landed in its slot.  The slot's full barrier alone cannot tell
// stage gs from stage gs - 2 NSLOT: a warp that skips stages may start waiting while the slot's
// previous stage (gs - NSLOT) is still in flight, and the parity test would then pass one phase
// early.  So the warp first waits until stage gs - NSLOT has been released (the slot's empty
// barrier completes that use's phase; its next phase needs this warp's own arrive for stage gs, so
// the parity identifies it).  From then on the full barrier's pending phase is stage gs's, and the
// second wait passes only when stage gs has landed.  Both waits are mbarrier tests, which suspend
// the warp while the phase is incomplete instead of spinning on the issue slots the other warps
// need.  Returns false after kStageWaitUs (the decision is the warp's, uniform).
template <int D, bool CP>
__device__ __forceinline__ bool wait_stage(uint32_t sb, int gs) {
    using C = Cfg<D, CP>;
    const int slot = gs % C::NSLOT, use = gs / C::NSLOT;
    if (use > 0 &&
        !uni(mbar_wait_bounded(ring_bar<D, CP>(sb, C::NSLOT + slot), uint32_t((use - 1) & 1), kStageWaitUs)))
        return false;
    return uni(mbar_wait_bounded(ring_bar<D, CP>(sb, slot), uint32_t(use & 1), kStageWaitUs));
}

// A consumer warp when every block takes the same number of stages (spb): stage s of the range is
// stage s mod spb of block fb0 + s / spb, so the warp goes straight to the stages of its tile
// groups (group j = w, w + NW, ... of the range; stage j / TPP, tiles NT (j mod TPP) ..), waits
// only on those, and arrives once per group (the slot's empty barrier counts TPP arrivals).  Its state is written
// when the unit of its next tile differs, and at the end of the range, to row
// row0 + (unit - the range's first unit); rows a warp never reaches keep m = -inf, l = 0.
template <int D, bool CP, bool BF16IN>
__device__ void consumer_by_tile(const AttnArgs &a, uint8_t *smem, int w, int lane, int fb0, int fb1,
                                 int row0) {
    using C = Cfg<D, CP>;
    const uint32_t sb = smem_u32(smem);
    const uint32_t xb = sb + uint32_t(C::O_TILE + w * C::TILE);
    StoreMap<D> sm;
    sm.init(xb, lane);
    uint32_t qb[C::KS][2];
    SoftState<D> st;
    st.reset();
    const int spb = a.stages_per_block;
    // stage of a block: gs mod spb (a mask when spb is a power of two, as it is for 128-token blocks)
    const int spb_mask = (spb & (spb - 1)) == 0 ? spb - 1 : -1;
    const int unit0 = __ldg(&a.desc[fb0].unit);
    int cur = -1;  // unit of the warp's state (-1: none yet)
    const int groups = (fb1 - fb0) * spb * C::TPP;
    for (int j = w; j < groups; j += C::NW) {
        const int gs = j / C::TPP, tw = (j % C::TPP) * C::NT;
        const int t0 = (spb_mask >= 0 ? (gs & spb_mask) : gs % spb) * C::TSB;
        const int slot = gs % C::NSLOT;
        const uint32_t empty = ring_bar<D, CP>(sb, C::NSLOT + slot);
        if (!wait_stage<D, CP>(sb, gs)) {
            if (lane == 0) report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
            return;
        }
        const uint8_t *sp = smem + slot * C::SLOT;
        const BlockDesc &bd = *reinterpret_cast<const BlockDesc *>(sp);
        const VisitDesc vd = load_visit(smem_u32(sp));
        const int valid = vd.valid(), unit = vd.unit;
        if (unit != cur) {
            if (cur >= 0) flush_state<D>(a, size_t(row0 + cur - unit0) * C::NW + size_t(w), st, lane);
            const UnitDev *U = a.units + unit;
            load_q<D>(U->q, U->n_q, U->q_stride, qb, lane);
            st.reset();
            cur = unit;
        }
        const int rows = valid - t0 - TT * tw;
        if (rows > 0) {
            tile_step<D, CP, BF16IN>(a, bd, vd, smem_u32(sp), empty, xb, sm, tw, t0, min(rows, C::NT * TT), qb, st,
                                 lane);
        } else {
            __syncwarp();  // every lane has read the descriptor
            if (lane == 0) mbar_arrive(empty);
        }
    }
    if (cur >= 0) flush_state<D>(a, size_t(row0 + cur - unit0) * C::NW + size_t(w), st, lane);
}

template <int D, bool CP, bool BF16IN>
__global__ void __launch_bounds__(Cfg<D, CP>::THREADS, 1) attn_kernel(const AttnArgs a) {
    using C = Cfg<D, CP>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int skip;
    // Launched as a programmatic dependent of the kernel before it in the stream (the previous
    // step's combine pass, or the plan's descriptor build): nothing is read before that grid has
    // completed and its writes are visible.  Only the launch itself overlaps it.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // A combine pass launched behind this grid (programmatic dependent launch) may start placing
    // its CTAs as soon as SMs free up; it waits for this grid's completion before reading.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int c = blockIdx.x;
    if (c >= a.n_ranges) return;
    const int fb0 = int(a.range_begin[c]), fb1 = int(a.range_begin[c + 1]);
    if (fb0 >= fb1) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool by_tile = a.stages_per_block > 0;
    if (threadIdx.x == 0) {
        const uint32_t sb = smem_u32(smem);
        for (int j = 0; j < C::NSLOT; ++j) {
            mbar_init(ring_bar<D, CP>(sb, j), 1);               // full: the producer's arrive + bytes
            // empty: one arrive per consumer warp, or per tile group when the warps go by tile
            mbar_init(ring_bar<D, CP>(sb, C::NSLOT + j), by_tile ? C::TPP : C::NW);
        }
        fence_mbar_init();
        // a step whose preparation reported an error (its escape records are incomplete) runs no work
        skip = *reinterpret_cast<volatile const int *>(a.status);
    }
    __syncthreads();
    if (skip != 0) return;
    if (warp >= C::NW) {
        if (a.stages != nullptr)
            producer_listed<D, CP, BF16IN>(a, smem, fb0, fb1, warp - C::NW, lane);
        else
            producer<D, CP, BF16IN>(a, smem, fb0, fb1, warp - C::NW, lane);
        return;
    }
    if (by_tile)
        consumer_by_tile<D, CP, BF16IN>(a, smem, warp, lane, fb0, fb1, a.seg_base[c]);
    else
        consumer<D, CP, BF16IN>(a, smem, warp, lane, fb0, fb1, a.seg_base[c]);
}

// ---- combine ------------------------------------------------------------------------------------

// Combine the partial states of one query of a unit: with M = max m_t over the unit's states,
// l = sum l_t e^(m_t - M) and acc = sum acc_t e^(m_t - M) (merge_state's arithmetic,
// src/softmax.hpp:16-30, applied to all states at once instead of a left fold), then
// out = acc * (1 / l) like finalize_state (src/softmax.hpp:32-41).  One CTA per (unit, query);
// the sums run over fixed slices of the states, so the result is deterministic.  A state of a
// warp that saw none of the unit's tokens has m = -inf and l = 0 (written so, or initialised so
// by init_partials_kernel and never written) and adds nothing; its accumulators are not read.
constexpr int kCombineThreads = 512;
constexpr int kMaxSegments = 4096;

template <int D>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const CombineArgs a) {
    constexpr int S = kCombineThreads / D;  // state slices summed in parallel
    constexpr int PRE = 8;                  // accumulator values a thread loads up front
    __shared__ float e[kMaxSegments];
    __shared__ float lw[kMaxSegments];
    __shared__ float red[kCombineThreads];
    // launched as a dependent of the attention grid: its partial states are complete and visible
    // after this wait (a no-op for an ordinary launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the next step's attention grid may be set up while this one runs (it waits for it)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const SplitUnit sp = a.split[blockIdx.x];
    const int g = blockIdx.y;
    if (g >= sp.n_q) return;
    const int nt = min(sp.n_states, kMaxSegments);
    const int ps = partial_stride(D);
    auto part = [&](int i) { return a.partials + (size_t(sp.first_state) + size_t(i)) * ps; };
    const int tid = threadIdx.x;
    const int d = tid % D, sl = tid / D;
    // every load that does not depend on M goes out first: (m, l) of the segments and the first
    // PRE accumulator values of this thread's slice
    float pre[PRE];
#pragma unroll
    for (int k = 0; k < PRE; ++k) {
        const int i = sl + k * S;
        pre[k] = (sl < S && i < nt) ? __ldg(part(i) + 16 + g * D + d) : 0.f;
    }
    float mx = -INFINITY;
    for (int i = tid; i < nt; i += kCombineThreads) {
        const float *pi = part(i);
        const float m = __ldg(pi + g);
        e[i] = m;
        lw[i] = __ldg(pi + 8 + g);
        mx = fmaxf(mx, m);
    }
    // maxima: within each warp by shuffles, then over the warps' results
    constexpr int NWC = kCombineThreads / 32;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < NWC; ++w) M = fmaxf(M, red[w]);
    float ls = 0.f;
    for (int i = tid; i < nt; i += kCombineThreads) {
        const float w = expf(e[i] - M);
        e[i] = w;
        ls = __fmaf_rn(lw[i], w, ls);
    }
    // sum of the weighted l: within each warp by shuffles, then over the warps in warp order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls = __fadd_rn(ls, __shfl_xor_sync(FULL, ls, o));
    __syncthreads();  // every thread has read the maxima from red
    if ((tid & 31) == 0) red[tid >> 5] = ls;
    __syncthreads();
    float lsum = red[0];
#pragma unroll
    for (int w = 1; w < NWC; ++w) lsum = __fadd_rn(lsum, red[w]);
    const float inv = __frcp_rn(lsum);
    __syncthreads();  // every thread has read the sums from red
    float acc = 0.f;
    if (sl < S) {
#pragma unroll
        for (int k = 0; k < PRE; ++k)
            if (sl + k * S < nt && e[sl + k * S] > 0.f) acc = __fmaf_rn(pre[k], e[sl + k * S], acc);
#pragma unroll 8
        for (int i = sl + PRE * S; i < nt; i += S)
            if (e[i] > 0.f) acc = __fmaf_rn(__ldg(part(i) + 16 + g * D + d), e[i], acc);
    }
    red[tid] = acc;
    __syncthreads();
    if (sl == 0) {
        float v = red[d];
        for (int j = 1; j < S; ++j) v = __fadd_rn(v, red[j * D + d]);
        sp.out[size_t(g) * sp.q_stride + d] = __fmul_rn(v, inv);
    }
    if (tid == 0 && sp.lse != nullptr) sp.lse[g] = M + logf(lsum);
}

// ---- fold of sequence shards --------------------------------------------------------------------

// Rank-ordered fold of the normalised outputs of sequence shards: per row (unit, query),
// M = max_r lse_r, w_r = exp(lse_r - M), out = (sum_r w_r o_r) * (1 / sum_r w_r).  This is the
// reference's thread fold (src/dispatch.cpp:98-103 with merge_state, src/softmax.hpp:16-30, and
// finalize_state, :32-41) carried over to outputs that are already normalised, where l_r is
// exp(lse_r - m_r).  Part r sits at parts + r * (n_rows * dim + n_rows): outputs [n_rows, dim],
// then lse [n_rows].  A part whose lse is -inf (an empty shard) is skipped, whatever its outputs
// hold.  One CTA per row; every thread folds the parts in rank order.
__global__ void fold_kernel(const float *__restrict__ parts, int n_parts, int n_rows, int dim,
                            float *__restrict__ out, float *__restrict__ lse_out) {
    const int row = blockIdx.x;
    const size_t stride = size_t(n_rows) * dim + n_rows;
    const float *lse = parts + size_t(n_rows) * dim + row;
    float M = -INFINITY;
    for (int r = 0; r < n_parts; ++r) M = fmaxf(M, lse[r * stride]);
    float den = 0.f;
    for (int r = 0; r < n_parts; ++r) den = __fadd_rn(den, expf(lse[r * stride] - M));
    const float inv = __frcp_rn(den);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        float acc = 0.f;
        for (int r = 0; r < n_parts; ++r) {
            const float l = lse[r * stride];
            if (l == -INFINITY) continue;
            acc = __fmaf_rn(expf(l - M), parts[r * stride + size_t(row) * dim + d], acc);
        }
        out[size_t(row) * dim + d] = __fmul_rn(acc, inv);
    }
    if (threadIdx.x == 0 && lse_out != nullptr) lse_out[row] = M + logf(den);
}

// ---- worker ranges -----------------------------------------------------------------------------

// Cost of one flat block for the worker split, per attended token and tensor: 4 with 4-bit
// residuals, 5 with 2- or 3-bit ones (more unpacking), 2 for raw rows; plus 1 per 8 escape words
// (a staged escape costs a lane one shared load and one store, about a thirtieth of a token's
// decode per tensor).  Heavier escape weights starved the CTAs that hold escape-dense blocks: at
// 1 per escape word the CTAs holding config[1]'s 2-bit layer-0 K blocks (8 % escapes) finished
// after 48 of the kernel's 74 us; at 1 per 8 the spread is 66-73 us.
__device__ __forceinline__ uint64_t mode_cost(int mode) { return mode == 4 ? 4u : (mode == 0 ? 2u : 5u); }
__device__ __forceinline__ uint64_t block_cost(const FlatBlock &b, bool by_tokens) {
    if (by_tokens) return uint64_t(b.valid);
    return uint64_t(b.valid) * (mode_cost(b.k_mode) + mode_cost(b.v_mode)) + (uint64_t(b.k_nesc) + b.v_nesc) / 8;
}

// One CTA: range_begin[w] = first block whose cost prefix reaches w * total / nw.
// Block b's cost plus unit_cost when it starts a unit: a CTA whose range reaches into another unit
// pays that unit's query loads, state flushes and fresh softmax states in every consumer warp
// (measured at config[1]: CTAs spanning two units took 1.4 us, about 1.7 blocks, longer).
__device__ __forceinline__ uint64_t range_cost(const FlatBlock *flat, int64_t b, bool by_tokens, uint64_t unit_cost) {
    const FlatBlock f = load_flat(flat, b);
    const bool first = b == 0 || load_flat(flat, b - 1).unit != f.unit;
    return block_cost(f, by_tokens) + (first ? unit_cost : 0u);
}

__global__ void __launch_bounds__(1024) split_kernel(const FlatBlock *flat, int64_t n, int nw,
                                                     bool by_tokens, uint64_t unit_cost, int64_t *range_begin) {
    __shared__ unsigned long long part[1024];
    const int t = threadIdx.x, T = blockDim.x;
    const int64_t chunk = (n + T - 1) / T;
    const int64_t lo = min(n, t * chunk), hi = min(n, lo + chunk);
    unsigned long long sum = 0;
    for (int64_t b = lo; b < hi; ++b) sum += range_cost(flat, b, by_tokens, unit_cost);
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
        const unsigned long long cn = c + range_cost(flat, b, by_tokens, unit_cost);
        while (w < nw && uint64_t(w) * total / nw <= c) ++w;
        while (w < nw && uint64_t(w) * total / nw <= cn) range_begin[w++] = b + 1;
        c = cn;
    }
    if (t == 0 && total == 0)
        for (int w2 = 1; w2 < nw; ++w2) range_begin[w2] = n;
}

template <int D, bool CP, bool BF16IN> void configure() {
    static bool done = false;
    if (done) return;
    cudaFuncSetAttribute(attn_kernel<D, CP, BF16IN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D, CP>::SMEM);
    done = true;
}

// ---- stage copy lists ------------------------------------------------------------------------------

// One thread per (flat block, stage): the stage's copy list (kStageRecWords words) from the block's
// descriptor -- the pieces a producer warp issues for the stage, where they land in the slot, and
// where the consumers find the staged escape-record entries.
template <int D, bool CP, bool BF16IN>
__global__ void stage_table_kernel(const BlockDesc *desc, const uint32_t *b7, const uint32_t *esc,
                                   int64_t n_blocks, int spb, uint4 *table) {
    using C = Cfg<D, CP>;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n_blocks * spb) return;
    const int64_t b = i / spb;
    const int t0 = int(i % spb) * C::TSB;
    const BlockDesc &d = desc[b];
    const int km = BF16IN ? 0 : d.k_mode, vm = BF16IN ? 0 : d.v_mode;
    const int n_tok = d.n_tok;
    const int n = min(C::TSB, int(d.valid) - t0);
    const bool whole = t0 == 0 && n == n_tok;
    uint4 w[kStageRecWords];
#pragma unroll
    for (int k = 0; k < kStageRecWords; ++k) w[k] = make_uint4(0u, 0u, 0u, 0u);
    uint32_t total = 0;
    // piece k: [src, src + len) to slot offset dst; returns the bytes copied
    auto put = [&](int k, const void *src, uint32_t len, uint32_t dst) -> uint32_t {
        if (len == 0u) return 0u;
        const Piece p = make_piece(static_cast<const uint8_t *>(src), len);
        const uint64_t a = reinterpret_cast<uint64_t>(p.src);
        w[k] = make_uint4(uint32_t(a), uint32_t(a >> 32), p.alloc, dst);
        total += p.alloc;
        return p.alloc;
    };
    put(0, desc + b, uint32_t(sizeof(BlockDesc)), 0u);
    if (!BF16IN && (km | vm) != 0 && n > 0) put(1, b7 + size_t(d.b7_block) * D, uint32_t(4 * D), uint32_t(C::S_B7));
    int rel[2] = {0, 0};
    uint32_t staged = 0;
    for (int T = 0; T < 2 && n > 0; ++T) {
        const uint8_t *blk = reinterpret_cast<const uint8_t *>(T ? d.v : d.k);
        const int mode = T ? vm : km;
        const uint32_t reg = uint32_t(C::S_T + T * C::T_BYTES);
        if (BF16IN) {
            put(2 + 3 * T, blk + size_t(t0) * 2 * D, uint32_t(n * 2 * D), reg);
        } else if (mode == 0) {
            put(2 + 3 * T, blk + kHeaderBytes + size_t(t0) * 2 * D, uint32_t(n * 2 * D), reg);
        } else {
            // rows, with the codes when the stage is the whole block (they follow the rows); `end`:
            // the first free byte of the tensor's region after them (16-byte aligned)
            uint32_t end = reg + put(2 + 3 * T, blk + kHeaderBytes + D + size_t(t0) * D,
                                     uint32_t(n * D + (whole ? n * D * mode / 8 : 0)), reg);
            if (!whole)
                end = reg + uint32_t(C::CODE_OFF) +
                      put(3 + 3 * T, blk + kHeaderBytes + D + size_t(n_tok) * D + size_t(t0) * D * mode / 8,
                          uint32_t(n * D * mode / 8), reg + uint32_t(C::CODE_OFF));
            // the escape-record entries go right behind, when they fit in the region (narrower codes
            // leave more room: a 2-bit stage of the compact ring takes about three times the entries
            // of a 4-bit one); otherwise the consumers read them from HBM
            const int e0 = esc_ms(d, T, t0 >> 4), e1 = esc_ms(d, T, min(16, (t0 + C::TSB) >> 4));
            if (e1 > e0) {
                const uint32_t r = T ? d.v_rec : d.k_rec;
                const uint32_t *src = esc + r + kEscRecHead + e0;
                const uint32_t len = uint32_t(4 * (e1 - e0));
                if (end + make_piece(reinterpret_cast<const uint8_t *>(src), len).alloc <= reg + uint32_t(C::T_BYTES)) {
                    put(4 + 3 * T, src, len, end);
                    rel[T] = int(end + esc_rec_line(r, e0)) - 4 * e0;
                    staged |= 1u << T;
                }
            }
        }
    }
    w[8] = make_uint4(uint32_t(rel[0]), uint32_t(rel[1]), total, staged);
    uint4 *out = table + size_t(i) * kStageRecWords;
#pragma unroll
    for (int k = 0; k < kStageRecWords; ++k) out[k] = w[k];
}

template <int D>
cudaError_t stage_table_d(bool bf16, bool compact, const BlockDesc *desc, const uint32_t *b7, const uint32_t *esc,
                          int64_t n_blocks, int spb, uint4 *table, cudaStream_t s) {
    const int64_t n = n_blocks * spb;
    if (n <= 0) return cudaSuccess;
    const unsigned grid = unsigned((n + 127) / 128);
    if (bf16)
        stage_table_kernel<D, false, true><<<grid, 128, 0, s>>>(desc, b7, esc, n_blocks, spb, table);
    else if (compact)
        stage_table_kernel<D, true, false><<<grid, 128, 0, s>>>(desc, b7, esc, n_blocks, spb, table);
    else
        stage_table_kernel<D, false, false><<<grid, 128, 0, s>>>(desc, b7, esc, n_blocks, spb, table);
    return cudaGetLastError();
}

// ---- block descriptors ---------------------------------------------------------------------------

__global__ void block_desc_kernel(const UnitDev *units, const FlatBlock *flat, const uint32_t *esc, int64_t n,
                                  int dim, bool bf16, BlockDesc *desc) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const FlatBlock f = flat[i];
    const UnitDev &U = units[f.unit];
    BlockDesc d = {};
    d.k_rec = f.k_rec;
    d.v_rec = f.v_rec;
    d.k_nesc = f.k_nesc;
    d.v_nesc = f.v_nesc;
    d.k_mode = bf16 ? 0 : f.k_mode;
    d.v_mode = bf16 ? 0 : f.v_mode;
    d.n_tok = f.n_tok;
    d.valid = f.valid;
    d.unit = f.unit;
    d.flags = uint8_t((i == U.block_begin ? kDescFirst : 0) | (i + 1 == U.block_begin + U.n_blocks ? kDescLast : 0));
    d.b7_block = f.src;
    for (int T = 0; T < 2; ++T) {
        const uint8_t *blob = T ? U.v : U.k;
        const uint32_t off = T ? f.v_off : f.k_off;
        const int mode = T ? d.v_mode : d.k_mode;
        const uint8_t *blk = bf16 ? blob + size_t(off) * 2 * dim : blob + off;
        const uint8_t *rows = bf16 ? blk : blk + kHeaderBytes + (mode != 0 ? dim : 0);
        const uint8_t *codes = rows + size_t(f.n_tok) * dim;
        (T ? d.v : d.k) = reinterpret_cast<uint64_t>(blk);
        d.align[2 * T] = uint8_t(reinterpret_cast<uintptr_t>(rows) & 15u);
        d.align[2 * T + 1] = mode != 0 ? uint8_t(reinterpret_cast<uintptr_t>(codes) & 15u) : uint8_t(0);
        const int nesc = T ? f.v_nesc : f.k_nesc;
        const uint32_t rec = T ? f.v_rec : f.k_rec;
        if (mode != 0 && nesc != 0)
            for (int j = 0; j < 16; ++j) d.em[T][j] = uint16_t(esc[rec + j]);
    }
    desc[i] = d;
}

// One warp per flat block: the merge words of its coded K and V (zeros for a raw tensor).  Blocks
// that share another block's K/V (src != itself) have none of their own.
__global__ void b7_kernel(const UnitDev *units, const FlatBlock *flat, int64_t n, int dim, uint32_t *b7) {
    const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= n) return;
    const FlatBlock f = flat[i];
    if (int64_t(f.src) != i) return;
    const UnitDev &U = units[f.unit];
    for (int T = 0; T < 2; ++T) {
        const int mode = T ? f.v_mode : f.k_mode;
        const uint16_t *base = reinterpret_cast<const uint16_t *>((T ? U.v : U.k) + (T ? f.v_off : f.k_off) + kHeaderBytes);
        uint32_t *w = b7 + size_t(i) * dim + size_t(T) * (dim / 2);
        for (int j = lane; j < dim / 2; j += 32) {
            const uint32_t x = mode != 0 ? uint32_t(__ldg(base + j)) : 0u;  // base[2j] | base[2j + 1] << 8
            w[j] = ((x & 0xFFu) << 7) | ((x >> 8) << 23);
        }
    }
}

// m = -inf and l = 0 in every partial state (its first 16 floats), so that a state no warp writes
// adds nothing in the combine pass.
__global__ void init_partials_kernel(float *partials, int64_t n_states, int stride) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n_states * 16) return;
    const int64_t st = i >> 4;
    const int f = int(i & 15);
    partials[st * stride + f] = f < 8 ? -INFINITY : 0.f;
}

// The largest number of attended tokens of any flat block (atomic max into out[0]) and whether any
// block has a raw K or V (out[1] != 0); both set to 0 first.
__global__ void max_valid_kernel(const FlatBlock *flat, int64_t n, int *out) {
    int m = 0, raw = 0;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const FlatBlock f = load_flat(flat, i);
        m = max(m, int(f.valid));
        raw |= (f.k_mode == 0 || f.v_mode == 0) ? 1 : 0;
    }
    m = __reduce_max_sync(FULL, m);
    raw = __reduce_or_sync(FULL, raw);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(out, m);
        if (raw) atomicOr(out + 1, 1);
    }
}

template <int D, bool CP, bool BF16IN>
cudaError_t launch_d(const AttnArgs &a, int grid, cudaStream_t s) {
    configure<D, CP, BF16IN>();
    // programmatic dependent launch: the grid may be set up while the kernel before it in the
    // stream drains (the kernel waits for that grid before it reads anything)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Cfg<D, CP>::THREADS);
    cfg.dynamicSmemBytes = size_t(Cfg<D, CP>::SMEM);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_kernel<D, CP, BF16IN>, a);
}

template <int D>
cudaError_t launch_dim(bool bf16, bool compact, const AttnArgs &a, int grid, cudaStream_t s) {
    if (bf16) return launch_d<D, false, true>(a, grid, s);
    if (compact) return launch_d<D, true, false>(a, grid, s);
    return launch_d<D, false, false>(a, grid, s);
}

}  // namespace

bool attention_dim_supported(int dim) {
    return dim == 32 || dim == 64 || dim == 128 || dim == 256;
}

cudaError_t launch_attention(int dim, bool bf16_input, bool compact, const AttnArgs &a, int grid,
                             cudaStream_t s) {
    switch (dim) {
    case 32: return launch_dim<32>(bf16_input, compact, a, grid, s);
    case 64: return launch_dim<64>(bf16_input, compact, a, grid, s);
    case 128: return launch_dim<128>(bf16_input, compact, a, grid, s);
    case 256: return launch_dim<256>(bf16_input, compact, a, grid, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_split(const FlatBlock *flat, int64_t n_blocks, int n_ranges, bool by_tokens, int dim,
                         int64_t *range_begin, cudaStream_t s) {
    // a unit start costs about 1.5 blocks of 128 tokens at dim 64 (2 x 4 per token and tensor), and
    // about as much time at other widths (its query loads and flushes are latency-bound)
    const uint64_t unit_cost = (by_tokens ? 192u : 1536u) * 64u / uint64_t(dim > 0 ? dim : 64);
    split_kernel<<<1, 1024, 0, s>>>(flat, n_blocks, n_ranges, by_tokens, unit_cost, range_begin);
    return cudaGetLastError();
}

cudaError_t launch_init_partials(float *partials, int64_t n_states, int dim, cudaStream_t s) {
    const int64_t n = n_states * 16;
    if (n <= 0) return cudaSuccess;
    init_partials_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(partials, n_states, partial_stride(dim));
    return cudaGetLastError();
}

cudaError_t launch_max_valid(const FlatBlock *flat, int64_t n_blocks, int *out, cudaStream_t s) {
    if (n_blocks <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(out, 0, 2 * sizeof(int), s);
    if (e != cudaSuccess) return e;
    const int64_t grid = (n_blocks + 255) / 256 < 1024 ? (n_blocks + 255) / 256 : 1024;
    max_valid_kernel<<<unsigned(grid), 256, 0, s>>>(flat, n_blocks, out);
    return cudaGetLastError();
}

cudaError_t launch_fold(const float *parts, int n_parts, int n_rows, int dim, float *out,
                        float *lse_out, cudaStream_t s) {
    fold_kernel<<<n_rows, dim < 256 ? dim : 256, 0, s>>>(parts, n_parts, n_rows, dim, out, lse_out);
    return cudaGetLastError();
}

cudaError_t launch_combine(int dim, const CombineArgs &a, int n_split, cudaStream_t s) {
    if (n_split <= 0) return cudaSuccess;
    // (split unit, query); units hold at most 8 queries.  Programmatic dependent launch: the grid
    // may be set up while the attention grid before it drains (the kernel waits for it).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_split, 8);
    cfg.blockDim = dim3(kCombineThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (dim) {
    case 32: return cudaLaunchKernelEx(&cfg, combine_kernel<32>, a);
    case 64: return cudaLaunchKernelEx(&cfg, combine_kernel<64>, a);
    case 128: return cudaLaunchKernelEx(&cfg, combine_kernel<128>, a);
    case 256: return cudaLaunchKernelEx(&cfg, combine_kernel<256>, a);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_b7(const UnitDev *units, const FlatBlock *flat, int64_t n_blocks, int dim,
                      uint32_t *b7, cudaStream_t s) {
    if (n_blocks <= 0) return cudaSuccess;
    b7_kernel<<<unsigned((n_blocks + 7) / 8), 256, 0, s>>>(units, flat, n_blocks, dim, b7);
    return cudaGetLastError();
}

cudaError_t launch_stage_table(int dim, bool bf16, bool compact, const BlockDesc *desc, const uint32_t *b7,
                               const uint32_t *esc, int64_t n_blocks, int stages_per_block,
                               uint4 *table, cudaStream_t s) {
    switch (dim) {
    case 32: return stage_table_d<32>(bf16, compact, desc, b7, esc, n_blocks, stages_per_block, table, s);
    case 64: return stage_table_d<64>(bf16, compact, desc, b7, esc, n_blocks, stages_per_block, table, s);
    case 128: return stage_table_d<128>(bf16, compact, desc, b7, esc, n_blocks, stages_per_block, table, s);
    case 256: return stage_table_d<256>(bf16, compact, desc, b7, esc, n_blocks, stages_per_block, table, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_block_desc(const UnitDev *units, const FlatBlock *flat, const uint32_t *esc, int64_t n,
                              int dim, bool bf16, BlockDesc *desc, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    block_desc_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(units, flat, esc, n, dim, bf16, desc);
    return cudaGetLastError();
}

}  // namespace kvx
