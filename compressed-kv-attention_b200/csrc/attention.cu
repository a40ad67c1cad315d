// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened; each worker warp owns a contiguous range and
//    streams stages of TS tokens of K and V through its own shared-memory ring: sign/mantissa
//    rows, packed exponent residuals, and the stage's escape words with their tile slots -- or raw
//    BF16 rows.  The pieces arrive as 1-D bulk copies of the TMA engine, issued in parallel by
//    ten lanes and completing on the ring slot's mbarrier.  A block's base exponents ride along
//    with its first stage.  Only the compressed bytes cross HBM (plus, for a coded block with
//    escapes, its escape record: 2 bytes per escape word and a 32-byte count header, built once
//    per plan), and no warp ever waits on another warp.
//  * Each lane rebuilds 8-element chunks of a stage's rows into BF16 words and stores them, 16
//    bytes at a time, into the warp's tile: TS rows of D BF16 values with 16-byte chunks swizzled
//    so that neither those stores nor the ldmatrix reads of the MMA conflict on shared-memory
//    banks.  A pair of elements costs four instructions: two byte permutes (sign/mantissa bytes;
//    exponent residuals), one multiply-add that adds the residual to the base exponent, and one
//    bit-select.  A block's sections start 0 or 2 bytes past a 4-byte boundary of the ring (every
//    size and offset in an XKV blob is even); the permutes take that shift in their selectors.
//  * Escape words are stored over their elements of the tile: one 16-bit store each, at the slot
//    the block's escape record gives.
//  * S = K Q^T runs on the tensor cores (mma.sync m16n8k16, tokens x queries, fp32 accumulate)
//    with K fragments from ldmatrix; the online softmax runs on the S fragments of a whole stage:
//    lane (g, t) holds queries 2t and 2t+1, which are also the output columns it accumulates, so
//    the rescale factors never leave the lane.  O^T += V^T P^T reads V^T with ldmatrix.trans; P^T
//    enters split into a bf16 part and a bf16 residual part (two MMAs), with 16 significant bits.
//  * Unit segments that span several workers leave (m, l, acc) partial states that combine_kernel
//    folds in worker order with merge_state semantics (src/softmax.hpp:16-30), then finalizes like
//    finalize_state (src/softmax.hpp:32-41: reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template reading [seq, dim] BF16 rows into the same
// tile; for the same blocks and worker ranges it produces bit-identical outputs to the XKV variant,
// because the tensor cores see identical BF16 tiles and everything after them is the same code.
// (Ranges are one block per worker whenever the step has no more blocks than workers; beyond
// that they are balanced by cost.)
#include "attention.cuh"

namespace kvx {
namespace {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int TT = 16;  // tokens per MMA tile (one m16 block of the QK MMA)
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
__host__ __device__ constexpr int cmin(int a, int b) { return a < b ? a : b; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

#ifndef KVX_MAXWARPS
#define KVX_MAXWARPS 12
#endif
template <int D> struct Cfg {
    static constexpr int KS = D / 16;             // k-steps of QK = M-tiles of PV
    static constexpr int TS = stage_tokens(D);    // tokens per ring stage
    static constexpr int SUBS = TS / TT;          // MMA tiles per stage
    static constexpr int C8 = D / 8;              // 8-element chunks per row
    static constexpr int NIT = TS * C8 / 32;      // chunk steps of a lane per stage and tensor
    // One tensor's stage: sign/mantissa rows | residual codes | escape record entries, or TS raw
    // BF16 rows -- both fit 2 TS D bytes (escapes beyond ESC_CAP stay in HBM).
    static constexpr int ESC_CAP = TS * D / 8;
    static constexpr int CODE_OFF = TS * D + 16;
    static constexpr int EE_OFF = CODE_OFF + TS * D / 2 + 16;
    static constexpr int TR = round16(cmax(EE_OFF + 4 * ESC_CAP + 16, TS * 2 * D + 16));
    // Ring of tensor-stages: K of stage s, V of stage s, K of stage s + 1, ...  A slot is free
    // again once its tensor is in the tile, so three slots keep one stage of copies in flight.
    static constexpr int NSLOT = 3;
    static constexpr int BASE = round16(D + 32);  // one block's base exponents (+ alignment slack)
    static constexpr int MSLOT = 2 * BASE;        // per-block meta slot: K base | V base
    static constexpr int XB = TS * 2 * D;         // the BF16 tile of one tensor's stage
    static constexpr int NDESC = 4;               // block descriptor ring
    // per-warp region: ring | meta x2 | tile | descriptors | one mbarrier per ring slot and
    // per descriptor
    static constexpr int W_META = NSLOT * TR;
    static constexpr int W_XB = W_META + 2 * MSLOT;
    static constexpr int W_DESC = W_XB + XB;
    static constexpr int W_BAR = W_DESC + NDESC * int(sizeof(BlockDesc));
    static constexpr int W_DBAR = W_BAR + 8 * NSLOT;
    static constexpr int WARP_BYTES = (W_DBAR + 8 * NDESC + 127) & ~127;
    static constexpr int MAXW = D <= 32 ? 16 : KVX_MAXWARPS;
    static constexpr int WARPS = cmin(MAXW, 232448 / WARP_BYTES);
    static_assert(WARPS >= 1, "worker does not fit in shared memory");
    static_assert(32 % C8 == 0 && NIT >= 1, "a warp step covers whole rows");
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

// Section pointers of one tensor of one block.
struct Sections {
    const uint8_t *rows;   // coded: sign/mantissa rows; raw / BF16: BF16 rows
    const uint8_t *codes;  // coded: packed residual codes
    const uint8_t *esc;    // coded: escape words
};

// blk: the block's header (BF16 input: its first row).
template <int D, bool BF16IN>
__device__ __forceinline__ Sections sections(const uint8_t *blk, int mode, int n_tok) {
    Sections s;
    if (BF16IN) {
        s.rows = blk;
        s.codes = s.esc = nullptr;
    } else if (mode == 0) {
        s.rows = blk + kHeaderBytes;
        s.codes = s.esc = nullptr;
    } else {
        s.rows = blk + kHeaderBytes + D;
        s.codes = s.rows + size_t(n_tok) * D;
        s.esc = s.codes + size_t(n_tok) * D * mode / 8;
    }
    return s;
}

// ---- escape records ----------------------------------------------------------------------------

// e(i) of tensor T (0 K, 1 V), i = 0..16; every lane of the warp calls it.
__device__ __forceinline__ int esc_at(uint32_t em, int T, int i) {
    const uint32_t v = __shfl_sync(FULL, em, (T << 4) + ((i + 15) & 15));
    return i == 0 ? 0 : int(v);
}

// e(i) of tensor T from a block descriptor's headers.
__device__ __forceinline__ int esc_ms(const BlockDesc &bd, int T, int i) {
    return i == 0 ? 0 : int(bd.em[T][i - 1]);
}

// Byte offset inside a 16-byte line of entry i of the escape record at `rec` (the record array is
// 16-byte aligned).
__device__ __forceinline__ uint32_t esc_rec_line(uint32_t rec, int i) {
    return (4u * (rec + uint32_t(kEscRecHead) + uint32_t(i))) & 15u;
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
// (head dims 8 c8 .. 8 c8 + 7) of rows t0 + RPI k.  Row sections start m = 0 or 2 bytes past a
// 4-byte boundary of the ring; the chunk adds a multiple of 4 to the sign/mantissa and raw rows,
// and 4 (4-bit) or 2 (2-bit) bytes per chunk to the residual rows.
struct Lay {
    uint32_t p0, p1;  // sign/mantissa bytes of element pairs 2q and 2q+1 from words q, q+1
    uint32_t w;       // one realigned word from two loaded ones (raw rows)
    uint32_t cs;      // one realigned word of residual codes
    uint32_t rows;    // byte offset of the lane's row window in the stage (4-aligned)
    uint32_t codes;   // byte offset of the lane's residual window in the stage (4-aligned)
};
// rd / cd: data offsets of the block's row and code pieces.
template <int D>
__device__ __forceinline__ Lay make_lay(uint32_t rd, uint32_t cd, int mode, int c8, bool bf16) {
    Lay l;
    const uint32_t m = rd & 3u;
    l.p0 = rep2(m);
    l.p1 = rep2(m + 2);
    l.w = shift4(m);
    l.rows = (rd & ~3u) + uint32_t((bf16 || mode == 0) ? 16 * c8 : 8 * c8);
    const uint32_t cb = (cd & 3u) + uint32_t(c8 * (mode == 0 ? 0 : mode));
    l.cs = shift4(cb & 3u);
    l.codes = uint32_t(Cfg<D>::CODE_OFF) + (cd & ~3u) + (cb & ~3u);
    return l;
}

// b7 of the lane's four dim pairs (c, c+1): base[c] << 7 | base[c+1] << 23.  `base` is the
// shared address of base[8 c8].
__device__ __forceinline__ void load_b7(uint32_t base, uint32_t (&b7)[4]) {
    const uint32_t m = base & 3u, q = base - m;
    const uint32_t B0 = lds_u32(q), B1 = lds_u32(q + 4u), B2 = lds_u32(q + 8u);
    const uint32_t s0 = rep2(m), s1 = rep2(m + 2);
    b7[0] = (prmt(B0, B1, s0) & 0x00FF00FFu) << 7;
    b7[1] = (prmt(B0, B1, s1) & 0x00FF00FFu) << 7;
    b7[2] = (prmt(B1, B2, s0) & 0x00FF00FFu) << 7;
    b7[3] = (prmt(B1, B2, s1) & 0x00FF00FFu) << 7;
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
            if constexpr (MODE == 4) X[g][1] = lds_u32(c + 4u);
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

// Chunk steps [K0, NIT) in groups of G: the loads of the next group are issued before the
// current group's arithmetic and stores (the shared-memory accesses keep their written order).
template <int D, int MODE, int G, int K0>
__device__ __forceinline__ void decode_groups(uint32_t qr, uint32_t qc, const Lay &ly, const uint32_t (&b7)[4],
                                              const StoreMap<D> &sm, uint32_t (&W)[G][MODE == 0 ? 5 : 3],
                                              uint32_t (&X)[G][2]) {
    constexpr int NIT = Cfg<D>::NIT;
    uint32_t Wn[G][MODE == 0 ? 5 : 3], Xn[G][2];
    if constexpr (K0 + G < NIT) load_chunks<D, MODE, G, K0 + G>(qr, qc, Wn, Xn);
    uint32_t w[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) build_chunk<MODE>(ly, b7, W[g], X[g], w[g]);
#pragma unroll
    for (int g = 0; g < G; ++g) sts_v4(sm.at(K0 + g), w[g][0], w[g][1], w[g][2], w[g][3]);
    if constexpr (K0 + G < NIT) decode_groups<D, MODE, G, K0 + G>(qr, qc, ly, b7, sm, Wn, Xn);
}

// Rebuild this lane's chunks of one tensor's stage into the tile (MODE 4 / 2 coded, 0 raw BF16).
template <int D, int MODE>
__device__ __forceinline__ void decode_stage(uint32_t stage, const Lay &ly, const uint32_t (&b7)[4],
                                             const StoreMap<D> &sm, int lane) {
    using C = Cfg<D>;
    // chunk steps per group (two groups' loads are live at a time)
    constexpr int G = C::NIT < 4 ? C::NIT : 4;
    const int r0 = lane / C::C8;
    const uint32_t qr = stage + ly.rows + uint32_t(r0 * (MODE == 0 ? 2 * D : D));
    const uint32_t qc = stage + ly.codes + uint32_t(r0 * (D * MODE / 8));
    uint32_t W[G][MODE == 0 ? 5 : 3], X[G][2];
    load_chunks<D, MODE, G, 0>(qr, qc, W, X);
    decode_groups<D, MODE, G, 0>(qr, qc, ly, b7, sm, W, X);
}

// Zero this lane's chunks of tile rows at or past `from` (V rows past the block's valid tokens:
// P is 0 there and V must be finite).
template <int D, int J = 0>
__device__ __forceinline__ void zero_rows(const StoreMap<D> &sm, int from, int lane) {
    if constexpr (J < Cfg<D>::NIT) {
        if (lane / Cfg<D>::C8 + J * StoreMap<D>::RPI >= from) sts_v4(sm.at(J), 0u, 0u, 0u, 0u);
        zero_rows<D, J + 1>(sm, from, lane);
    }
}

// Store escapes [e0, e1) of a block over their elements of the stage's tile: record entry i (tile
// byte | escape word << 16) is the u32 at ents + 4 i -- a shared address of the staged copy, or
// (HBM variant) the record in global memory.  Slots at or past the stage's valid rows (lim bytes)
// are skipped; slots are even.
template <int D>
__device__ __forceinline__ void esc_patch(uint32_t xb, uint32_t ents, int e0, int e1, uint32_t lim, int lane) {
    for (int i = e0 + lane; i < e1; i += 32) {
        const uint32_t e = lds_u32(ents + 4u * uint32_t(i));
        if ((e & 0xFFFFu) < lim) sts_u16(xb + (e & 0xFFFEu), e >> 16);
    }
}
template <int D>
__device__ __noinline__ void esc_patch_hbm(uint32_t xb, const uint32_t *ents, int e0, int e1, uint32_t lim,
                                           int lane) {
    for (int i = e0 + lane; i < e1; i += 32) {
        const uint32_t e = __ldg(ents + i);
        if ((e & 0xFFFFu) < lim) sts_u16(xb + (e & 0xFFFEu), e >> 16);
    }
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

// O^T += V^T P^T for the 16-token tile at tile row r0 (P^T as B fragments: bh = bf16(p),
// bm = bf16(p - bh), bl = bf16(p - bh - bm): three bf16 terms carry p's 24 significant bits, so the
// tensor cores see the fp32 softmax weight exactly).  V^T A fragments by ldmatrix.trans: matrix i
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

// ---- the worker -------------------------------------------------------------------------------

__device__ __forceinline__ const uint8_t *desc_ptr(uint64_t a) { return reinterpret_cast<const uint8_t *>(a); }

// Copy side of the worker's ring.  Block descriptors arrive in a ring of NDESC slots, fetched one
// block ahead of their first stage (block fb0 + i uses slot i % NDESC); the producer reads a block's descriptor when
// it issues the block's first stage, the consumer while it works on the block.
template <int D, bool BF16IN> struct Producer {
    using C = Cfg<D>;
    int fb, fb0, fb1;  // next block to start; the worker's range
    int pf;            // next block whose descriptor is fetched
    int dwait;         // next block whose descriptor is waited for
    int tile = 0, q = 0, bseq = 0;  // q: tensor-stages issued (2 per stage, K first)
    int valid = 0;     // tokens of the block being issued
    uint32_t em = 0u;  // lane l: entry l % 16 of its K (l < 16) / V count header
    // This lane's piece of every stage of the current block.  Lane 4 T + j (j < 4) copies piece j
    // of tensor T: rows (j 0) and residual codes (j 1) are [src + t0 stride, + n stride) for the
    // stage's tokens [t0, t0 + n); the escape record entries (j 2) of the stage's escapes
    // [e0, e1) are at src + 4 e0, copied when they fit the slot.  Lanes 8 and 9 copy the K and V base
    // exponents (D bytes at src) with the block's first stage.  dst: offset in the ring slot or
    // (base exponents) in the meta slot.
    const uint8_t *src = nullptr;
    uint32_t stride = 0, dst = 0;
    int kind = 0;  // 0 none, 1 strided, 2 escapes, 3 base exponents

    // Fetch descriptors up to the block after the next one to start (lane 0 issues).  A block
    // starts when the consumer is at most one block behind, so the slot a fetch overwrites (its
    // block four earlier) is no longer read.
    __device__ __forceinline__ void fetch(const AttnArgs &a, uint8_t *R, int lane) {
        while (pf < fb1 && pf <= fb + 1) {
            const int i = (pf - fb0) % C::NDESC;
            const uint32_t bar = smem_u32(R + C::W_DBAR + 8 * i);
            if (lane == 0) {
                mbar_arrive_expect_tx(bar, uint32_t(sizeof(BlockDesc)));
                bulk_g2s(smem_u32(R + C::W_DESC + i * int(sizeof(BlockDesc))),
                         reinterpret_cast<const uint8_t *>(a.desc + pf), uint32_t(sizeof(BlockDesc)), bar);
            }
            ++pf;
        }
    }

    __device__ __forceinline__ bool start_block(const AttnArgs &a, uint8_t *R, int lane) {
        const int i = (fb - fb0) % C::NDESC;
        if (!uni(mbar_wait_bounded(smem_u32(R + C::W_DBAR + 8 * i), ((fb - fb0) / C::NDESC) & 1, kStageWaitUs)))
            return false;
        dwait = fb + 1;
        const BlockDesc &bd = *reinterpret_cast<const BlockDesc *>(R + C::W_DESC + i * int(sizeof(BlockDesc)));
        const int T = (lane >> 2) & 1, j = lane & 3;
        const int km = BF16IN ? 0 : bd.k_mode, vm = BF16IN ? 0 : bd.v_mode;
        const int mode = T ? vm : km;
        const uint8_t *blk = desc_ptr(T ? bd.v : bd.k);
        const Sections sc = sections<D, BF16IN>(blk, mode, bd.n_tok);
        valid = bd.valid;
        em = bd.em[lane >> 4][lane & 15];
        src = nullptr;
        stride = 0;
        kind = 0;
        dst = 0u;
        if (lane < 8) {
            if (j == 0) {
                src = sc.rows;
                stride = (BF16IN || mode == 0) ? 2 * D : D;
                kind = 1;
            } else if (!BF16IN && mode != 0) {
                if (j == 1) {
                    src = sc.codes;
                    stride = uint32_t(D * mode / 8);
                    dst += C::CODE_OFF;
                    kind = 1;
                } else if (j == 2) {
                    src = reinterpret_cast<const uint8_t *>(a.esc + (T ? bd.v_rec : bd.k_rec) + kEscRecHead);
                    dst += C::EE_OFF;
                    kind = 2;
                }
            }
        } else if (!BF16IN && lane < 10 && (lane == 8 ? km : vm) != 0) {
            src = desc_ptr(lane == 8 ? bd.k : bd.v) + kHeaderBytes;
            dst = uint32_t((lane - 8) * C::BASE);
            kind = 3;
        }
        return true;
    }

    // Issue tensor-stages while a ring slot is free (the consumer is done with every one before
    // c_q); a block start waits until the consumer is at most one block behind, so a meta slot is
    // never overwritten while in use.  A slot's previous tensor was read by the whole warp before
    // this call (__syncwarp after every tensor's decode).  The pieces of a tensor-stage go out in
    // parallel, one bulk copy per lane (lanes 4 T .. 4 T + 2, and 8 and 9 with a block's first K);
    // lane 0 first tells the slot's barrier how many bytes to expect.  False when a descriptor
    // did not arrive in time.
    __device__ __forceinline__ bool produce(const AttnArgs &a, uint8_t *R, int c_q, int c_fb, int lane) {
        while (fb < fb1 && q - c_q < C::NSLOT) {
            const int T = q & 1;
            if (T == 0 && tile == 0) {
                if (fb - c_fb >= 2) break;
                if (!start_block(a, R, lane)) return false;
            }
            const int slot = q % C::NSLOT;
            const uint32_t bar = smem_u32(R + C::W_BAR + 8 * slot);
            const uint32_t ms = smem_u32(R + C::W_META + (bseq & 1) * C::MSLOT);
            const int t0 = tile * C::TS;
            const int n = min(C::TS, valid - t0);
            const int LT = (lane >> 2) & 1;  // the tensor of lanes 0-7's pieces
            const int e0 = esc_at(em, LT, t0 >> 4), e1 = esc_at(em, LT, min(16, (t0 + C::TS) >> 4));
            const bool now = lane < 8 ? LT == T : (T == 0 && tile == 0);
            const uint8_t *p;
            uint32_t len;
            if (kind == 2) {
                p = src + 4 * e0;
                len = e1 - e0 <= C::ESC_CAP ? uint32_t(4 * (e1 - e0)) : 0u;
            } else {
                p = src + size_t(t0) * stride;
                len = kind == 1 ? uint32_t(n) * stride : (kind == 3 ? uint32_t(D) : 0u);
            }
            if (!now) len = 0u;
            const uint32_t d = kind == 3 ? ms + dst : smem_u32(R + slot * C::TR) + dst;
            const Piece pc = make_piece(p, len);
            const uint32_t bytes = len != 0 ? pc.alloc : 0u;
            const uint32_t total = __reduce_add_sync(FULL, bytes);
            fence_proxy_async();
            if (lane == 0) mbar_arrive_expect_tx(bar, total);
            __syncwarp();
            if (bytes != 0) bulk_g2s(d, pc.src, bytes, bar);
            ++q;
            if (T == 1) {
                if (t0 + C::TS >= valid) {
                    tile = 0;
                    ++bseq;
                    ++fb;
                    fetch(a, R, lane);
                } else {
                    ++tile;
                }
            }
        }
        return true;
    }
};

// One tensor of a stage into the tile, escapes included.
template <int D>
__device__ __forceinline__ void stage_tile(const AttnArgs &a, const BlockDesc &bd, int T, int mode,
                                           uint32_t tstage, uint32_t xb, const StoreMap<D> &sm, const Lay &ly,
                                           const uint32_t (&b7)[4], int ia, int ib, int rows,
                                           int zero_from, int lane) {
    if (mode == 4) decode_stage<D, 4>(tstage, ly, b7, sm, lane);
    else if (mode == 2) decode_stage<D, 2>(tstage, ly, b7, sm, lane);
    else decode_stage<D, 0>(tstage, ly, b7, sm, lane);
    if (zero_from < Cfg<D>::TS) zero_rows<D>(sm, zero_from, lane);
    const int e0 = esc_ms(bd, T, ia), e1 = esc_ms(bd, T, ib);
    if (e1 > e0) {
        using C = Cfg<D>;
        const uint32_t rec = T ? bd.v_rec : bd.k_rec;
        const uint32_t lim = uint32_t(rows) * (2 * D);
        __syncwarp();  // the decoded words are in place before escapes overwrite some
        if (e1 - e0 <= C::ESC_CAP)  // staged by the producer
            esc_patch<D>(xb, tstage + C::EE_OFF + esc_rec_line(rec, e0) - 4u * uint32_t(e0), e0, e1, lim, lane);
        else
            esc_patch_hbm<D>(xb, a.esc + rec + kEscRecHead, e0, e1, lim, lane);
    }
    __syncwarp();
}

template <int D, bool BF16IN>
__device__ __forceinline__ void worker(const AttnArgs &a, uint8_t *R, int wk, int fb0, int fb1,
                                       int lane) {
    using C = Cfg<D>;
    const int gi = lane >> 2, tig = lane & 3, c8 = lane % C::C8;
    uint8_t *ring = R;
    uint8_t *metas = R + C::W_META;
    const uint32_t xb = smem_u32(R + C::W_XB);
    uint8_t *bars = R + C::W_BAR;
    StoreMap<D> smap;
    smap.init(xb, lane);
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j < C::NSLOT; ++j) mbar_init(smem_u32(bars + 8 * j), 1);
#pragma unroll
        for (int j = 0; j < C::NDESC; ++j) mbar_init(smem_u32(R + C::W_DBAR + 8 * j), 1);
        fence_mbar_init();
    }
    __syncwarp();
    Producer<D, BF16IN> pp;
    pp.fb = pp.fb0 = pp.pf = pp.dwait = fb0;
    pp.fb1 = fb1;
    pp.fetch(a, R, lane);
    int fb = fb0, tile = 0, cq = 0, bseq = 0;  // cq: the next tensor-stage to consume
    int seg_begin = fb0;
    uint32_t flags = 0u, whole = 0u;  // the block's flags; the segment began at its unit's start
    Lay lk{}, lv{};
    uint32_t b7k[4] = {0u, 0u, 0u, 0u}, b7v[4] = {0u, 0u, 0u, 0u};
    uint32_t qb[C::KS][2];
    float acc[C::KS][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // Tensor-stage q's slot barrier and its phase for that use.
    auto slot_bar = [&](int q) { return smem_u32(bars + 8 * (q % C::NSLOT)); };
    auto slot_par = [&](int q) { return uint32_t((q / C::NSLOT) & 1); };
    // After a timeout: report it and let the copies already issued land before this CTA's
    // shared memory goes away.
    auto fail = [&]() {
        if (lane == 0) report(a.status, KVX_ERR_TIMEOUT, DERR_TIMEOUT);
        for (int q = cq; q < pp.q; ++q) mbar_wait_bounded(slot_bar(q), slot_par(q), kStageWaitUs);
        for (int b = pp.dwait; b < pp.pf; ++b)
            mbar_wait_bounded(smem_u32(R + C::W_DBAR + 8 * ((b - fb0) % C::NDESC)),
                              ((b - fb0) / C::NDESC) & 1, kStageWaitUs);
    };

    while (fb < fb1) {
        if (!pp.produce(a, R, cq, fb, lane) || !uni(mbar_wait_bounded(slot_bar(cq), slot_par(cq), kStageWaitUs))) {
            fail();
            return;
        }
        __syncwarp();
        const uint8_t *ms = metas + (bseq & 1) * C::MSLOT;
        const BlockDesc &bd =
            *reinterpret_cast<const BlockDesc *>(R + C::W_DESC + ((fb - fb0) % C::NDESC) * int(sizeof(BlockDesc)));
        const int kmode = BF16IN ? 0 : bd.k_mode, vmode = BF16IN ? 0 : bd.v_mode;
        const int valid = bd.valid;
        if (tile == 0) {
            const uint32_t al = *reinterpret_cast<const uint32_t *>(bd.align);
            flags = bd.flags;
            const uint32_t kd = al & 15u, kc = (al >> 8) & 15u, vd = (al >> 16) & 15u, vc = (al >> 24) & 15u;
            lk = make_lay<D>(kd, kc, kmode, c8, BF16IN);
            lv = make_lay<D>(vd, vc, vmode, c8, BF16IN);
            if (kmode != 0) load_b7(smem_u32(ms) + kd + 8 * c8, b7k);
            if (vmode != 0) load_b7(smem_u32(ms) + C::BASE + vd + 8 * c8, b7v);
            if (fb == seg_begin) {
                const UnitDev *U = a.units + bd.unit;
                whole = flags & kDescFirst;
                load_q<D>(U->q, U->n_q, U->q_stride, qb, lane);
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
#pragma unroll
                for (int m = 0; m < C::KS; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
            }
        }
        const uint32_t kst = smem_u32(ring + (cq % C::NSLOT) * C::TR);
        const uint32_t vst = smem_u32(ring + ((cq + 1) % C::NSLOT) * C::TR);
        const int t0 = tile * C::TS;
        const int rows = min(C::TS, valid - t0);
        const bool last_tile = t0 + C::TS >= valid;
        const bool seg_end = last_tile && (fb + 1 == fb1 || (flags & kDescLast) != 0u);
        const int ia = t0 >> 4, ib = min(16, (t0 + C::TS) >> 4);

        // S^T = K Q^T for every tile of the stage
        stage_tile<D>(a, bd, 0, kmode, kst, xb, smap, lk, b7k, ia, ib, rows, C::TS, lane);
        ++cq;  // K's slot is free: the next copies can go out while the tensor cores work
        if (!pp.produce(a, R, cq, fb, lane)) {
            fail();
            return;
        }
        // (a stage's rows past `rows` hold stale words: their scores are dropped below)
        float s[C::SUBS][4];
        qk_tiles<D, C::SUBS>(xb, qb, lane, s);
        if (rows < C::TS) {
#pragma unroll
            for (int sub = 0; sub < C::SUBS; ++sub) {
                const int rr = rows - sub * TT;
                if (gi >= rr) s[sub][0] = s[sub][1] = -INFINITY;
                if (gi + 8 >= rr) s[sub][2] = s[sub][3] = -INFINITY;
            }
        }

        // online softmax over the stage's tokens; p = 2^(s log2e - m log2e).  The warp-wide
        // maximum is only taken when some score exceeds the running one; otherwise m stays and
        // the accumulators are not rescaled (alpha is exactly 1).
        float t0m = fmaxf(s[0][0], s[0][2]), t1m = fmaxf(s[0][1], s[0][3]);
#pragma unroll
        for (int sub = 1; sub < C::SUBS; ++sub) {
            t0m = fmaxf(t0m, fmaxf(s[sub][0], s[sub][2]));
            t1m = fmaxf(t1m, fmaxf(s[sub][1], s[sub][3]));
        }
        const bool grow = __any_sync(FULL, t0m > m0 || t1m > m1);
        float mn0 = m0, mn1 = m1, al0 = 1.0f, al1 = 1.0f;
        if (grow) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                t0m = fmaxf(t0m, __shfl_xor_sync(FULL, t0m, o));
                t1m = fmaxf(t1m, __shfl_xor_sync(FULL, t1m, o));
            }
            mn0 = fmaxf(m0, t0m);
            mn1 = fmaxf(m1, t1m);
            al0 = ex2(__fmaf_rn(m0, kLog2e, -__fmul_rn(mn0, kLog2e)));
            al1 = ex2(__fmaf_rn(m1, kLog2e, -__fmul_rn(mn1, kLog2e)));
        }
        const float ml0 = __fmul_rn(mn0, kLog2e), ml1 = __fmul_rn(mn1, kLog2e);
        float ps0 = 0.f, ps1 = 0.f;
        uint32_t bh[C::SUBS][2], bm[C::SUBS][2], bl[C::SUBS][2];
#pragma unroll
        for (int sub = 0; sub < C::SUBS; ++sub) {
            const float p0 = ex2(__fmaf_rn(s[sub][0], kLog2e, -ml0)), p1 = ex2(__fmaf_rn(s[sub][1], kLog2e, -ml1));
            const float p2 = ex2(__fmaf_rn(s[sub][2], kLog2e, -ml0)), p3 = ex2(__fmaf_rn(s[sub][3], kLog2e, -ml1));
            ps0 = __fadd_rn(ps0, __fadd_rn(p0, p2));
            ps1 = __fadd_rn(ps1, __fadd_rn(p1, p3));
            // P^T B fragments: p = h + m + l exactly, h = bf16(p), m = bf16(p - h),
            // l = bf16(p - h - m) (each difference is exact in fp32; 3 x 8 significant bits)
            const uint32_t h01 = pack_bf16x2(p1, p0), h23 = pack_bf16x2(p3, p2);
            const float r0 = __fsub_rn(p0, bf16lo_to_f32(h01)), r1 = __fsub_rn(p1, bf16hi_to_f32(h01));
            const float r2 = __fsub_rn(p2, bf16lo_to_f32(h23)), r3 = __fsub_rn(p3, bf16hi_to_f32(h23));
            const uint32_t m01 = pack_bf16x2(r1, r0), m23 = pack_bf16x2(r3, r2);
            const float u0 = __fsub_rn(r0, bf16lo_to_f32(m01)), u1 = __fsub_rn(r1, bf16hi_to_f32(m01));
            const float u2 = __fsub_rn(r2, bf16lo_to_f32(m23)), u3 = __fsub_rn(r3, bf16hi_to_f32(m23));
            bh[sub][0] = movm_t(h01);
            bh[sub][1] = movm_t(h23);
            bm[sub][0] = movm_t(m01);
            bm[sub][1] = movm_t(m23);
            bl[sub][0] = movm_t(pack_bf16x2(u1, u0));
            bl[sub][1] = movm_t(pack_bf16x2(u3, u2));
        }
        l0 = __fmaf_rn(l0, al0, ps0);
        l1 = __fmaf_rn(l1, al1, ps1);
        m0 = mn0;
        m1 = mn1;
        if (grow) {
#pragma unroll
            for (int m = 0; m < C::KS; ++m) {
                acc[m][0] = __fmul_rn(acc[m][0], al0);
                acc[m][1] = __fmul_rn(acc[m][1], al1);
                acc[m][2] = __fmul_rn(acc[m][2], al0);
                acc[m][3] = __fmul_rn(acc[m][3], al1);
            }
        }

        // O^T += V^T P^T for every tile of the stage (the tile's K reads are done: stage_tile
        // ends with __syncwarp, and the K tiles were read before the softmax)
        if (!uni(mbar_wait_bounded(slot_bar(cq), slot_par(cq), kStageWaitUs))) {
            fail();
            return;
        }
        __syncwarp();
        stage_tile<D>(a, bd, 1, vmode, vst, xb, smap, lv, b7v, ia, ib, rows, rows, lane);
        ++cq;
#pragma unroll
        for (int sub = 0; sub < C::SUBS; ++sub)
            if (sub * TT < rows) pv_tile<D>(xb, sub * TT, bh[sub], bm[sub], bl[sub], lane, acc);

        if (seg_end) {
            float lt0 = l0, lt1 = l1;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                lt0 = __fadd_rn(lt0, __shfl_xor_sync(FULL, lt0, o));
                lt1 = __fadd_rn(lt1, __shfl_xor_sync(FULL, lt1, o));
            }
            const int qa = 2 * tig, qc = 2 * tig + 1;
            // acc[m][0 / 1]: dim 16 m + g of queries qa / qc; acc[m][2 / 3]: dim 16 m + g + 8
            if (whole != 0u && (flags & kDescLast) != 0u) {
                const UnitDev *U = a.units + bd.unit;
                const int n_q = U->n_q, stride = U->q_stride;
                float *out = U->out;
                float *lse = U->lse;
                const float inv0 = __frcp_rn(lt0), inv1 = __frcp_rn(lt1);
                if (lse != nullptr && gi == 0) {
                    if (qa < n_q) lse[qa] = m0 + logf(lt0);
                    if (qc < n_q) lse[qc] = m1 + logf(lt1);
                }
                if (qa < n_q) {
                    float *o = out + size_t(qa) * stride + gi;
#pragma unroll
                    for (int m = 0; m < C::KS; ++m) {
                        o[16 * m] = __fmul_rn(acc[m][0], inv0);
                        o[16 * m + 8] = __fmul_rn(acc[m][2], inv0);
                    }
                }
                if (qc < n_q) {
                    float *o = out + size_t(qc) * stride + gi;
#pragma unroll
                    for (int m = 0; m < C::KS; ++m) {
                        o[16 * m] = __fmul_rn(acc[m][1], inv1);
                        o[16 * m + 8] = __fmul_rn(acc[m][3], inv1);
                    }
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
                float *oa = part + 16 + qa * D + gi;
                float *oc = part + 16 + qc * D + gi;
#pragma unroll
                for (int m = 0; m < C::KS; ++m) {
                    oa[16 * m] = acc[m][0];
                    oa[16 * m + 8] = acc[m][2];
                    oc[16 * m] = acc[m][1];
                    oc[16 * m + 8] = acc[m][3];
                }
            }
        }
        __syncwarp();  // every lane is done with this ring slot and the tile before they are reused
        if (last_tile) {
            tile = 0;
            ++bseq;
            if (seg_end) seg_begin = fb + 1;
            ++fb;
        } else {
            ++tile;
        }
    }
}

template <int D, bool BF16IN>
__global__ void __launch_bounds__(32 * Cfg<D>::WARPS, 1) attn_kernel(const AttnArgs a) {
    using C = Cfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    // Launched as a programmatic dependent of the kernel before it in the stream (the previous
    // step's combine pass, or the plan's descriptor build): nothing is read before that grid has
    // completed and its writes are visible.  Only the launch itself overlaps it.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // A combine pass launched behind this grid (programmatic dependent launch) may start placing
    // its CTAs as soon as SMs free up; it waits for this grid's completion before reading.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // consecutive workers on different SMs: neighbouring ranges often share a cost profile
    const int wk = warp * gridDim.x + blockIdx.x;
    if (wk >= a.n_workers) return;
    // a step whose preparation reported an error (its escape records are incomplete) runs no work
    if (*reinterpret_cast<volatile const int *>(a.status) != 0) return;
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
    const int t0 = sp.first_worker;  // first worker of the unit and the number of workers
    const int nt = min(sp.n_workers, kMaxSegments);
    const int ps = partial_stride(D);
    // only the unit's first worker can hold it in its second partial slot (its range began in an
    // earlier unit); the host worked that out
    auto part = [&](int i) {
        const int t = t0 + i;
        return a.partials + (size_t(t) * 2 + (i == 0 ? sp.first_slot : 0)) * ps;
    };
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
        ls = __fmaf_rn(lw[i], w, ls);
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
    float acc = 0.f;
    if (sl < S) {
#pragma unroll
        for (int k = 0; k < PRE; ++k)
            if (sl + k * S < nt) acc = __fmaf_rn(pre[k], e[sl + k * S], acc);
#pragma unroll 8
        for (int i = sl + PRE * S; i < nt; i += S) acc = __fmaf_rn(__ldg(part(i) + 16 + g * D + d), e[i], acc);
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
// residuals, 5 with 2-bit ones (more unpacking), 2 for raw rows; plus 1 per escape word, which
// costs a lane one staged load and one store.  (Weighting escapes near a token's cost, as an
// earlier model did, starved the workers that hold escape-dense blocks and left the others
// about 10 % more work than a balanced split.)
__device__ __forceinline__ uint64_t mode_cost(int mode) { return mode == 4 ? 4u : (mode == 2 ? 5u : 2u); }
__device__ __forceinline__ uint64_t block_cost(const FlatBlock &b) {
    return uint64_t(b.valid) * (mode_cost(b.k_mode) + mode_cost(b.v_mode)) + uint64_t(b.k_nesc) + b.v_nesc;
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

template <int D>
cudaError_t launch_d(bool bf16, const AttnArgs &a, int grid, cudaStream_t s) {
    configure<D>(bf16);
    // programmatic dependent launch: the grid may be set up while the kernel before it in the
    // stream drains (the kernel waits for that grid before it reads anything)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * Cfg<D>::WARPS);
    cfg.dynamicSmemBytes = size_t(Cfg<D>::WARP_BYTES) * Cfg<D>::WARPS;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (bf16) return cudaLaunchKernelEx(&cfg, attn_kernel<D, true>, a);
    return cudaLaunchKernelEx(&cfg, attn_kernel<D, false>, a);
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

cudaError_t launch_block_desc(const UnitDev *units, const FlatBlock *flat, const uint32_t *esc, int64_t n,
                              int dim, bool bf16, BlockDesc *desc, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    block_desc_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(units, flat, esc, n, dim, bf16, desc);
    return cudaGetLastError();
}

}  // namespace kvx
