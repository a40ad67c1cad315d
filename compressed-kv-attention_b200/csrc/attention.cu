// attention.cu -- fused XKV decode + GQA decode attention for sm_100a.
//
// Hot path of kvexp::attention_decode (reference src/dispatch.cpp:27-104 with the per-token kernels
// src/attention_{scalar,avx2,avx512}.cpp and the online softmax of src/softmax.hpp), restructured
// for the GPU:
//
//  * The step's (unit, block) pairs are flattened; each worker warp owns a contiguous range and
//    streams stages of TS tokens of K and V through its own shared-memory ring with cp.async, one
//    cp.async group per stage: sign/mantissa rows, packed exponent residuals, and the stage's
//    escape words with their element positions -- or raw BF16 rows.  A block's base exponents ride
//    along with its first stage.  Only the compressed bytes cross HBM (plus, for a coded block
//    with escapes, its escape record: 2 bytes per escape word and a 32-byte count header, built
//    once per plan), and no warp ever waits on another warp.
//  * K rows are rebuilt straight into mma.sync A fragments: lane (g, t) rebuilds tokens g and g+8,
//    head dims [t D/4, (t+1) D/4).  The MMA's k index runs over the head dims in that permuted
//    order and the query B fragments use the same order, so S = K Q^T (tokens x queries, fp32
//    accumulate) needs no BF16 tile in shared memory.  A pair of elements costs four instructions:
//    two byte permutes (sign/mantissa bytes; exponent residuals), one multiply-add that adds the
//    residual to the base exponent, and one bit-select.  A block's sections start 0 or 2 bytes
//    past a 4-byte boundary of the ring (every size and offset in an XKV blob is even); the
//    permutes take that shift in their selectors.
//  * The online softmax runs on the S fragments of a whole stage: lane (g, t) holds queries 2t and
//    2t+1, which are also the output columns it accumulates, so the rescale factors never leave
//    the lane.
//  * V rows are rebuilt into A fragments of V^T: lane (g, t) rebuilds tokens 2t, 2t+1, 2t+8, 2t+9,
//    head dims [g D/8, (g+1) D/8).  O^T += V^T P^T with P^T split into a bf16 part and a bf16
//    residual part (two MMAs), so P enters with 16 significant bits.
//  * Exponent escapes: a row half whose tokens hold escape words goes to scratch, each escape word
//    is stored over its element (one 16-bit store, at the position the block's escape record
//    gives) and the half is read back.  Halves without escapes skip all of it.
//  * Unit segments that span several workers leave (m, l, acc) partial states that combine_kernel
//    folds in worker order with merge_state semantics (src/softmax.hpp:16-30), then finalizes like
//    finalize_state (src/softmax.hpp:32-41: reciprocal, then multiply).
//
// The BF16-input variant (BF16IN) is the same template reading [seq, dim] BF16 rows; for the same
// blocks and worker ranges it produces bit-identical outputs to the XKV variant, because both
// rebuild identical BF16 fragments and run identical arithmetic afterwards.  (Ranges are one block
// per worker whenever the step has no more blocks than workers; beyond that they are balanced by
// cost.)
#include "attention.cuh"

namespace kvx {
namespace {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int TT = 16;  // tokens per MMA tile (one m16 block of the QK MMA)
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

#ifndef KVX_MAXWARPS
#define KVX_MAXWARPS 12
#endif

template <int D> struct Cfg {
    static constexpr int DK = D / 4;        // head dims per lane in a K row
    static constexpr int NK = D / 8;        // K fragment registers per row (dim pairs)
    static constexpr int DV = D / 8;        // head dims per lane in a V token (= V registers)
    static constexpr int KS = D / 16;       // k-steps of QK = M-tiles of PV
    static constexpr bool SPLIT = D > 128;  // rebuild and multiply row halves one at a time
    static constexpr int TS = D <= 64 ? 32 : 16;  // tokens per ring stage
    static constexpr int SUBS = TS / TT;          // MMA tiles per stage
    // One tensor's stage: sign/mantissa rows | residual codes | escape words | their positions,
    // or TS raw BF16 rows -- both fit 2 TS D bytes (escapes beyond ESC_CAP stay in HBM).
    static constexpr int ESC_CAP = TS * D / 8;
    static constexpr int CODE_OFF = TS * D + 16;
    static constexpr int EV_OFF = CODE_OFF + TS * D / 2 + 16;
    static constexpr int EP_OFF = EV_OFF + 2 * ESC_CAP + 16;
    static constexpr int TR = round16(cmax(EP_OFF + 2 * ESC_CAP + 16, TS * 2 * D + 16));
    static constexpr int SLOT = 2 * TR;  // K stage | V stage
    static constexpr int NSTAGE = D <= 32 ? 3 : 2;
    static_assert(NSTAGE >= 2 && NSTAGE <= 4, "stage waits cover at most 3 younger groups");
    static constexpr int BASE = round16(D + 32);  // one block's base exponents (+ alignment slack)
    // Per-block meta slot: K base | V base | the block's FlatBlock | its escape count headers.
    static constexpr int M_FB = 2 * BASE;
    static constexpr int M_EM = M_FB + 32;
    static constexpr int MSLOT = M_EM + 64;
    static constexpr int SCR = 16 * D;            // escape scratch: one row half of fragments
    static constexpr int W_META = NSTAGE * SLOT;  // per-warp region: ring | meta x2 | scratch
    static constexpr int W_SCR = W_META + 2 * MSLOT;
    static constexpr int WARP_BYTES = (W_SCR + SCR + 127) & ~127;
    // Register budget 65536 / (32 WARPS): 12 warps leave 168 per thread, 10 leave 204.
    static constexpr int MAXW = D <= 32 ? 16 : D <= 64 ? KVX_MAXWARPS : 10;
    static constexpr int WARPS = cmin(MAXW, 232448 / WARP_BYTES);
    static_assert(WARPS >= 1, "worker does not fit in shared memory");
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

// ---- escape records ----------------------------------------------------------------------------

// Lane l < 16 holds entry l of the block's K count header, lane 16 + l entry l of V's (0 without
// a record): e(i) = escape words of tokens [0, 16 i).
__device__ __forceinline__ uint32_t load_em(const uint16_t *esc, const FlatBlock &f, int lane) {
    const bool v = lane >= 16;
    const int mode = v ? f.v_mode : f.k_mode;
    const int n = v ? f.v_nesc : f.k_nesc;
    const uint32_t rec = v ? f.v_rec : f.k_rec;
    return (mode != 0 && n != 0) ? uint32_t(__ldg(esc + rec + (lane & 15))) : 0u;
}
// e(i) of tensor T (0 K, 1 V), i = 0..16; every lane of the warp calls it.
__device__ __forceinline__ int esc_at(uint32_t em, int T, int i) {
    const uint32_t v = __shfl_sync(FULL, em, (T << 4) + ((i + 15) & 15));
    return i == 0 ? 0 : int(v);
}

// e(i) of tensor T from a meta slot's copy of the headers.
__device__ __forceinline__ int esc_ms(const uint8_t *em, int T, int i) {
    return i == 0 ? 0 : int(*reinterpret_cast<const uint16_t *>(em + 2 * (16 * T + i - 1)));
}

// Byte offset inside a 16-byte line of escape word i of a coded block (the blob is 16-byte
// aligned) and of its position in the escape records (16-byte aligned allocation).
template <int D>
__device__ __forceinline__ uint32_t esc_word_line(uint32_t off, int n_tok, int mode, int i) {
    return (off + uint32_t(kHeaderBytes + D) + uint32_t(n_tok * D) + uint32_t(n_tok * D * mode / 8) +
            2u * uint32_t(i)) & 15u;
}
__device__ __forceinline__ uint32_t esc_pos_line(uint32_t rec, int i) {
    return (2u * (rec + uint32_t(kEscRecHead) + uint32_t(i))) & 15u;
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
__host__ __device__ constexpr uint32_t sel_cross(int b) {  // byte b of A -> 0, 1; of B -> 2, 3
    return uint32_t(b) | (uint32_t(b) << 4) | (uint32_t(4 + b) << 8) | (uint32_t(4 + b) << 12);
}

// Two BF16 values from sign/mantissa bytes (byte 0 and 1 of each half hold the element's byte:
// bits 0-6 give the mantissa, bit 15 the sign) and exponent residuals in bytes 0 and 2 of cw.
// Exponent = base + residual modulo 256 like bf16_from_delta's uint8 sum (reference
// include/kvexp/bf16.hpp:35-37).  Bytes 1 and 3 of cw may hold other residuals (< 16): times 128
// they land in bits 15-18 of each half, which the select drops, and no carry reaches bit 23.
__device__ __forceinline__ uint32_t merge(uint32_t sg, uint32_t cw, uint32_t b7) {
    return (sg & 0x807F807Fu) | ((cw * 128u + b7) & 0x7F807F80u);
}

// How this lane reads one tensor of the current block from a ring stage.  Row sections start
// m = 0 or 2 bytes past a 4-byte boundary; the lane's columns add a multiple of 4 to the sign/
// mantissa and raw rows, and any byte count to the residual rows.
struct Lay {
    uint32_t p0, p1;  // sign/mantissa bytes of element pairs 2q and 2q+1 from words q, q+1
    uint32_t w;       // one realigned word from two loaded ones (sign/mantissa, raw rows)
    uint32_t cs;      // one realigned word of residual codes
    int rows;         // byte offset of the lane's row window in the stage (4-aligned)
    int codes;        // byte offset of the lane's residual window in the stage (4-aligned)
};
// rd / cd: data offsets of the block's row and code pieces; col: the lane's first head dim.
template <int D>
__device__ __forceinline__ Lay make_lay(uint32_t rd, uint32_t cd, int mode, int col, bool bf16) {
    Lay l;
    const uint32_t m = rd & 3u;
    l.p0 = rep2(m);
    l.p1 = rep2(m + 2);
    l.w = shift4(m);
    const int rcol = (bf16 || mode == 0) ? 2 * col : col;
    l.rows = int(rd & ~3u) + rcol;
    const uint32_t cb = (cd & 3u) + uint32_t(col * (mode == 0 ? 0 : mode) / 8);
    l.cs = shift4(cb & 3u);
    l.codes = Cfg<D>::CODE_OFF + int(cd & ~3u) + int(cb & ~3u);
    return l;
}

// b7 of a K register (dims d, d+1): base[d] << 7 | base[d+1] << 23.  `base` points at the
// block's staged base exponents (data offset applied), the lane's first dim c0.
template <int D>
__device__ __forceinline__ void load_b7k(const uint8_t *base, uint32_t (&b7)[Cfg<D>::NK]) {
    constexpr int NB = Cfg<D>::DK / 4;
    const uint32_t m = uint32_t(reinterpret_cast<uintptr_t>(base)) & 3u;
    const uint32_t *q = reinterpret_cast<const uint32_t *>(base - m);
    uint32_t B[NB + 1];
#pragma unroll
    for (int i = 0; i <= NB; ++i) B[i] = q[i];
    const uint32_t s0 = rep2(m), s1 = rep2(m + 2);
#pragma unroll
    for (int p = 0; p < Cfg<D>::NK; ++p)
        b7[p] = (prmt(B[p >> 1], B[(p >> 1) + 1], (p & 1) ? s1 : s0) & 0x00FF00FFu) << 7;
}
// b7 of a V register (one dim, two tokens): base[d] << 7 | base[d] << 23.
template <int D>
__device__ __forceinline__ void load_b7v(const uint8_t *base, uint32_t (&b7)[Cfg<D>::DV]) {
    constexpr int NB = Cfg<D>::DV / 4;
    const uint32_t m = uint32_t(reinterpret_cast<uintptr_t>(base)) & 3u;
    const uint32_t *q = reinterpret_cast<const uint32_t *>(base - m);
    uint32_t B[NB + 1];
#pragma unroll
    for (int i = 0; i <= NB; ++i) B[i] = q[i];
    const uint32_t sw = shift4(m);
#pragma unroll
    for (int e = 0; e < Cfg<D>::DV; ++e) {
        const uint32_t w = prmt(B[e >> 2], B[(e >> 2) + 1], sw);
        b7[e] = (prmt(w, 0u, uint32_t(e & 3) * 0x1111u) & 0x00FF00FFu) << 7;
    }
}

// ---- row rebuild -------------------------------------------------------------------------------

// One K row of this lane (token r of the stage, dims c0 .. c0 + DK - 1).  MODE 4 / 2: coded,
// 0: raw BF16 rows.
template <int D, int MODE>
__device__ __forceinline__ void k_row(const uint8_t *stage, const Lay &ly, int r,
                                      const uint32_t (&b7)[Cfg<D>::NK], uint32_t (&o)[Cfg<D>::NK]) {
    using C = Cfg<D>;
    if constexpr (MODE == 0) {
        const uint32_t *q = reinterpret_cast<const uint32_t *>(stage + ly.rows + r * (2 * D));
        uint32_t W[C::NK + 1];
#pragma unroll
        for (int i = 0; i <= C::NK; ++i) W[i] = q[i];
#pragma unroll
        for (int p = 0; p < C::NK; ++p) o[p] = prmt(W[p], W[p + 1], ly.w);
    } else {
        constexpr int NS = C::DK / 4;
        const uint32_t *qs = reinterpret_cast<const uint32_t *>(stage + ly.rows + r * D);
        uint32_t W[NS + 1];
#pragma unroll
        for (int i = 0; i <= NS; ++i) W[i] = qs[i];
        const uint32_t *qc = reinterpret_cast<const uint32_t *>(stage + ly.codes + r * (D * MODE / 8));
        if constexpr (MODE == 4) {
            constexpr int NC = C::DK / 8;  // words of 8 residuals
            uint32_t X[NC + 1], lo[NC], hi[NC];
#pragma unroll
            for (int i = 0; i <= NC; ++i) X[i] = qc[i];
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const uint32_t x = prmt(X[k], X[k + 1], ly.cs);
                lo[k] = x & 0x0F0F0F0Fu;
                hi[k] = (x >> 4) & 0x0F0F0F0Fu;
            }
#pragma unroll
            for (int p = 0; p < C::NK; ++p)
                o[p] = merge(prmt(W[p >> 1], W[(p >> 1) + 1], (p & 1) ? ly.p1 : ly.p0),
                             prmt(lo[p >> 2], hi[p >> 2], sel_code(p & 3)), b7[p]);
        } else {
            constexpr int NC = (C::DK + 15) / 16;  // words of 16 residuals
            uint32_t X[NC + 1], el[NC], eh[NC], ol[NC], oh[NC];
#pragma unroll
            for (int i = 0; i <= NC; ++i) X[i] = qc[i];
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const uint32_t x = prmt(X[k], X[k + 1], ly.cs);
                const uint32_t ev = x & 0x33333333u, od = (x >> 2) & 0x33333333u;
                el[k] = ev & 0x0F0F0F0Fu;  // even elements of pairs 0, 2, 4, 6
                eh[k] = (ev >> 4) & 0x0F0F0F0Fu;
                ol[k] = od & 0x0F0F0F0Fu;
                oh[k] = (od >> 4) & 0x0F0F0F0Fu;
            }
#pragma unroll
            for (int p = 0; p < C::NK; ++p) {
                const int k = p >> 3, j = (p & 7) >> 1;
                const uint32_t cw = (p & 1) ? prmt(eh[k], oh[k], sel_code(j)) : prmt(el[k], ol[k], sel_code(j));
                o[p] = merge(prmt(W[p >> 1], W[(p >> 1) + 1], (p & 1) ? ly.p1 : ly.p0), cw, b7[p]);
            }
        }
    }
}

// Two V tokens of this lane (token a of the stage -> low halves, a + 1 -> high halves; dims
// v0 .. v0 + DV - 1).
template <int D, int MODE>
__device__ __forceinline__ void v_pair(const uint8_t *stage, const Lay &ly, int a,
                                       const uint32_t (&b7)[Cfg<D>::DV], uint32_t (&o)[Cfg<D>::DV]) {
    using C = Cfg<D>;
    if constexpr (MODE == 0) {
        constexpr int NW = C::DV / 2;
        const uint32_t *qa = reinterpret_cast<const uint32_t *>(stage + ly.rows + a * (2 * D));
        const uint32_t *qb = qa + D / 2;
        uint32_t A[NW + 1], B[NW + 1];
#pragma unroll
        for (int i = 0; i <= NW; ++i) {
            A[i] = qa[i];
            B[i] = qb[i];
        }
#pragma unroll
        for (int e = 0; e < C::DV; ++e) {
            const uint32_t x = prmt(A[e >> 1], A[(e >> 1) + 1], ly.w);
            const uint32_t y = prmt(B[e >> 1], B[(e >> 1) + 1], ly.w);
            o[e] = prmt(x, y, (e & 1) ? 0x7632u : 0x5410u);
        }
    } else {
        constexpr int NS = C::DV / 4;
        const uint32_t *sa = reinterpret_cast<const uint32_t *>(stage + ly.rows + a * D);
        const uint32_t *sb = sa + D / 4;
        uint32_t A[NS + 1], B[NS + 1], SA[NS], SB[NS];
#pragma unroll
        for (int i = 0; i <= NS; ++i) {
            A[i] = sa[i];
            B[i] = sb[i];
        }
#pragma unroll
        for (int k = 0; k < NS; ++k) {
            SA[k] = prmt(A[k], A[k + 1], ly.w);
            SB[k] = prmt(B[k], B[k + 1], ly.w);
        }
        constexpr int CR = D * MODE / 8;  // residual bytes per row
        const uint32_t *ca = reinterpret_cast<const uint32_t *>(stage + ly.codes + a * CR);
        const uint32_t *cb = reinterpret_cast<const uint32_t *>(stage + ly.codes + (a + 1) * CR);
        if constexpr (MODE == 4) {
            constexpr int NC = (C::DV + 7) / 8;
            uint32_t XA[NC + 1], XB[NC + 1], la[NC], ha[NC], lb[NC], hb[NC];
#pragma unroll
            for (int i = 0; i <= NC; ++i) {
                XA[i] = ca[i];
                XB[i] = cb[i];
            }
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const uint32_t x = prmt(XA[k], XA[k + 1], ly.cs), y = prmt(XB[k], XB[k + 1], ly.cs);
                la[k] = x & 0x0F0F0F0Fu;
                ha[k] = (x >> 4) & 0x0F0F0F0Fu;
                lb[k] = y & 0x0F0F0F0Fu;
                hb[k] = (y >> 4) & 0x0F0F0F0Fu;
            }
#pragma unroll
            for (int e = 0; e < C::DV; ++e) {
                const int k = e >> 3, j = (e & 7) >> 1;
                const uint32_t cw = (e & 1) ? prmt(ha[k], hb[k], sel_code(j)) : prmt(la[k], lb[k], sel_code(j));
                o[e] = merge(prmt(SA[e >> 2], SB[e >> 2], sel_cross(e & 3)), cw, b7[e]);
            }
        } else {
            constexpr int NC = (C::DV + 15) / 16;
            uint32_t XA[NC + 1], XB[NC + 1], ca4[4][NC], cb4[4][NC];
#pragma unroll
            for (int i = 0; i <= NC; ++i) {
                XA[i] = ca[i];
                XB[i] = cb[i];
            }
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const uint32_t x = prmt(XA[k], XA[k + 1], ly.cs), y = prmt(XB[k], XB[k + 1], ly.cs);
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    ca4[s][k] = (x >> (2 * s)) & 0x03030303u;
                    cb4[s][k] = (y >> (2 * s)) & 0x03030303u;
                }
            }
#pragma unroll
            for (int e = 0; e < C::DV; ++e) {
                const int k = e >> 4, s = e & 3, j = (e & 15) >> 2;
                o[e] = merge(prmt(SA[e >> 2], SB[e >> 2], sel_cross(e & 3)),
                             prmt(ca4[s][k], cb4[s][k], sel_code(j)), b7[e]);
            }
        }
    }
}

// Zero the halves of tokens past the tile's valid rows (P is 0 there, V must be finite).
template <int D>
__device__ __forceinline__ void v_tail(int t, int rows, uint32_t (&va)[Cfg<D>::DV]) {
    const uint32_t keep = (t < rows ? 0x0000FFFFu : 0u) | (t + 1 < rows ? 0xFFFF0000u : 0u);
#pragma unroll
    for (int e = 0; e < Cfg<D>::DV; ++e) va[e] &= keep;
}

// ---- escapes -----------------------------------------------------------------------------------

// The escape words of one tensor of a stage: word i of the block is val[i - off], its element
// position pos[i - off] (shared memory when the stage staged them, else the block's words in HBM
// with off = 0).
struct StageEsc {
    const uint16_t *val;
    const uint16_t *pos;
    int off;
};

// A row half of N fragment registers per lane goes to scratch as N / 4 chunks of 512 bytes, chunk
// k holding lane l's registers 4k .. 4k+3 at byte 16 l (16-byte stores without bank conflicts).
template <int N> __device__ __forceinline__ void regs_to(uint8_t *scr, const uint32_t (&o)[N], int lane) {
#pragma unroll
    for (int k = 0; k < N / 4; ++k)
        *reinterpret_cast<uint4 *>(scr + 512 * k + 16 * lane) =
            make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
}
template <int N> __device__ __forceinline__ void regs_from(const uint8_t *scr, uint32_t (&o)[N], int lane) {
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
        const uint4 v = *reinterpret_cast<const uint4 *>(scr + 512 * k + 16 * lane);
        o[4 * k] = v.x;
        o[4 * k + 1] = v.y;
        o[4 * k + 2] = v.z;
        o[4 * k + 3] = v.w;
    }
}
__device__ __forceinline__ uint32_t scr_addr(int owner, int p, int half) {
    return uint32_t(512 * (p >> 2) + 16 * owner + 4 * (p & 3) + 2 * half);
}

// Scratch byte of element (token r of the 16-token tile, dim c) in its row half's layout.
template <int D, bool K> __device__ __forceinline__ uint32_t esc_slot(int r, int c) {
    using C = Cfg<D>;
    if (K) {  // lane (r & 7, c / DK) register (c % DK) / 2, half c & 1
        const int q = c % C::DK;
        return scr_addr(4 * (r & 7) + c / C::DK, q >> 1, q & 1);
    }
    // V: lane (c / DV, (r & 7) / 2) register c % DV, half r & 1
    return scr_addr(4 * (c / C::DV) + ((r & 7) >> 1), c % C::DV, r & 1);
}

// Which row halves of the tile (tokens t0 .. t0+15 of the block) hold escapes [i0, i1): bit h.
template <int D>
__device__ __forceinline__ uint32_t esc_halves(const StageEsc &se, int i0, int i1, int t0, int lane) {
    uint32_t f = 0;
    for (int i = i0 + lane; i < i1; i += 32) {
        const int r = int(se.pos[i - se.off]) / D - t0;
        f |= 1u << ((r >> 3) & 1);
    }
    return __reduce_or_sync(FULL, f);
}

// Store escapes [i0, i1) of row half h over their elements: the half's registers round-trip
// through scratch.
template <int D, bool K, int N>
__device__ __forceinline__ void esc_patch(uint32_t (&o)[N], uint8_t *scr, const StageEsc &se, int i0,
                                          int i1, int t0, int h, int lane) {
    __syncwarp();
    regs_to(scr, o, lane);
    __syncwarp();
    for (int i = i0 + lane; i < i1; i += 32) {
        const int pos = int(se.pos[i - se.off]);
        const int r = pos / D - t0, c = pos % D;
        if ((r >> 3) == h) *reinterpret_cast<uint16_t *>(scr + esc_slot<D, K>(r, c)) = se.val[i - se.off];
    }
    __syncwarp();
    regs_from(scr, o, lane);
}

// ---- per-tile stages ----------------------------------------------------------------------------

// S^T fragment of a 16-token tile (tile row r0 of the stage): s0/s1 token g (queries 2t, 2t+1),
// s2/s3 token g + 8.
template <int D, int MODE>
__device__ __forceinline__ void qk_tile(const uint8_t *stage, const Lay &ly, int r0,
                                        const uint32_t (&b7)[Cfg<D>::NK],
                                        const uint32_t (&qb)[Cfg<D>::KS][2], const StageEsc &se,
                                        int i0, int i1, int tb, uint8_t *scr, int lane, float (&s)[4]) {
    using C = Cfg<D>;
    const int gi = lane >> 2;
    s[0] = s[1] = s[2] = s[3] = 0.f;
    const uint32_t halves = (MODE != 0 && i1 > i0) ? esc_halves<D>(se, i0, i1, tb, lane) : 0u;
    if (!C::SPLIT) {
        uint32_t ka0[C::NK], ka1[C::NK];
        k_row<D, MODE>(stage, ly, r0 + gi, b7, ka0);
        k_row<D, MODE>(stage, ly, r0 + gi + 8, b7, ka1);
        if (MODE != 0) {
            if (halves & 1u) esc_patch<D, true>(ka0, scr, se, i0, i1, tb, 0, lane);
            if (halves & 2u) esc_patch<D, true>(ka1, scr, se, i0, i1, tb, 1, lane);
        }
#pragma unroll
        for (int k = 0; k < C::KS; ++k)
            mma_bf16(s[0], s[1], s[2], s[3], ka0[2 * k], ka1[2 * k], ka0[2 * k + 1], ka1[2 * k + 1],
                     qb[k][0], qb[k][1]);
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t ka[C::NK];
            k_row<D, MODE>(stage, ly, r0 + gi + 8 * h, b7, ka);
            if (MODE != 0 && (halves >> h & 1u)) esc_patch<D, true>(ka, scr, se, i0, i1, tb, h, lane);
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

// O^T += V^T P^T for a 16-token tile (P^T as B fragments: bh = bf16 part, bm = residual part).
template <int D, int MODE>
__device__ __forceinline__ void pv_tile(const uint8_t *stage, const Lay &ly, int r0, int rows,
                                        const uint32_t (&b7)[Cfg<D>::DV], const uint32_t (&bh)[2],
                                        const uint32_t (&bm)[2], const StageEsc &se, int i0, int i1,
                                        int tb, uint8_t *scr, int lane, float (&acc)[Cfg<D>::KS][4]) {
    using C = Cfg<D>;
    const int t = 2 * (lane & 3);
    const uint32_t halves = (MODE != 0 && i1 > i0) ? esc_halves<D>(se, i0, i1, tb, lane) : 0u;
    if (!C::SPLIT) {
        uint32_t va0[C::DV], va1[C::DV];
        v_pair<D, MODE>(stage, ly, r0 + t, b7, va0);
        v_pair<D, MODE>(stage, ly, r0 + t + 8, b7, va1);
        if (MODE != 0) {
            if (halves & 1u) esc_patch<D, false>(va0, scr, se, i0, i1, tb, 0, lane);
            if (halves & 2u) esc_patch<D, false>(va1, scr, se, i0, i1, tb, 1, lane);
        }
        if (rows < TT) {
            v_tail<D>(t, rows, va0);
            v_tail<D>(t + 8, rows, va1);
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
            v_pair<D, MODE>(stage, ly, r0 + t + 8 * h, b7, va);
            if (MODE != 0 && (halves >> h & 1u)) esc_patch<D, false>(va, scr, se, i0, i1, tb, h, lane);
            if (rows < TT) v_tail<D>(t + 8 * h, rows, va);
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
// refuses larger steps), together with this lane's entry of each block's escape count headers.
struct Walker {
    int fb, fb1;
    FlatBlock cur, nxt;
    uint32_t em, emn;
    __device__ __forceinline__ void init(const AttnArgs &a, int b0, int b1, int lane) {
        fb = b0;
        fb1 = b1;
        cur = load_flat(a.flat, fb);
        em = load_em(a.esc, cur, lane);
        if (fb + 1 < fb1) {
            nxt = load_flat(a.flat, fb + 1);
            emn = load_em(a.esc, nxt, lane);
        }
    }
    __device__ __forceinline__ void next(const AttnArgs &a, int lane) {
        ++fb;
        if (fb < fb1) {
            cur = nxt;
            em = emn;
            if (fb + 1 < fb1) {
                nxt = load_flat(a.flat, fb + 1);
                emn = load_em(a.esc, nxt, lane);
            }
        }
    }
};

// Copy side of the worker's ring.  At a block's first stage it also leaves the block's FlatBlock
// and escape count headers in the block's meta slot for the consumer side.
template <int D, bool BF16IN> struct Producer {
    using C = Cfg<D>;
    Walker w;
    int tile = 0, stage = 0, bseq = 0;
    const uint8_t *kb = nullptr, *vb = nullptr;  // the current unit's K and V blobs

    __device__ __forceinline__ static void tensor(uint8_t *dst, const Sections &s, const uint16_t *pos,
                                                  int mode, int t0, int n, int e0, int e1, int lane) {
        if (BF16IN || mode == 0) {
            copy_piece<C::TS * 2 * D + 16>(
                dst, make_piece(s.rows + size_t(t0) * (2 * D), uint32_t(n * 2 * D)), lane);
        } else {
            copy_piece<C::TS * D + 16>(dst, make_piece(s.rows + size_t(t0) * D, uint32_t(n * D)), lane);
            copy_piece<C::TS * D / 2 + 16>(
                dst + C::CODE_OFF,
                make_piece(s.codes + size_t(t0) * D * mode / 8, uint32_t(n * D * mode / 8)), lane);
            const int cnt = e1 - e0;
            if (cnt > 0 && cnt <= C::ESC_CAP) {
                copy_piece<2 * C::ESC_CAP + 16>(dst + C::EV_OFF, make_piece(s.esc + 2 * e0, uint32_t(2 * cnt)), lane);
                copy_piece<2 * C::ESC_CAP + 16>(
                    dst + C::EP_OFF, make_piece(reinterpret_cast<const uint8_t *>(pos + e0), uint32_t(2 * cnt)),
                    lane);
            }
        }
    }

    // Issue stages while a ring slot is free; a block start waits until the consumer is at most
    // one block behind, so a meta slot is never overwritten while in use.
    __device__ __forceinline__ void produce(const AttnArgs &a, uint8_t *ring, uint8_t *metas,
                                            int c_stage, int c_fb, int lane) {
        while (w.fb < w.fb1 && stage - c_stage < C::NSTAGE) {
            if (tile == 0 && w.fb - c_fb >= 2) break;
            const FlatBlock &f = w.cur;
            const int km = BF16IN ? 0 : f.k_mode, vm = BF16IN ? 0 : f.v_mode;
            if (tile == 0) {
                const UnitDev *U = a.units + f.unit;
                kb = U->k;
                vb = U->v;
                uint8_t *ms = metas + (bseq & 1) * C::MSLOT;
                if (lane == 0) {
                    const uint4 *src = reinterpret_cast<const uint4 *>(&f);
                    reinterpret_cast<uint4 *>(ms + C::M_FB)[0] = src[0];
                    reinterpret_cast<uint4 *>(ms + C::M_FB)[1] = src[1];
                }
                reinterpret_cast<uint16_t *>(ms + C::M_EM)[lane] = uint16_t(w.em);
                if (!BF16IN) {
                    if (km != 0) copy_piece<D + 32>(ms, make_piece(kb + f.k_off + kHeaderBytes, D), lane);
                    if (vm != 0) copy_piece<D + 32>(ms + C::BASE, make_piece(vb + f.v_off + kHeaderBytes, D), lane);
                }
            }
            const int t0 = tile * C::TS;
            const int n = min(C::TS, int(f.valid) - t0);
            const int ia = t0 >> 4, ib = min(16, (t0 + C::TS) >> 4);
            uint8_t *slot = ring + (stage % C::NSTAGE) * C::SLOT;
            tensor(slot, sections<D, BF16IN>(kb, f.k_off, km, f.n_tok), a.esc + f.k_rec + kEscRecHead,
                   km, t0, n, esc_at(w.em, 0, ia), esc_at(w.em, 0, ib), lane);
            tensor(slot + C::TR, sections<D, BF16IN>(vb, f.v_off, vm, f.n_tok),
                   a.esc + f.v_rec + kEscRecHead, vm, t0, n, esc_at(w.em, 1, ia), esc_at(w.em, 1, ib), lane);
            cp_async_commit();
            ++stage;
            if (t0 + C::TS >= int(f.valid)) {
                tile = 0;
                ++bseq;
                w.next(a, lane);
            } else {
                ++tile;
            }
        }
    }
};

// The escape words of tensor T (0 K, 1 V) of the block's stage holding escapes [e0, e1):
// the producer's staged copies when they fit, else the block's words in HBM.
template <int D>
__device__ __forceinline__ StageEsc stage_esc(const AttnArgs &a, const FlatBlock &f, int T,
                                              const uint8_t *tstage, int e0, int e1) {
    using C = Cfg<D>;
    const uint32_t off = T ? f.v_off : f.k_off, rec = T ? f.v_rec : f.k_rec;
    const int mode = T ? f.v_mode : f.k_mode;
    StageEsc se;
    if (e1 - e0 <= C::ESC_CAP) {
        se.val = reinterpret_cast<const uint16_t *>(tstage + C::EV_OFF + esc_word_line<D>(off, f.n_tok, mode, e0));
        se.pos = reinterpret_cast<const uint16_t *>(tstage + C::EP_OFF + esc_pos_line(rec, e0));
        se.off = e0;
    } else {
        const UnitDev *U = a.units + f.unit;
        se.val = reinterpret_cast<const uint16_t *>(sections<D, false>(T ? U->v : U->k, off, mode, f.n_tok).esc);
        se.pos = a.esc + rec + kEscRecHead;
        se.off = 0;
    }
    return se;
}

template <int D, bool BF16IN>
__device__ __forceinline__ void worker(const AttnArgs &a, uint8_t *R, int wk, int fb0, int fb1,
                                       int lane) {
    using C = Cfg<D>;
    const int gi = lane >> 2, tig = lane & 3;
    uint8_t *ring = R;
    uint8_t *metas = R + C::W_META;
    uint8_t *scr = R + C::W_SCR;
    Producer<D, BF16IN> pp;
    pp.w.init(a, fb0, fb1, lane);
    int fb = fb0, tile = 0, stage = 0, bseq = 0;
    int ubeg = 0, uend = 0, seg_begin = fb0;  // the current unit's flat block range
    Lay lk{}, lv{};
    uint32_t b7k[C::NK], b7v[C::DV];
#pragma unroll
    for (int p = 0; p < C::NK; ++p) b7k[p] = 0u;
#pragma unroll
    for (int e = 0; e < C::DV; ++e) b7v[e] = 0u;
    uint32_t qb[C::KS][2];
    float acc[C::KS][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    while (fb < fb1) {
        pp.produce(a, ring, metas, stage, fb, lane);
        cp_async_wait(pp.stage - stage - 1);
        __syncwarp();
        const uint8_t *ms = metas + (bseq & 1) * C::MSLOT;
        const FlatBlock f = *reinterpret_cast<const FlatBlock *>(ms + C::M_FB);
        const uint8_t *em = ms + C::M_EM;
        const int kmode = BF16IN ? 0 : f.k_mode, vmode = BF16IN ? 0 : f.v_mode;
        if (tile == 0) {
            const UnitDev *U = a.units + f.unit;
            ubeg = int(U->block_begin);
            uend = ubeg + U->n_blocks;
            const Sections sk = sections<D, BF16IN>(U->k, f.k_off, kmode, f.n_tok);
            const Sections sv = sections<D, BF16IN>(U->v, f.v_off, vmode, f.n_tok);
            const uint32_t kd = uint32_t(reinterpret_cast<uintptr_t>(sk.rows) & 15u);
            const uint32_t vd = uint32_t(reinterpret_cast<uintptr_t>(sv.rows) & 15u);
            const uint32_t kc = kmode ? uint32_t(reinterpret_cast<uintptr_t>(sk.codes) & 15u) : 0u;
            const uint32_t vc = vmode ? uint32_t(reinterpret_cast<uintptr_t>(sv.codes) & 15u) : 0u;
            lk = make_lay<D>(kd, kc, kmode, tig * C::DK, BF16IN);
            lv = make_lay<D>(vd, vc, vmode, gi * C::DV, BF16IN);
            if (kmode != 0) load_b7k<D>(ms + kd + tig * C::DK, b7k);
            if (vmode != 0) load_b7v<D>(ms + C::BASE + vd + gi * C::DV, b7v);
            if (fb == seg_begin) {
                load_q<D>(U->q, U->n_q, U->q_stride, qb, lane);
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
#pragma unroll
                for (int m = 0; m < C::KS; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
            }
        }
        uint8_t *slot = ring + (stage % C::NSTAGE) * C::SLOT;
        const int t0 = tile * C::TS;
        const int rows = min(C::TS, int(f.valid) - t0);
        const bool last_tile = t0 + C::TS >= int(f.valid);
        const bool seg_end = last_tile && (fb + 1 == fb1 || fb + 1 == uend);
        const int ia = t0 >> 4, ib = min(16, (t0 + C::TS) >> 4);

        // S^T = K Q^T for every tile of the stage
        float s[C::SUBS][4];
        {
            const StageEsc se = stage_esc<D>(a, f, 0, slot, esc_ms(em, 0, ia), esc_ms(em, 0, ib));
#pragma unroll
            for (int sub = 0; sub < C::SUBS; ++sub) {
                if (sub * TT < rows) {
                    const int i0 = esc_ms(em, 0, ia + sub), i1 = esc_ms(em, 0, ia + sub + 1);
                    const int tb = t0 + sub * TT;
                    if (kmode == 4) qk_tile<D, 4>(slot, lk, sub * TT, b7k, qb, se, i0, i1, tb, scr, lane, s[sub]);
                    else if (kmode == 2) qk_tile<D, 2>(slot, lk, sub * TT, b7k, qb, se, i0, i1, tb, scr, lane, s[sub]);
                    else qk_tile<D, 0>(slot, lk, sub * TT, b7k, qb, se, i0, i1, tb, scr, lane, s[sub]);
                    const int rr = rows - sub * TT;
                    if (gi >= rr) s[sub][0] = s[sub][1] = -INFINITY;
                    if (gi + 8 >= rr) s[sub][2] = s[sub][3] = -INFINITY;
                } else {
                    s[sub][0] = s[sub][1] = s[sub][2] = s[sub][3] = -INFINITY;
                }
            }
        }

        // online softmax over the stage's tokens; p = 2^(s log2e - m log2e)
        float t0m = fmaxf(s[0][0], s[0][2]), t1m = fmaxf(s[0][1], s[0][3]);
#pragma unroll
        for (int sub = 1; sub < C::SUBS; ++sub) {
            t0m = fmaxf(t0m, fmaxf(s[sub][0], s[sub][2]));
            t1m = fmaxf(t1m, fmaxf(s[sub][1], s[sub][3]));
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            t0m = fmaxf(t0m, __shfl_xor_sync(FULL, t0m, o));
            t1m = fmaxf(t1m, __shfl_xor_sync(FULL, t1m, o));
        }
        const float mn0 = fmaxf(m0, t0m), mn1 = fmaxf(m1, t1m);
        const float ml0 = __fmul_rn(mn0, kLog2e), ml1 = __fmul_rn(mn1, kLog2e);
        const float al0 = ex2(__fmaf_rn(m0, kLog2e, -ml0)), al1 = ex2(__fmaf_rn(m1, kLog2e, -ml1));
        float ps0 = 0.f, ps1 = 0.f;
        uint32_t bh[C::SUBS][2], bm[C::SUBS][2];
#pragma unroll
        for (int sub = 0; sub < C::SUBS; ++sub) {
            const float p0 = ex2(__fmaf_rn(s[sub][0], kLog2e, -ml0)), p1 = ex2(__fmaf_rn(s[sub][1], kLog2e, -ml1));
            const float p2 = ex2(__fmaf_rn(s[sub][2], kLog2e, -ml0)), p3 = ex2(__fmaf_rn(s[sub][3], kLog2e, -ml1));
            ps0 = __fadd_rn(ps0, __fadd_rn(p0, p2));
            ps1 = __fadd_rn(ps1, __fadd_rn(p1, p3));
            // P^T B fragments: bf16(p) and bf16(p - bf16(p))
            const uint32_t h01 = pack_bf16x2(p1, p0), h23 = pack_bf16x2(p3, p2);
            const float r0 = __fsub_rn(p0, bf16lo_to_f32(h01)), r1 = __fsub_rn(p1, bf16hi_to_f32(h01));
            const float r2 = __fsub_rn(p2, bf16lo_to_f32(h23)), r3 = __fsub_rn(p3, bf16hi_to_f32(h23));
            bh[sub][0] = movm_t(h01);
            bh[sub][1] = movm_t(h23);
            bm[sub][0] = movm_t(pack_bf16x2(r1, r0));
            bm[sub][1] = movm_t(pack_bf16x2(r3, r2));
        }
        l0 = __fmaf_rn(l0, al0, ps0);
        l1 = __fmaf_rn(l1, al1, ps1);
        m0 = mn0;
        m1 = mn1;
        if (__any_sync(FULL, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
            for (int m = 0; m < C::KS; ++m) {
                acc[m][0] = __fmul_rn(acc[m][0], al0);
                acc[m][1] = __fmul_rn(acc[m][1], al1);
                acc[m][2] = __fmul_rn(acc[m][2], al0);
                acc[m][3] = __fmul_rn(acc[m][3], al1);
            }
        }

        // O^T += V^T P^T for every tile of the stage
        {
            const uint8_t *vstage = slot + C::TR;
            const StageEsc se = stage_esc<D>(a, f, 1, vstage, esc_ms(em, 1, ia), esc_ms(em, 1, ib));
#pragma unroll
            for (int sub = 0; sub < C::SUBS; ++sub) {
                if (sub * TT < rows) {
                    const int i0 = esc_ms(em, 1, ia + sub), i1 = esc_ms(em, 1, ia + sub + 1);
                    const int tb = t0 + sub * TT;
                    const int rr = min(TT, rows - sub * TT);
                    if (vmode == 4) pv_tile<D, 4>(vstage, lv, sub * TT, rr, b7v, bh[sub], bm[sub], se, i0, i1, tb, scr, lane, acc);
                    else if (vmode == 2) pv_tile<D, 2>(vstage, lv, sub * TT, rr, b7v, bh[sub], bm[sub], se, i0, i1, tb, scr, lane, acc);
                    else pv_tile<D, 0>(vstage, lv, sub * TT, rr, b7v, bh[sub], bm[sub], se, i0, i1, tb, scr, lane, acc);
                }
            }
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
            if (seg_begin == ubeg && fb + 1 == uend) {
                const UnitDev *U = a.units + f.unit;
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

cudaError_t launch_fold(const float *parts, int n_parts, int n_rows, int dim, float *out,
                        float *lse_out, cudaStream_t s) {
    fold_kernel<<<n_rows, dim < 256 ? dim : 256, 0, s>>>(parts, n_parts, n_rows, dim, out, lse_out);
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
