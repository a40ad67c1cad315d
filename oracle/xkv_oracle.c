/*
 * xkv_oracle.c -- CPU restatement of kvexp's XKV codec and scalar decode attention.
 *
 * TEST INFRASTRUCTURE ONLY (the checker; never the thing measured or shipped).
 * Each function names the reference file:line it follows.  Compile with
 * -ffp-contract=off -fno-fast-math so every fmaf / expf / + / * rounds as in the
 * reference's scalar kernel (reference CMakeLists.txt:48).
 *
 * One extension has no reference code: the 3-bit residual mode (mode byte 3), which the
 * reference measured and did not implement (README.md:35, :200).  Its size model is the one of
 * python/analyze_exponents.py:101-103 (width 7 = 2^3 - 1 exponents per window, sentinel 7) and
 * :129-138 (the same best-window search and tie rules as 2 and 4 bits); its layout is this
 * library's: element i's code in bits [3 i, 3 i + 3) of the little-endian code bytes, the code
 * section padded with one zero byte to an even length when 3 n dim / 8 is odd (so every section
 * of a blob stays 2-byte aligned).  The reference's own encoder never writes it: 3-bit blocks are
 * emitted only when the caller's mode mask asks for them.
 */
#include "xkv_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define OX_MAX_DIM 256 /* kMaxHeadDim, include/kvexp/bf16.hpp:13 */

static __thread char g_err[256];

const char *ox_last_error(void) { return g_err; }

static int fail(int code, const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return code;
}

/* ---- BF16 helpers, include/kvexp/bf16.hpp:15-37 ---------------------------------- */

static float bf16_to_fp32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static uint8_t bf16_exponent(uint16_t bits) { return (uint8_t)((bits >> 7) & 0xFF); }

static uint8_t bf16_sm(uint16_t bits) { return (uint8_t)(((bits >> 8) & 0x80) | (bits & 0x7F)); }

static uint16_t bf16_from_delta(uint8_t base, uint8_t delta, uint8_t sm) {
    uint8_t e = (uint8_t)((uint16_t)base + (uint16_t)delta);
    return (uint16_t)(((uint16_t)(sm & 0x80) << 8) | ((uint16_t)e << 7) | (uint16_t)(sm & 0x7F));
}

int ox_exp_payload_bytes(int n_tokens, int dim, int bits) {
    if (bits == 3) return (n_tokens * dim * 3 + 15) / 16 * 2; /* extension: padded to even */
    return (n_tokens * dim * bits + 7) / 8;
}

int ox_coded_block_bytes(int n_tokens, int dim, int bits, int n_escape) {
    return 8 + dim + n_tokens * dim + ox_exp_payload_bytes(n_tokens, dim, bits) + 2 * n_escape;
}

int ox_raw_block_bytes(int n_tokens, int dim) { return 8 + 2 * n_tokens * dim; }

size_t ox_encode_bound(int seq, int dim, int block_tokens) {
    if (seq <= 0 || dim <= 0 || block_tokens <= 0) return 0;
    size_t nblk = ((size_t)seq + (size_t)block_tokens - 1) / (size_t)block_tokens;
    /* the encoder never emits a block larger than its raw form */
    return nblk * 8u + 2u * (size_t)seq * (size_t)dim;
}

/* ---- block parsing, include/kvexp/scan.hpp:24-75 ---------------------------------- */

static int u16_le(const uint8_t *p) { return (int)p[0] | ((int)p[1] << 8); }

int ox_parse_block(const uint8_t *blob, size_t bytes, size_t offset, int dim, ox_block *b) {
    if (offset > bytes || bytes - offset < 8) return fail(OX_RUNTIME, "truncated xkv block header");
    const uint8_t *p = blob + offset;
    b->mode = p[0];
    b->n_tokens = p[1];
    b->n_escape = u16_le(p + 2);
    b->offset = offset;
    int hdim = u16_le(p + 4);
    if (hdim != dim || b->n_tokens <= 0)
        return fail(OX_RUNTIME, "xkv block dimension or length mismatch");
    size_t rest = bytes - offset - 8;
    if (b->mode == 0) {
        size_t nbytes = (size_t)b->n_tokens * (size_t)dim * 2u;
        if (rest < nbytes) return fail(OX_RUNTIME, "truncated raw xkv block");
        b->next = offset + 8 + nbytes;
        return OX_OK;
    }
    /* mode 3 (3-bit residuals) is this library's extension; the reference knows 2 and 4 */
    if (b->mode != 2 && b->mode != 3 && b->mode != 4) return fail(OX_RUNTIME, "unknown xkv block mode");
    size_t sm_bytes = (size_t)b->n_tokens * (size_t)dim;
    size_t exp_bytes = (size_t)ox_exp_payload_bytes(b->n_tokens, dim, b->mode);
    size_t esc_bytes = (size_t)b->n_escape * 2u;
    size_t need = (size_t)dim + sm_bytes + exp_bytes + esc_bytes;
    if (rest < need) return fail(OX_RUNTIME, "truncated coded xkv block");
    b->next = offset + 8 + need;
    return OX_OK;
}

static int residual_code(const uint8_t *exp, int index, int bits) {
    if (bits == 4) {
        uint8_t byte = exp[index >> 1];
        return (index & 1) ? (byte >> 4) : (byte & 0x0F);
    }
    if (bits == 3) { /* extension: bits [3 index, 3 index + 3), little-endian */
        const int bit = 3 * index, sh = bit & 7;
        int v = exp[bit >> 3] >> sh;
        if (sh > 5) v |= exp[(bit >> 3) + 1] << (8 - sh);
        return v & 7;
    }
    uint8_t byte = exp[index >> 2];
    return (byte >> ((index & 3) * 2)) & 0x03;
}

int ox_block_walk(const uint8_t *blob, size_t bytes, int dim, int seq, ox_block *blocks, int cap,
                  int *n_blocks) {
    size_t off = 0;
    int n = 0;
    long long tokens = 0;
    while (off < bytes) {
        ox_block b;
        int rc = ox_parse_block(blob, bytes, off, dim, &b);
        if (rc) return rc;
        if (blocks && n < cap) blocks[n] = b;
        ++n;
        tokens += b.n_tokens;
        off = b.next;
    }
    *n_blocks = n;
    if (seq > 0 && tokens < seq) return fail(OX_RUNTIME, "xkv decode ran out of blocks");
    return OX_OK;
}

/* Reader state: XkvReader, include/kvexp/scan.hpp:79-165. */
typedef struct {
    const uint8_t *data;
    size_t size;
    int dim;
    ox_block blk;
    int local, di;
    size_t esc; /* byte offset of the next escape word */
    int done;
} reader;

static size_t block_base(const reader *r) { return r->blk.offset + 8; }

static int reader_open_block(reader *r, size_t off) {
    int rc = ox_parse_block(r->data, r->size, off, r->dim, &r->blk);
    if (rc) return rc;
    r->local = 0;
    r->di = 0;
    if (r->blk.mode != 0) {
        size_t sm = (size_t)r->blk.n_tokens * (size_t)r->dim;
        size_t ex = (size_t)ox_exp_payload_bytes(r->blk.n_tokens, r->dim, r->blk.mode);
        r->esc = block_base(r) + (size_t)r->dim + sm + ex;
    }
    r->done = 0;
    return OX_OK;
}

/* XkvReader::seek, scan.hpp:94-123 */
static int reader_seek(reader *r, const uint8_t *data, size_t size, int dim, int token) {
    r->data = data;
    r->size = size;
    r->dim = dim;
    r->done = 1;
    if (token < 0) return fail(OX_RUNTIME, "negative token");
    size_t p = 0;
    int pos = 0;
    while (pos < token) {
        if (p >= size) return fail(OX_RUNTIME, "xkv seek past end");
        ox_block b;
        int rc = ox_parse_block(data, size, p, dim, &b);
        if (rc) return rc;
        if (pos + b.n_tokens > token)
            return fail(OX_RUNTIME, "token split is not aligned to an encoded block");
        pos += b.n_tokens;
        p = b.next;
    }
    if (p >= size) {
        r->done = 1;
        r->local = 0;
        return OX_OK;
    }
    return reader_open_block(r, p);
}

/* XkvReader::read_next, scan.hpp:125-155 */
static int reader_next(reader *r, uint16_t *value) {
    if (r->done) return fail(OX_RUNTIME, "xkv decode ran out of blocks");
    const uint8_t *base = r->data + block_base(r);
    if (r->blk.mode == 0) {
        size_t idx = (size_t)r->local * (size_t)r->dim + (size_t)r->di;
        *value = (uint16_t)u16_le(base + 2 * idx);
    } else {
        const int index = r->local * r->dim + r->di;
        const uint8_t *bases = base;
        const uint8_t *sm = base + r->dim;
        const uint8_t *exp = sm + (size_t)r->blk.n_tokens * (size_t)r->dim;
        const int code = residual_code(exp, index, r->blk.mode);
        const int sentinel = (1 << r->blk.mode) - 1;
        if (code == sentinel) {
            /* The reference trusts n_escape here (a well-formed blob never runs past it);
             * the oracle refuses instead of reading past the buffer. */
            if (r->esc + 2 > r->size) return fail(OX_RUNTIME, "xkv escape stream overrun");
            *value = (uint16_t)u16_le(r->data + r->esc);
            r->esc += 2;
        } else {
            *value = bf16_from_delta(bases[r->di], (uint8_t)code, sm[index]);
        }
    }
    ++r->di;
    if (r->di == r->dim) {
        r->di = 0;
        ++r->local;
        if (r->local == r->blk.n_tokens) {
            if (r->blk.next >= r->size) {
                r->done = 1;
            } else {
                int rc = reader_open_block(r, r->blk.next);
                if (rc) return rc;
            }
        }
    }
    return OX_OK;
}

int ox_decode_bf16(const uint8_t *blob, size_t bytes, int seq, int dim, uint16_t *out) {
    reader r;
    int rc = reader_seek(&r, blob, bytes, dim, 0);
    if (rc) return rc;
    const long long n = (long long)seq * (long long)dim;
    for (long long i = 0; i < n; ++i) {
        rc = reader_next(&r, &out[i]);
        if (rc) return rc;
    }
    return OX_OK;
}

/* ---- encoder, src/codec.cpp:18-164 ------------------------------------------------ */

/* best_base, codec.cpp:18-35: smallest base maximising the window count. */
static int best_base(const int *hist, int width) {
    int prefix[257];
    prefix[0] = 0;
    for (int i = 0; i < 256; ++i) prefix[i + 1] = prefix[i] + hist[i];
    int best_c = -1, best_b = 0;
    const int nbase = 256 - width + 1;
    for (int base = 0; base < nbase; ++base) {
        const int c = prefix[base + width] - prefix[base];
        if (c > best_c) {
            best_c = c;
            best_b = base;
        }
    }
    return best_b;
}

static void put_u16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xFF);
    p[1] = (uint8_t)(v >> 8);
}

int ox_encode_bf16(const uint16_t *kv, int seq, int dim, int block_tokens, uint8_t *out,
                   size_t out_cap, size_t *out_bytes, uint8_t *modes) {
    return ox_encode_bf16_modes(kv, seq, dim, block_tokens, OX_MODES_REFERENCE, out, out_cap,
                                out_bytes, modes);
}

int ox_encode_bf16_modes(const uint16_t *kv, int seq, int dim, int block_tokens, int mode_mask,
                         uint8_t *out, size_t out_cap, size_t *out_bytes, uint8_t *modes) {
    /* validation, codec.cpp:40-52 */
    if (kv == NULL || seq <= 0 || dim <= 0 || block_tokens <= 0)
        return fail(OX_INVALID_ARGUMENT, "encode_bf16: empty input");
    if (dim % 4 != 0 || dim > OX_MAX_DIM)
        return fail(OX_INVALID_ARGUMENT,
                    "encode_bf16: head_dim must be a multiple of 4 and at most 256");
    if (block_tokens > 255)
        return fail(OX_INVALID_ARGUMENT, "encode_bf16: block_tokens must fit in a byte");
    if ((long long)block_tokens * dim > 65535)
        return fail(OX_INVALID_ARGUMENT, "encode_bf16: block escape count would not fit in u16");
    if ((mode_mask & ~OX_MODES_ALL) != 0 || (mode_mask & OX_MODES_REFERENCE) != OX_MODES_REFERENCE)
        return fail(OX_INVALID_ARGUMENT, "encode_bf16: mode mask must hold 2 and 4 bits, and may add 3");

    int *hist = (int *)malloc(sizeof(int) * (size_t)dim * 256u);
    uint8_t *base_exp = (uint8_t *)malloc((size_t)dim);
    uint8_t *packed = (uint8_t *)malloc((size_t)block_tokens * (size_t)dim);
    uint16_t *escapes = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)block_tokens * (size_t)dim);
    if (!hist || !base_exp || !packed || !escapes) {
        free(hist); free(base_exp); free(packed); free(escapes);
        return fail(OX_RUNTIME, "encode_bf16: out of memory");
    }
    size_t w = 0;
    int rc = OX_OK;
    int blk = 0;
    for (int t0 = 0; t0 < seq; t0 += block_tokens, ++blk) {
        const int n = (block_tokens < seq - t0) ? block_tokens : seq - t0;
        const uint16_t *src = kv + (size_t)t0 * (size_t)dim;
        /* histogram, codec.cpp:68-73 */
        memset(hist, 0, sizeof(int) * (size_t)dim * 256u);
        for (int t = 0; t < n; ++t)
            for (int d = 0; d < dim; ++d) ++hist[(size_t)d * 256 + bf16_exponent(src[(size_t)t * dim + d])];

        /* mode choice with tie rules, codec.cpp:75-103 (candidates narrowest first, so a tie
         * between coded modes keeps fewer escapes, then the narrower code) */
        int best_mode = 0, best_bytes = ox_raw_block_bytes(n, dim), best_esc = 0;
        for (int bits = 2; bits <= 4; ++bits) {
            if (!(mode_mask & (1 << bits))) continue;
            const int width = (1 << bits) - 1;
            int n_esc = 0;
            for (int d = 0; d < dim; ++d) {
                const int *h = hist + (size_t)d * 256;
                const int b = best_base(h, width);
                int covered = 0;
                for (int e = b; e < b + width; ++e) covered += h[e];
                n_esc += n - covered;
            }
            const int c_bytes = ox_coded_block_bytes(n, dim, bits, n_esc);
            const int better_size = c_bytes < best_bytes;
            const int tie = c_bytes == best_bytes;
            const int better_tie =
                tie && best_mode != 0 &&
                (n_esc < best_esc || (n_esc == best_esc && bits < best_mode));
            if (better_size || better_tie) {
                best_mode = bits;
                best_bytes = c_bytes;
                best_esc = n_esc;
            }
        }
        if (modes) modes[blk] = (uint8_t)best_mode;
        if (w + (size_t)best_bytes > out_cap) {
            rc = fail(OX_RUNTIME, "encode_bf16: output capacity too small");
            break;
        }
        /* header, codec.cpp:105-109 */
        uint8_t *hdr = out + w;
        hdr[0] = (uint8_t)best_mode;
        hdr[1] = (uint8_t)n;
        put_u16(hdr + 2, (uint16_t)(best_mode == 0 ? 0 : best_esc));
        put_u16(hdr + 4, (uint16_t)dim);
        put_u16(hdr + 6, 0);
        w += 8;
        if (best_mode == 0) { /* raw payload, codec.cpp:111-116 */
            for (int i = 0; i < n * dim; ++i) put_u16(out + w + 2 * (size_t)i, src[i]);
            w += 2u * (size_t)n * (size_t)dim;
            continue;
        }
        /* coded payload, codec.cpp:118-161 */
        const int bits = best_mode;
        const int width = (1 << bits) - 1;
        for (int d = 0; d < dim; ++d) base_exp[d] = (uint8_t)best_base(hist + (size_t)d * 256, width);
        uint8_t *obase = out + w;
        uint8_t *osm = obase + dim;
        const size_t nel = (size_t)n * (size_t)dim;
        const size_t exp_bytes = (size_t)ox_exp_payload_bytes(n, dim, bits);
        memset(packed, 0, exp_bytes);
        int n_escapes = 0;
        for (int t = 0; t < n; ++t) {
            for (int d = 0; d < dim; ++d) {
                const int index = t * dim + d;
                const uint16_t h = src[index];
                osm[index] = bf16_sm(h);
                const int delta = (int)bf16_exponent(h) - (int)base_exp[d];
                int code;
                if (delta >= 0 && delta < width) {
                    code = delta;
                } else {
                    code = width; /* sentinel */
                    escapes[n_escapes++] = h;
                }
                if (bits == 4) {
                    if ((index & 1) == 0) packed[index >> 1] = (uint8_t)code;
                    else packed[index >> 1] |= (uint8_t)(code << 4);
                } else if (bits == 3) { /* extension: bits [3 index, 3 index + 3) */
                    const int bit = 3 * index, sh = bit & 7;
                    packed[bit >> 3] |= (uint8_t)(code << sh);
                    if (sh > 5) packed[(bit >> 3) + 1] |= (uint8_t)(code >> (8 - sh));
                } else {
                    packed[index >> 2] |= (uint8_t)(code << ((index & 3) * 2));
                }
            }
        }
        if (n_escapes != best_esc) { /* drift check, codec.cpp:153-155 */
            rc = fail(OX_LOGIC, "escape count drifted from the size model");
            break;
        }
        memcpy(obase, base_exp, (size_t)dim);
        memcpy(osm + nel, packed, exp_bytes);
        uint8_t *oesc = osm + nel + exp_bytes;
        for (int i = 0; i < n_escapes; ++i) put_u16(oesc + 2 * (size_t)i, escapes[i]);
        w += (size_t)best_bytes - 8u;
    }
    free(hist);
    free(base_exp);
    free(packed);
    free(escapes);
    if (rc == OX_OK && out_bytes) *out_bytes = w;
    return rc;
}

/* ---- scalar attention, src/attention_scalar.cpp + src/softmax.hpp + src/dispatch.cpp */

/* hsum8, attention_scalar.cpp:13-17 */
static float hsum8(const float lane[8]) {
    const float a = (lane[0] + lane[4]) + (lane[1] + lane[5]);
    const float b = (lane[2] + lane[6]) + (lane[3] + lane[7]);
    return a + b;
}

static float max_f(float a, float b) { return (a < b) ? b : a; } /* std::max semantics */

/* softmax_coeff, softmax.hpp:8-14 */
static void softmax_coeff(float *m, float *l, float score, float *alpha, float *e) {
    const float m2 = max_f(*m, score);
    *alpha = expf(*m - m2);
    *e = expf(score - m2);
    *l = fmaf(*l, *alpha, *e);
    *m = m2;
}

/* merge_state, softmax.hpp:16-30 */
static void merge_state(float *m, float *l, float *acc, const float *mb, const float *lb,
                        const float *accb, int n_q, int dim) {
    for (int g = 0; g < n_q; ++g) {
        const float mm = max_f(m[g], mb[g]);
        const float e1 = expf(m[g] - mm);
        const float e2 = expf(mb[g] - mm);
        l[g] = fmaf(l[g], e1, lb[g] * e2);
        float *a = acc + (size_t)g * (size_t)dim;
        const float *b = accb + (size_t)g * (size_t)dim;
        for (int d = 0; d < dim; ++d) a[d] = fmaf(a[d], e1, b[d] * e2);
        m[g] = mm;
    }
}

/* finalize_state, softmax.hpp:32-41: reciprocal then multiply */
static void finalize_state(const float *l, const float *acc, float *out, int n_q, int dim) {
    for (int g = 0; g < n_q; ++g) {
        const float inv = 1.0f / l[g];
        const float *a = acc + (size_t)g * (size_t)dim;
        float *o = out + (size_t)g * (size_t)dim;
        for (int d = 0; d < dim; ++d) o[d] = a[d] * inv;
    }
}

/* apply_token, attention_scalar.cpp:19-42 */
static void apply_token(const float *qfp, const uint16_t *k, const uint16_t *v, int n_q, int dim,
                        float *score, float *alpha, float *e, float *m, float *l, float *acc) {
    for (int g = 0; g < n_q; ++g) {
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const float *qg = qfp + (size_t)g * (size_t)dim;
        for (int d = 0; d < dim; d += 8)
            for (int j = 0; j < 8; ++j) lane[j] = fmaf(qg[d + j], bf16_to_fp32(k[d + j]), lane[j]);
        score[g] = hsum8(lane);
    }
    for (int g = 0; g < n_q; ++g) softmax_coeff(&m[g], &l[g], score[g], &alpha[g], &e[g]);
    for (int g = 0; g < n_q; ++g) {
        float *ag = acc + (size_t)g * (size_t)dim;
        const float eg = e[g], al = alpha[g];
        for (int d = 0; d < dim; ++d) ag[d] = fmaf(eg, bf16_to_fp32(v[d]), ag[d] * al);
    }
}

/* range_scalar, attention_scalar.cpp:46-85 */
static int range_scalar(const float *qfp, const uint16_t *k_raw, const uint16_t *v_raw,
                        const uint8_t *k_xkv, size_t k_bytes, const uint8_t *v_xkv, size_t v_bytes,
                        int n_q, int dim, int t0, int t1, float *m, float *l, float *acc,
                        float *scratch) {
    if (t0 >= t1) return OX_OK;
    float *score = scratch, *alpha = scratch + n_q, *e = scratch + 2 * n_q;
    if (k_raw != NULL) {
        for (int t = t0; t < t1; ++t)
            apply_token(qfp, k_raw + (size_t)t * dim, v_raw + (size_t)t * dim, n_q, dim, score,
                        alpha, e, m, l, acc);
        return OX_OK;
    }
    uint16_t kt[OX_MAX_DIM], vt[OX_MAX_DIM];
    reader kc, vc;
    int rc = reader_seek(&kc, k_xkv, k_bytes, dim, t0);
    if (rc) return rc;
    rc = reader_seek(&vc, v_xkv, v_bytes, dim, t0);
    if (rc) return rc;
    for (int t = t0; t < t1; ++t) {
        for (int d = 0; d < dim; ++d) {
            if ((rc = reader_next(&kc, &kt[d]))) return rc;
            if ((rc = reader_next(&vc, &vt[d]))) return rc;
        }
        apply_token(qfp, kt, vt, n_q, dim, score, alpha, e, m, l, acc);
    }
    return OX_OK;
}

/* token_bounds, dispatch.cpp:17-23 */
static void token_bounds(int seq, int tile, int tid, int nthreads, int *a, int *b) {
    const int ntiles = (seq + tile - 1) / tile;
    const int b0 = (int)((long long)tid * ntiles / nthreads);
    const int b1 = (int)((long long)(tid + 1) * ntiles / nthreads);
    *a = (seq < b0 * tile) ? seq : b0 * tile;
    *b = (seq < b1 * tile) ? seq : b1 * tile;
}

/* attention_decode, dispatch.cpp:27-104 (Scalar backend; ranges run in thread order) */
int ox_attention_decode(const uint16_t *q, const uint16_t *k_raw, const uint16_t *v_raw,
                        const uint8_t *k_xkv, size_t k_bytes, const uint8_t *v_xkv,
                        size_t v_bytes, float *out, int n_q, int dim, int seq, int n_threads,
                        int split_tokens) {
    if (q == NULL || out == NULL || n_q <= 0 || dim <= 0 || seq <= 0 || split_tokens <= 0)
        return fail(OX_INVALID_ARGUMENT, "attention_decode: bad argument");
    const int raw = k_raw != NULL, xkv = k_xkv != NULL;
    if (raw == xkv || (v_raw != NULL) != raw || (v_xkv != NULL) != xkv)
        return fail(OX_INVALID_ARGUMENT,
                    "attention_decode: pass raw K and V or xkv K and V, not both");
    /* range_scalar shape check, attention_scalar.cpp:50-52 */
    if (dim % 8 != 0 || dim <= 0 || dim > OX_MAX_DIM || n_q <= 0)
        return fail(OX_INVALID_ARGUMENT, "scalar attention: bad shape");
    const int ntiles = (seq + split_tokens - 1) / split_tokens;
    int threads = n_threads < 1 ? 1 : n_threads;
    if (threads > ntiles) threads = ntiles;

    const size_t sq = (size_t)n_q, sa = (size_t)n_q * (size_t)dim;
    float *qfp = (float *)malloc(sizeof(float) * sa);
    float *m = (float *)malloc(sizeof(float) * sq * (size_t)threads);
    float *l = (float *)malloc(sizeof(float) * sq * (size_t)threads);
    float *acc = (float *)malloc(sizeof(float) * sa * (size_t)threads);
    float *scratch = (float *)malloc(sizeof(float) * 3 * sq);
    int rc = OX_OK;
    if (!qfp || !m || !l || !acc || !scratch) {
        rc = fail(OX_RUNTIME, "attention_decode: out of memory");
        goto done;
    }
    for (size_t i = 0; i < sa; ++i) qfp[i] = bf16_to_fp32(q[i]);
    for (size_t i = 0; i < sq * (size_t)threads; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
    }
    memset(acc, 0, sizeof(float) * sa * (size_t)threads);
    if (threads == 1) {
        rc = range_scalar(qfp, k_raw, v_raw, k_xkv, k_bytes, v_xkv, v_bytes, n_q, dim, 0, seq, m,
                          l, acc, scratch);
        if (rc == OX_OK) finalize_state(l, acc, out, n_q, dim);
        goto done;
    }
    for (int tid = 0; tid < threads && rc == OX_OK; ++tid) {
        int a, b;
        token_bounds(seq, split_tokens, tid, threads, &a, &b);
        if (a < b)
            rc = range_scalar(qfp, k_raw, v_raw, k_xkv, k_bytes, v_xkv, v_bytes, n_q, dim, a, b,
                              m + (size_t)tid * sq, l + (size_t)tid * sq, acc + (size_t)tid * sa,
                              scratch);
    }
    if (rc == OX_OK) {
        for (int t = 1; t < threads; ++t)
            merge_state(m, l, acc, m + (size_t)t * sq, l + (size_t)t * sq, acc + (size_t)t * sa,
                        n_q, dim);
        finalize_state(l, acc, out, n_q, dim);
    }
done:
    free(qfp);
    free(m);
    free(l);
    free(acc);
    free(scratch);
    return rc;
}

int ox_model_heads(int n_units, const uint16_t *const *q, const uint8_t *const *k_xkv,
                   const size_t *k_bytes, const uint8_t *const *v_xkv, const size_t *v_bytes,
                   float *const *out, int n_q, int dim, int seq) {
    for (int u = 0; u < n_units; ++u) {
        int rc = ox_attention_decode(q[u], NULL, NULL, k_xkv[u], k_bytes[u], v_xkv[u], v_bytes[u],
                                     out[u], n_q, dim, seq, 1, 128);
        if (rc) return rc;
    }
    return OX_OK;
}
