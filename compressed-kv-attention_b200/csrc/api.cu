// api.cu -- host side of the C ABI (include/kvexp_b200.h).
//
// Mirrors the reference's public API and error behaviour (include/kvexp/attention.hpp,
// include/kvexp/codec.hpp): the same argument checks in the same order, with each C++
// exception type turned into a status code and its message kept in kvx_last_error().
// Everything that computes runs on the GPU; host code only validates, walks block headers of
// host-resident blobs (the same walk the reference does in include/kvexp/scan.hpp), moves
// buffers and launches kernels.
#include "codec.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace kvx {
namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

#define KVX_CUDA(call)                                                                         \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(KVX_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
    } while (0)

const char *detail_message(int code, int detail) {
    switch (detail) {
    case DERR_TRUNC_HEADER: return "truncated xkv block header";
    case DERR_DIM_LEN: return "xkv block dimension or length mismatch";
    case DERR_TRUNC_RAW: return "truncated raw xkv block";
    case DERR_MODE: return "unknown xkv block mode";
    case DERR_TRUNC_CODED: return "truncated coded xkv block";
    case DERR_OUT_OF_TOKENS: return "xkv decode ran out of blocks";
    case DERR_ESC_OVERRUN:
        return code == KVX_ERR_LOGIC ? "escape count drifted from the size model"
                                     : "xkv escape stream overrun";
    case DERR_KV_MISMATCH: return "xkv K and V blocks cover different token counts";
    case DERR_TIMEOUT: return "a bounded device wait timed out";
    case DERR_INDEX_CAP: return "xkv block index capacity exceeded";
    case DERR_RANGE: return "xkv block index entry outside its blob";
    case DERR_ESC_CAP:
        return "kvx_attention_decode_noalloc: the blobs' escape positions exceed the fixed scratch";
    default: return "device error";
    }
}


// RAII device buffer (stream-ordered allocator).
struct DevBuf {
    void *p = nullptr;
    cudaStream_t s = nullptr;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf() {
        if (p) cudaFreeAsync(p, s);
    }
    cudaError_t alloc(size_t n, cudaStream_t st) {
        s = st;
        return cudaMallocAsync(&p, n ? n : 16, st);
    }
    template <class T> T *as() const { return static_cast<T *>(p); }
};

struct EventGuard {
    cudaEvent_t e = nullptr;
    ~EventGuard() {
        if (e) cudaEventDestroy(e);
    }
};

// Drains two streams when it goes out of scope: buffers declared before it outlive every kernel
// and copy that either stream may still run, on every return path.
struct DrainGuard {
    cudaStream_t a, b;
    ~DrainGuard() {
        cudaStreamSynchronize(a);
        cudaStreamSynchronize(b);
    }
};

bool is_device_ptr(const void *p) {
    if (p == nullptr) return false;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

constexpr int kMaxDevices = 64;

int check_device() {
    int dev = 0;
    KVX_CUDA(cudaGetDevice(&dev));
    int major = 0;
    KVX_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return fail(KVX_ERR_RUNTIME, "kvexp_b200 needs an sm_100 (B200) device");
    // The host-buffer entry points take their per-call arenas from the device's default memory
    // pool; let the pool keep up to 1 GiB between calls instead of returning it to the driver at
    // every synchronisation (re-mapping a few hundred MB each call costs milliseconds).
    static std::once_flag pool_once[kMaxDevices];
    if (dev >= 0 && dev < kMaxDevices)
        std::call_once(pool_once[dev], [dev] {
            cudaMemPool_t pool;
            if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
                uint64_t keep = uint64_t(1) << 30;
                cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
            }
            cudaGetLastError();
        });
    return KVX_OK;
}

// A pinned host buffer per device for the outputs of the host-buffer entry points: one
// device -> host copy per chunk of units instead of one per unit; held (locked) by one call at a
// time, grown when a call needs more.
struct PinnedStage {
    std::mutex mu;
    void *p = nullptr;
    size_t bytes = 0;
};
PinnedStage &pinned_stage(int dev) {
    static PinnedStage stages[kMaxDevices];
    return stages[dev];
}

// A non-blocking stream per device for host -> device copies of the host-buffer entry points, so
// that work on the legacy stream (plan creation) does not wait for them.
int copy_stream(cudaStream_t *out) {
    static std::mutex mu;
    static cudaStream_t streams[kMaxDevices] = {};
    int dev = 0;
    KVX_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(KVX_ERR_RUNTIME, "kvexp_b200: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (streams[dev] == nullptr) KVX_CUDA(cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking));
    *out = streams[dev];
    return KVX_OK;
}

int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// ---- host header walk (include/kvexp/scan.hpp:28-66, :94-123) ----------------------------------

struct HostIndex {
    std::vector<kvx_block> blocks;
    std::vector<long long> tok_start;  // first token of each block
    long long tokens = 0;
};

int host_walk(const uint8_t *blob, size_t bytes, int dim, HostIndex &idx) {
    idx.blocks.clear();
    idx.tok_start.clear();
    idx.tokens = 0;
    size_t off = 0;
    while (off < bytes) {
        if (bytes - off < 8) return fail(KVX_ERR_RUNTIME, "truncated xkv block header");
        const uint8_t *p = blob + off;
        const int mode = p[0], nt = p[1];
        const int nesc = int(p[2]) | (int(p[3]) << 8);
        const int hdim = int(p[4]) | (int(p[5]) << 8);
        if (hdim != dim || nt <= 0) return fail(KVX_ERR_RUNTIME, "xkv block dimension or length mismatch");
        const size_t rest = bytes - off - 8;
        size_t need;
        if (mode == 0) {
            need = size_t(nt) * dim * 2;
            if (rest < need) return fail(KVX_ERR_RUNTIME, "truncated raw xkv block");
        } else if (mode != 2 && mode != 3 && mode != 4) {  // 3: the library's 3-bit extension
            return fail(KVX_ERR_RUNTIME, "unknown xkv block mode");
        } else {
            need = size_t(dim) + size_t(nt) * dim + size_t(exp_payload_bytes(nt, dim, mode)) +
                   2u * size_t(nesc);
            if (rest < need) return fail(KVX_ERR_RUNTIME, "truncated coded xkv block");
        }
        if (off > 0xFFFFFFFFull)
            return fail(KVX_ERR_UNSUPPORTED, "xkv blob larger than 4 GiB per tensor");
        kvx_block b;
        b.offset = uint32_t(off);
        b.n_escape = uint16_t(mode == 0 ? 0 : nesc);
        b.mode = uint8_t(mode);
        b.n_tokens = uint8_t(nt);
        idx.blocks.push_back(b);
        idx.tok_start.push_back(idx.tokens);
        idx.tokens += nt;
        off += 8 + need;
    }
    return KVX_OK;
}

// token_bounds, reference src/dispatch.cpp:17-23
void token_bounds(int seq, int tile, int tid, int nthreads, int &a, int &b) {
    const int ntiles = (seq + tile - 1) / tile;
    const int b0 = int((long long)tid * ntiles / nthreads);
    const int b1 = int((long long)(tid + 1) * ntiles / nthreads);
    a = std::min(seq, b0 * tile);
    b = std::min(seq, b1 * tile);
}

// The reference throws when a thread's range starts inside an encoded block
// (include/kvexp/scan.hpp:107-109); reproduce that check for the caller's n_threads/split.
int check_split(const std::vector<long long> &tok_start, long long tokens, int seq, int n_threads,
                int split) {
    const int ntiles = (seq + split - 1) / split;
    int threads = std::max(1, n_threads);
    threads = std::min(threads, ntiles);
    if (threads == 1) return KVX_OK;
    for (int t = 0; t < threads; ++t) {
        int a, b;
        token_bounds(seq, split, t, threads, a, b);
        if (a >= b || a == 0) continue;
        if (a > tokens) return fail(KVX_ERR_RUNTIME, "xkv seek past end");
        if (a == tokens) continue;
        if (!std::binary_search(tok_start.begin(), tok_start.end(), (long long)a))
            return fail(KVX_ERR_RUNTIME, "token split is not aligned to an encoded block");
    }
    return KVX_OK;
}

// ---- shape rules of the reference backends --------------------------------------------------------

int check_attention_args(int backend, const uint16_t *q, const uint16_t *k_raw,
                         const uint16_t *v_raw, const uint8_t *k_xkv, const uint8_t *v_xkv,
                         const float *out, int n_q, int dim, int seq, int split_tokens) {
    // src/dispatch.cpp:31-38
    if (q == nullptr || out == nullptr || n_q <= 0 || dim <= 0 || seq <= 0 || split_tokens <= 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, "attention_decode: bad argument");
    const bool raw = k_raw != nullptr, xkv = k_xkv != nullptr;
    if (raw == xkv || (v_raw != nullptr) != raw || (v_xkv != nullptr) != xkv)
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    "attention_decode: pass raw K and V or xkv K and V, not both");
    if (backend != KVX_BACKEND_SCALAR && backend != KVX_BACKEND_AVX2 &&
        backend != KVX_BACKEND_AVX512BF16)
        return fail(KVX_ERR_INVALID_ARGUMENT, "attention_decode: unknown backend");
    // range_* shape checks (src/attention_scalar.cpp:50-52, avx2 :142-144, avx512 :157-159)
    if (backend == KVX_BACKEND_AVX512BF16) {
        if (dim % 32 != 0 || dim > kMaxHeadDim)
            return fail(KVX_ERR_INVALID_ARGUMENT,
                        "avx512 attention: head_dim must be a multiple of 32");
    } else if (dim % 8 != 0 || dim > kMaxHeadDim) {
        return fail(KVX_ERR_INVALID_ARGUMENT, backend == KVX_BACKEND_AVX2
                                                  ? "avx2 attention: bad shape"
                                                  : "scalar attention: bad shape");
    }
    return KVX_OK;
}

// The fused kernels' head dims: 32, 64, 128, 256.  The drop-in single-head call takes every
// head_dim the reference's backends take (a multiple of 8, or of 32 for AVX-512, up to 256) and
// runs the others zero-padded to the next of these.
int padded_dim(int dim) { return dim <= 32 ? 32 : dim <= 64 ? 64 : dim <= 128 ? 128 : 256; }

}  // namespace
}  // namespace kvx

using namespace kvx;

// ---- plans -------------------------------------------------------------------------------------------

struct kvx_plan_s {
    int dim = 0;
    bool bf16 = false;
    int n_units = 0;      // device units (query groups of <= 8)
    int64_t n_blocks = 0;
    int n_ranges = 0;     // CTA ranges of the attention grid (one CTA each)
    int64_t n_rows = 0;   // partial-state rows (one per unit segment of a CTA range)
    int stages_per_block = 0;  // ring stages of every block in the attention kernel (0: by block)
    bool compact = false;      // every block is coded: the attention kernel's compact ring
    cudaStream_t s = nullptr;
    UnitDev *units = nullptr;
    FlatBlock *flat = nullptr;
    BlockDesc *desc = nullptr;  // per flat block, for the attention kernel
    uint4 *stages = nullptr;    // stage copy lists ([n_blocks][stages_per_block][kStageRecWords])
    uint32_t *esc = nullptr;  // escape records of the step's coded blocks
    uint32_t *b7 = nullptr;   // merge words of the step's coded blocks ([n_blocks][dim])
    int64_t *range_begin = nullptr;
    int32_t *seg_base = nullptr;
    float *partials = nullptr;
    SplitUnit *split_units = nullptr;  // every unit, as the combine pass sees it
    int *status = nullptr;
    // Internal plans of the host-buffer entry points take their arrays from the device's memory
    // pool (stream-ordered on the legacy stream) and are destroyed only after that stream has
    // drained; plans made by kvx_plan_create use cudaMalloc / cudaFree.
    bool pooled = false;
    unsigned long long esc_total = 0;  // escape record entries (u32)
    std::vector<void *> owned;
    ~kvx_plan_s() {
        for (void *p : owned) {
            if (pooled) cudaFreeAsync(p, nullptr);
            else cudaFree(p);
        }
    }
};

namespace {

template <class T> cudaError_t plan_alloc(kvx_plan_s *p, T **dst, size_t n) {
    void *q = nullptr;
    cudaError_t e = p->pooled ? cudaMallocAsync(&q, n ? n * sizeof(T) : 16, nullptr)
                              : cudaMalloc(&q, n ? n * sizeof(T) : 16);
    if (e == cudaSuccess) {
        p->owned.push_back(q);
        *dst = static_cast<T *>(q);
    }
    return e;
}

// The partial-state rows of a step from its CTA ranges: seg_base per CTA and, per unit, the
// combine pass's view (its run of states: one per consumer warp of each of its rows).
int64_t plan_segments(const std::vector<int64_t> &tb, int n_ranges, const std::vector<UnitDev> &ud,
                      int dim, std::vector<int32_t> &seg_base, std::vector<SplitUnit> &split) {
    const size_t n = ud.size();
    std::vector<int64_t> ub(n);
    std::vector<int32_t> nb(n), first(n), rows(n);
    for (size_t u = 0; u < n; ++u) {
        ub[u] = ud[u].block_begin;
        nb[u] = ud[u].n_blocks;
    }
    seg_base.assign(size_t(n_ranges), 0);
    const int64_t total = segment_rows(tb.data(), n_ranges, ub.data(), nb.data(), int(n),
                                       seg_base.data(), first.data(), rows.data());
    const int nw = attention_consumer_warps(dim);
    split.resize(n);
    for (size_t u = 0; u < n; ++u) {
        SplitUnit &x = split[u];
        x = SplitUnit{};
        x.out = ud[u].out;
        x.lse = ud[u].lse;
        x.first_state = first[u] * nw;
        x.n_states = rows[u] * nw;
        x.n_q = ud[u].n_q;
        x.q_stride = ud[u].q_stride;
    }
    return total;
}

struct PlanGuard {
    kvx_plan_s *p;
    ~PlanGuard() { delete p; }
};

int read_status(int *dev_status, bool reset) {
    int st[2] = {0, 0};
    KVX_CUDA(cudaMemcpy(st, dev_status, sizeof st, cudaMemcpyDeviceToHost));
    if (st[0] == 0) return KVX_OK;
    if (reset) cudaMemset(dev_status, 0, sizeof st);
    return fail(st[0], detail_message(st[0], st[1]));
}

}  // namespace

extern "C" {

const char *kvx_last_error(void) { return g_err.c_str(); }

const char *kvx_version(void) { return "kvexp_b200 0.1 (sm_100a)"; }

int kvx_device_info(int *sm_major, int *sm_minor, int *sms, size_t *hbm_bytes) {
    int dev = 0;
    KVX_CUDA(cudaGetDevice(&dev));
    int ma = 0, mi = 0, n = 0;
    KVX_CUDA(cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, dev));
    KVX_CUDA(cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, dev));
    KVX_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    size_t fr = 0, tot = 0;
    KVX_CUDA(cudaMemGetInfo(&fr, &tot));
    if (sm_major) *sm_major = ma;
    if (sm_minor) *sm_minor = mi;
    if (sms) *sms = n;
    if (hbm_bytes) *hbm_bytes = tot;
    if (ma != 10) return fail(KVX_ERR_RUNTIME, "kvexp_b200 needs an sm_100 (B200) device");
    g_err.clear();
    return KVX_OK;
}

// Plan creation.  `pooled`: the plan's arrays come from the device's memory pool (internal
// plans).  `blobs_ready`: when given, the blob contents may still be in flight on another stream;
// everything that reads only the block indexes (flat list, escape record sizes, worker split) is
// done at once, and the escape records and block descriptors, which read the blobs, are enqueued
// on the legacy stream behind the event, without waiting on the host; their errors then surface
// at kvx_plan_check after the run.
// The plan work that reads the blobs: escape records, then block descriptors (legacy stream,
// behind `blobs_ready` when given).
static cudaError_t plan_blob_work(kvx_plan_s *p, cudaEvent_t blobs_ready) {
    cudaError_t e = cudaSuccess;
    if (blobs_ready != nullptr) e = cudaStreamWaitEvent(nullptr, blobs_ready, 0);
    if (e == cudaSuccess && p->esc_total > 0)
        e = launch_esc_fill(p->units, p->flat, p->n_blocks, p->dim, p->esc, p->esc_total, p->status, nullptr);
    if (e == cudaSuccess && !p->bf16) e = launch_b7(p->units, p->flat, p->n_blocks, p->dim, p->b7, nullptr);
    if (e == cudaSuccess)
        e = launch_block_desc(p->units, p->flat, p->esc, p->n_blocks, p->dim, p->bf16, p->desc, nullptr);
    if (e == cudaSuccess && p->stages != nullptr)
        e = launch_stage_table(p->dim, p->bf16, p->compact, p->desc, p->b7, p->esc, p->n_blocks,
                               p->stages_per_block, p->stages, nullptr);
    return e;
}

// `defer_blob_work`: return once the blob-independent part is done; the caller enqueues
// plan_blob_work later (so that preparing several plans never waits on a copy).  `by_tokens`: cut
// the CTA ranges by token counts alone (an XKV plan and a BF16 plan over the same tokens then get
// the same ranges, and bit-identical outputs); otherwise by decode cost (residual width, raw rows,
// escape words).
static int plan_create_impl(const kvx_unit *units, int n_units, int n_q, int dim, int block_tokens,
                            kvx_plan *out, bool pooled, cudaEvent_t blobs_ready,
                            bool defer_blob_work = false, bool by_tokens = false) {
    if (out == nullptr || units == nullptr || n_units <= 0 || n_q <= 0 || block_tokens <= 0 ||
        block_tokens > 255)
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_create: bad argument");
    *out = nullptr;
    if (int rc = check_device()) return rc;
    if (!attention_dim_supported(dim))
        return fail(KVX_ERR_UNSUPPORTED,
                    "kvexp_b200: head_dim must be 32, 64, 128 or 256 for the GPU kernels");
    const bool bf16 = units[0].k_index == nullptr;
    if (bf16) by_tokens = true;
    const int groups = (n_q + 7) / 8;
    std::vector<kvx_unit> vu;
    std::vector<UnitDev> ud;
    std::vector<int64_t> begin, src;
    int64_t total = 0;
    vu.reserve(size_t(n_units) * groups);
    for (int u = 0; u < n_units; ++u) {
        const kvx_unit &x = units[u];
        if ((x.k_index == nullptr) != bf16 || (x.v_index == nullptr) != bf16)
            return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_create: mixed raw and xkv units");
        if (x.k == nullptr || x.v == nullptr || x.q == nullptr || x.out == nullptr || x.seq <= 0)
            return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_create: bad unit");
        if ((reinterpret_cast<uintptr_t>(x.k) | reinterpret_cast<uintptr_t>(x.v)) & 15u)
            return fail(KVX_ERR_INVALID_ARGUMENT,
                        "kvx_plan_create: K/V buffers must be 16-byte aligned");
        const int nb = bf16 ? (x.seq + block_tokens - 1) / block_tokens : x.n_blocks;
        if (nb <= 0) return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_create: unit without blocks");
        for (int g = 0; g < groups; ++g) {
            kvx_unit y = x;
            y.n_blocks = nb;
            vu.push_back(y);
            UnitDev d{};
            d.k = static_cast<const uint8_t *>(x.k);
            d.v = static_cast<const uint8_t *>(x.v);
            d.q = x.q + size_t(8) * g * dim;
            d.out = x.out + size_t(8) * g * dim;
            d.lse = x.lse != nullptr ? x.lse + size_t(8) * g : nullptr;
            d.block_begin = total;
            d.n_blocks = nb;
            d.n_q = std::min(8, n_q - 8 * g);
            d.q_stride = dim;
            ud.push_back(d);
            // query groups of one unit share its K/V blocks and their escape records
            src.push_back(g == 0 ? total : begin[begin.size() - size_t(g)]);
            begin.push_back(total);
            total += nb;
        }
    }
    if (total > int64_t(0x7FFFFFFF))
        return fail(KVX_ERR_UNSUPPORTED, "kvx_plan_create: more than 2^31 - 1 blocks in one step");
    auto *p = new kvx_plan_s();
    p->pooled = pooled;
    p->dim = dim;
    p->bf16 = bf16;
    p->n_units = int(vu.size());
    p->n_blocks = total;
    // one CTA per SM, each with a cost-balanced range of flat blocks
    p->n_ranges = int(std::min<int64_t>(sm_count(), total));
    std::vector<int64_t> tb(size_t(p->n_ranges) + 1);
    kvx_unit *dvu = nullptr;
    int64_t *dbegin = nullptr, *dsrc = nullptr;
    unsigned long long *desc_total = nullptr;
    cudaError_t e = cudaSuccess;
    if ((e = plan_alloc(p, &p->units, ud.size())) != cudaSuccess ||
        (e = plan_alloc(p, &p->flat, size_t(total))) != cudaSuccess ||
        (e = plan_alloc(p, &p->desc, size_t(total))) != cudaSuccess ||
        (e = plan_alloc(p, &p->b7, bf16 ? size_t(0) : size_t(total) * size_t(dim))) != cudaSuccess ||
        (e = plan_alloc(p, &p->range_begin, tb.size())) != cudaSuccess ||
        (e = plan_alloc(p, &p->seg_base, size_t(p->n_ranges))) != cudaSuccess ||
        (e = plan_alloc(p, &p->split_units, ud.size())) != cudaSuccess ||
        (e = plan_alloc(p, &p->status, 2)) != cudaSuccess ||
        (e = plan_alloc(p, &dvu, vu.size())) != cudaSuccess ||
        (e = plan_alloc(p, &dbegin, begin.size())) != cudaSuccess ||
        (e = plan_alloc(p, &dsrc, src.size())) != cudaSuccess ||
        (e = plan_alloc(p, &desc_total, 2)) != cudaSuccess) {
        delete p;
        return fail(KVX_ERR_CUDA, std::string("kvx_plan_create: ") + cudaGetErrorString(e));
    }
    cudaMemcpy(p->units, ud.data(), ud.size() * sizeof(UnitDev), cudaMemcpyHostToDevice);
    cudaMemcpy(dvu, vu.data(), vu.size() * sizeof(kvx_unit), cudaMemcpyHostToDevice);
    cudaMemcpy(dbegin, begin.data(), begin.size() * sizeof(int64_t), cudaMemcpyHostToDevice);
    cudaMemcpy(dsrc, src.data(), src.size() * sizeof(int64_t), cudaMemcpyHostToDevice);
    cudaMemset(p->status, 0, 2 * sizeof(int));
    e = launch_build_flat(dvu, dbegin, dsrc, p->n_units, dim, block_tokens, bf16, p->flat,
                          p->status, nullptr);
    // every block takes the same number of ring stages in the attention kernel (enough for the
    // longest block; shorter ones get empty stages), so a consumer warp goes straight to the stage
    // of each of its tiles
    int max_valid[2] = {0, 0};  // longest block, any raw block
    if (e == cudaSuccess)
        e = launch_max_valid(p->flat, total, reinterpret_cast<int *>(desc_total + 1), nullptr);
    if (e == cudaSuccess)
        e = cudaMemcpy(max_valid, desc_total + 1, sizeof max_valid, cudaMemcpyDeviceToHost);
    {
        const int tsb = attention_stage_tokens(dim);
        p->stages_per_block = max_valid[0] > 0 ? (max_valid[0] + tsb - 1) / tsb : 0;
        p->compact = !bf16 && max_valid[1] == 0;
    }
    // escape records: offsets, then (with the array sized) the records
    unsigned long long esc_total = 0;
    if (e == cudaSuccess && !bf16)
        e = launch_esc_layout(p->flat, total, desc_total, ~0ull, p->status, nullptr);
    if (e == cudaSuccess && !bf16)
        e = cudaMemcpy(&esc_total, desc_total, sizeof esc_total, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && esc_total > 0xFFFFFFFFull) {
        delete p;
        return fail(KVX_ERR_UNSUPPORTED, "kvx_plan_create: more than 2^32 escape record entries");
    }
    // (+4 entries: the kernel's 16-byte aligned bulk copies may read up to 12 bytes past the end)
    if (e == cudaSuccess) e = plan_alloc(p, &p->esc, size_t(esc_total) + 4);
    if (e == cudaSuccess && p->stages_per_block > 0)
        e = plan_alloc(p, &p->stages, size_t(total) * size_t(p->stages_per_block) * kStageRecWords);
    if (e != cudaSuccess) {
        delete p;
        return fail(KVX_ERR_CUDA, std::string("kvx_plan_create: ") + cudaGetErrorString(e));
    }
    // CTA ranges of about equal cost; with no more blocks than CTAs every block is its own range.
    if (total <= p->n_ranges) {
        for (int t = 0; t <= p->n_ranges; ++t) tb[size_t(t)] = t;
        e = cudaMemcpy(p->range_begin, tb.data(), tb.size() * sizeof(int64_t), cudaMemcpyHostToDevice);
    } else {
        e = launch_split(p->flat, total, p->n_ranges, by_tokens, dim, p->range_begin, nullptr);
        if (e == cudaSuccess)
            e = cudaMemcpy(tb.data(), p->range_begin, tb.size() * sizeof(int64_t),
                           cudaMemcpyDeviceToHost);
    }
    // the partial-state rows of every unit segment of every range, and the combine's unit list
    std::vector<int32_t> seg_base;
    std::vector<SplitUnit> split;
    if (e == cudaSuccess) {
        p->n_rows = plan_segments(tb, p->n_ranges, ud, dim, seg_base, split);
        e = cudaMemcpy(p->seg_base, seg_base.data(), seg_base.size() * sizeof(int32_t),
                       cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess)
        e = cudaMemcpy(p->split_units, split.data(), split.size() * sizeof(SplitUnit),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = plan_alloc(p, &p->partials,
                       size_t(p->n_rows) * attention_consumer_warps(dim) * partial_stride(dim));
    if (e == cudaSuccess)
        e = launch_init_partials(p->partials, p->n_rows * attention_consumer_warps(dim), dim, nullptr);
    if (e != cudaSuccess) {
        delete p;
        return fail(KVX_ERR_CUDA, std::string("kvx_plan_create: ") + cudaGetErrorString(e));
    }
    // errors of the flat list and the record layout (the copies above waited for those kernels)
    if (int rc = read_status(p->status, true)) {
        delete p;
        return rc;
    }
    p->esc_total = esc_total;
    if (defer_blob_work) {
        *out = p;
        g_err.clear();
        return KVX_OK;
    }
    // escape records and block descriptors read the blobs
    e = plan_blob_work(p, blobs_ready);
    if (e == cudaSuccess && blobs_ready == nullptr) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        delete p;
        return fail(KVX_ERR_CUDA, std::string("kvx_plan_create: ") + cudaGetErrorString(e));
    }
    if (blobs_ready == nullptr) {
        if (int rc = read_status(p->status, true)) {
            delete p;
            return rc;
        }
    }
    *out = p;
    g_err.clear();
    return KVX_OK;
}

int kvx_plan_create(const kvx_unit *units, int n_units, int n_q, int dim, int block_tokens,
                    kvx_plan *out) {
    return plan_create_impl(units, n_units, n_q, dim, block_tokens, out, false, nullptr);
}

int kvx_plan_run(kvx_plan p, void *stream) {
    if (int rc = kvx_plan_run_part(p, 0, stream)) return rc;
    return kvx_plan_run_part(p, 1, stream);
}

int kvx_plan_run_part(kvx_plan p, int part, void *stream) {
    if (p == nullptr) return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_run: null plan");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (part == 1) {
        CombineArgs c{};
        c.split = p->split_units;
        c.partials = p->partials;
        KVX_CUDA(launch_combine(p->dim, c, p->n_units, s));
        return KVX_OK;
    }
    if (part != 0) return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_run_part: part is 0 or 1");
    AttnArgs a{};
    a.units = p->units;
    a.flat = p->flat;
    a.desc = p->desc;
    a.stages = p->stages;
    a.esc = p->esc;
    a.b7 = p->b7;
    a.range_begin = p->range_begin;
    a.seg_base = p->seg_base;
    a.partials = p->partials;
    a.status = p->status;
    a.n_ranges = p->n_ranges;
    a.stages_per_block = p->stages_per_block;
    KVX_CUDA(launch_attention(p->dim, p->bf16, p->compact, a, p->n_ranges, s));
    return KVX_OK;
}

int kvx_plan_check(kvx_plan p) {
    if (p == nullptr) return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_plan_check: null plan");
    KVX_CUDA(cudaDeviceSynchronize());
    if (int rc = read_status(p->status, true)) return rc;
    g_err.clear();
    return KVX_OK;
}

int kvx_plan_launches(kvx_plan p) { return p ? 2 : 0; }

int kvx_plan_split_units(kvx_plan p) { return p ? p->n_units : 0; }

void kvx_plan_destroy(kvx_plan p) { delete p; }

}  // extern "C"

// ---- drop-in attention ---------------------------------------------------------------------------

namespace {

// Device-side copy of one XKV blob (or its original pointer when already on the device) plus
// its block index on the device.
struct DevBlob {
    DevBuf buf;                 // owned copy of a host blob (16-byte padded)
    DevBuf idx;                 // device index
    const uint8_t *ptr = nullptr;
    int n_blocks = 0;
    long long tokens = 0;
    std::vector<long long> tok_start;
};

int prepare_blob(const uint8_t *blob, size_t bytes, int dim, int seq, DevBlob &db,
                 cudaStream_t s) {
    HostIndex hi;
    if (!is_device_ptr(blob)) {
        if (int rc = host_walk(blob, bytes, dim, hi)) return rc;
        KVX_CUDA(db.buf.alloc((bytes + 31) & ~size_t(15), s));
        KVX_CUDA(cudaMemcpyAsync(db.buf.p, blob, bytes, cudaMemcpyHostToDevice, s));
        db.ptr = db.buf.as<uint8_t>();
    } else {
        if (reinterpret_cast<uintptr_t>(blob) & 15u) {
            // keep the 16-byte alignment the bulk copies rely on
            KVX_CUDA(db.buf.alloc((bytes + 31) & ~size_t(15), s));
            KVX_CUDA(cudaMemcpyAsync(db.buf.p, blob, bytes, cudaMemcpyDeviceToDevice, s));
            db.ptr = db.buf.as<uint8_t>();
        } else {
            db.ptr = blob;
        }
        // device walk, then bring the index home for the split check
        const int cap = int(std::min<size_t>(bytes / 8 + 1, size_t(1) << 30));
        DevBuf d_idx, d_tok, d_cnt;
        KVX_CUDA(d_idx.alloc(size_t(cap) * sizeof(kvx_block), s));
        KVX_CUDA(d_tok.alloc(size_t(cap) * sizeof(uint32_t), s));
        KVX_CUDA(d_cnt.alloc(4 * sizeof(long long), s));
        KVX_CUDA(cudaMemsetAsync(d_cnt.p, 0, 4 * sizeof(long long), s));
        int *counts = d_cnt.as<int>();
        long long *ntok = d_cnt.as<long long>() + 1;
        int *status = d_cnt.as<int>() + 4;
        KVX_CUDA(launch_index_walk(db.ptr, bytes, dim, d_idx.as<kvx_block>(), d_tok.as<uint32_t>(),
                                   cap, counts, ntok, status, s));
        long long host_cnt[4];
        KVX_CUDA(cudaMemcpyAsync(host_cnt, d_cnt.p, sizeof host_cnt, cudaMemcpyDeviceToHost, s));
        KVX_CUDA(cudaStreamSynchronize(s));
        const int *hc = reinterpret_cast<const int *>(host_cnt);
        if (hc[4] != 0) return fail(hc[4], detail_message(hc[4], hc[5]));
        const int nb = hc[0];
        hi.blocks.resize(static_cast<size_t>(nb));
        std::vector<uint32_t> ts(static_cast<size_t>(nb));
        KVX_CUDA(cudaMemcpy(hi.blocks.data(), d_idx.p, size_t(nb) * sizeof(kvx_block),
                            cudaMemcpyDeviceToHost));
        KVX_CUDA(cudaMemcpy(ts.data(), d_tok.p, size_t(nb) * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost));
        hi.tok_start.assign(ts.begin(), ts.end());
        hi.tokens = host_cnt[1];
    }
    if (hi.tokens < seq) return fail(KVX_ERR_RUNTIME, "xkv decode ran out of blocks");
    // blocks covering [0, seq)
    int nb = 0;
    while (nb < int(hi.blocks.size()) && hi.tok_start[size_t(nb)] < seq) ++nb;
    db.n_blocks = nb;
    db.tokens = hi.tokens;
    db.tok_start = hi.tok_start;
    KVX_CUDA(db.idx.alloc(size_t(std::max(nb, 1)) * sizeof(kvx_block), s));
    if (nb > 0)
        KVX_CUDA(cudaMemcpyAsync(db.idx.p, hi.blocks.data(), size_t(nb) * sizeof(kvx_block),
                                 cudaMemcpyHostToDevice, s));
    // the host copy above reads hi.blocks: finish before it goes out of scope
    KVX_CUDA(cudaStreamSynchronize(s));
    return KVX_OK;
}

// Copy (or alias) a host/device array to the device.
int to_device(const void *src, size_t bytes, DevBuf &buf, const void *&dptr, cudaStream_t s) {
    if (is_device_ptr(src) && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        dptr = src;
        return KVX_OK;
    }
    KVX_CUDA(buf.alloc((bytes + 31) & ~size_t(15), s));
    KVX_CUDA(cudaMemcpyAsync(buf.p, src, bytes,
                             is_device_ptr(src) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                             s));
    dptr = buf.p;
    return KVX_OK;
}

int run_units(std::vector<kvx_unit> &units, int n_q, int dim, int block_tokens, cudaStream_t s);

// kvx_attention_decode for a head_dim the fused kernels do not take: K and V as [seq, dim] BF16 on
// the device (XKV blobs decoded by the GPU decoder), zero-padded with Q to the next fused width
// and run through the BF16-input kernel in tiles of split_tokens rows.  Zero columns add exact
// zeros to every score and only the first dim output columns are returned; raw and XKV inputs
// reach the tensor cores as the same tiles, so their outputs are bit-identical (the reference's
// invariant, include/kvexp/attention.hpp:48-50).
int attention_decode_padded(const uint16_t *q, const uint16_t *k_raw, const uint16_t *v_raw,
                            const uint8_t *k_xkv, size_t k_bytes, const uint8_t *v_xkv,
                            size_t v_bytes, float *out, int n_q, int dim, int seq, int n_threads,
                            int split_tokens) {
    cudaStream_t s = nullptr;
    const int dp = padded_dim(dim);
    const bool xkv = k_xkv != nullptr;
    DevBuf kv_dense[2], kv_pad[2], st, tok, qb, qp, ob;
    const void *dense[2] = {nullptr, nullptr};
    if (xkv) {
        DevBlob kb, vb;
        if (int rc = prepare_blob(k_xkv, k_bytes, dim, seq, kb, s)) return rc;
        if (int rc = prepare_blob(v_xkv, v_bytes, dim, seq, vb, s)) return rc;
        if (int rc = check_split(kb.tok_start, kb.tokens, seq, n_threads, split_tokens)) return rc;
        if (int rc = check_split(vb.tok_start, vb.tokens, seq, n_threads, split_tokens)) return rc;
        if (kb.n_blocks != vb.n_blocks)
            return fail(KVX_ERR_RUNTIME, "xkv K and V blocks cover different token counts");
        KVX_CUDA(st.alloc(2 * sizeof(int), s));
        KVX_CUDA(cudaMemsetAsync(st.p, 0, 2 * sizeof(int), s));
        DevBlob *blobs[2] = {&kb, &vb};
        for (int t = 0; t < 2; ++t) {
            DevBlob &b = *blobs[t];
            std::vector<uint32_t> ts(b.tok_start.begin(), b.tok_start.begin() + b.n_blocks);
            DevBuf tk;
            KVX_CUDA(tk.alloc(std::max<size_t>(ts.size(), 1) * 4, s));
            KVX_CUDA(cudaMemcpyAsync(tk.p, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice, s));
            KVX_CUDA(kv_dense[t].alloc(size_t(seq) * dim * 2, s));
            KVX_CUDA(launch_decode(b.ptr, b.idx.as<kvx_block>(), tk.as<uint32_t>(), b.n_blocks, dim,
                                   seq, kv_dense[t].as<uint16_t>(), st.as<int>(), s));
            KVX_CUDA(cudaStreamSynchronize(s));  // ts and tk go out of scope
            dense[t] = kv_dense[t].p;
        }
        if (int rc = read_status(st.as<int>(), false)) return rc;
    } else {
        if (int rc = to_device(k_raw, size_t(seq) * dim * 2, kv_dense[0], dense[0], s)) return rc;
        if (int rc = to_device(v_raw, size_t(seq) * dim * 2, kv_dense[1], dense[1], s)) return rc;
    }
    for (int t = 0; t < 2; ++t) {
        KVX_CUDA(kv_pad[t].alloc(size_t(seq) * dp * 2, s));
        KVX_CUDA(launch_pad_rows(static_cast<const uint16_t *>(dense[t]), seq, dim, dp,
                                 kv_pad[t].as<uint16_t>(), s));
    }
    const void *qd = nullptr;
    if (int rc = to_device(q, size_t(n_q) * dim * 2, qb, qd, s)) return rc;
    KVX_CUDA(qp.alloc(size_t(n_q) * dp * 2, s));
    KVX_CUDA(launch_pad_rows(static_cast<const uint16_t *>(qd), n_q, dim, dp, qp.as<uint16_t>(), s));
    KVX_CUDA(ob.alloc(size_t(n_q) * dp * 4, s));
    kvx_unit u{};
    u.k = kv_pad[0].p;
    u.v = kv_pad[1].p;
    u.q = qp.as<uint16_t>();
    u.out = ob.as<float>();
    u.seq = seq;
    std::vector<kvx_unit> us{u};
    if (int rc = run_units(us, n_q, dp, std::min(split_tokens, 255), s)) return rc;
    // the first dim columns of each output row
    KVX_CUDA(cudaMemcpy2D(out, size_t(dim) * 4, ob.p, size_t(dp) * 4, size_t(dim) * 4, size_t(n_q),
                          is_device_ptr(out) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost));
    g_err.clear();
    return KVX_OK;
}

int run_units(std::vector<kvx_unit> &units, int n_q, int dim, int block_tokens, cudaStream_t s) {
    KVX_CUDA(cudaStreamSynchronize(s));
    kvx_plan plan = nullptr;
    if (int rc = plan_create_impl(units.data(), int(units.size()), n_q, dim, block_tokens, &plan,
                                  false, nullptr, false, true))
        return rc;
    int rc = kvx_plan_run(plan, s);
    if (rc == KVX_OK) rc = kvx_plan_check(plan);
    kvx_plan_destroy(plan);
    return rc;
}

}  // namespace

extern "C" int kvx_attention_decode(int backend, const uint16_t *q, const uint16_t *k_raw,
                                    const uint16_t *v_raw, const uint8_t *k_xkv, size_t k_bytes,
                                    const uint8_t *v_xkv, size_t v_bytes, float *out, int n_q,
                                    int dim, int seq, int n_threads, int split_tokens) {
    if (int rc = check_attention_args(backend, q, k_raw, v_raw, k_xkv, v_xkv, out, n_q, dim, seq,
                                      split_tokens))
        return rc;
    if (int rc = check_device()) return rc;
    if (!attention_dim_supported(dim))
        return attention_decode_padded(q, k_raw, v_raw, k_xkv, k_bytes, v_xkv, v_bytes, out, n_q,
                                       dim, seq, n_threads, split_tokens);
    cudaStream_t s = nullptr;
    const bool xkv = k_xkv != nullptr;
    DevBlob kb, vb;
    DevBuf kr, vr, qb, ob;
    kvx_unit u{};
    int block = split_tokens;
    if (xkv) {
        if (int rc = prepare_blob(k_xkv, k_bytes, dim, seq, kb, s)) return rc;
        if (int rc = prepare_blob(v_xkv, v_bytes, dim, seq, vb, s)) return rc;
        if (int rc = check_split(kb.tok_start, kb.tokens, seq, n_threads, split_tokens)) return rc;
        if (int rc = check_split(vb.tok_start, vb.tokens, seq, n_threads, split_tokens)) return rc;
        if (kb.n_blocks != vb.n_blocks)
            return fail(KVX_ERR_RUNTIME, "xkv K and V blocks cover different token counts");
        u.k = kb.ptr;
        u.v = vb.ptr;
        u.k_index = kb.idx.as<kvx_block>();
        u.v_index = vb.idx.as<kvx_block>();
        u.k_bytes = k_bytes;
        u.v_bytes = v_bytes;
        u.n_blocks = kb.n_blocks;
        block = 128;
    } else {
        if (block > 255) block = 255;
        const void *kp = nullptr, *vp = nullptr;
        if (int rc = to_device(k_raw, size_t(seq) * dim * 2, kr, kp, s)) return rc;
        if (int rc = to_device(v_raw, size_t(seq) * dim * 2, vr, vp, s)) return rc;
        u.k = kp;
        u.v = vp;
    }
    const void *qp = nullptr;
    if (int rc = to_device(q, size_t(n_q) * dim * 2, qb, qp, s)) return rc;
    const bool out_dev = is_device_ptr(out) && (reinterpret_cast<uintptr_t>(out) & 3u) == 0;
    float *op = out;
    if (!out_dev) {
        KVX_CUDA(ob.alloc(size_t(n_q) * dim * 4, s));
        op = ob.as<float>();
    }
    u.q = static_cast<const uint16_t *>(qp);
    u.out = op;
    u.seq = seq;
    std::vector<kvx_unit> us{u};
    if (int rc = run_units(us, n_q, dim, block, s)) return rc;
    if (!out_dev) KVX_CUDA(cudaMemcpy(out, op, size_t(n_q) * dim * 4, cudaMemcpyDeviceToHost));
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_attention_decode_units(int backend, int n_units, const uint16_t *const *q,
                                          const uint8_t *const *k_xkv, const size_t *k_bytes,
                                          const uint8_t *const *v_xkv, const size_t *v_bytes,
                                          float *const *out, int n_q, int dim, int seq,
                                          int split_tokens) {
    if (n_units <= 0 || q == nullptr || k_xkv == nullptr || v_xkv == nullptr ||
        k_bytes == nullptr || v_bytes == nullptr || out == nullptr)
        return fail(KVX_ERR_INVALID_ARGUMENT, "attention_decode: bad argument");
    for (int u = 0; u < n_units; ++u)
        if (int rc = check_attention_args(backend, q[u], nullptr, nullptr, k_xkv[u], v_xkv[u],
                                          out[u], n_q, dim, seq, split_tokens))
            return rc;
    if (!attention_dim_supported(dim))
        return fail(KVX_ERR_UNSUPPORTED,
                    "kvexp_b200: head_dim must be 32, 64, 128 or 256 for the batched GPU kernels");
    if (int rc = check_device()) return rc;
    cudaStream_t s = nullptr;
    // One device arena for every host blob and query, copied with one transfer per buffer on the
    // copy stream; the host walks the headers and builds the plans while the copies run.  With 8
    // or more units the call runs as two chunks of units, each with its own plan behind its own
    // copies, so the first chunk's records and kernels overlap the second chunk's copies.
    cudaStream_t sc = nullptr;
    if (int rc = copy_stream(&sc)) return rc;
    std::vector<size_t> koff(static_cast<size_t>(n_units)), voff(static_cast<size_t>(n_units)), qoff(static_cast<size_t>(n_units));
    size_t arena = 0;
    auto place = [&](size_t bytes) {
        const size_t at = arena;
        arena += (bytes + 31) & ~size_t(15);
        return at;
    };
    for (int u = 0; u < n_units; ++u) {
        koff[size_t(u)] = is_device_ptr(k_xkv[u]) ? SIZE_MAX : place(k_bytes[u]);
        voff[size_t(u)] = is_device_ptr(v_xkv[u]) ? SIZE_MAX : place(v_bytes[u]);
        qoff[size_t(u)] = is_device_ptr(q[u]) ? SIZE_MAX : place(size_t(n_q) * dim * 2);
    }
    const size_t out_bytes = size_t(n_q) * dim * 4;
    const size_t out_at = arena;
    arena += size_t(n_units) * out_bytes;
    DevBuf ar;
    KVX_CUDA(ar.alloc(arena, sc));
    DrainGuard drain{s, sc};
    uint8_t *A = ar.as<uint8_t>();
    std::vector<HostIndex> kidx(static_cast<size_t>(n_units)), vidx(static_cast<size_t>(n_units));
    const int nchunk = n_units >= 8 ? 2 : 1;
    auto chunk_begin = [&](int c) { return int(int64_t(c) * n_units / nchunk); };
    EventGuard copied[2];
    for (int c = 0; c < nchunk; ++c) {
        for (int u = chunk_begin(c); u < chunk_begin(c + 1); ++u) {
            if (koff[size_t(u)] != SIZE_MAX)
                KVX_CUDA(cudaMemcpyAsync(A + koff[size_t(u)], k_xkv[u], k_bytes[u], cudaMemcpyHostToDevice, sc));
            if (voff[size_t(u)] != SIZE_MAX)
                KVX_CUDA(cudaMemcpyAsync(A + voff[size_t(u)], v_xkv[u], v_bytes[u], cudaMemcpyHostToDevice, sc));
            if (qoff[size_t(u)] != SIZE_MAX)
                KVX_CUDA(cudaMemcpyAsync(A + qoff[size_t(u)], q[u], size_t(n_q) * dim * 2,
                                         cudaMemcpyHostToDevice, sc));
        }
        KVX_CUDA(cudaEventCreateWithFlags(&copied[c].e, cudaEventDisableTiming));
        KVX_CUDA(cudaEventRecord(copied[c].e, sc));
    }
    // header walks of the host blobs overlap the transfers
    std::vector<DevBlob> dk(static_cast<size_t>(n_units)), dv(static_cast<size_t>(n_units));
    std::vector<kvx_unit> units(static_cast<size_t>(n_units));
    std::vector<std::vector<kvx_block>> hostblocks;
    size_t idx_entries = 0;
    for (int u = 0; u < n_units; ++u) {
        for (int t = 0; t < 2; ++t) {
            const uint8_t *blob = t == 0 ? k_xkv[u] : v_xkv[u];
            const size_t bytes = t == 0 ? k_bytes[u] : v_bytes[u];
            const size_t at = t == 0 ? koff[size_t(u)] : voff[size_t(u)];
            HostIndex &hi = t == 0 ? kidx[size_t(u)] : vidx[size_t(u)];
            if (at == SIZE_MAX) {
                DevBlob &db = t == 0 ? dk[size_t(u)] : dv[size_t(u)];
                if (int rc = prepare_blob(blob, bytes, dim, seq, db, s)) return rc;
                hi.tok_start = db.tok_start;
                hi.tokens = db.tokens;
                hi.blocks.resize(size_t(db.n_blocks));
                KVX_CUDA(cudaMemcpy(hi.blocks.data(), db.idx.p,
                                    size_t(db.n_blocks) * sizeof(kvx_block), cudaMemcpyDeviceToHost));
            } else {
                if (int rc = host_walk(blob, bytes, dim, hi)) return rc;
                if (hi.tokens < seq) return fail(KVX_ERR_RUNTIME, "xkv decode ran out of blocks");
                int nb = 0;
                while (nb < int(hi.blocks.size()) && hi.tok_start[size_t(nb)] < seq) ++nb;
                hi.blocks.resize(static_cast<size_t>(nb));
            }
            idx_entries += hi.blocks.size();
        }
        if (kidx[size_t(u)].blocks.size() != vidx[size_t(u)].blocks.size())
            return fail(KVX_ERR_RUNTIME, "xkv K and V blocks cover different token counts");
    }
    std::vector<kvx_block> all;
    all.reserve(idx_entries);
    std::vector<size_t> kstart(static_cast<size_t>(n_units)), vstart(static_cast<size_t>(n_units));
    for (int u = 0; u < n_units; ++u) {
        kstart[size_t(u)] = all.size();
        all.insert(all.end(), kidx[size_t(u)].blocks.begin(), kidx[size_t(u)].blocks.end());
        vstart[size_t(u)] = all.size();
        all.insert(all.end(), vidx[size_t(u)].blocks.begin(), vidx[size_t(u)].blocks.end());
    }
    DevBuf didx;
    KVX_CUDA(didx.alloc(std::max<size_t>(all.size(), 1) * sizeof(kvx_block), s));
    KVX_CUDA(cudaMemcpyAsync(didx.p, all.data(), all.size() * sizeof(kvx_block),
                             cudaMemcpyHostToDevice, s));
    for (int u = 0; u < n_units; ++u) {
        kvx_unit &x = units[size_t(u)];
        x.k = koff[size_t(u)] == SIZE_MAX ? dk[size_t(u)].ptr : A + koff[size_t(u)];
        x.v = voff[size_t(u)] == SIZE_MAX ? dv[size_t(u)].ptr : A + voff[size_t(u)];
        x.k_index = didx.as<kvx_block>() + kstart[size_t(u)];
        x.v_index = didx.as<kvx_block>() + vstart[size_t(u)];
        x.q = qoff[size_t(u)] == SIZE_MAX ? q[u]
                                          : reinterpret_cast<const uint16_t *>(A + qoff[size_t(u)]);
        x.out = reinterpret_cast<float *>(A + out_at + size_t(u) * out_bytes);
        x.k_bytes = k_bytes[u];
        x.v_bytes = v_bytes[u];
        x.n_blocks = int(kidx[size_t(u)].blocks.size());
        x.seq = seq;
    }
    // Plans first (their host-side steps wait only for blob-independent work), then per chunk:
    // the blob readers behind its copies, the run and its output copies, all on the legacy
    // stream; one synchronisation at the end, then the plans' status.
    PlanGuard pg[2] = {{nullptr}, {nullptr}};
    for (int c = 0; c < nchunk; ++c) {
        const int u0 = chunk_begin(c);
        if (int rc = plan_create_impl(units.data() + u0, chunk_begin(c + 1) - u0, n_q, dim, 128, &pg[c].p,
                                      true, nullptr, true))
            return rc;
    }
    // Outputs in host memory come back through the device's pinned staging buffer, one copy per
    // chunk (the outputs sit together in the arena); outputs in device memory are copied one by one.
    bool all_host = true;
    for (int u = 0; u < n_units && all_host; ++u) all_host = !is_device_ptr(out[u]);
    int dev = 0;
    KVX_CUDA(cudaGetDevice(&dev));
    PinnedStage *ps = all_host && dev >= 0 && dev < kMaxDevices ? &pinned_stage(dev) : nullptr;
    std::unique_lock<std::mutex> stage_lock;
    const size_t out_total = size_t(n_units) * out_bytes;
    if (ps != nullptr) {
        stage_lock = std::unique_lock<std::mutex>(ps->mu);
        if (ps->bytes < out_total) {
            if (ps->p != nullptr) cudaFreeHost(ps->p);
            ps->p = nullptr;
            ps->bytes = 0;
            KVX_CUDA(cudaHostAlloc(&ps->p, out_total, cudaHostAllocDefault));
            ps->bytes = out_total;
        }
    }
    int rc = KVX_OK;
    for (int c = 0; c < nchunk && rc == KVX_OK; ++c) {
        const cudaError_t e = plan_blob_work(pg[c].p, copied[c].e);
        if (e != cudaSuccess) return fail(KVX_ERR_CUDA, std::string("attention_decode: ") + cudaGetErrorString(e));
        rc = kvx_plan_run(pg[c].p, s);
        const int u0 = chunk_begin(c), u1 = chunk_begin(c + 1);
        if (rc == KVX_OK && ps != nullptr)
            KVX_CUDA(cudaMemcpyAsync(static_cast<uint8_t *>(ps->p) + size_t(u0) * out_bytes,
                                     A + out_at + size_t(u0) * out_bytes, size_t(u1 - u0) * out_bytes,
                                     cudaMemcpyDeviceToHost, s));
        for (int u = u0; rc == KVX_OK && ps == nullptr && u < u1; ++u)
            KVX_CUDA(cudaMemcpyAsync(out[u], A + out_at + size_t(u) * out_bytes, out_bytes,
                                     is_device_ptr(out[u]) ? cudaMemcpyDeviceToDevice
                                                           : cudaMemcpyDeviceToHost,
                                     s));
    }
    KVX_CUDA(cudaStreamSynchronize(s));
    KVX_CUDA(cudaStreamSynchronize(sc));
    for (int c = 0; c < nchunk && rc == KVX_OK; ++c) rc = kvx_plan_check(pg[c].p);
    if (rc != KVX_OK) return rc;
    if (ps != nullptr)
        for (int u = 0; u < n_units; ++u)
            std::memcpy(out[u], static_cast<const uint8_t *>(ps->p) + size_t(u) * out_bytes, out_bytes);
    g_err.clear();
    return KVX_OK;
}

// ---- codec -----------------------------------------------------------------------------------------

namespace {

int check_encode_args(const void *kv, int seq_len, int head_dim, int block_tokens) {
    // src/codec.cpp:40-52
    if (kv == nullptr || seq_len <= 0 || head_dim <= 0 || block_tokens <= 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, "encode_bf16: empty input");
    if (head_dim % 4 != 0 || head_dim > kMaxHeadDim)
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    "encode_bf16: head_dim must be a multiple of 4 and at most 256");
    if (block_tokens > 255)
        return fail(KVX_ERR_INVALID_ARGUMENT, "encode_bf16: block_tokens must fit in a byte");
    if ((long long)block_tokens * head_dim > 65535)
        return fail(KVX_ERR_INVALID_ARGUMENT, "encode_bf16: block escape count would not fit in u16");
    return KVX_OK;
}

int check_code_bits(int code_bits) {
    if ((code_bits & ~KVX_CODE_BITS_ALL) != 0 ||
        (code_bits & KVX_CODE_BITS_REFERENCE) != KVX_CODE_BITS_REFERENCE)
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    "encode_bf16: mode mask must hold 2 and 4 bits, and may add 3");
    return KVX_OK;
}

size_t blob_bound(int seq, int dim, int bt) {
    const size_t nb = (size_t(seq) + size_t(bt) - 1) / size_t(bt);
    return nb * 8u + 2u * size_t(seq) * size_t(dim);
}

// Encode n device tensors: analyze, lay out, emit.  Offsets are relative to `arena`.
int encode_device(const uint16_t *const *dev_tensors_host, int n, int seq, int dim, int bt,
                  int code_bits, uint8_t *arena, size_t cap, kvx_block *index, uint64_t *blob_off,
                  uint64_t *blob_bytes, cudaStream_t s) {
    const int nb_per = (seq + bt - 1) / bt;
    const size_t nb = size_t(n) * size_t(nb_per);
    DevBuf tens, blocks, bases, boff, toff, status;
    KVX_CUDA(tens.alloc(size_t(n) * sizeof(void *), s));
    KVX_CUDA(cudaMemcpyAsync(tens.p, dev_tensors_host, size_t(n) * sizeof(void *),
                             cudaMemcpyHostToDevice, s));
    KVX_CUDA(blocks.alloc(nb * sizeof(EncBlock), s));
    KVX_CUDA(bases.alloc(nb * size_t(dim), s));
    KVX_CUDA(status.alloc(2 * sizeof(int), s));
    KVX_CUDA(cudaMemsetAsync(status.p, 0, 2 * sizeof(int), s));
    const uint16_t *const *dt = tens.as<const uint16_t *const>();
    KVX_CUDA(launch_encode_analyze(dt, n, seq, dim, bt, code_bits, blocks.as<EncBlock>(),
                                   bases.as<uint8_t>(), s));
    std::vector<EncBlock> hb(nb);
    KVX_CUDA(cudaMemcpyAsync(hb.data(), blocks.p, nb * sizeof(EncBlock), cudaMemcpyDeviceToHost, s));
    KVX_CUDA(cudaStreamSynchronize(s));
    std::vector<uint64_t> bo(nb), to(static_cast<size_t>(n));
    uint64_t at = 0;
    for (int t = 0; t < n; ++t) {
        to[size_t(t)] = at;
        uint64_t sz = 0;
        for (int b = 0; b < nb_per; ++b) {
            bo[size_t(t) * nb_per + b] = at + sz;
            sz += hb[size_t(t) * nb_per + b].bytes;
        }
        if (sz > 0xFFFFFFFFull)
            return fail(KVX_ERR_UNSUPPORTED, "xkv blob larger than 4 GiB per tensor");
        blob_bytes[t] = sz;
        blob_off[t] = at;
        at += (sz + 16 + 15) & ~uint64_t(15);
    }
    if (at > cap) return fail(KVX_ERR_INVALID_ARGUMENT, "encode: arena capacity too small");
    KVX_CUDA(boff.alloc(nb * sizeof(uint64_t), s));
    KVX_CUDA(toff.alloc(size_t(n) * sizeof(uint64_t), s));
    KVX_CUDA(cudaMemcpyAsync(boff.p, bo.data(), nb * sizeof(uint64_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(toff.p, to.data(), size_t(n) * sizeof(uint64_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(launch_encode_emit(dt, n, seq, dim, bt, blocks.as<EncBlock>(), bases.as<uint8_t>(),
                                boff.as<uint64_t>(), arena, index, toff.as<uint64_t>(),
                                status.as<int>(), s));
    KVX_CUDA(cudaStreamSynchronize(s));
    return read_status(status.as<int>(), false);
}

}  // namespace

extern "C" size_t kvx_encode_bound(int seq_len, int head_dim, int block_tokens) {
    if (seq_len <= 0 || head_dim <= 0 || block_tokens <= 0) return 0;
    return blob_bound(seq_len, head_dim, block_tokens);
}

extern "C" int kvx_encode_bf16(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                               uint8_t *out, size_t out_capacity, size_t *out_bytes) {
    return kvx_encode_bf16_bits(kv, seq_len, head_dim, block_tokens, KVX_CODE_BITS_REFERENCE, out,
                                out_capacity, out_bytes);
}

extern "C" int kvx_encode_bf16_bits(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                                    int code_bits, uint8_t *out, size_t out_capacity,
                                    size_t *out_bytes) {
    if (int rc = check_encode_args(kv, seq_len, head_dim, block_tokens)) return rc;
    if (int rc = check_code_bits(code_bits)) return rc;
    if (out == nullptr) return fail(KVX_ERR_INVALID_ARGUMENT, "encode_bf16: null output");
    if (int rc = check_device()) return rc;
    cudaStream_t s = nullptr;
    DevBuf src, arena, index;
    const void *dsrc = nullptr;
    if (int rc = to_device(kv, size_t(seq_len) * head_dim * 2, src, dsrc, s)) return rc;
    const size_t cap = blob_bound(seq_len, head_dim, block_tokens) + 64;
    KVX_CUDA(arena.alloc(cap, s));
    const int nb = (seq_len + block_tokens - 1) / block_tokens;
    KVX_CUDA(index.alloc(size_t(nb) * sizeof(kvx_block), s));
    const uint16_t *tp = static_cast<const uint16_t *>(dsrc);
    uint64_t boff = 0, bbytes = 0;
    if (int rc = encode_device(&tp, 1, seq_len, head_dim, block_tokens, code_bits,
                               arena.as<uint8_t>(), cap, index.as<kvx_block>(), &boff, &bbytes, s))
        return rc;
    if (bbytes > out_capacity) return fail(KVX_ERR_INVALID_ARGUMENT, "encode_bf16: output capacity too small");
    KVX_CUDA(cudaMemcpy(out, arena.as<uint8_t>() + boff, bbytes,
                        is_device_ptr(out) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost));
    if (out_bytes) *out_bytes = bbytes;
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_exponent_stats(const uint16_t *kv, int seq_len, int head_dim, int block_tokens,
                                  int *best, float *entropy) {
    if (kv == nullptr || best == nullptr || entropy == nullptr || seq_len <= 0 || head_dim <= 0 ||
        block_tokens <= 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, "exponent_stats: bad argument");
    if (int rc = check_device()) return rc;
    cudaStream_t s = nullptr;
    const size_t nb = size_t((seq_len + block_tokens - 1) / block_tokens);
    const size_t best_bytes = 3 * nb * size_t(head_dim) * sizeof(int);
    const size_t ent_bytes = nb * size_t(head_dim) * sizeof(float);
    DevBuf kb, bb, eb;
    const void *kp = nullptr;
    if (int rc = to_device(kv, size_t(seq_len) * head_dim * 2, kb, kp, s)) return rc;
    const bool best_dev = is_device_ptr(best), ent_dev = is_device_ptr(entropy);
    int *bp = best;
    float *ep = entropy;
    if (!best_dev) {
        KVX_CUDA(bb.alloc(best_bytes, s));
        bp = bb.as<int>();
    }
    if (!ent_dev) {
        KVX_CUDA(eb.alloc(ent_bytes, s));
        ep = eb.as<float>();
    }
    KVX_CUDA(launch_exp_stats(static_cast<const uint16_t *>(kp), seq_len, head_dim, block_tokens, bp, ep, s));
    if (!best_dev) KVX_CUDA(cudaMemcpyAsync(best, bp, best_bytes, cudaMemcpyDeviceToHost, s));
    if (!ent_dev) KVX_CUDA(cudaMemcpyAsync(entropy, ep, ent_bytes, cudaMemcpyDeviceToHost, s));
    KVX_CUDA(cudaStreamSynchronize(s));
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_decode_bf16(const uint8_t *blob, size_t bytes, int seq_len, int head_dim,
                               uint16_t *out) {
    if (blob == nullptr || out == nullptr || seq_len <= 0 || head_dim <= 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, "decode_bf16: bad argument");
    if (int rc = check_device()) return rc;
    cudaStream_t s = nullptr;
    DevBlob db;
    if (int rc = prepare_blob(blob, bytes, head_dim, seq_len, db, s)) return rc;
    DevBuf tok, ob, st;
    std::vector<uint32_t> ts(db.tok_start.begin(), db.tok_start.begin() + db.n_blocks);
    KVX_CUDA(tok.alloc(std::max<size_t>(ts.size(), 1) * 4, s));
    KVX_CUDA(cudaMemcpyAsync(tok.p, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice, s));
    const size_t ob_bytes = size_t(seq_len) * head_dim * 2;
    const bool out_dev = is_device_ptr(out);
    uint16_t *op = out;
    if (!out_dev) {
        KVX_CUDA(ob.alloc(ob_bytes, s));
        op = ob.as<uint16_t>();
    }
    KVX_CUDA(st.alloc(2 * sizeof(int), s));
    KVX_CUDA(cudaMemsetAsync(st.p, 0, 2 * sizeof(int), s));
    KVX_CUDA(launch_decode(db.ptr, db.idx.as<kvx_block>(), tok.as<uint32_t>(), db.n_blocks,
                           head_dim, seq_len, op, st.as<int>(), s));
    KVX_CUDA(cudaStreamSynchronize(s));
    if (int rc = read_status(st.as<int>(), false)) return rc;
    if (!out_dev) KVX_CUDA(cudaMemcpy(out, op, ob_bytes, cudaMemcpyDeviceToHost));
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_xkv_index(const uint8_t *blob, size_t bytes, int head_dim, kvx_block *index,
                             int max_blocks, int *n_blocks, long long *n_tokens) {
    if (blob == nullptr || index == nullptr || max_blocks <= 0 || head_dim <= 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_xkv_index: bad argument");
    if (!is_device_ptr(blob) || !is_device_ptr(index))
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_xkv_index: blob and index must be device memory");
    cudaStream_t s = nullptr;
    DevBuf cnt;
    KVX_CUDA(cnt.alloc(4 * sizeof(long long), s));
    KVX_CUDA(cudaMemsetAsync(cnt.p, 0, 4 * sizeof(long long), s));
    KVX_CUDA(launch_index_walk(blob, bytes, head_dim, index, nullptr, max_blocks, cnt.as<int>(),
                               cnt.as<long long>() + 1, cnt.as<int>() + 4, s));
    long long h[4];
    KVX_CUDA(cudaMemcpyAsync(h, cnt.p, sizeof h, cudaMemcpyDeviceToHost, s));
    KVX_CUDA(cudaStreamSynchronize(s));
    const int *hc = reinterpret_cast<const int *>(h);
    if (hc[4] != 0) return fail(hc[4], detail_message(hc[4], hc[5]));
    if (n_blocks) *n_blocks = hc[0];
    if (n_tokens) *n_tokens = h[1];
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_encode_batch_bounds(int n_tensors, int seq, int head_dim, int block_tokens,
                                       size_t *arena_bytes, size_t *index_entries) {
    if (n_tensors <= 0) return fail(KVX_ERR_INVALID_ARGUMENT, "encode_batch: bad argument");
    if (int rc = check_encode_args(reinterpret_cast<const void *>(1), seq, head_dim, block_tokens))
        return rc;
    const size_t per = (blob_bound(seq, head_dim, block_tokens) + 16 + 15) & ~size_t(15);
    if (arena_bytes) *arena_bytes = per * size_t(n_tensors) + 64;
    if (index_entries)
        *index_entries = size_t(n_tensors) * size_t((seq + block_tokens - 1) / block_tokens);
    return KVX_OK;
}

extern "C" int kvx_encode_batch(int n_tensors, const uint16_t *const *kv, int seq, int head_dim,
                                int block_tokens, uint8_t *arena, size_t arena_capacity,
                                kvx_block *index, uint64_t *blob_offset, uint64_t *blob_bytes,
                                void *stream) {
    return kvx_encode_batch_bits(n_tensors, kv, seq, head_dim, block_tokens, KVX_CODE_BITS_REFERENCE,
                                 arena, arena_capacity, index, blob_offset, blob_bytes, stream);
}

extern "C" int kvx_encode_batch_bits(int n_tensors, const uint16_t *const *kv, int seq, int head_dim,
                                     int block_tokens, int code_bits, uint8_t *arena,
                                     size_t arena_capacity, kvx_block *index, uint64_t *blob_offset,
                                     uint64_t *blob_bytes, void *stream) {
    if (n_tensors <= 0 || kv == nullptr || arena == nullptr || index == nullptr ||
        blob_offset == nullptr || blob_bytes == nullptr)
        return fail(KVX_ERR_INVALID_ARGUMENT, "encode_batch: bad argument");
    if (int rc = check_encode_args(kv[0], seq, head_dim, block_tokens)) return rc;
    if (int rc = check_code_bits(code_bits)) return rc;
    if (reinterpret_cast<uintptr_t>(arena) & 15u)
        return fail(KVX_ERR_INVALID_ARGUMENT, "encode_batch: arena must be 16-byte aligned");
    if (int rc = encode_device(kv, n_tensors, seq, head_dim, block_tokens, code_bits, arena,
                               arena_capacity, index, blob_offset, blob_bytes,
                               static_cast<cudaStream_t>(stream)))
        return rc;
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_cache_append(const uint16_t *kv_new, int n_new, int head_dim, int block_tokens,
                                uint8_t *blob, size_t at, size_t capacity, kvx_block *index,
                                size_t *bytes_written, int *blocks_written, void *stream) {
    return kvx_cache_append_bits(kv_new, n_new, head_dim, block_tokens, KVX_CODE_BITS_REFERENCE, blob,
                                 at, capacity, index, bytes_written, blocks_written, stream);
}

extern "C" int kvx_cache_append_bits(const uint16_t *kv_new, int n_new, int head_dim, int block_tokens,
                                     int code_bits, uint8_t *blob, size_t at, size_t capacity,
                                     kvx_block *index, size_t *bytes_written, int *blocks_written,
                                     void *stream) {
    if (int rc = check_encode_args(kv_new, n_new, head_dim, block_tokens)) return rc;
    if (int rc = check_code_bits(code_bits)) return rc;
    if (blob == nullptr || index == nullptr)
        return fail(KVX_ERR_INVALID_ARGUMENT, "cache_append: bad argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t cap = blob_bound(n_new, head_dim, block_tokens) + 64;
    DevBuf tmp;
    KVX_CUDA(tmp.alloc(cap, s));
    uint64_t boff = 0, bbytes = 0;
    const int nb = (n_new + block_tokens - 1) / block_tokens;
    if (int rc = encode_device(&kv_new, 1, n_new, head_dim, block_tokens, code_bits,
                               tmp.as<uint8_t>(), cap, index, &boff, &bbytes, s))
        return rc;
    if (at + bbytes > capacity) return fail(KVX_ERR_INVALID_ARGUMENT, "cache_append: blob capacity too small");
    KVX_CUDA(cudaMemcpyAsync(blob + at, tmp.as<uint8_t>() + boff, bbytes, cudaMemcpyDeviceToDevice, s));
    // shift the new index entries by `at`
    std::vector<kvx_block> hi(static_cast<size_t>(nb));
    KVX_CUDA(cudaMemcpyAsync(hi.data(), index, size_t(nb) * sizeof(kvx_block), cudaMemcpyDeviceToHost, s));
    KVX_CUDA(cudaStreamSynchronize(s));
    for (auto &b : hi) {
        if (uint64_t(b.offset) + at > 0xFFFFFFFFull)
            return fail(KVX_ERR_UNSUPPORTED, "xkv blob larger than 4 GiB per tensor");
        b.offset = uint32_t(b.offset + at);
    }
    KVX_CUDA(cudaMemcpyAsync(index, hi.data(), size_t(nb) * sizeof(kvx_block), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaStreamSynchronize(s));
    if (bytes_written) *bytes_written = bbytes;
    if (blocks_written) *blocks_written = nb;
    g_err.clear();
    return KVX_OK;
}

extern "C" int kvx_synth_bf16(uint16_t *out, int seq, int dim, uint64_t seed, uint64_t stream_id,
                              int profile, uint32_t rate, void *stream) {
    if (out == nullptr || seq <= 0 || dim <= 0 || profile < 0 || profile > 5)
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_synth_bf16: bad argument");
    KVX_CUDA(launch_synth(out, seq, dim, seed, stream_id, profile, rate,
                          static_cast<cudaStream_t>(stream)));
    return KVX_OK;
}

extern "C" int kvx_hbm_read_probe(const void *buf, size_t bytes, int reps, double *gbps) {
    if (buf == nullptr || bytes < 16 || reps <= 0 || gbps == nullptr)
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_hbm_read_probe: bad argument");
    DevBuf sink;
    KVX_CUDA(sink.alloc(16, nullptr));
    const size_t n16 = bytes / 16;
    const int grid = sm_count() * 4;
    cudaEvent_t a, b;
    KVX_CUDA(cudaEventCreate(&a));
    KVX_CUDA(cudaEventCreate(&b));
    KVX_CUDA(launch_read_probe(static_cast<const uint4 *>(buf), n16, sink.as<uint32_t>(), grid, nullptr));
    float best = 1e30f;
    for (int r = 0; r < reps; ++r) {
        cudaEventRecord(a, nullptr);
        launch_read_probe(static_cast<const uint4 *>(buf), n16, sink.as<uint32_t>(), grid, nullptr);
        cudaEventRecord(b, nullptr);
        cudaEventSynchronize(b);
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        best = std::min(best, ms);
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    KVX_CUDA(cudaGetLastError());
    *gbps = double(n16) * 16.0 / (double(best) * 1e-3) / 1e9;
    return KVX_OK;
}

// ---- fold of sequence shards ---------------------------------------------------------------

extern "C" int kvx_fold_shards(const float *parts, int n_parts, int n_rows, int dim, float *out,
                               float *lse_out, void *stream) {
    if (parts == nullptr || out == nullptr || n_parts <= 0 || n_rows <= 0 || dim <= 0 ||
        dim > kMaxHeadDim)
        return fail(KVX_ERR_INVALID_ARGUMENT, "kvx_fold_shards: bad argument");
    KVX_CUDA(launch_fold(parts, n_parts, n_rows, dim, out, lse_out,
                         static_cast<cudaStream_t>(stream)));
    return KVX_OK;
}

// ---- decode attention without allocation ---------------------------------------------------
//
// kvx_attention_decode_noalloc is for callers that must not allocate GPU memory once they are
// running: serving engines that reserve the device's memory for their KV-cache pool at start-up
// and treat any later cudaMalloc as a failure, and decode loops that cannot afford the
// device-wide synchronisation that cudaFree implies.  All of its scratch (the flat block list,
// block descriptors, worker ranges, partial softmax states and the error word) lives in the file-scope device array
// below, which every device that loads this library holds until the process exits.

namespace kvx {
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(40) << 20;  // 40 MiB per device
constexpr size_t kNoAllocEscEntries = size_t(3) << 20;      // escape record entries (12 MiB)
constexpr int kNoAllocMaxBlocks = 8192;                   // XKV blocks per tensor
constexpr int kNoAllocMaxQueries = 64;                    // queries per call (8 groups of 8)
constexpr int kNoAllocMaxRanges = 1024;                   // CTA ranges of the attention grid
constexpr int kNoAllocMaxGroups = kNoAllocMaxQueries / 8;  // query groups of <= 8

constexpr size_t up256c(size_t x) { return (x + 255) & ~size_t(255); }
// Bytes of the fixed part of the scratch layout (everything before the partial states), in the
// order kvx_attention_decode_noalloc carves it.
constexpr size_t kNoAllocFixedBytes =
    up256c(2 * sizeof(int)) + up256c(kNoAllocMaxGroups * sizeof(UnitDev)) +
    up256c(kNoAllocMaxGroups * sizeof(kvx_unit)) + up256c(kNoAllocMaxGroups * sizeof(int64_t)) +
    up256c(kNoAllocMaxGroups * sizeof(int64_t)) + up256c(kNoAllocMaxGroups * sizeof(SplitUnit)) +
    up256c(size_t(kNoAllocMaxGroups) * kNoAllocMaxBlocks * sizeof(FlatBlock)) +
    up256c(size_t(kNoAllocMaxGroups) * kNoAllocMaxBlocks * sizeof(BlockDesc)) +
    up256c((kNoAllocMaxRanges + 1) * sizeof(int64_t)) + up256c(kNoAllocMaxRanges * sizeof(int32_t)) +
    up256c(sizeof(unsigned long long)) + up256c((kNoAllocEscEntries + 4) * sizeof(uint32_t)) +
    up256c(size_t(kNoAllocMaxBlocks) * kMaxHeadDim * sizeof(uint32_t));
// One partial-state row (every consumer warp's m, l and acc) at its largest, over the head dims.
constexpr size_t noalloc_row_bytes(int dim) {
    return size_t(attention_consumer_warps(dim)) * size_t(16 + 8 * dim) * sizeof(float);
}
constexpr size_t kNoAllocMaxRowBytes =
    noalloc_row_bytes(128) > noalloc_row_bytes(256) ? noalloc_row_bytes(128) : noalloc_row_bytes(256);
static_assert(kNoAllocFixedBytes + (64 + kNoAllocMaxGroups) * kNoAllocMaxRowBytes <= kNoAllocScratchBytes,
              "the fixed scratch must leave room for the partial states of at least 64 CTAs");
}  // namespace
}  // namespace kvx

static __device__ __align__(256) unsigned char kvx_noalloc_scratch[kvx::kNoAllocScratchBytes];

namespace kvx {
namespace {

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of the scratch array on the current device.  The array's name in host code is
// only a host-side stand-in, so the address comes from cudaGetSymbolAddress, looked up once per
// device (the first call on a device also loads the module there).
int noalloc_scratch(uint8_t **out) {
    static std::mutex mu;
    static uint8_t *addr[64] = {};
    int dev = 0;
    KVX_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(KVX_ERR_RUNTIME, "kvx_attention_decode_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, kvx_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(KVX_ERR_CUDA,
                        std::string("kvx_attention_decode_noalloc: cudaGetSymbolAddress: ") +
                            cudaGetErrorString(e));
        addr[dev] = static_cast<uint8_t *>(p);
    }
    *out = addr[dev];
    return KVX_OK;
}

}  // namespace
}  // namespace kvx

extern "C" int kvx_attention_decode_noalloc(const uint16_t *q, const uint8_t *k_xkv, size_t k_bytes,
                                            const kvx_block *k_index, const uint8_t *v_xkv,
                                            size_t v_bytes, const kvx_block *v_index, int n_blocks,
                                            float *out, int n_q, int dim, int seq, void *stream) {
    const char *fn = "kvx_attention_decode_noalloc: ";
    if (q == nullptr || k_xkv == nullptr || v_xkv == nullptr || k_index == nullptr ||
        v_index == nullptr || out == nullptr)
        return fail(KVX_ERR_INVALID_ARGUMENT, std::string(fn) + "null pointer");
    if (n_q <= 0 || dim <= 0 || seq <= 0 || n_blocks <= 0 || k_bytes == 0 || v_bytes == 0)
        return fail(KVX_ERR_INVALID_ARGUMENT, std::string(fn) + "sizes must be positive");
    if (n_q > kNoAllocMaxQueries)
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    std::string(fn) + "n_q exceeds the limit of 64 queries per call");
    if (n_blocks > kNoAllocMaxBlocks)
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    std::string(fn) + "n_blocks exceeds the scratch limit of 8192 blocks per tensor");
    if (!attention_dim_supported(dim))
        return fail(KVX_ERR_UNSUPPORTED,
                    std::string(fn) + "head_dim must be 32, 64, 128 or 256 for the GPU kernels");
    if (int rc = check_device()) return rc;
    if (!is_device_ptr(q) || !is_device_ptr(k_xkv) || !is_device_ptr(v_xkv) ||
        !is_device_ptr(k_index) || !is_device_ptr(v_index) || !is_device_ptr(out))
        return fail(KVX_ERR_INVALID_ARGUMENT, std::string(fn) + "every pointer must be device memory");
    if (((reinterpret_cast<uintptr_t>(k_xkv) | reinterpret_cast<uintptr_t>(v_xkv)) & 15u) ||
        (reinterpret_cast<uintptr_t>(q) & 3u) || (reinterpret_cast<uintptr_t>(out) & 7u))
        return fail(KVX_ERR_INVALID_ARGUMENT,
                    std::string(fn) + "K/V blobs must be 16-byte aligned, q 4-byte, out 8-byte");
    uint8_t *base = nullptr;
    if (int rc = noalloc_scratch(&base)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // Scratch layout (256-byte aligned pieces): status | units | unit descriptors | block
    // begins | record sources | split units | flat blocks | block descriptors | CTA ranges | row
    // bases | record size | escape records | merge words | partial states.
    const int groups = (n_q + 7) / 8;
    const int64_t total = int64_t(groups) * n_blocks;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += up256(bytes);
        return base + o;
    };
    int *status = reinterpret_cast<int *>(take(2 * sizeof(int)));
    UnitDev *d_units = reinterpret_cast<UnitDev *>(take(kNoAllocMaxGroups * sizeof(UnitDev)));
    kvx_unit *d_vu = reinterpret_cast<kvx_unit *>(take(kNoAllocMaxGroups * sizeof(kvx_unit)));
    int64_t *d_begin = reinterpret_cast<int64_t *>(take(kNoAllocMaxGroups * sizeof(int64_t)));
    int64_t *d_src = reinterpret_cast<int64_t *>(take(kNoAllocMaxGroups * sizeof(int64_t)));
    SplitUnit *d_split = reinterpret_cast<SplitUnit *>(take(kNoAllocMaxGroups * sizeof(SplitUnit)));
    FlatBlock *d_flat = reinterpret_cast<FlatBlock *>(
        take(size_t(kNoAllocMaxGroups) * kNoAllocMaxBlocks * sizeof(FlatBlock)));
    BlockDesc *d_desc = reinterpret_cast<BlockDesc *>(
        take(size_t(kNoAllocMaxGroups) * kNoAllocMaxBlocks * sizeof(BlockDesc)));
    int64_t *d_range = reinterpret_cast<int64_t *>(take((kNoAllocMaxRanges + 1) * sizeof(int64_t)));
    int32_t *d_seg = reinterpret_cast<int32_t *>(take(kNoAllocMaxRanges * sizeof(int32_t)));
    unsigned long long *d_esc_total =
        reinterpret_cast<unsigned long long *>(take(sizeof(unsigned long long)));
    uint32_t *d_esc = reinterpret_cast<uint32_t *>(take((kNoAllocEscEntries + 4) * sizeof(uint32_t)));
    // merge words: only the first query group's blocks have their own (the others share them)
    uint32_t *d_b7 = reinterpret_cast<uint32_t *>(take(size_t(kNoAllocMaxBlocks) * kMaxHeadDim * sizeof(uint32_t)));
    if (off != kNoAllocFixedBytes)
        return fail(KVX_ERR_RUNTIME, std::string(fn) + "scratch layout out of step with its size");
    float *d_partials = reinterpret_cast<float *>(base + off);
    // A range holds at most one more unit segment than it crosses unit starts, so the rows are at
    // most n_ranges + groups - 1: cap the ranges so that they fit the rest of the scratch.
    const int64_t fit_rows = int64_t((kNoAllocScratchBytes - off) / noalloc_row_bytes(dim));
    const int n_ranges = int(std::max<int64_t>(1, std::min<int64_t>(
        std::min<int64_t>(total, sm_count()), std::min<int64_t>(fit_rows - groups + 1, kNoAllocMaxRanges))));

    // Host-side descriptors (plain stack / vector memory, copied into the scratch).
    std::vector<kvx_unit> vu(static_cast<size_t>(groups));
    std::vector<UnitDev> ud(static_cast<size_t>(groups));
    std::vector<int64_t> begin(static_cast<size_t>(groups));
    // every query group reads the same K/V blocks: their escape records are built once
    const std::vector<int64_t> srcs(static_cast<size_t>(groups), 0);
    for (int g = 0; g < groups; ++g) {
        kvx_unit &x = vu[size_t(g)];
        x.k = k_xkv;
        x.v = v_xkv;
        x.k_index = k_index;
        x.v_index = v_index;
        x.q = q + size_t(8) * g * dim;
        x.out = out + size_t(8) * g * dim;
        x.k_bytes = k_bytes;
        x.v_bytes = v_bytes;
        x.n_blocks = n_blocks;
        x.seq = seq;
        UnitDev &d = ud[size_t(g)];
        d = UnitDev{};
        d.k = k_xkv;
        d.v = v_xkv;
        d.q = x.q;
        d.out = x.out;
        d.block_begin = int64_t(g) * n_blocks;
        d.n_blocks = n_blocks;
        d.n_q = std::min(8, n_q - 8 * g);
        d.q_stride = dim;
        begin[size_t(g)] = d.block_begin;
    }
    // CTA ranges: one block each when they fit, else an even split of the blocks; then the
    // partial-state rows of every unit segment and the combine's unit list.
    std::vector<int64_t> tb(static_cast<size_t>(n_ranges) + 1);
    for (int t = 0; t <= n_ranges; ++t) tb[size_t(t)] = int64_t(t) * total / n_ranges;
    std::vector<int32_t> seg_base;
    std::vector<SplitUnit> split;
    const int64_t rows = plan_segments(tb, n_ranges, ud, dim, seg_base, split);
    if (rows > fit_rows) return fail(KVX_ERR_RUNTIME, std::string(fn) + "partial states exceed the scratch");

    // Every call shares the scratch and finds the previous call's contents there: the status
    // word is cleared here; everything else is fully written before it is read.
    KVX_CUDA(cudaMemsetAsync(status, 0, 2 * sizeof(int), s));
    KVX_CUDA(cudaMemcpyAsync(d_units, ud.data(), ud.size() * sizeof(UnitDev), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_vu, vu.data(), vu.size() * sizeof(kvx_unit), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_begin, begin.data(), begin.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_src, srcs.data(), srcs.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_range, tb.data(), tb.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_seg, seg_base.data(), seg_base.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    KVX_CUDA(cudaMemcpyAsync(d_split, split.data(), split.size() * sizeof(SplitUnit),
                             cudaMemcpyHostToDevice, s));
    KVX_CUDA(launch_build_flat(d_vu, d_begin, d_src, groups, dim, kDefaultBlock, false, d_flat,
                               status, s));
    KVX_CUDA(launch_esc_layout(d_flat, total, d_esc_total, kNoAllocEscEntries, status, s));
    KVX_CUDA(launch_esc_fill(d_units, d_flat, total, dim, d_esc, kNoAllocEscEntries, status, s));
    KVX_CUDA(launch_b7(d_units, d_flat, total, dim, d_b7, s));
    KVX_CUDA(launch_block_desc(d_units, d_flat, d_esc, total, dim, false, d_desc, s));
    AttnArgs a{};
    a.units = d_units;
    a.flat = d_flat;
    a.desc = d_desc;
    a.esc = d_esc;
    a.b7 = d_b7;
    a.range_begin = d_range;
    a.seg_base = d_seg;
    a.partials = d_partials;
    a.status = status;
    a.n_ranges = n_ranges;
    KVX_CUDA(launch_attention(dim, false, false, a, n_ranges, s));
    CombineArgs c{};
    c.split = d_split;
    c.partials = d_partials;
    KVX_CUDA(launch_combine(dim, c, groups, s));
    // The host descriptors above are pageable stack/vector memory: wait for the stream before
    // they go out of scope, then report device-side errors like kvx_attention_decode.
    KVX_CUDA(cudaStreamSynchronize(s));
    int st[2] = {0, 0};
    KVX_CUDA(cudaMemcpy(st, status, sizeof st, cudaMemcpyDeviceToHost));
    if (st[0] != 0) return fail(st[0], std::string(detail_message(st[0], st[1])));
    g_err.clear();
    return KVX_OK;
}
