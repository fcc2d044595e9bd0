// Host side of the insitu_b200 C ABI: the cache handle, its paged pool and
// page tables, argument checking, and the kernel launches.
//
// The host owns the cache metadata (lengths, page tables, the free-page
// list), as the reference's CompressedCache owns its buffer and length
// (cache/compressed.py:42-86). Kernels read device mirrors of it that every
// mutating call refreshes with stream-ordered copies before its launch.

#include <climits>
#include <cstdio>
#include <cstring>
#include <string>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "scan_chunked.cuh"
#include "scan_fused.cuh"
#include "project.cuh"

using namespace ins;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

#define CK(call)                                                                       \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return fail(INS_ECUDA, std::string(#call " failed: ") + cudaGetErrorString(e_)); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Per-call uploads (sequence ids, slots, plans, positions) go through a ring
// of pinned host / device buffer pairs. reserve() moves to the next slot and
// waits only for that slot's previous copy, so the host can run NSLOT calls
// ahead of the GPU rather than one; host writes into a slot wait on that
// slot's last copy, so an enqueued copy never reads a half-rewritten area. A
// slot that must grow takes the whole ring with it, so that steady-state
// calls never allocate.
struct Staging {
    static constexpr int NSLOT = 4;
    struct Slot {
        void *h = nullptr;
        void *d = nullptr;
        cudaEvent_t done = nullptr;
    };
    Slot ring[NSLOT];
    size_t cap = 0;                     // every slot's size
    int cur = NSLOT - 1;
    void *h = nullptr;                  // the current slot's buffers
    void *d = nullptr;
    int64_t *launches = nullptr;        // the cache's kernel count (an upload may be a launch)

    int reserve(size_t bytes) {
        cur = (cur + 1) % NSLOT;
        Slot &sl = ring[cur];
        if (!sl.done) CK(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
        CK(cudaEventSynchronize(sl.done));
        if (bytes > cap) {
            size_t want = cap ? cap : 4096;
            while (want < bytes) want *= 2;
            for (Slot &o : ring) {
                if (o.done) CK(cudaEventSynchronize(o.done));
                if (o.h) cudaFreeHost(o.h);
                if (o.d) cudaFree(o.d);
                o.h = o.d = nullptr;
            }
            cap = 0;
            for (Slot &o : ring) {
                CK(cudaHostAlloc(&o.h, want, cudaHostAllocDefault));
                CK(cudaMalloc(&o.d, want));
            }
            cap = want;
        }
        h = sl.h;
        d = sl.d;
        return INS_OK;
    }
    int upload(size_t bytes, cudaStream_t s) {
        int launched = 0;
        CK(small_upload(d, h, bytes, s, &launched));
        if (launched && launches) *launches += 1;
        CK(cudaEventRecord(ring[cur].done, s));
        return INS_OK;
    }
    void release() {
        for (Slot &o : ring) {
            if (o.done) cudaEventSynchronize(o.done), cudaEventDestroy(o.done);
            if (o.h) cudaFreeHost(o.h);
            if (o.d) cudaFree(o.d);
            o = Slot();
        }
        h = d = nullptr;
        cap = 0;
    }
};

}  // namespace

struct ins_cache {
    ins_config cfg;
    Geo g;
    int device = 0;
    DevTables *d_tables = nullptr;
    uint8_t *d_pool = nullptr;
    int32_t *d_page_table = nullptr;   // [max_seqs, max_pages]
    int32_t *d_status = nullptr;
    unsigned long long *d_redo_total = nullptr;   // items the sequential kernel recomputed, running
    // host mirrors (pinned, so their copies can be asynchronous)
    int32_t *h_page_table = nullptr;
    int32_t *h_seq_lens = nullptr;
    cudaEvent_t mirror_done = nullptr;
    std::vector<int32_t> free_pages;
    Staging stage_a;                    // per-call index uploads
    Staging stage_b;
    Staging stage_c;                    // positions of ins_seam
    ChunkScratch chunk;                 // scratch of the context-parallel scan
    uint64_t gen = 0;                   // bumped by every call that rewrites `chunk`
    struct {                            // context split: phase 1 waiting for phase 2
        bool armed = false;
        uint64_t gen = 0;
        int32_t B = 0;
        std::vector<int32_t> seq;
        std::vector<int64_t> T;
        const int32_t *q_rot = nullptr;
        int32_t rs = 0;                 // rows-per-thread instantiation phase 1 used
        ChunkArgs a{};
    } split;
};

namespace {

bool valid_bits(int b) { return b >= 1 && b <= 8; }

int check_config(const ins_config *c) {
    if (!c) return fail(INS_EINVAL, "config is NULL");
    if (c->head_dim != D) return fail(INS_EINVAL, "this build supports head_dim 64 only");
    if (c->n_kv_heads < 1 || c->n_kv_heads > 1024) return fail(INS_EINVAL, "n_kv_heads out of range");
    if (!(c->kv_groups == 1 || c->kv_groups == 2 || c->kv_groups == 4 || c->kv_groups == 8))
        return fail(INS_EINVAL, "kv_groups must be 1, 2, 4 or 8");
    if (!valid_bits(c->key_bits) || !valid_bits(c->value_bits))
        return fail(INS_EINVAL, "key_bits/value_bits outside 1..8");
    if (c->norm_bits != 16) return fail(INS_EINVAL, "this build stores 16-bit norms only");
    if (c->norm_frac < 0 || c->norm_frac >= c->norm_bits) return fail(INS_EINVAL, "norm_frac");
    if (c->centroid_frac + c->norm_frac < c->qk_frac)
        return fail(INS_EINVAL, "centroid_frac + norm_frac below qk_frac: the threshold "
                                "comparison would truncate x (ops/quantize.py:150-156)");
    if (c->acc_width < 2 || c->acc_width > 32 || c->score_width < 2 || c->score_width > 62)
        return fail(INS_EINVAL, "acc_width/score_width");
    if (c->exp_lut_bits < 1 || c->exp_lut_bits > 8 || c->acc_frac - c->exp_lut_bits < 0)
        return fail(INS_EINVAL, "exp_lut_bits");
    if (c->prob_frac < 1 || c->prob_frac > 16) return fail(INS_EINVAL, "prob_frac");
    if (c->rot_rounds < 0 || c->rot_rounds > MAX_ROUNDS) return fail(INS_EINVAL, "rot_rounds 0..8");
    if (c->page_tokens < 16 || c->page_tokens % 16 || c->page_tokens > 1024)
        return fail(INS_EINVAL, "page_tokens must be a multiple of 16 in [16, 1024]");
    if (c->max_seqs < 1 || c->max_pages_per_seq < 1 || c->n_pages < 1)
        return fail(INS_EINVAL, "max_seqs, max_pages_per_seq and n_pages must be positive");
    if (c->n_pages > INT32_MAX) return fail(INS_EINVAL, "n_pages above 2^31");
    if ((int64_t)c->max_seqs * c->max_pages_per_seq > INT32_MAX)
        return fail(INS_EINVAL, "max_seqs x max_pages_per_seq above 2^31 page-table entries");
    return INS_OK;
}

Geo make_geo(const ins_config &c) {
    Geo g{};
    g.n_kv = c.n_kv_heads;
    g.H = c.kv_groups;
    g.kb = c.key_bits;
    g.vb = c.value_bits;
    g.kbytes = D * c.key_bits / 8;
    g.vbytes = D * c.value_bits / 8;
    g.row_bytes = g.kbytes + g.vbytes + 2 * (c.norm_bits / 8);
    g.P = c.page_tokens;
    g.p_log2 = (c.page_tokens & (c.page_tokens - 1)) ? -1 : __builtin_ctz((unsigned)c.page_tokens);
    g.max_pages = c.max_pages_per_seq;
    g.norm_bits = c.norm_bits;
    g.norm_frac = c.norm_frac;
    g.qk_frac = c.qk_frac;
    g.centroid_frac = c.centroid_frac;
    g.acc_frac = c.acc_frac;
    g.acc_width = c.acc_width;
    g.score_width = c.score_width;
    g.prob_frac = c.prob_frac;
    g.exp_lut_bits = c.exp_lut_bits;
    g.saturate = c.saturate;
    g.rounds = c.rot_rounds;
    g.rot_shift = c.rot_shift;
    g.rot_inv = c.rot_inv_sqrt_q15;
    g.score_shift = c.qk_frac + c.centroid_frac + c.norm_frac - c.acc_frac;   // config.py:249-250
    g.acc_shift = c.centroid_frac + c.norm_frac + c.prob_frac - c.acc_frac;   // config.py:252-254
    g.enc_shift = c.centroid_frac + c.norm_frac - c.qk_frac;                  // ops/quantize.py:190
    g.head_bytes = (int64_t)g.P * (g.kbytes + g.vbytes + 4);
    g.page_bytes = g.head_bytes * g.n_kv;
    return g;
}

int sync_mirrors(ins_cache *c) {
    CK(cudaEventSynchronize(c->mirror_done));
    return INS_OK;
}

// Copy the page-table rows of sequences seq_lo .. seq_hi-1 to the device
// (after a reset or an import; ingress ships only the entries it adds).
int push_mirrors(ins_cache *c, cudaStream_t s, int32_t seq_lo, int32_t seq_hi) {
    const size_t row = (size_t)c->cfg.max_pages_per_seq;
    CK(cudaMemcpyAsync(c->d_page_table + (size_t)seq_lo * row, c->h_page_table + (size_t)seq_lo * row,
                       sizeof(int32_t) * row * (size_t)(seq_hi - seq_lo), cudaMemcpyHostToDevice, s));
    CK(cudaEventRecord(c->mirror_done, s));
    return INS_OK;
}

int64_t capacity_of(const ins_cache *c) {
    return (int64_t)c->cfg.max_pages_per_seq * c->cfg.page_tokens;
}

// Reserve slots for n tokens appended to their sequences in order. On
// failure nothing changes (the reference raises before it writes,
// cache/base.py:67-73).
int reserve_slots(ins_cache *c, int32_t n, const int32_t *seq_ids, int64_t *slots,
                  int32_t *lo, int32_t *hi, int2 *pt_new = nullptr, int32_t *n_new = nullptr) {
    const int P = c->cfg.page_tokens;
    std::vector<int64_t> len_after;
    std::vector<int32_t> touched;
    int64_t need_pages = 0;
    {
        std::vector<int64_t> extra(c->cfg.max_seqs, 0);
        for (int32_t i = 0; i < n; ++i) {
            const int32_t s = seq_ids[i];
            if (s < 0 || s >= c->cfg.max_seqs)
                return fail(INS_EINVAL, "sequence id " + std::to_string(s) + " out of range");
            extra[s] += 1;
        }
        for (int32_t s = 0; s < c->cfg.max_seqs; ++s) {
            if (!extra[s]) continue;
            const int64_t len = c->h_seq_lens[s], after = len + extra[s];
            if (after > capacity_of(c))
                return fail(INS_EBADLEN, "cache holds " + std::to_string(len) + " of " +
                                             std::to_string(capacity_of(c)) +
                                             " tokens for sequence " + std::to_string(s) +
                                             "; cannot append " + std::to_string(extra[s]));
            need_pages += (after + P - 1) / P - (len + P - 1) / P;
        }
        if (need_pages > (int64_t)c->free_pages.size())
            return fail(INS_EBADLEN, "page pool exhausted: need " + std::to_string(need_pages) +
                                         " pages, " + std::to_string(c->free_pages.size()) + " free");
    }
    int32_t smin = INT32_MAX, smax = -1;
    const size_t row = (size_t)c->cfg.max_pages_per_seq;
    if (n_new) *n_new = 0;
    for (int32_t i = 0; i < n; ++i) {
        const int32_t s = seq_ids[i];
        const int64_t pos = c->h_seq_lens[s];
        const size_t at = (size_t)s * row + (size_t)(pos / P);
        int32_t &pg = c->h_page_table[at];
        if (pos % P == 0) {
            pg = c->free_pages.back();
            c->free_pages.pop_back();
            if (pt_new) pt_new[(*n_new)++] = make_int2((int32_t)at, pg);
        }
        slots[i] = (int64_t)pg * P + pos % P;
        c->h_seq_lens[s] = (int32_t)(pos + 1);
        smin = s < smin ? s : smin;
        smax = s > smax ? s : smax;
    }
    *lo = smin;
    *hi = smax + 1;
    return INS_OK;
}

template <int H>
int launch_scan_h(ins_cache *c, int32_t B, const int32_t *d_seq, const int64_t *d_T,
                  const int64_t *h_T, const int32_t *q_rot, int64_t *out, ins_stats *stats,
                  ins_softmax mode, cudaStream_t s, const int32_t *h_seq) {
    const Geo &g = c->g;
    const int threads = H * 64;
    const dim3 grid(B * g.n_kv);
    if (mode == INS_SOFTMAX_TWO_PASS) {
        const size_t smem = (size_t)H * g.P * 8 + (size_t)2 * H * g.P * 4 + (size_t)g.P * g.vbytes +
                            (size_t)g.P * 4;
        auto fn = (g.kb == 4 && g.vb == 2) ? k_scan_two_pass<H, 4, 2>
                  : (g.kb == 3 && g.vb == 3) ? k_scan_two_pass<H, 3, 3>
                                             : k_scan_two_pass<H, 0, 0>;
        CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        fn<<<grid, threads, smem, s>>>(g, c->d_tables, d_seq, d_T, c->d_page_table,
                                       c->d_pool, q_rot, out, stats);
        CK(cudaGetLastError());
        c->chunk.launches += 1;
        return INS_OK;
    }
    return launch_online(c->chunk, g, c->d_tables, B, d_seq, d_T, h_T, c->d_page_table,
                         c->d_pool, q_rot, out, stats, c->d_status, H, s, h_seq);
}

}  // namespace

// ---------------------------------------------------------------------------
// launch_online picks the exact sequential kernel or the context-parallel
// chunked scan; it is defined in scan_chunked.cuh and instantiated here.
// ---------------------------------------------------------------------------

extern "C" {

int32_t ins_abi_version(void) { return 1; }

const char *ins_last_error(void) { return g_err.c_str(); }

int32_t ins_bytes_per_token(const ins_config *cfg) {
    if (!cfg || cfg->head_dim <= 0) return -1;
    const int32_t bits = cfg->head_dim * (cfg->key_bits + cfg->value_bits);
    if (bits % 8 || (cfg->head_dim * cfg->key_bits) % 8 || cfg->norm_bits % 8) return -1;
    return bits / 8 + 2 * (cfg->norm_bits / 8);
}

int ins_cache_create(const ins_config *cfg, const ins_tables *tb, int32_t device, ins_cache **out) {
    if (!out) return fail(INS_EINVAL, "out is NULL");
    *out = nullptr;
    if (int rc = check_config(cfg)) return rc;
    if (!tb || !tb->k_centroids || !tb->k_bounds || !tb->v_centroids || !tb->v_bounds ||
        !tb->exp_table || (cfg->rot_rounds && !tb->signs))
        return fail(INS_EINVAL, "tables incomplete");
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(INS_EINVAL, "no such device");
    DeviceGuard dg(device);

    DevTables ht;
    std::memset(&ht, 0, sizeof(ht));
    const int nk = 1 << cfg->key_bits, nv = 1 << cfg->value_bits;
    for (int i = 0; i < nk; ++i) {
        ht.k_cent[i] = tb->k_centroids[i];
        ht.k_cent_f64[i] = (double)tb->k_centroids[i];
        if (tb->k_centroids[i] >= (1ll << 20) || tb->k_centroids[i] <= -(1ll << 20))
            return fail(INS_EINVAL, "key centroid beyond 20 bits");
    }
    for (int i = 0; i + 1 < nk; ++i) ht.k_bound[i] = tb->k_bounds[i];
    for (int i = 0; i < nv; ++i) ht.v_cent[i] = tb->v_centroids[i];
    for (int i = 0; i + 1 < nv; ++i) ht.v_bound[i] = tb->v_bounds[i];
    for (int i = 0; i < (1 << cfg->exp_lut_bits); ++i) ht.exp_tab[i] = (int32_t)tb->exp_table[i];
    for (int r = 0; r < cfg->rot_rounds; ++r) {
        uint64_t m = 0;
        for (int j = 0; j < D; ++j) {
            const int64_t s = tb->signs[r * D + j];
            if (s != 1 && s != -1) return fail(INS_EINVAL, "signs must be +-1");
            if (s < 0) m |= 1ull << j;
        }
        ht.sign_mask[r] = m;
    }

    ins_cache *c = new ins_cache();
    c->cfg = *cfg;
    c->g = make_geo(*cfg);
    c->g.log2e = tb->log2e;
    c->g.delta_max = tb->delta_max;
    {
        int64_t cmax = 1;
        for (int i = 0; i < nk; ++i) {
            const int64_t x = tb->k_centroids[i] < 0 ? -tb->k_centroids[i] : tb->k_centroids[i];
            cmax = x > cmax ? x : cmax;
        }
        const int64_t lim = (1ll << 47) / cmax;
        c->g.q_lim = lim < (1ll << 30) ? lim : (1ll << 30);
    }
    c->device = device;
    auto cleanup = [&](int rc) {
        ins_cache_destroy(c);
        return rc;
    };
    const size_t pool_bytes = (size_t)cfg->n_pages * (size_t)c->g.page_bytes;
    const size_t pt = (size_t)cfg->max_seqs * (size_t)cfg->max_pages_per_seq;
    if (cudaMalloc(&c->d_tables, sizeof(DevTables)) != cudaSuccess ||
        cudaMalloc(&c->d_pool, pool_bytes) != cudaSuccess ||
        cudaMalloc(&c->d_page_table, sizeof(int32_t) * pt) != cudaSuccess ||
        cudaMalloc(&c->d_status, sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&c->d_redo_total, sizeof(unsigned long long)) != cudaSuccess ||
        cudaHostAlloc(&c->h_page_table, sizeof(int32_t) * pt, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc(&c->h_seq_lens, sizeof(int32_t) * cfg->max_seqs, cudaHostAllocDefault) !=
            cudaSuccess) {
        cudaGetLastError();
        return cleanup(fail(INS_ENOMEM, "allocation of " + std::to_string(pool_bytes) +
                                            " B of cache pool (or its tables) failed"));
    }
    if (cudaEventCreateWithFlags(&c->mirror_done, cudaEventDisableTiming) != cudaSuccess)
        return cleanup(fail(INS_ECUDA, "event creation failed"));
    c->chunk.redo_total = c->d_redo_total;
    c->stage_a.launches = c->stage_b.launches = c->stage_c.launches = &c->chunk.launches;
    std::memset(c->h_page_table, 0xff, sizeof(int32_t) * pt);
    std::memset(c->h_seq_lens, 0, sizeof(int32_t) * cfg->max_seqs);
    c->free_pages.reserve((size_t)cfg->n_pages);
    for (int64_t p = cfg->n_pages - 1; p >= 0; --p) c->free_pages.push_back((int32_t)p);
    if (cudaMemcpy(c->d_tables, &ht, sizeof(ht), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(c->d_page_table, c->h_page_table, sizeof(int32_t) * pt, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemset(c->d_status, 0, sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(c->d_redo_total, 0, sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(c->d_pool, 0, pool_bytes) != cudaSuccess)
        return cleanup(fail(INS_ECUDA, "initial copies failed"));
    if (cudaDeviceSynchronize() != cudaSuccess) return cleanup(fail(INS_ECUDA, "init sync failed"));
    *out = c;
    return INS_OK;
}

int ins_cache_destroy(ins_cache *c) {
    if (!c) return INS_OK;
    DeviceGuard dg(c->device);
    cudaDeviceSynchronize();
    c->stage_a.release();
    c->stage_b.release();
    c->stage_c.release();
    c->chunk.release();
    if (c->mirror_done) cudaEventDestroy(c->mirror_done);
    cudaFree(c->d_tables);
    cudaFree(c->d_pool);
    cudaFree(c->d_page_table);
    cudaFree(c->d_status);
    cudaFree(c->d_redo_total);
    if (c->h_page_table) cudaFreeHost(c->h_page_table);
    if (c->h_seq_lens) cudaFreeHost(c->h_seq_lens);
    delete c;
    return INS_OK;
}

int64_t ins_cache_length(const ins_cache *c, int32_t seq) {
    if (!c || seq < 0 || seq >= c->cfg.max_seqs) return -1;
    return c->h_seq_lens[seq];
}

int64_t ins_cache_capacity(const ins_cache *c) { return c ? capacity_of(c) : -1; }

int64_t ins_cache_launches(const ins_cache *c) { return c ? c->chunk.launches : -1; }

int ins_cache_set_tiles(ins_cache *c, int32_t mode) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (mode != INS_TILES_AUTO && mode != INS_TILES_LARGE && mode != INS_TILES_SMALL)
        return fail(INS_EINVAL, "tile mode must be INS_TILES_AUTO, _LARGE or _SMALL");
    c->chunk.tiles_mode = mode;
    return INS_OK;
}

int ins_cache_set_scan_kernel(ins_cache *c, int32_t mode) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (mode != INS_SCAN_FUSED && mode != INS_SCAN_SPLIT)
        return fail(INS_EINVAL, "scan kernel must be INS_SCAN_FUSED or INS_SCAN_SPLIT");
    c->chunk.scan_kernel = mode;
    return INS_OK;
}

int ins_cache_set_wait_test(ins_cache *c, int32_t poll_limit, int32_t item, int32_t chunk, int32_t head) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (poll_limit < 1 || head < 0 || head >= c->g.H || chunk < 0)
        return fail(INS_EINVAL, "wait test arguments");
    c->chunk.poll_limit = poll_limit;
    c->chunk.hold_item = item;
    c->chunk.hold_chunk = chunk;
    c->chunk.hold_head = head;
    return INS_OK;
}

int ins_cache_reset(ins_cache *c, int32_t seq) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    DeviceGuard dg(c->device);
    if (int rc = sync_mirrors(c)) return rc;
    const int32_t lo = seq < 0 ? 0 : seq, hi = seq < 0 ? c->cfg.max_seqs : seq + 1;
    if (seq >= c->cfg.max_seqs) return fail(INS_EINVAL, "sequence id out of range");
    const size_t row = (size_t)c->cfg.max_pages_per_seq;
    for (int32_t s = lo; s < hi; ++s) {
        for (size_t p = 0; p < row; ++p) {
            int32_t &pg = c->h_page_table[(size_t)s * row + p];
            if (pg >= 0) c->free_pages.push_back(pg);
            pg = -1;
        }
        c->h_seq_lens[s] = 0;
    }
    if (int rc = push_mirrors(c, 0, lo, hi)) return rc;
    CK(cudaStreamSynchronize(0));
    return INS_OK;
}

// The ingress launch shared by ins_ingress and ins_ingress_lanes: `lanes`,
// when set, replaces q, k and v with the board's packed 24-bit stream.
static int ingress_launch(ins_cache *c, int32_t n, const int32_t *seq_ids, const int32_t *q,
                          const int32_t *k, const int32_t *v, const uint8_t *lanes, int32_t *q_rot,
                          uint32_t flags, void *stream) {
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    if (int rc = sync_mirrors(c)) return rc;
    // staging: [slot of every token (n int64)][pages opened: (page-table index, page) (<= n int2)]
    if (int rc = c->stage_a.reserve(sizeof(int64_t) * (size_t)n + sizeof(int2) * (size_t)n)) return rc;
    int32_t lo, hi, n_new = 0;
    int64_t *h_slots = (int64_t *)c->stage_a.h;
    int2 *h_new = (int2 *)(h_slots + n);
    if (int rc = reserve_slots(c, n, seq_ids, h_slots, &lo, &hi, h_new, &n_new)) return rc;
    if (int rc = c->stage_a.upload(sizeof(int64_t) * (size_t)n + sizeof(int2) * (size_t)n_new, s))
        return rc;
    const int per_tok = ((q || lanes) ? c->g.n_kv * c->g.H : 0) + 2 * c->g.n_kv;
    const int64_t warps = (int64_t)n * per_tok;
    const int wpb = 8;
    const int64_t blocks = (warps + wpb - 1) / wpb;
    CK(launch_after(k_ingress, (unsigned)blocks, (unsigned)(wpb * 32), 0, s, c->g, (const DevTables *)c->d_tables,
                    n, (const int64_t *)c->stage_a.d, q, k, v, q_rot, c->d_pool, flags, c->d_status,
                    (const int2 *)((const int64_t *)c->stage_a.d + n), n_new, c->d_page_table, lanes));
    c->chunk.launches += 1;
    return INS_OK;
}

int ins_ingress(ins_cache *c, int32_t n, const int32_t *seq_ids, const int32_t *q,
                const int32_t *k, const int32_t *v, int32_t *q_rot, uint32_t flags,
                void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || (n > 0 && (!seq_ids || !k || !v))) return fail(INS_EINVAL, "ingress arguments");
    if (q && !q_rot) return fail(INS_EINVAL, "q given without q_rot");
    if (n == 0) return INS_OK;
    auto aligned = [](const void *p) { return ((uintptr_t)p & 7u) == 0; };
    if (!aligned(k) || !aligned(v) || (q && (!aligned(q) || !aligned(q_rot))))
        return fail(INS_EINVAL, "q/k/v buffers must be 8-byte aligned");
    return ingress_launch(c, n, seq_ids, q, k, v, nullptr, q_rot, flags, stream);
}

int ins_ingress_lanes(ins_cache *c, int32_t n, const int32_t *seq_ids, const uint8_t *lanes,
                      int32_t *q_rot, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || (n > 0 && (!seq_ids || !lanes || !q_rot))) return fail(INS_EINVAL, "ingress arguments");
    if (n == 0) return INS_OK;
    if (((uintptr_t)lanes & 1u) || ((uintptr_t)q_rot & 7u))
        return fail(INS_EINVAL, "lanes must be 2-byte aligned, q_rot 8-byte aligned");
    return ingress_launch(c, n, seq_ids, nullptr, nullptr, nullptr, lanes, q_rot, 0, stream);
}

int64_t ins_lanes_bytes_per_token(const ins_cache *c) {
    return c ? (int64_t)c->g.n_kv * (2 + c->g.H) * D * 3 : -1;
}

// The planes of the board's DDR layout for this cache's row format
// (DdrLayout.for_quant / planes, hw/ddr_layout.py:111-179): fields first, then
// beats of 16 bytes; every plane must be a whole beat or a whole fraction of one.
static int ddr_planes(const ins_cache *c, DdrPlanes &pl, int &maxw) {
    const int f[4] = {0, c->g.kbytes, c->g.kbytes + c->g.vbytes, c->g.row_bytes};
    pl.n = 0;
    maxw = 0;
    for (int i = 0; i < 3; ++i)
        for (int a = f[i]; a < f[i + 1];) {
            const int b = a + 16 < f[i + 1] ? a + 16 : f[i + 1], w = b - a;
            if (pl.n == 16 || w > 16 || 16 % w || w % 4 || a % 4)
                return fail(INS_EINVAL, "row fields do not split into beat planes of whole 32-bit words");
            pl.lo[pl.n] = a;
            pl.width[pl.n] = w;
            ++pl.n;
            maxw = w > maxw ? w : maxw;
            a = b;
        }
    return INS_OK;
}

int64_t ins_ddr_image_bytes(const ins_cache *c, int64_t capacity) {
    if (!c || capacity < 0) return -1;
    DdrPlanes pl;
    int maxw;
    if (ddr_planes(c, pl, maxw)) return -1;
    const int64_t span = (capacity * maxw + 4095) / 4096 * 4096;   // plane_span, 4 KB pages
    return (int64_t)c->g.n_kv * pl.n * span;
}

int ins_cache_ddr_image(ins_cache *c, int32_t seq, int64_t capacity, uint8_t *img, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(INS_EINVAL, "sequence id out of range");
    if (!img) return fail(INS_EINVAL, "image buffer is NULL");
    const int64_t n = c->h_seq_lens[seq];
    if (capacity < n)
        return fail(INS_EBADLEN, std::to_string(n) + " tokens exceeds capacity " + std::to_string(capacity));
    DdrPlanes pl;
    int maxw;
    if (int rc = ddr_planes(c, pl, maxw)) return rc;
    const int64_t span = (capacity * maxw + 4095) / 4096 * 4096;
    const int64_t total = (int64_t)c->g.n_kv * pl.n * span;
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemsetAsync(img, 0, (size_t)total, s));
    const int64_t threads = n * c->g.n_kv * pl.n;
    if (threads) {
        k_ddr_image<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
            c->g, c->d_pool, c->d_page_table + (size_t)seq * c->cfg.max_pages_per_seq, n, pl, span, img);
        CK(cudaGetLastError());
    }
    return INS_OK;
}

static int seam_launch(ins_cache *c, int32_t n, const float *q, const float *k, const float *v,
                       const int64_t *positions, bool host_positions, const ins_seam_cfg *cfg,
                       int32_t *wq, int32_t *wk, int32_t *wv, int64_t *conv, void *stream) {
    if (!c || !cfg) return fail(INS_EINVAL, "cache or seam config is NULL");
    if (n < 0 || (n > 0 && (!q || !k || !v || !positions || !wq || !wk || !wv || !conv)))
        return fail(INS_EINVAL, "seam arguments");
    if (!cfg->rope_cos || !cfg->rope_sin || cfg->max_position < 1 || cfg->rope_frac < 0 ||
        cfg->rope_frac > 30)
        return fail(INS_EINVAL, "seam RoPE tables");
    if (n == 0) return INS_OK;
    if (host_positions)
        for (int32_t i = 0; i < n; ++i)
            if (positions[i] < 0 || positions[i] >= cfg->max_position)
                return fail(INS_EINVAL, "position " + std::to_string(positions[i]) + " beyond the table's " +
                                            std::to_string(cfg->max_position));
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    SeamArgs a;
    if (host_positions) {
        if (int rc = c->stage_c.reserve(sizeof(int64_t) * (size_t)n)) return rc;
        std::memcpy(c->stage_c.h, positions, sizeof(int64_t) * (size_t)n);
        if (int rc = c->stage_c.upload(sizeof(int64_t) * (size_t)n, s)) return rc;
        a.pos = (const int64_t *)c->stage_c.d;
    } else {
        a.pos = positions;
    }
    a.max_position = cfg->max_position;
    a.status = c->d_status;
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_norm = cfg->q_norm;
    a.k_norm = cfg->k_norm;
    a.eps = cfg->norm_eps;
    a.attn_scale = cfg->attn_scale;
    a.cos_t = cfg->rope_cos;
    a.sin_t = cfg->rope_sin;
    a.frac = cfg->rope_frac;
    a.cast_after_rope = cfg->cast_after_rope;
    a.wire_bits = 24;
    a.wq = wq;
    a.wk = wk;
    a.wv = wv;
    a.conv = (unsigned long long *)conv;
    const int64_t warps = (int64_t)n * (c->g.n_kv * c->g.H + 2 * c->g.n_kv);
    k_seam<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(c->g, a, n);
    CK(cudaGetLastError());
    c->chunk.launches += 1;
    return INS_OK;
}

int ins_seam(ins_cache *c, int32_t n, const float *q, const float *k, const float *v,
             const int64_t *positions, const ins_seam_cfg *cfg, int32_t *wq, int32_t *wk, int32_t *wv,
             int64_t *conv, void *stream) {
    return seam_launch(c, n, q, k, v, positions, true, cfg, wq, wk, wv, conv, stream);
}

int ins_seam_device_positions(ins_cache *c, int32_t n, const float *q, const float *k, const float *v,
                              const int64_t *positions, const ins_seam_cfg *cfg, int32_t *wq,
                              int32_t *wk, int32_t *wv, int64_t *conv, void *stream) {
    return seam_launch(c, n, q, k, v, positions, false, cfg, wq, wk, wv, conv, stream);
}

int ins_scan(ins_cache *c, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
             const int32_t *q_rot, int64_t *out, ins_stats *stats, ins_softmax mode,
             void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (B < 0 || (B > 0 && (!seq_ids || !q_rot || !out))) return fail(INS_EINVAL, "scan arguments");
    if (mode != INS_SOFTMAX_ONLINE && mode != INS_SOFTMAX_TWO_PASS)
        return fail(INS_EINVAL, "unknown softmax mode");
    if (B == 0) return INS_OK;
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    // staging: [T (B int64)][seq ids (B int32)]
    const size_t bytes = sizeof(int64_t) * (size_t)B + sizeof(int32_t) * (size_t)B;
    if (int rc = c->stage_b.reserve(bytes)) return rc;
    int64_t *hT = (int64_t *)c->stage_b.h;
    int32_t *hS = (int32_t *)(hT + B);
    for (int32_t i = 0; i < B; ++i) {
        const int32_t sq = seq_ids[i];
        if (sq < 0 || sq >= c->cfg.max_seqs) return fail(INS_EINVAL, "sequence id out of range");
        const int64_t len = c->h_seq_lens[sq];
        int64_t T = len;
        if (lengths) {
            T = lengths[i];
            if (T < 0 || T > len)
                return fail(INS_EBADLEN, "scan length " + std::to_string(T) +
                                             " outside the sequence's " + std::to_string(len) +
                                             " cached tokens");
        }
        hT[i] = T;
        hS[i] = sq;
    }
    // the context-parallel online scan uploads the lengths and ids with its
    // tile plan (one copy); the other kernels read them from this upload
    const int64_t *d_T = nullptr;
    const int32_t *d_seq = nullptr;
    if (mode != INS_SOFTMAX_ONLINE || !chunk_variant(c->g, c->g.H)) {
        if (int rc = c->stage_b.upload(bytes, s)) return rc;
        d_T = (const int64_t *)c->stage_b.d;
        d_seq = (const int32_t *)(d_T + B);
    }
    ++c->gen;
    switch (c->g.H) {
        case 1: return launch_scan_h<1>(c, B, d_seq, d_T, hT, q_rot, out, stats, mode, s, hS);
        case 2: return launch_scan_h<2>(c, B, d_seq, d_T, hT, q_rot, out, stats, mode, s, hS);
        case 4: return launch_scan_h<4>(c, B, d_seq, d_T, hT, q_rot, out, stats, mode, s, hS);
        case 8: return launch_scan_h<8>(c, B, d_seq, d_T, hT, q_rot, out, stats, mode, s, hS);
    }
    return fail(INS_EINVAL, "kv_groups");
}

int ins_rotate(ins_cache *c, int64_t n, const int32_t *x, int32_t *y, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || (n > 0 && (!x || !y))) return fail(INS_EINVAL, "rotate arguments");
    if (n == 0) return INS_OK;
    if (((uintptr_t)x & 7u) || ((uintptr_t)y & 7u)) return fail(INS_EINVAL, "x/y must be 8-byte aligned");
    DeviceGuard dg(c->device);
    const int wpb = 8;
    k_rotate<<<(unsigned)((n + wpb - 1) / wpb), wpb * 32, 0, (cudaStream_t)stream>>>(
        c->g, c->d_tables, n, x, y, c->d_status);
    CK(cudaGetLastError());
    return INS_OK;
}

int ins_scores(ins_cache *c, int32_t seq, int32_t head, int64_t t0, int64_t n,
               const int32_t *q_rot, int64_t *s_out, int64_t *ovf, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (seq < 0 || seq >= c->cfg.max_seqs || head < 0 || head >= c->g.n_kv)
        return fail(INS_EINVAL, "sequence or head out of range");
    if (t0 < 0 || n < 0 || t0 + n > c->h_seq_lens[seq])
        return fail(INS_EBADLEN, "rows outside the sequence's length");
    if (n > 0 && (!q_rot || !s_out)) return fail(INS_EINVAL, "scores arguments");
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    if (ovf) CK(cudaMemsetAsync(ovf, 0, sizeof(int64_t), s));
    if (n == 0) return INS_OK;
    const int32_t *pt = c->d_page_table + (size_t)seq * c->cfg.max_pages_per_seq;
    unsigned long long *o = (unsigned long long *)ovf;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    const Geo &g = c->g;
#define INS_SCORES(HH)                                                                    \
    {                                                                                     \
        auto fn = g.kb == 4 ? k_scores<HH, 4> : g.kb == 3 ? k_scores<HH, 3> : k_scores<HH, 0>; \
        fn<<<blocks, 256, 0, s>>>(g, c->d_tables, pt, head, t0, n, c->d_pool, q_rot, s_out, o); \
    }
    switch (g.H) {
        case 1: INS_SCORES(1) break;
        case 2: INS_SCORES(2) break;
        case 4: INS_SCORES(4) break;
        case 8: INS_SCORES(8) break;
    }
#undef INS_SCORES
    CK(cudaGetLastError());
    return INS_OK;
}

int ins_cache_export(ins_cache *c, int32_t seq, int32_t head, int64_t t0, int64_t n, uint8_t *rows) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (seq < 0 || seq >= c->cfg.max_seqs || head < 0 || head >= c->g.n_kv)
        return fail(INS_EINVAL, "sequence or head out of range");
    if (t0 < 0 || n < 0 || t0 + n > c->h_seq_lens[seq])
        return fail(INS_EBADLEN, "rows outside the sequence's length");
    if (n == 0) return INS_OK;
    if (!rows) return fail(INS_EINVAL, "rows is NULL");
    DeviceGuard dg(c->device);
    if (int rc = sync_mirrors(c)) return rc;
    const int P = c->cfg.page_tokens;
    const size_t row = (size_t)c->cfg.max_pages_per_seq;
    std::vector<int64_t> slots((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t pos = t0 + i;
        slots[(size_t)i] = (int64_t)c->h_page_table[(size_t)seq * row + (size_t)(pos / P)] * P + pos % P;
    }
    int64_t *d_slots = nullptr;
    uint8_t *d_rows = nullptr;
    CK(cudaMalloc(&d_slots, sizeof(int64_t) * (size_t)n));
    if (cudaMalloc(&d_rows, (size_t)n * c->g.row_bytes) != cudaSuccess) {
        cudaFree(d_slots);
        return fail(INS_ENOMEM, "export buffer");
    }
    cudaMemcpy(d_slots, slots.data(), sizeof(int64_t) * (size_t)n, cudaMemcpyHostToDevice);
    const int64_t total = n * c->g.row_bytes;
    k_export_rows<<<(unsigned)((total + 255) / 256), 256>>>(c->g, c->d_pool, d_slots, n, head, d_rows);
    cudaError_t e = cudaMemcpy(rows, d_rows, (size_t)total, cudaMemcpyDeviceToHost);
    cudaFree(d_slots);
    cudaFree(d_rows);
    if (e != cudaSuccess) return fail(INS_ECUDA, std::string("export: ") + cudaGetErrorString(e));
    return INS_OK;
}

int ins_cache_import(ins_cache *c, int32_t seq, int64_t n, const uint8_t *rows) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || n > INT32_MAX) return fail(INS_EINVAL, "row count");
    if (n == 0) return INS_OK;
    if (!rows) return fail(INS_EINVAL, "rows is NULL");
    DeviceGuard dg(c->device);
    if (int rc = sync_mirrors(c)) return rc;
    std::vector<int32_t> ids((size_t)n, seq);
    std::vector<int64_t> slots((size_t)n);
    int32_t lo, hi;
    if (int rc = reserve_slots(c, (int32_t)n, ids.data(), slots.data(), &lo, &hi)) return rc;
    if (int rc = push_mirrors(c, 0, lo, hi)) return rc;
    const size_t bytes = (size_t)n * c->g.n_kv * c->g.row_bytes;
    int64_t *d_slots = nullptr;
    uint8_t *d_rows = nullptr;
    CK(cudaMalloc(&d_slots, sizeof(int64_t) * (size_t)n));
    if (cudaMalloc(&d_rows, bytes) != cudaSuccess) {
        cudaFree(d_slots);
        return fail(INS_ENOMEM, "import buffer");
    }
    cudaMemcpy(d_slots, slots.data(), sizeof(int64_t) * (size_t)n, cudaMemcpyHostToDevice);
    cudaMemcpy(d_rows, rows, bytes, cudaMemcpyHostToDevice);
    k_import_rows<<<(unsigned)((bytes + 255) / 256), 256>>>(c->g, c->d_pool, d_slots, n, d_rows);
    cudaError_t e = cudaDeviceSynchronize();
    cudaFree(d_slots);
    cudaFree(d_rows);
    if (e != cudaSuccess) return fail(INS_ECUDA, std::string("import: ") + cudaGetErrorString(e));
    return INS_OK;
}

int64_t ins_scan_recomputed(ins_cache *c, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL"), -1;
    DeviceGuard dg(c->device);
    const int n = c->chunk.last_items;
    if (n <= 0 || !c->chunk.redo) return 0;
    std::vector<int32_t> redo(n);
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess ||
        cudaMemcpy(redo.data(), c->chunk.redo, sizeof(int32_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(INS_ECUDA, "reading the recompute flags"), -1;
    int64_t k = 0;
    for (int i = 0; i < n; ++i) k += redo[i] != 0;
    return k;
}

int64_t ins_scan_recomputed_total(ins_cache *c, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL"), -1;
    DeviceGuard dg(c->device);
    unsigned long long k = 0;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess ||
        cudaMemcpy(&k, c->d_redo_total, sizeof(k), cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(INS_ECUDA, "reading the recompute count"), -1;
    return (int64_t)k;
}

int ins_cache_status(ins_cache *c, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    DeviceGuard dg(c->device);
    int32_t st = 0;
    CK(cudaStreamSynchronize((cudaStream_t)stream));
    CK(cudaMemcpy(&st, c->d_status, sizeof(st), cudaMemcpyDeviceToHost));
    CK(cudaMemset(c->d_status, 0, sizeof(st)));
    if (st & ST_TIMEOUT) return fail(INS_ETIMEOUT, "a bounded device wait gave up");
    if (st & ST_RANGE) return fail(INS_ERANGE, "a value escaped its fixed-point format");
    if (st & ST_INTERNAL) return fail(INS_EINVAL, "internal consistency check failed");
    if (st & ST_POSITION)
        return fail(INS_EINVAL, "a seam position lay outside the RoPE table (ins_seam_device_positions); "
                                "that token's lanes were written as zero");
    if (st & ST_SPLIT)
        return fail(INS_ERANGE, "a context-split merge could not prove its result exact (a shard held "
                                "more rescales of one head than its composite can carry, or the 32-bit "
                                "accumulator could have clamped); those items' outputs were not written");
    return INS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The scan's scalar stages on their own: the finalize and the exp lookup, run
// by the same device functions the scan kernels call, over caller arrays.
// ---------------------------------------------------------------------------
namespace ins {

__global__ void k_finalize_rows(Geo g, int64_t n, const int64_t *__restrict__ acc,
                                const int64_t *__restrict__ l, int64_t *__restrict__ out,
                                int64_t *__restrict__ recip, int64_t *__restrict__ shift) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * D) return;
    const int64_t row = i / D;
    out[i] = finalize_out(g, acc[i], l[row]);
    if ((i % D) == 0 && (recip || shift)) {
        int64_t r;
        int sh;
        reciprocal(g, l[row], r, sh);
        if (recip) recip[row] = r;
        if (shift) shift[row] = sh;
    }
}

// Row 0: exp_lut (the sequential and two-pass kernels); row 1: exp_lut32;
// row 2: exp_lut_def (the context-parallel scan, default format only, else 0).
// A negative distance, which the reference refuses (ops/attention.py:156-157),
// latches ST_RANGE and gives -1.
__global__ void k_exp_values(Geo g, const DevTables *__restrict__ tb, int64_t n,
                             const int64_t *__restrict__ delta, int32_t *__restrict__ p,
                             int32_t def_fmt, int32_t *status) {
    __shared__ int32_t tab[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = tb->exp_tab[i];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = delta[i];
        if (d < 0) {
            atomicOr(status, ST_RANGE);
            p[i] = p[n + i] = p[2 * n + i] = -1;
            continue;
        }
        p[i] = exp_lut(g, tab, d);
        p[n + i] = exp_lut32(g, tab, d);
        p[2 * n + i] = def_fmt ? (int32_t)exp_lut_def(tab, d) : 0;
    }
}

}  // namespace ins

extern "C" {

int ins_project(int32_t n, int32_t in_dim, int32_t out_dim, const uint16_t *w16, const float *x,
                const float *bias, float *y, void *stream) {
    if (n < 0 || in_dim < 8 || in_dim % 8 || in_dim > 8192 || out_dim < 1)
        return fail(INS_EINVAL, "project: n >= 0, in_dim a multiple of 8 in [8, 8192], out_dim >= 1");
    if (n == 0) return INS_OK;
    if (!w16 || !x || !y) return fail(INS_EINVAL, "project: NULL buffer");
    if ((uintptr_t)w16 & 15u) return fail(INS_EINVAL, "project: weights must be 16-byte aligned");
    const size_t smem = (size_t)PROJ_TT * in_dim * sizeof(__half);
    CK(cudaFuncSetAttribute(k_project, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int rows_per_cta = PROJ_WARPS;
    int grid = (out_dim + rows_per_cta - 1) / rows_per_cta;
    grid = grid < 2 * sms ? grid : 2 * sms;
    k_project<<<grid, PROJ_WARPS * 32, smem, (cudaStream_t)stream>>>(n, in_dim, out_dim,
                                                                     reinterpret_cast<const __half *>(w16), x,
                                                                     bias, y);
    CK(cudaGetLastError());
    return INS_OK;
}

int ins_finalize(ins_cache *c, int64_t n, const int64_t *acc, const int64_t *l, int64_t *out,
                 int64_t *recip, int64_t *shift, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || (n > 0 && (!acc || !l || !out))) return fail(INS_EINVAL, "finalize arguments");
    if (n == 0) return INS_OK;
    DeviceGuard dg(c->device);
    const int64_t threads = n * D;
    k_finalize_rows<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(c->g, n, acc, l, out,
                                                                                     recip, shift);
    CK(cudaGetLastError());
    return INS_OK;
}

int ins_exp_lut(ins_cache *c, int64_t n, const int64_t *delta, int32_t *p, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (n < 0 || (n > 0 && (!delta || !p))) return fail(INS_EINVAL, "exp arguments");
    if (n == 0) return INS_OK;
    DeviceGuard dg(c->device);
    const int64_t blocks = (n + 255) / 256;
    k_exp_values<<<(unsigned)(blocks < 1184 ? blocks : 1184), 256, 0, (cudaStream_t)stream>>>(
        c->g, c->d_tables, n, delta, p, is_def_fmt(c->g) ? 1 : 0, c->d_status);
    CK(cudaGetLastError());
    return INS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Context split: one sequence's tokens held by several shards (GPUs), each a
// causal range. Phase 1 gives each shard's per-item maxima; the caller
// exchanges them; phase 2, knowing the running maximum entering the shard,
// writes one composite per item; the caller gathers the composites and
// ins_merge_parts folds them in causal order.
// ---------------------------------------------------------------------------
namespace {

// Stage T and sequence ids of a scan call (the checks of ins_scan).
int stage_scan_args(ins_cache *c, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                    cudaStream_t s, std::vector<int32_t> *seq_out, std::vector<int64_t> *T_out,
                    const int64_t **d_T, const int32_t **d_seq) {
    const size_t bytes = sizeof(int64_t) * (size_t)B + sizeof(int32_t) * (size_t)B;
    if (int rc = c->stage_b.reserve(bytes)) return rc;
    int64_t *hT = (int64_t *)c->stage_b.h;
    int32_t *hS = (int32_t *)(hT + B);
    for (int32_t i = 0; i < B; ++i) {
        const int32_t sq = seq_ids[i];
        if (sq < 0 || sq >= c->cfg.max_seqs) return fail(INS_EINVAL, "sequence id out of range");
        const int64_t len = c->h_seq_lens[sq];
        int64_t T = len;
        if (lengths) {
            T = lengths[i];
            if (T < 0 || T > len)
                return fail(INS_EBADLEN, "scan length " + std::to_string(T) + " outside the sequence's " +
                                             std::to_string(len) + " cached tokens");
        }
        hT[i] = T;
        hS[i] = sq;
    }
    if (seq_out) seq_out->assign(hS, hS + B);
    if (T_out) T_out->assign(hT, hT + B);
    if (int rc = c->stage_b.upload(bytes, s)) return rc;
    *d_T = (const int64_t *)c->stage_b.d;
    *d_seq = (const int32_t *)(*d_T + B);
    return INS_OK;
}

template <int H, int KB, int VB, int RS>
int split_maxima_t(ins_cache *c, int32_t B, const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                   const int32_t *q_rot, int64_t *maxima, cudaStream_t s) {
    ChunkArgs a;
    c->split.rs = RS;
    if (int rc = prepare_chunked<H, KB, VB, RS>(c->chunk, c->g, c->d_tables, B, d_seq, d_T, h_T,
                                            c->d_page_table, c->d_pool, q_rot, nullptr, nullptr,
                                            c->d_status, a, s))
        return fail(rc, "context-split scan scratch");
    a.maxima = (long long *)maxima;
    if (int rc = launch_split_maxima<H, KB, VB, RS>(a, s)) return fail(rc, "context-split scores launch");
    c->split.a = a;
    return INS_OK;
}

template <int H, int KB, int VB, int RS>
int split_part_t(ins_cache *c, const int64_t *m_in, void *part, cudaStream_t s) {
    ChunkArgs a = c->split.a;
    a.m_init = (const long long *)m_in;
    a.parts = (PartRec *)part;
    if (int rc = launch_split_part<H, KB, VB, RS>(a, s)) return fail(rc, "context-split values launch");
    return INS_OK;
}

// The tile size of a context split is chosen by phase 1 and kept for phase 2.
template <int H, int KB, int VB>
int split_maxima_pick(ins_cache *c, int32_t B, const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                      const int32_t *q_rot, int64_t *maxima, cudaStream_t s) {
    if constexpr (ChunkCfg<H, KB, VB>::R == 4)
        if (small_tiles<H, KB, VB>(c->chunk, c->g, B, h_T))
            return split_maxima_t<H, KB, VB, 2>(c, B, d_seq, d_T, h_T, q_rot, maxima, s);
    return split_maxima_t<H, KB, VB, 0>(c, B, d_seq, d_T, h_T, q_rot, maxima, s);
}

template <int H, int KB, int VB>
int split_part_pick(ins_cache *c, const int64_t *m_in, void *part, cudaStream_t s) {
    if constexpr (ChunkCfg<H, KB, VB>::R == 4)
        if (c->split.rs == 2) return split_part_t<H, KB, VB, 2>(c, m_in, part, s);
    return split_part_t<H, KB, VB, 0>(c, m_in, part, s);
}

int split_maxima(ins_cache *c, int variant, int32_t B, const int32_t *d_seq, const int64_t *d_T,
                 const int64_t *h_T, const int32_t *q_rot, int64_t *maxima, cudaStream_t s) {
#define CALL(HH, KK, VV) split_maxima_pick<HH, KK, VV>(c, B, d_seq, d_T, h_T, q_rot, maxima, s)
    switch (variant) {
        case 142: return CALL(1, 4, 2);
        case 242: return CALL(2, 4, 2);
        case 442: return CALL(4, 4, 2);
        case 842: return CALL(8, 4, 2);
        case 433: return CALL(4, 3, 3);
        case 833: return CALL(8, 3, 3);
    }
#undef CALL
    return fail(INS_EINVAL, "no context-parallel scan for this cache");
}

int split_part(ins_cache *c, int variant, const int64_t *m_in, void *part, cudaStream_t s) {
#define CALL(HH, KK, VV) split_part_pick<HH, KK, VV>(c, m_in, part, s)
    switch (variant) {
        case 142: return CALL(1, 4, 2);
        case 242: return CALL(2, 4, 2);
        case 442: return CALL(4, 4, 2);
        case 842: return CALL(8, 4, 2);
        case 433: return CALL(4, 3, 3);
        case 833: return CALL(8, 3, 3);
    }
#undef CALL
    return fail(INS_EINVAL, "no context-parallel scan for this cache");
}
}  // namespace

extern "C" {

int64_t ins_part_bytes(ins_cache *c, int32_t B) {
    if (!c || B < 0) return fail(INS_EINVAL, "part size arguments"), -1;
    return (int64_t)B * c->g.n_kv * (int64_t)sizeof(PartRec);
}

int ins_scan_maxima(ins_cache *c, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                    const int32_t *q_rot, int64_t *maxima, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (B <= 0 || !seq_ids || !q_rot || !maxima) return fail(INS_EINVAL, "scan_maxima arguments");
    const int variant = chunk_variant(c->g, c->g.H);
    if (!variant)
        return fail(INS_EINVAL, "the context split needs the context-parallel scan (4b/2b or 3b/3b "
                                "codes, the default fixed-point format)");
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    c->split.armed = false;
    const int64_t *d_T;
    const int32_t *d_seq;
    if (int rc = stage_scan_args(c, B, seq_ids, lengths, s, &c->split.seq, &c->split.T, &d_T, &d_seq))
        return rc;
    ++c->gen;
    if (int rc = split_maxima(c, variant, B, d_seq, d_T, c->split.T.data(), q_rot, maxima, s)) return rc;
    c->split.armed = true;
    c->split.gen = c->gen;
    c->split.B = B;
    c->split.q_rot = q_rot;
    return INS_OK;
}

int ins_scan_part(ins_cache *c, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                  const int32_t *q_rot, const int64_t *m_in, void *part, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (B <= 0 || !seq_ids || !q_rot || !m_in || !part) return fail(INS_EINVAL, "scan_part arguments");
    if (((uintptr_t)part & 7u) || ((uintptr_t)m_in & 7u)) return fail(INS_EINVAL, "part/m_in must be 8-byte aligned");
    auto &sp = c->split;
    bool same = sp.armed && sp.gen == c->gen && sp.B == B && sp.q_rot == q_rot;
    for (int32_t i = 0; same && i < B; ++i) {
        const int32_t sq = seq_ids[i];
        const int64_t T = lengths ? lengths[i] : (sq >= 0 && sq < c->cfg.max_seqs ? c->h_seq_lens[sq] : -1);
        same = sq == sp.seq[i] && T == sp.T[i];
    }
    if (!same)
        return fail(INS_EINVAL, "ins_scan_part must follow ins_scan_maxima on this cache with the same "
                                "sequences, lengths and q_rot, with no scan in between");
    DeviceGuard dg(c->device);
    sp.armed = false;
    return split_part(c, chunk_variant(c->g, c->g.H), m_in, part, (cudaStream_t)stream);
}

int ins_merge_parts(ins_cache *c, int32_t B, int32_t n_parts, const void *parts, int64_t *out,
                    ins_stats *stats, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (B <= 0 || n_parts <= 0 || !parts || !out) return fail(INS_EINVAL, "merge_parts arguments");
    if ((uintptr_t)parts & 7u) return fail(INS_EINVAL, "parts must be 8-byte aligned");
    DeviceGuard dg(c->device);
    cudaStream_t s = (cudaStream_t)stream;
    const int n_items = B * c->g.n_kv;
    const PartRec *p = (const PartRec *)parts;
    switch (c->g.H) {
        case 1: k_merge_parts<1><<<n_items, CHUNK_THREADS, 0, s>>>(c->g, p, n_items, n_parts, out, stats, c->d_status); break;
        case 2: k_merge_parts<2><<<n_items, CHUNK_THREADS, 0, s>>>(c->g, p, n_items, n_parts, out, stats, c->d_status); break;
        case 4: k_merge_parts<4><<<n_items, CHUNK_THREADS, 0, s>>>(c->g, p, n_items, n_parts, out, stats, c->d_status); break;
        case 8: k_merge_parts<8><<<n_items, CHUNK_THREADS, 0, s>>>(c->g, p, n_items, n_parts, out, stats, c->d_status); break;
        default: return fail(INS_EINVAL, "kv_groups");
    }
    CK(cudaGetLastError());
    return INS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// ins_scan_noalloc: the online scan without any device allocation.
//
// Some callers cannot allocate device memory once they are running: a serving
// engine that hands the whole of HBM to its own pool at start-up, a runtime
// whose allocator is not reentrant from the thread that calls the scan, or
// host code that must not block on an allocation in its decode loop. ins_scan
// grows its scratch (chunk records, look-back flags, segment pool) with
// cudaMalloc the first time a larger batch or context arrives; this entry
// point runs the same chunked scan with that scratch carved from one
// file-scope device array of NOALLOC_BYTES, which every GPU that loads this
// library holds until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t NOALLOC_BYTES = (size_t)192 << 20;
constexpr int NOALLOC_MAX_B = 4096;           // sequences per call

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

struct NoallocState {
    void *ptr = nullptr;                      // device address of g_noalloc_scratch
};
std::mutex g_noalloc_mu;
NoallocState g_noalloc[256];                  // per device ordinal
// host staging of one call, reused under the lock
int64_t g_na_T[NOALLOC_MAX_B];
int32_t g_na_seq[NOALLOC_MAX_B];
TilePlan g_na_plan;
std::vector<uint8_t> g_na_desc;

template <int H, int KB, int VB, int RS = 0>
int noalloc_chunked(ins_cache *c, int32_t B, const int32_t *q_rot, int64_t *out, ins_stats *stats,
                    cudaStream_t s, NoallocState &st) {
    if constexpr (RS == 0 && ChunkCfg<H, KB, VB>::R == 4)
        if (small_tiles<H, KB, VB>(c->chunk, c->g, B, g_na_T))
            return noalloc_chunked<H, KB, VB, 2>(c, B, q_rot, out, stats, s, st);
    using CF = ChunkCfg<H, KB, VB, RS>;
    const Geo &g = c->g;
    const int n_items = B * g.n_kv;
    if (n_items > NOALLOC_MAX_B * 8) return fail(INS_EBADLEN, "too many (sequence, KV head) items");
    TilePlan &tp = g_na_plan;
    tp.build(g, B, g_na_T, CF::C);
    const int64_t n_tiles = tp.n_tiles;
    if (n_tiles > INT32_MAX / 2) return fail(INS_EBADLEN, "too many tiles for one scan");
    const int tiles = (int)(n_tiles < 1 ? 1 : n_tiles);
    const size_t staging = ((sizeof(int64_t) * (size_t)B + 255) & ~(size_t)255) + sizeof(int32_t) * (size_t)B;
    // The single-launch scan keeps scores in shared memory, so the carve needs
    // no per-row area: records per tile and per item, look-back words, and the
    // rescale-segment pool, which takes what the rest leaves, up to what
    // ins_scan would reserve; an item whose segments do not fit is recomputed
    // by the sequential kernel (still exact, only slower).
    const ScratchLayout L0(n_items, tp.max_nc, 0, tiles, H, CF::CW, 0);
    if (L0.total + staging > NOALLOC_BYTES)
        return fail(INS_EBADLEN, "this scan needs " + std::to_string(L0.total + staging) + " B of scratch; "
                                 "ins_scan_noalloc holds " + std::to_string(NOALLOC_BYTES) + " B");
    const int64_t seg_want = 2 * (64 * (int64_t)n_items * H) + 4 * (int64_t)tiles;
    const int64_t seg_fit = (int64_t)((NOALLOC_BYTES - L0.total - staging - 256) / sizeof(SegEntry));
    const int seg_cap = (int)std::min<int64_t>(std::min(seg_want, seg_fit), INT32_MAX);
    // the carve, in the same order ins_scan's scratch uses
    const ScratchLayout L(n_items, tp.max_nc, seg_cap, tiles, H, CF::CW, 0);
    const size_t o_T = L.total;
    const size_t o_seq = o_T + ((sizeof(int64_t) * (size_t)B + 255) & ~(size_t)255);
    const size_t o_end = o_seq + sizeof(int32_t) * (size_t)B;
    if (o_end > NOALLOC_BYTES)
        return fail(INS_EBADLEN, "this scan needs " + std::to_string(o_end) + " B of scratch; "
                                 "ins_scan_noalloc holds " + std::to_string(NOALLOC_BYTES) + " B");
    const TileDesc TD(n_items);
    g_na_desc.assign(TD.total, 0);
    tp.write(g_na_desc.data(), TD);
    uint8_t *p = (uint8_t *)st.ptr;
    // what the kernel expects at zero, since the array keeps whatever the
    // previous call left in it, laid out for that call's shape: the segment
    // counter, the per-item accumulators, the look-back words (read with
    // epoch 1, which a cleared word never carries) and the fold counters
    CK(cudaMemsetAsync(p + L.top, 0, 8, s));
    CK(cudaMemsetAsync(p + L.items, 0, sizeof(ItemAcc) * (size_t)n_items, s));
    CK(cudaMemsetAsync(p + L.lbw, 0, L.sdone + sizeof(unsigned int) - L.lbw, s));
    CK(cudaMemcpyAsync(p + L.desc, g_na_desc.data(), g_na_desc.size(), cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(p + o_T, g_na_T, sizeof(int64_t) * (size_t)B, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(p + o_seq, g_na_seq, sizeof(int32_t) * (size_t)B, cudaMemcpyHostToDevice, s));
    ChunkArgs a{};
    a.g = g;
    a.tb = c->d_tables;
    a.runs = (const int4 *)(p + L.desc + TD.runs);
    a.n_runs = (int32_t)tp.runs.size();
    a.order = (const int32_t *)(p + L.desc + TD.ord);
    a.tile_rows = CF::C;
    a.n_tiles = (int32_t)n_tiles;
    a.max_chunks = tp.max_nc;
    a.max_blocks = (tp.max_nc + GBLK - 1) / GBLK;
    a.n_items = n_items;
    a.row_base = (const int64_t *)(p + L.desc + TD.rb);
    a.seq_ids = (const int32_t *)(p + o_seq);
    a.T = (const int64_t *)(p + o_T);
    a.page_table = c->d_page_table;
    a.pool = c->d_pool;
    a.q_rot = q_rot;
    a.out = out;
    a.stats = stats;
    a.recs = (ChunkRec *)(p + L.rec);
    a.blks = (BlockRec *)(p + L.blk);
    a.segs = (SegEntry *)(p + L.seg);
    a.seg_top = (unsigned int *)(p + L.top);
    a.seg_cap = seg_cap;
    a.items = (ItemAcc *)(p + L.items);
    a.redo = (int32_t *)(p + L.redo);
    a.redo_total = c->d_redo_total;
    a.status = c->d_status;
    FusedExtra x;
    x.lbw = (unsigned long long *)(p + L.lbw);
    a.item_done = (unsigned int *)(p + L.idone);
    a.scan_done = (unsigned int *)(p + L.sdone);
    a.poll_limit = c->chunk.poll_limit;
    a.hold_rec = -1;
    x.epoch = 1;
    x.poll_limit = c->chunk.poll_limit;
    x.hold_word = -1;
    const int rc = launch_fused_kernels<H, KB, VB, RS>(a, x, B, a.seq_ids, a.T, s);
    if (rc) return fail(rc, "scan launch");
    c->chunk.launches += 3;                    // the scan, the fold, the exact re-run
    return INS_OK;
}

template <int H>
int noalloc_dispatch(ins_cache *c, int32_t B, const int32_t *q_rot, int64_t *out,
                     ins_stats *stats, cudaStream_t s, NoallocState &st) {
    const Geo &g = c->g;
    if (is_def_fmt(g) && g.kb == 4 && g.vb == 2) return noalloc_chunked<H, 4, 2>(c, B, q_rot, out, stats, s, st);
    if constexpr (H == 4 || H == 8)
        if (is_def_fmt(g) && g.kb == 3 && g.vb == 3)
            return noalloc_chunked<H, 3, 3>(c, B, q_rot, out, stats, s, st);
    // other widths scan with the sequential body, which needs no scratch
    uint8_t *p = (uint8_t *)st.ptr;
    CK(cudaMemcpyAsync(p, g_na_T, sizeof(int64_t) * (size_t)B, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(p + ((sizeof(int64_t) * (size_t)B + 255) & ~(size_t)255), g_na_seq,
                       sizeof(int32_t) * (size_t)B, cudaMemcpyHostToDevice, s));
    const int32_t *d_seq = (const int32_t *)(p + ((sizeof(int64_t) * (size_t)B + 255) & ~(size_t)255));
    CK(launch_seq<H>(g, c->d_tables, B, d_seq, (const int64_t *)p, c->d_page_table, c->d_pool,
                     q_rot, out, stats, nullptr, s));
    c->chunk.launches += 1;
    return INS_OK;
}

}  // namespace

extern "C" int ins_scan_noalloc(ins_cache *c, int32_t B, const int32_t *seq_ids,
                                const int64_t *lengths, const int32_t *q_rot, int64_t *out,
                                ins_stats *stats, void *stream) {
    if (!c) return fail(INS_EINVAL, "cache is NULL");
    if (B < 0 || (B > 0 && (!seq_ids || !q_rot || !out))) return fail(INS_EINVAL, "scan arguments");
    if (B == 0) return INS_OK;
    if (B > NOALLOC_MAX_B)
        return fail(INS_EBADLEN, "ins_scan_noalloc takes at most " + std::to_string(NOALLOC_MAX_B) +
                                     " sequences per call");
    if (c->device < 0 || c->device >= 256) return fail(INS_EINVAL, "device ordinal");
    DeviceGuard dg(c->device);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoallocState &st = g_noalloc[c->device];
    if (!st.ptr) {
        // once per device, with that device current: the array's device address
        void *ptr = nullptr;
        CK(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        st.ptr = ptr;
    }
    for (int32_t i = 0; i < B; ++i) {
        const int32_t sq = seq_ids[i];
        if (sq < 0 || sq >= c->cfg.max_seqs) return fail(INS_EINVAL, "sequence id out of range");
        const int64_t len = c->h_seq_lens[sq];
        int64_t T = len;
        if (lengths) {
            T = lengths[i];
            if (T < 0 || T > len)
                return fail(INS_EBADLEN, "scan length outside the sequence's cached tokens");
        }
        g_na_T[i] = T;
        g_na_seq[i] = sq;
    }
    cudaStream_t s = (cudaStream_t)stream;
    switch (c->g.H) {
        case 1: return noalloc_dispatch<1>(c, B, q_rot, out, stats, s, st);
        case 2: return noalloc_dispatch<2>(c, B, q_rot, out, stats, s, st);
        case 4: return noalloc_dispatch<4>(c, B, q_rot, out, stats, s, st);
        case 8: return noalloc_dispatch<8>(c, B, q_rot, out, stats, s, st);
    }
    return fail(INS_EINVAL, "kv_groups");
}
