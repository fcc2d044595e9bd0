// The context-parallel online scan.
//
// attend_online (ops/attention.py:451-513) is a sequential recurrence: a
// running maximum m, and at every token whose score exceeds it, a rescale
// acc = floor(acc * exp(s - m) / 2^15) before the token's own term is added.
// This scan splits every (sequence, KV head) item into tiles of C rows and
// still returns the reference's bits. It is three launches, and no CTA ever
// waits on another:
//
//  1. k_scan_scores: the scores of every tile (exact FP64 FMA on integer
//     operands; the K rows staged in shared memory by bulk copies one tile
//     ahead). Each is kept as its offset below its 32-row block's maximum;
//     the block and tile maxima are kept too.
//  2. k_scan_values, per tile: the running maximum entering it (m_in, the
//     maximum of the earlier tiles' maxima), the exact rescale points (tokens
//     above the running maximum), p = exp(m - s) for every token, and its
//     tokens split into segments at the rescale points. Within a segment
//     every term is a fixed integer, so its contribution is a plain sum; the
//     tile writes a record of its segments.
//  3. k_fold: a CTA per block of 32 tiles folds their records in causal
//     order, and the one that completes an item's last block folds the blocks
//     and finalizes: acc = floor(acc * f / 2^15) at each rescale, + segment
//     sums.
//     That fold equals the per-token recurrence provided the reference's
//     32-bit clamp never fires; the fold proves it per tile with
//     |acc at tile start| + sum_t max_k |term(t, k)| <= 2^31 - 1, which bounds
//     every partial sum inside the tile (a rescale never grows |acc|).
//
// An item that fails the proof, overflows the segment pool or meets a value
// outside the formats these kernels assume is recomputed by the exact
// sequential kernel (a last launch that only touches flagged items), so the
// result is bit-exact in every case.
#pragma once

#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace ins {

constexpr int HMAX = 8;
constexpr int SEGMAX = 32;               // rescales one head's tile can hold
constexpr int GBLK = 64;                 // tiles folded per level-1 block
constexpr int CHUNK_THREADS = 256;
constexpr int FB = 8;                     // block records an item fold loads at once

struct SegEntry {          // a rescale and the translation that follows it
    int64_t S[D];          // sum of terms after the rescale (per channel)
    int64_t l;             // sum of p over the same tokens
    int32_t f;             // factor applied to acc and l at the rescale
    int32_t pad;
};

struct ChunkRec {          // one (item, tile)
    int32_t S0[HMAX][D];   // terms of the tokens before the tile's first rescale
    int64_t l0[HMAX];
    int64_t B[HMAX];       // sum over tokens of max over codes of |term|
    int32_t nseg[HMAX];
    int32_t seg_base[HMAX];
};

struct BlockRec {          // GBLK consecutive tiles of one item, folded
    int64_t Spre[HMAX][D]; // translation before the block's first rescale
    int64_t Y[HMAX][D];    // max over the block of |local partial sum| (clamp proof)
    int64_t lpre[HMAX];
    int32_t nent[HMAX];
    int32_t ent_base[HMAX];
};

struct ItemAcc {
    unsigned long long done_blocks;
    unsigned long long resc;
    unsigned long long sovf;
    long long maxs;
    int32_t fail;
    int32_t pad;
};

// The fixed-point format the chunked kernels are compiled for: FixedFormat()
// with QuantConfig's norm_frac of 9 -- qk Q8.16, centroid Q1.15, acc Q16, prob
// Q15, an 8-bit exp LUT, 48-bit saturating scores (config.py:214-254). Other
// formats scan with the exact sequential kernel.
struct DefFmt {
    static constexpr int SCORE_SHIFT = 24, ACC_SHIFT = 23, ACC_FRAC = 16, LUT_BITS = 8, PROB_FRAC = 15;
    static constexpr int SCORE_WIDTH = 48;
    static constexpr int64_t LOG2E = 94548, DELTA_MAX = 772248;
    static constexpr int64_t S_LO = -(1ll << (SCORE_WIDTH - 1)), S_HI = (1ll << (SCORE_WIDTH - 1)) - 1;
};

inline bool is_def_fmt(const Geo &g) {
    return g.score_shift == DefFmt::SCORE_SHIFT && g.acc_shift == DefFmt::ACC_SHIFT &&
           g.acc_frac == DefFmt::ACC_FRAC && g.exp_lut_bits == DefFmt::LUT_BITS &&
           g.prob_frac == DefFmt::PROB_FRAC && g.score_width == DefFmt::SCORE_WIDTH &&
           g.saturate && g.log2e == DefFmt::LOG2E && g.delta_max == DefFmt::DELTA_MAX;
}

// exp_lut for a distance known to be non-negative, in the default format
// (ExpLut.__call__, ops/attention.py:153-159; the nested floors of exp_lut32).
__device__ __forceinline__ uint32_t exp_lut_def(const int32_t *tab, int64_t delta) {
    const uint32_t d = delta < DefFmt::DELTA_MAX ? (uint32_t)delta : (uint32_t)DefFmt::DELTA_MAX;
    const uint32_t u =
        (uint32_t)(((uint64_t)d * (uint64_t)DefFmt::LOG2E) >> (2 * DefFmt::ACC_FRAC - DefFmt::LUT_BITS));
    constexpr uint32_t SPAN = (uint32_t)(DefFmt::PROB_FRAC + 2) << DefFmt::LUT_BITS;
    return u >= SPAN ? 0u : ((uint32_t)tab[u & ((1u << DefFmt::LUT_BITS) - 1u)] >> (u >> DefFmt::LUT_BITS));
}

// Page slot and row of position `pr` of a sequence's rows.
__device__ __forceinline__ void page_row(const Geo &g, int pr, int &pi, int &lr) {
    if (g.p_log2 >= 0) {
        pi = pr >> g.p_log2;
        lr = pr & (g.P - 1);
    } else {
        pi = pr / g.P;
        lr = pr - pi * g.P;
    }
}

// One item's contribution from one context shard (a rank holding a causal
// range of a sequence): its tiles folded into one composite -- the sums before
// its first rescale, every rescale (factor, following sums) in order, the
// clamp-proof bound Y -- and its share of the statistics. Folding the shards'
// records in causal order is the recurrence over the whole sequence.
constexpr int PART_MAXE = 64;            // rescales one head's shard can hold

struct PartEntry {
    int32_t S[D];          // within a shard |S| <= Y, which the merge needs below 2^31
    int64_t l;
    int32_t f;
    int32_t pad;
};

struct PartRec {
    int64_t Spre[HMAX][D];
    int64_t Y[HMAX][D];
    int64_t lpre[HMAX];
    int32_t nent[HMAX];
    int32_t fail;                          // the shard could not build an exact composite
    int32_t pad;
    int64_t n_tokens, resc, sovf, maxs;
    PartEntry ent[HMAX][PART_MAXE];
};

struct ChunkArgs {
    Geo g;
    const DevTables *tb;
    // The tiles, chunk-major: every item's chunk 0, then every item's chunk
    // 1, ... (items with fewer chunks drop out). `order` lists the items by
    // chunk count, most first; run r covers the chunks from runs[r].x on, in
    // which the first runs[r].z items of `order` have a tile each, and its
    // first tile is tile runs[r].y.
    const int4 *runs;
    int32_t n_runs;
    const int32_t *order;
    int32_t tile_rows;            // rows per tile (the last tile of an item may hold fewer)
    int32_t n_tiles;
    int32_t max_chunks;
    int32_t max_blocks;
    int32_t n_items;
    const int64_t *row_base;      // [n_items]: first row of the item in `sc`
    const int32_t *seq_ids;
    const int64_t *T;
    const int32_t *page_table;
    const uint8_t *pool;
    const int32_t *q_rot;
    int64_t *out;
    ins_stats *stats;
    uint32_t *sc;                 // [rows][H]: score offset below its block maximum
    long long *bmg;               // [n_tiles][H][CW]: block maxima
    long long *cmx;               // [n_items * max_chunks][2][HMAX]: tile maximum, m_in
    ChunkRec *recs;               // [n_items * max_chunks]
    BlockRec *blks;               // [n_items * max_blocks]
    SegEntry *segs;
    unsigned int *seg_top;
    int32_t seg_cap;
    ItemAcc *items;               // [n_items]
    int32_t *redo;                // [n_items]: 1 = recompute with the sequential body
    int32_t *status;
    const long long *m_init;      // [n_items][H] running maximum entering the first tile, or null
    long long *maxima;            // [n_items][H] k_item_maxima writes each item's maximum, or null
    PartRec *parts;               // [n_items] composites instead of finalized outputs, or null
    unsigned long long *redo_total;  // running count of items handed to the sequential kernel, or null
    // counters of the fold launch that reset themselves on the last arrival
    unsigned int *item_done;      // [n_items] blocks folded into each item so far
    unsigned int *scan_done;      // items finished in this launch
    // the test of the bounded waits: polls before a wait gives up, and the
    // tile (item * max_chunks + chunk) whose staged rows are announced 16
    // bytes larger than the copies that land (its wait cannot complete), or -1
    int32_t poll_limit;
    int64_t hold_rec;
};

// Chunks of an item: one per tile_rows rows, and one (empty) for an empty item.
__device__ __forceinline__ int item_chunks(const ChunkArgs &a, int item) {
    const int64_t T = a.T[item / a.g.n_kv];
    return T ? (int)((T + a.tile_rows - 1) / a.tile_rows) : 1;
}

// Tile `tile` of the plan as (item, chunk, first row, rows). With one run all
// items have the same chunk count and `order` is the identity, so the common
// case reads nothing but T.
__device__ __forceinline__ int4 tile_at(const ChunkArgs &a, int tile) {
    int4 r;
    int item;
    if (a.n_runs == 1) {
        r = a.runs[0];
        item = (tile - r.y) % r.z;
    } else {
        int lo = 0, hi = a.n_runs - 1;              // the last run starting at or before `tile`
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (a.runs[mid].y <= tile) lo = mid;
            else hi = mid - 1;
        }
        r = a.runs[lo];
        item = a.order[(tile - r.y) % r.z];
    }
    const int c = r.x + (tile - r.y) / r.z;
    const int64_t T = a.T[item / a.g.n_kv], t0 = (int64_t)c * a.tile_rows;
    const int64_t n = T - t0 < a.tile_rows ? T - t0 : a.tile_rows;
    return make_int4(item, c, (int)t0, (int)(n > 0 ? n : 0));
}

// Pinned host buffers for the per-call uploads (the tile plan), used in turn:
// a buffer is rewritten only after the copy that read it four calls ago has
// run, so the host never waits for the stream to drain (a copy from pageable
// memory would). The slots live in one allocation that grows for all of them
// at once, so a warmed-up ring never allocates again.
struct PinnedRing {
    static constexpr int N = 4;
    uint8_t *base = nullptr;
    size_t slot_bytes = 0;
    cudaEvent_t ev[N] = {};
    int next = 0;

    void *take(size_t bytes, int &slot) {
        if (bytes > slot_bytes) {
            for (int i = 0; i < N; ++i)
                if (ev[i] && cudaEventSynchronize(ev[i]) != cudaSuccess) return nullptr;
            if (base) cudaFreeHost(base);
            base = nullptr;
            slot_bytes = 0;
            size_t want = 4096;
            while (want < bytes) want *= 2;
            if (cudaHostAlloc((void **)&base, want * N, cudaHostAllocDefault) != cudaSuccess) return nullptr;
            slot_bytes = want;
        }
        slot = next;
        next = (next + 1) % N;
        if (!ev[slot]) {
            if (cudaEventCreateWithFlags(&ev[slot], cudaEventDisableTiming) != cudaSuccess) return nullptr;
        } else if (cudaEventSynchronize(ev[slot]) != cudaSuccess) {
            return nullptr;
        }
        return base + (size_t)slot * slot_bytes;
    }
    int done(int slot, cudaStream_t s) { return cudaEventRecord(ev[slot], s) == cudaSuccess ? 0 : -1; }
    void release() {
        for (int i = 0; i < N; ++i) {
            if (ev[i]) cudaEventSynchronize(ev[i]), cudaEventDestroy(ev[i]);
            ev[i] = nullptr;
        }
        if (base) cudaFreeHost(base);
        base = nullptr;
        slot_bytes = 0;
    }
};

// Device layout of the tile plan of `ni` items: the runs, each item's first
// row in the score-offset array, the item order (see ChunkArgs::runs).
struct TileDesc {
    size_t runs, rb, ord, lens, seqs, total;
    // ni items; B > 0: the scan's lengths and sequence ids ride in the same
    // upload (one copy per scan)
    explicit TileDesc(int ni, int B = 0) {
        auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
        runs = 0;
        rb = al(sizeof(int4) * (size_t)(ni + 1));
        ord = rb + al(sizeof(int64_t) * (size_t)ni);
        lens = al(ord + sizeof(int32_t) * (size_t)ni);
        seqs = lens + sizeof(int64_t) * (size_t)B;
        total = seqs + sizeof(int32_t) * (size_t)B;
    }
};

// The tile plan of one scan, built on the host: items in chunk-count order
// and the runs of chunk levels that the same items reach. A batch of equal
// lengths is one run; B distinct lengths give at most B runs.
struct TilePlan {
    std::vector<int32_t> nc, order;
    std::vector<int64_t> rb;
    std::vector<int4> runs;
    int max_nc = 1;
    int64_t n_tiles = 0, rows = 0;

    void build(const Geo &g, int32_t B, const int64_t *h_T, int C) {
        const int ni = B * g.n_kv;
        nc.resize(ni);
        rb.resize(ni);
        order.resize(ni);
        rows = 0;
        max_nc = 1;
        bool uniform = true;
        for (int it = 0; it < ni; ++it) {
            const int64_t T = h_T[it / g.n_kv];
            nc[it] = T ? (int)((T + C - 1) / C) : 1;
            rb[it] = rows;
            rows += T;
            max_nc = nc[it] > max_nc ? nc[it] : max_nc;
            uniform = uniform && nc[it] == nc[0];
            order[it] = it;
        }
        if (!uniform)
            std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return nc[x] > nc[y]; });
        runs.clear();
        n_tiles = 0;
        int c = 0, k = ni;
        while (k > 0) {
            const int cend = nc[order[k - 1]];        // chunks c .. cend-1 hold the first k items
            if (cend > c) {
                runs.push_back(make_int4(c, (int)n_tiles, k, 0));
                n_tiles += (int64_t)k * (cend - c);
                c = cend;
            }
            while (k > 0 && nc[order[k - 1]] == cend) --k;
        }
    }
    // the plan in TileDesc layout at host address h
    void write(uint8_t *h, const TileDesc &L) const {
        memcpy(h + L.runs, runs.data(), sizeof(int4) * runs.size());
        memcpy(h + L.rb, rb.data(), sizeof(int64_t) * rb.size());
        memcpy(h + L.ord, order.data(), sizeof(int32_t) * order.size());
    }
};

// Device scratch of the chunked scan, owned by the cache handle and grown on
// demand. Everything in it is either rewritten each launch or reset by the
// kernels themselves, so launches need no memsets.
struct ChunkScratch {
    void *base = nullptr;
    size_t bytes = 0;
    int32_t n_items = 0, max_chunks = 0, seg_cap = 0, tile_cap = 0;
    int32_t last_items = 0;       // items of the last chunked launch (their redo flags)
    int32_t tiles_mode = 0;       // TILES_AUTO / TILES_LARGE / TILES_SMALL
    int32_t scan_kernel = 1;      // SCAN_FUSED (one launch) / SCAN_SPLIT (separate launches, the default)
    int32_t poll_limit = 1 << 22; // polls before a look-back wait of the fused scan gives up
    int32_t hold_item = -1, hold_chunk = 0, hold_head = 0;   // a look-back word left unpublished
                                                              // (the test of the bounded wait)
    unsigned long long *lbw = nullptr;   // look-back words of the fused scan
    size_t lbw_words = 0;
    unsigned int *idone = nullptr, *sdone = nullptr;
    unsigned int epoch = 0;       // of the last fused scan, 1 .. 4095
    int64_t launches = 0;         // kernels launched by ingress, seam and scan calls (a count)
    int64_t sc_rows = 0;          // rows * H capacity of `sc`, in 32-bit words
    uint32_t *sc = nullptr;
    long long *bmg = nullptr, *cmx = nullptr;
    ChunkRec *recs = nullptr;
    BlockRec *blks = nullptr;
    SegEntry *segs = nullptr;
    unsigned int *seg_top = nullptr;
    ItemAcc *items = nullptr;
    int32_t *redo = nullptr;
    unsigned long long *redo_total = nullptr;   // set by the cache: its running recompute count
    uint8_t *desc = nullptr;      // the tile plan (TileDesc layout), uploaded per call
    PinnedRing up;                // host side of the tile-plan uploads
    TilePlan plan;                // the last call's plan (its vectors keep their capacity)

    void release() {
        up.release();
        if (base) cudaFree(base);
        base = nullptr;
        bytes = 0;
        n_items = max_chunks = seg_cap = tile_cap = 0;
        sc_rows = 0;
    }
};

// ---------------------------------------------------------------------------
// Geometry of the tiles
//
// One CTA of 256 threads owns a tile of C rows of one (sequence, KV head)
// item. In k_scan_values shared memory holds, for the tile: the scores [H][C]
// (int64, later w = v_norm * p in place), the V codes transposed to one
// 32-bit word per (channel, 8 table units) -- nibble j of a word is the table
// index of unit j --, the v norms, two term tables (double-buffered
// sub-tiles of SUBT tokens) and the per-32-row block state of the online
// control. The V codes arrive row-major in a staging area that the term
// tables later reuse.
//
// A term-table unit is TPE consecutive tokens. For 2-bit V codes a unit is a
// token pair: its 16 entries hold term(t, k0) + term(t+1, k1) for every code
// pair, so one 16-byte lookup adds two tokens' terms for four heads. For 3-bit
// codes a unit is one token with 8 entries.
// ---------------------------------------------------------------------------
template <int H, int KB, int VB, int RS = 0>
struct ChunkCfg {
    static constexpr int NT = CHUNK_THREADS;
    // rows per thread in the score phase: RS, or the default for the shape
    static constexpr int R = RS ? RS : ((H == 8 || VB == 3) ? 2 : 4);
    static constexpr int C = R * NT;                         // rows per tile
    static constexpr int CW = C / 32;                        // 32-row blocks per tile
    static constexpr int NC = 1 << VB;                       // V codes
    static constexpr int VW = VB * 2;                        // 32-bit words per V row
    static constexpr int TPE = VB == 2 ? 2 : 1;              // tokens per table unit
    static constexpr int NE = 1 << (VB * TPE);               // entries per unit
    static constexpr int HL = H >= 4 ? 4 : H;                // heads per accumulating lane
    static constexpr int HG = H / HL;                        // head groups in the accumulate
    static constexpr int SUBT = (NT / 64) * 32 / HG;         // tokens per table sub-tile
    static constexpr int UNITS = SUBT / TPE;                 // units per sub-tile
    // A unit's entries are grouped by head pair: [head pair][index][2 heads],
    // 8 bytes an entry, so a warp's lookups of one unit (16 distinct entries at
    // most) fall in distinct banks. HPS pads a head pair's block by one entry
    // so that the build's stores (lanes = 8 units x 4 heads) are conflict-free
    // too. A single head (H == 1) keeps 4-byte entries.
    static constexpr int HPS = 2 * NE + 2;                   // words per head pair
    static constexpr int USTR = H == 1 ? NE + 1 : (H / 2) * HPS;   // words per unit
    static constexpr int TPW = 8 * TPE;                      // tokens per code word
    static constexpr int TWS = C / TPW + 1;                  // words per channel of the code matrix
    static constexpr int VS = (C + C / 16) / 32 * 32 + 48;   // words per V staging plane, = 16 mod 32
    static constexpr int STREAMS = (NT / 64) / HG;           // 32-token streams per sub-tile
    static constexpr size_t TAB_WORDS = (size_t)UNITS * USTR;
    static constexpr size_t STAGE_BYTES = (size_t)VW * VS * 4;
    static constexpr size_t TABS_BYTES =
        2 * TAB_WORDS * 4 > STAGE_BYTES ? 2 * TAB_WORDS * 4 : STAGE_BYTES;
    // byte offsets in dynamic shared memory
    static constexpr size_t OFF_S = 0;                                           // u32 [H][C]
    static constexpr size_t OFF_TW = OFF_S + (size_t)H * C * 4;                  // u32 [64][TWS]
    static constexpr size_t OFF_VN = OFF_TW + (size_t)64 * TWS * 4;              // int32 [C]
    static constexpr size_t OFF_TAB = (OFF_VN + (size_t)C * 4 + 15) & ~(size_t)15;
    static constexpr size_t OFF_GREW = OFF_TAB + TABS_BYTES;                     // u32 [H+1][CW]
    static constexpr size_t OFF_PRE = OFF_GREW + (size_t)(H + 1) * CW * 4;       // int32 [H][CW]
    static constexpr size_t OFF_BMAX = (OFF_PRE + (size_t)H * CW * 4 + 7) & ~(size_t)7;  // int64 [H][CW]
    static constexpr size_t OFF_BCAR = OFF_BMAX + (size_t)H * CW * 8;            // int64 [H][CW]
    static constexpr size_t OFF_DB = OFF_BCAR + (size_t)H * CW * 8;              // int64 [H][CW]
    static constexpr size_t OFF_S0 = OFF_DB + (size_t)H * CW * 8;                // int32 [H][64]
    // the next tile's V rows and norm words, staged by bulk copies
    static constexpr size_t OFF_VB = (OFF_S0 + (size_t)H * D * 4 + 15) & ~(size_t)15;
    static constexpr size_t OFF_NB = OFF_VB + (size_t)C * VW * 4;
    static constexpr size_t BYTES = OFF_NB + (size_t)C * 4 + 16;
    static_assert(C % 32 == 0 && SUBT % 32 == 0 && (UNITS * H) % 32 == 0, "tile shape");
    static_assert(H == 1 || (USTR % 2 == 0 && TAB_WORDS % 2 == 0), "8-byte entries stay aligned");
    static_assert(CW <= 32, "the control phase gives one lane to each 32-row block");
};

// Shared memory of k_scan_scores: the replicated pair table, then two tile
// buffers (the tile's K rows, then their norm words) that bulk copies fill one
// tile ahead of the arithmetic.
template <int H, int KB, int VB, int RS = 0>
struct ScoreCfg {
    static constexpr int C = ChunkCfg<H, KB, VB, RS>::C;
    static constexpr size_t CTAB = (size_t)(1 << (2 * KB)) * 8 * 16;
    static constexpr size_t KPL = (size_t)C * KB * 8;              // K rows of a tile
    static constexpr size_t BUF = KPL + (size_t)C * 4;             // + their norm words
    static constexpr size_t BYTES = CTAB + 2 * BUF;
    static constexpr int PGMAX = C / 16 + 1;                       // pages a tile touches (P >= 16)
    static_assert(CTAB % 16 == 0 && KPL % 16 == 0 && BUF % 16 == 0, "bulk copies need 16-byte alignment");
};

// The 16 x 16 transpose of 2-bit fields held in 16 words: on entry A[i] has
// field c = element (i, c); on exit A[c] has field i = element (i, c). Four
// block-swap stages (8, 4, 2, 1 fields), each pairing rows i and i + bs.
__device__ __forceinline__ void transpose16x2(uint32_t (&A)[16]) {
#pragma unroll
    for (int st = 0; st < 4; ++st) {
        const int bs = 8 >> st, s = 2 * bs;
        const uint32_t m = st == 0 ? 0x0000FFFFu : st == 1 ? 0x00FF00FFu : st == 2 ? 0x0F0F0F0Fu : 0x33333333u;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (!(i & bs)) {
                const uint32_t t = ((A[i] >> s) ^ A[i + bs]) & m;
                A[i + bs] ^= t;
                A[i] ^= t << s;
            }
    }
}

// One row's K code words (KB words per 32 channels) and its norm word.
template <int KB>
__device__ __forceinline__ void load_krow(const Geo &g, const uint8_t *reg, int lr,
                                          uint32_t (&kw)[KB * 2], uint32_t &nw) {
    const uint8_t *kp = reg + (int64_t)lr * (KB * 8);
    if constexpr (KB == 4) {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(kp));
        const uint4 b = __ldg(reinterpret_cast<const uint4 *>(kp) + 1);
        kw[0] = a.x; kw[1] = a.y; kw[2] = a.z; kw[3] = a.w;
        kw[4] = b.x; kw[5] = b.y; kw[6] = b.z; kw[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < KB; ++i) {
            const uint2 a = __ldg(reinterpret_cast<const uint2 *>(kp) + i);
            kw[2 * i] = a.x;
            kw[2 * i + 1] = a.y;
        }
    }
    nw = __ldg(reinterpret_cast<const uint32_t *>(reg + nplane_off(g) + (int64_t)lr * 4));
}

// One row's V code words and its norm word.
template <int VB>
__device__ __forceinline__ void load_vrow(const Geo &g, const uint8_t *reg, int lr,
                                          uint32_t (&vw)[VB * 2], uint32_t &nw) {
    const uint8_t *vp = reg + vplane_off(g) + (int64_t)lr * (VB * 8);
    if constexpr (VB == 2) {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(vp));
        vw[0] = a.x; vw[1] = a.y; vw[2] = a.z; vw[3] = a.w;
    } else {
#pragma unroll
        for (int i = 0; i < VB; ++i) {
            const uint2 a = __ldg(reinterpret_cast<const uint2 *>(vp) + i);
            vw[2 * i] = a.x;
            vw[2 * i + 1] = a.y;
        }
    }
    nw = __ldg(reinterpret_cast<const uint32_t *>(reg + nplane_off(g) + (int64_t)lr * 4));
}

// Code j (0..63) of a row held as KB*2 words (32 codes of KB bits = KB words).
// The extraction is a volatile asm statement so that the compiler keeps it
// next to its lookup instead of computing all 64 x R of them up front, which
// would need more registers than the kernel has.
template <int KB>
__device__ __forceinline__ uint32_t kcode(const uint32_t (&kw)[KB * 2], int j);

// The codes of channels 2p and 2p+1 of a row held as KB*2 words, as one index
// code(2p) + code(2p+1) << KB (bits 2p*KB .. 2p*KB + 2KB - 1 of the row; no
// 32-channel group boundary falls inside a pair). Pinned like kcode.
template <int KB>
__device__ __forceinline__ uint32_t kpair(const uint32_t (&kw)[KB * 2], int p) {
    const int pos = (p >> 4) * 32 * KB + (p & 15) * 2 * KB;
    const int wi = pos >> 5, sh = pos & 31;
    uint32_t v;
    if (sh + 2 * KB <= 32) {
        asm volatile("bfe.u32 %0, %1, %2, %3;" : "=r"(v) : "r"(kw[wi]), "r"(sh), "r"(2 * KB));
    } else {
        asm volatile("{\n\t.reg .u32 t;\n\tshf.r.clamp.b32 t, %1, %2, %3;\n\tand.b32 %0, t, %4;\n\t}"
                     : "=r"(v) : "r"(kw[wi]), "r"(kw[wi + 1]), "r"(sh), "r"((1u << (2 * KB)) - 1u));
    }
    return v;
}

template <int KB>
__device__ __forceinline__ uint32_t kcode(const uint32_t (&kw)[KB * 2], int j) {
    const int pos = (j >> 5) * 32 * KB + (j & 31) * KB;   // bit position in the row
    const int wi = pos >> 5, sh = pos & 31;
    uint32_t v;
    if (sh + KB <= 32) {
        asm volatile("bfe.u32 %0, %1, %2, %3;" : "=r"(v) : "r"(kw[wi]), "r"(sh), "r"(KB));
    } else {
        asm volatile("{\n\t.reg .u32 t;\n\tshf.r.clamp.b32 t, %1, %2, %3;\n\tand.b32 %0, t, %4;\n\t}"
                     : "=r"(v) : "r"(kw[wi]), "r"(kw[wi + 1]), "r"(sh), "r"((1u << KB) - 1u));
    }
    return v;
}

template <class T>
__device__ __forceinline__ T ldcg(const T *p) {
    return __ldcg(p);
}

// Max over the CTA of non-negative values < 2^51, with two 32-bit warp
// reductions per warp and one slot per warp. Every thread calls it.
__device__ __forceinline__ long long cta_max_nonneg(long long v, long long *slots /* [NT/32] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hi = (int)(v >> 20);
    const int mhi = __reduce_max_sync(FULL, hi);
    const unsigned mlo = __reduce_max_sync(FULL, hi == mhi ? (unsigned)(v & 0xFFFFF) : 0u);
    __syncthreads();
    if (lane == 0) slots[warp] = (long long)mhi * (1ll << 20) + (long long)mlo;
    __syncthreads();
    long long m = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = slots[w] > m ? slots[w] : m;
    return m;
}

// The folds stage what they read in shared memory, so that a fold costs a few
// rounds of loads instead of one round per record with rescales.
//
// Rescale entries: up to ECAP per head (the first ones in causal order) of up
// to NR consecutive records (the tiles of a block, or 32 blocks of an item)
// are staged; an entry past that is read from global memory where it is
// applied.
template <int H>
struct FoldCfg {
    static constexpr int ECAP = 128 / H;                           // staged entries per head
    static constexpr size_t OFF_ES = 0;                            // int64 [H][ECAP][D]: S
    static constexpr size_t OFF_S0 = OFF_ES + (size_t)H * ECAP * D * 8;  // int32 [GBLK][H][D]: tile sums
    static constexpr size_t BYTES = OFF_S0 + (size_t)GBLK * H * D * 4;
};

// The staged entries of one fold step; `cnt`/`bas`: per (head, record) the
// entry count and first entry index, for nrec <= NR records.
template <int H, int NR>
struct EntStage {
    static constexpr int ECAP = FoldCfg<H>::ECAP;
    int ex[H][NR + 1];          // entries before each record; [h][NR] = the head's total
    int idx[H * ECAP];
    int32_t f[H * ECAP];
    long long l[H * ECAP];
};

template <int H, int NR>
__device__ void stage_entries(const ChunkArgs &a, const int (*cnt)[NR], const int (*bas)[NR], int nrec,
                              EntStage<H, NR> &st, long long *eS /* [H][ECAP][D] */) {
    constexpr int ECAP = FoldCfg<H>::ECAP;
    static_assert(NR % 32 == 0, "records in whole warps");
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (w < H) {                               // warp h: head h, records lane, lane + 32, ...
        int before = 0;
#pragma unroll
        for (int i = 0; i < NR / 32; ++i) {
            const int r = i * 32 + lane;
            const int c = r < nrec ? cnt[w][r] : 0;
            int x = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(FULL, x, off);
                if (lane >= off) x += y;
            }
            const int ex = before + x - c;
            st.ex[w][r] = ex;
            for (int j = 0; j < c && ex + j < ECAP; ++j) st.idx[w * ECAP + ex + j] = bas[w][r] + j;
            before += __shfl_sync(FULL, x, 31);
        }
        if (lane == 0) st.ex[w][NR] = before;
    }
    __syncthreads();
    // only the staged entries, all heads in one index space, eight loads a
    // thread issued before any is stored
    int start[H + 1];
    start[0] = 0;
#pragma unroll
    for (int h = 0; h < H; ++h) start[h + 1] = start[h] + min(st.ex[h][NR], ECAP) * D;
    const int tot = start[H];
    constexpr int U = 8;
    for (int base = (int)threadIdx.x; base < tot; base += U * (int)blockDim.x) {
        long long v[U];
        int dst[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * (int)blockDim.x;
            dst[u] = -1;
            if (i < tot) {
                int h = 0, s0 = 0;
#pragma unroll
                for (int hh = 1; hh < H; ++hh)
                    if (i >= start[hh]) {
                        h = hh;
                        s0 = start[hh];
                    }
                const int k = (i - s0) / D, ch = (i - s0) % D;
                const SegEntry &se = a.segs[st.idx[h * ECAP + k]];
                v[u] = ldcg(&se.S[ch]);
                dst[u] = (h * ECAP + k) * D + ch;
                if (ch == 0) {
                    st.f[h * ECAP + k] = ldcg(&se.f);
                    st.l[h * ECAP + k] = ldcg(&se.l);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (dst[u] >= 0) eS[dst[u]] = v[u];
    }
    __syncthreads();
}

// Entry j of record r of head h (f, S[ch], l), staged or from global memory.
template <int H, int NR>
__device__ __forceinline__ void entry_at(const ChunkArgs &a, const EntStage<H, NR> &st, const long long *eS,
                                         const int (*bas)[NR], int h, int r, int j, int ch,
                                         int64_t &f, int64_t &S, int64_t &l) {
    constexpr int ECAP = FoldCfg<H>::ECAP;
    const int k = st.ex[h][r] + j;
    if (k < ECAP) {
        f = st.f[h * ECAP + k];
        S = eS[((size_t)h * ECAP + k) * D + ch];
        l = st.l[h * ECAP + k];
    } else {
        const SegEntry &se = a.segs[bas[h][r] + j];
        f = ldcg(&se.f);
        S = ldcg(&se.S[ch]);
        l = ldcg(&se.l);
    }
}

// The end of an item's fold: the item goes to the exact sequential kernel if
// any thread's proof failed (or the item was flagged), else its outputs are
// finalized and its statistics written. Called by every thread of the CTA.
template <int H>
__device__ __forceinline__ void finalize_item(const ChunkArgs &a, int item, int64_t T, int64_t qbase,
                                              const int64_t (&acc)[(H * D + CHUNK_THREADS - 1) / CHUNK_THREADS],
                                              const int64_t (&l)[(H * D + CHUNK_THREADS - 1) / CHUNK_THREADS],
                                              bool bad, long long *slots /* [NT/32] */) {
    constexpr int NP = (H * D + CHUNK_THREADS - 1) / CHUNK_THREADS;
    const int tid = threadIdx.x;
    bad = __syncthreads_or(bad);
    if (tid == 0) {
        a.redo[item] = bad ? 1 : 0;
        if (bad && a.redo_total) atomicAdd(a.redo_total, 1ull);
    }
    if (bad) return;
    int64_t *out_row = a.out + qbase;
    long long mx = 0;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        const int pr = tid + k * CHUNK_THREADS;
        if (pr >= H * D) continue;
        out_row[pr] = finalize_out(a.g, acc[k], l[k]);
        const long long ab = acc[k] < 0 ? -acc[k] : acc[k];
        mx = ab > mx ? ab : mx;
    }
    // the fold already proved |acc| <= 2^31 - 1
    mx = cta_max_nonneg(mx, slots);
    if (tid == 0 && a.stats) {
        const volatile ItemAcc &ia = a.items[item];
        ins_stats st;
        st.n_tokens = T;
        st.rescale_events = (int64_t)ia.resc;
        st.score_overflows = (int64_t)ia.sovf;
        st.acc_overflows = 0;
        st.max_abs_score = ia.maxs;
        st.max_abs_acc = mx;
        a.stats[item] = st;
    }
}

// Items of at most this many tiles are folded and finalized by one CTA in one
// pass over their tiles (GBLK at a time), without block records.
constexpr int DIRECT_TILES = 4 * GBLK;

// Level 1: fold the tiles of block `blk` of `item` into a BlockRec. The
// records come into shared memory first (the scalars by one warp per head,
// the sums S0 and the rescale entries by the whole CTA); then each thread
// takes a (head, channel) pair and walks the tiles in order. `direct`: the
// CTA walks all the item's tiles (GBLK at a time) and, the walk's running
// accumulator being the item's, proves and finalizes it here.
template <int H>
__device__ void merge_block(const ChunkArgs &a, int item, int blk, int nchunks, int *base_sm /* [H] */,
                            uint8_t *dyn /* FoldCfg<H>::BYTES */, bool direct, long long *slots) {
    constexpr int NR = GBLK;
    constexpr int NP = (H * D + CHUNK_THREADS - 1) / CHUNK_THREADS;   // pairs per thread
    const ChunkRec *recs = a.recs + (int64_t)item * a.max_chunks;
    int32_t *s0_sm = reinterpret_cast<int32_t *>(dyn + FoldCfg<H>::OFF_S0);
    long long *eS = reinterpret_cast<long long *>(dyn + FoldCfg<H>::OFF_ES);
    __shared__ long long bk_s[H][NR], l0_s[H][NR];
    __shared__ int ns_s[H][NR], sb_s[H][NR];
    __shared__ unsigned long long quiet_s[H];          // bit u: tile u has no entry for the head
    __shared__ EntStage<H, NR> st;
    static_assert(NR == 64 && HMAX <= CHUNK_THREADS / 32, "one warp per head, two tiles per lane");
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // per (head, channel) pair: the running fold
    int64_t loc[NP], Y[NP], curS[NP], curl[NP], Spre[NP], lpre[NP], lrun[NP];
    int ne[NP];
    bool opened[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        loc[k] = Y[k] = curS[k] = curl[k] = Spre[k] = lpre[k] = lrun[k] = 0;
        ne[k] = 0;
        opened[k] = false;
    }
    if (w < H && lane == 0) base_sm[w] = -1;
    const int cbeg = direct ? 0 : blk * GBLK, cend = direct ? nchunks : min(nchunks, blk * GBLK + GBLK);
    for (int c0 = cbeg; c0 < cend; c0 += GBLK) {
        const int nt = min(GBLK, cend - c0);
        // warp h: head h's scalars, tiles lane and lane + 32, and (one block)
        // the entries the head's block record needs = the rescales in its tiles
        if (w < H) {
            int need = 0;
            unsigned long long qm = 0;
#pragma unroll
            for (int i = 0; i < NR / 32; ++i) {
                const int r = i * 32 + lane, c = c0 + r;
                int ns = 0, sb = 0;
                if (c < c0 + nt) {
                    bk_s[w][r] = ldcg(&recs[c].B[w]);
                    l0_s[w][r] = ldcg(&recs[c].l0[w]);
                    ns = ldcg(&recs[c].nseg[w]);
                    sb = ldcg(&recs[c].seg_base[w]);
                }
                ns_s[w][r] = ns;
                sb_s[w][r] = sb;
                need += ns;
                qm |= (unsigned long long)__ballot_sync(FULL, ns == 0) << (32 * i);
            }
            need = __reduce_add_sync(FULL, need);
            if (lane == 0) {
                quiet_s[w] = qm;
                if (!direct) {
                    unsigned b = 0;
                    if (need) b = atomicAdd(a.seg_top, (unsigned)need);
                    if (need && b + need > (unsigned)a.seg_cap) {
                        atomicExch(&a.items[item].fail, 1);
                        need = 0;
                    }
                    base_sm[w] = need ? (int)b : -1;
                }
            }
        }
        // S0 of every tile, 16 bytes a load: [tile][head][channel]
        {
            constexpr int Q = D / 4;                   // 16-byte pieces per (tile, head)
            constexpr int U = 8;                       // loads a thread issues before it stores
            const int n16 = nt * H * Q;
            for (int base = (int)threadIdx.x; base < n16; base += U * (int)blockDim.x) {
                int4 x[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int i = base + j * (int)blockDim.x;
                    if (i < n16) {
                        const int u = i / (H * Q), r = i % (H * Q), h = r / Q, q = r % Q;
                        x[j] = ldcg(reinterpret_cast<const int4 *>(&recs[c0 + u].S0[h][0]) + q);
                    }
                }
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int i = base + j * (int)blockDim.x;
                    if (i < n16) {
                        const int u = i / (H * Q), r = i % (H * Q), h = r / Q, q = r % Q;
                        reinterpret_cast<int4 *>(s0_sm + ((size_t)u * H + h) * D)[q] = x[j];
                    }
                }
            }
        }
        __syncthreads();
        // the tiles' entries; the block's own entries written below are a
        // separate allocation, so these read what the values launch wrote
        stage_entries<H, NR>(a, ns_s, sb_s, nt, st, eS);
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            const int pr = threadIdx.x + k * CHUNK_THREADS;
            if (pr >= H * D) continue;
            const int h = pr / D, ch = pr % D;
            const int eb = base_sm[h];
            const unsigned long long qm = quiet_s[h];
            const int32_t *s0h = s0_sm + (size_t)h * D + ch;      // tile u at s0h[u * H * D]
            int u = 0;
            while (u < nt) {
                // four tiles with no rescale for the head: plain translations
                if (u + 4 <= nt && ((qm >> u) & 15ull) == 15ull) {
                    int32_t S[4];
                    long long Bv[4], lv[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        S[j] = s0h[(size_t)(u + j) * H * D];
                        Bv[j] = bk_s[h][u + j];
                        lv[j] = l0_s[h][u + j];
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int64_t al = loc[k] < 0 ? -loc[k] : loc[k];
                        Y[k] = max(Y[k], al + (int64_t)Bv[j]);
                        loc[k] += S[j];
                        curS[k] += S[j];
                        curl[k] += lv[j];
                        lrun[k] += lv[j];
                    }
                    u += 4;
                    continue;
                }
                const int32_t S0 = s0h[(size_t)u * H * D];
                const int64_t al = loc[k] < 0 ? -loc[k] : loc[k];
                Y[k] = max(Y[k], al + (int64_t)bk_s[h][u]);
                loc[k] += S0;
                curS[k] += S0;
                curl[k] += l0_s[h][u];
                lrun[k] += l0_s[h][u];
                const int ns = ns_s[h][u];
                for (int j = 0; j < ns; ++j) {
                    int64_t f, sS, sl;
                    entry_at<H, NR>(a, st, eS, sb_s, h, u, j, ch, f, sS, sl);
                    if (eb >= 0) {
                        if (!opened[k]) {
                            Spre[k] = curS[k];
                            lpre[k] = curl[k];
                            opened[k] = true;
                        } else {
                            a.segs[eb + ne[k] - 1].S[ch] = curS[k];
                            if (ch == 0) a.segs[eb + ne[k] - 1].l = curl[k];
                        }
                        if (ch == 0) a.segs[eb + ne[k]].f = (int32_t)f;
                        ++ne[k];
                    }
                    curS[k] = sS;
                    curl[k] = sl;
                    loc[k] = ((loc[k] * f) >> a.g.prob_frac) + sS;
                    lrun[k] = ((lrun[k] * f) >> a.g.prob_frac) + sl;
                }
                ++u;
            }
        }
        __syncthreads();                  // the stage is reused by the next GBLK tiles
    }
    if (direct) {
        // the item's recurrence from zero: its proof is the walk's Y
        bool bad = *reinterpret_cast<volatile int32_t *>(&a.items[item].fail) != 0;
#pragma unroll
        for (int k = 0; k < NP; ++k) bad |= threadIdx.x + k * CHUNK_THREADS < H * D && Y[k] > INT32_MAX;
        finalize_item<H>(a, item, a.T[item / a.g.n_kv], (int64_t)item * H * D, loc, lrun, bad, slots);
        return;
    }
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        const int pr = threadIdx.x + k * CHUNK_THREADS;
        if (pr >= H * D) continue;
        const int h = pr / D, ch = pr % D;
        const int eb = base_sm[h];
        if (!opened[k]) {
            Spre[k] = curS[k];
            lpre[k] = curl[k];
        } else if (eb >= 0) {
            a.segs[eb + ne[k] - 1].S[ch] = curS[k];
            if (ch == 0) a.segs[eb + ne[k] - 1].l = curl[k];
        }
        BlockRec &br = a.blks[(int64_t)item * a.max_blocks + blk];
        br.Spre[h][ch] = Spre[k];
        br.Y[h][ch] = Y[k];
        if (ch == 0) {
            br.lpre[h] = lpre[k];
            br.nent[h] = eb >= 0 ? ne[k] : 0;
            br.ent_base[h] = eb >= 0 ? eb : 0;
        }
    }
}

// Level 2: fold the item's blocks; finalize or mark the item for the exact
// sequential recomputation. The blocks go 32 at a time: their scalars (one
// warp per head, one block per lane) and rescale entries into shared memory,
// each thread's Y and Spre in batches of FB loads issued together.
template <int H>
__device__ void merge_item(const ChunkArgs &a, int item, int nblocks, int64_t T,
                           int64_t qbase, long long *slots /* [NT/32] */, uint8_t *dyn) {
    constexpr int NP = (H * D + CHUNK_THREADS - 1) / CHUNK_THREADS;   // pairs per thread
    const int tid = threadIdx.x;
    const BlockRec *blks = a.blks + (int64_t)item * a.max_blocks;
    long long *eS = reinterpret_cast<long long *>(dyn + FoldCfg<H>::OFF_ES);
    __shared__ long long lp_s[H][32];
    __shared__ int ne_s[H][32], eb_s[H][32];
    __shared__ EntStage<H, 32> st;
    int64_t acc[NP], l[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) acc[k] = l[k] = 0;
    bool bad = *reinterpret_cast<volatile int32_t *>(&a.items[item].fail) != 0;
    bad = __syncthreads_or(bad);
    for (int g0 = 0; g0 < nblocks; g0 += 32) {
        if (bad) break;                    // the same for every thread
        const int nb = min(32, nblocks - g0);
        {
            const int w = tid >> 5, lane = tid & 31;
            if (w < H) {
                const int b = g0 + lane;
                long long lp = 0;
                int ne = 0, eb = 0;
                if (lane < nb) {
                    lp = ldcg(&blks[b].lpre[w]);
                    ne = ldcg(&blks[b].nent[w]);
                    eb = ldcg(&blks[b].ent_base[w]);
                }
                lp_s[w][lane] = lp;
                ne_s[w][lane] = ne;
                eb_s[w][lane] = eb;
            }
        }
        __syncthreads();
        stage_entries<H, 32>(a, ne_s, eb_s, nb, st, eS);
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            const int pr = tid + k * CHUNK_THREADS;
            if (pr >= H * D) continue;
            const int h = pr / D, ch = pr % D;
            for (int u0 = 0; u0 < nb; u0 += FB) {
                int64_t Yv[FB], Sv[FB];
#pragma unroll
                for (int u = 0; u < FB; ++u) {
                    if (u0 + u < nb) {
                        const BlockRec &br = blks[g0 + u0 + u];
                        Yv[u] = ldcg(&br.Y[h][ch]);
                        Sv[u] = ldcg(&br.Spre[h][ch]);
                    }
                }
#pragma unroll
                for (int u = 0; u < FB; ++u) {
                    if (u0 + u >= nb) break;
                    const int r = u0 + u;
                    const int64_t aa = acc[k] < 0 ? -acc[k] : acc[k];
                    if (aa + Yv[u] > INT32_MAX) bad = true;
                    acc[k] += Sv[u];
                    l[k] += lp_s[h][r];
                    const int ne = ne_s[h][r];
                    for (int j = 0; j < ne; ++j) {
                        int64_t f, sS, sl;
                        entry_at<H, 32>(a, st, eS, eb_s, h, r, j, ch, f, sS, sl);
                        acc[k] = ((acc[k] * f) >> a.g.prob_frac) + sS;
                        l[k] = ((l[k] * f) >> a.g.prob_frac) + sl;
                    }
                }
            }
        }
        // the stage is reused by the next 32 blocks; a failed proof ends the fold
        bad = __syncthreads_or(bad);
    }
    finalize_item<H>(a, item, T, qbase, acc, l, bad, slots);
}

// A context shard's item: fold its blocks into the item's PartRec instead of
// finalizing. The same translation-and-rescale fold as merge_block, over the
// item's blocks; Y composes as max(Y, |partial at block start| + Y_block).
template <int H>
__device__ void fold_part(const ChunkArgs &a, int item, int nblocks, int64_t T, long long *slots) {
    PartRec &pr = a.parts[item];
    const BlockRec *blks = a.blks + (int64_t)item * a.max_blocks;
    bool over = false;
    for (int pi = threadIdx.x; pi < H * D; pi += blockDim.x) {
        const int h = pi / D, ch = pi % D;
        int64_t loc = 0, Y = 0, curS = 0, curl = 0, Spre = 0, lpre = 0;
        int ne = 0;
        bool opened = false;
        // the block records in batches of 8, their loads issued together
        for (int b0 = 0; b0 < nblocks; b0 += FB) {
            int64_t Yv[FB], Sv[FB], lv[FB];
            int nev[FB], ebv[FB];
#pragma unroll
            for (int u = 0; u < FB; ++u) {
                if (b0 + u < nblocks) {
                    const BlockRec &br = blks[b0 + u];
                    Yv[u] = ldcg(&br.Y[h][ch]);
                    Sv[u] = ldcg(&br.Spre[h][ch]);
                    lv[u] = ldcg(&br.lpre[h]);
                    nev[u] = ldcg(&br.nent[h]);
                    ebv[u] = ldcg(&br.ent_base[h]);
                }
            }
#pragma unroll
            for (int u = 0; u < FB; ++u) {
                if (b0 + u >= nblocks) break;
                const int64_t al = loc < 0 ? -loc : loc;
                Y = max(Y, al + Yv[u]);
                loc += Sv[u];
                curS += Sv[u];
                curl += lv[u];
                // the entries four at a time (loads together, then in order);
                // the composite written below is separate memory
                for (int e0 = 0; e0 < nev[u]; e0 += 4) {
                  int64_t fv[4], sv[4], lw[4];
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                      if (e0 + j < nev[u]) {
                          const SegEntry &se = a.segs[ebv[u] + e0 + j];
                          fv[j] = ldcg(&se.f);
                          sv[j] = ldcg(&se.S[ch]);
                          lw[j] = ldcg(&se.l);
                      }
                  }
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    if (e0 + j >= nev[u]) break;
                    const int64_t f = fv[j];
                    if (!opened) {
                        Spre = curS;
                        lpre = curl;
                        opened = true;
                    } else if (ne - 1 < PART_MAXE) {
                        over |= curS < INT32_MIN || curS > INT32_MAX;
                        pr.ent[h][ne - 1].S[ch] = (int32_t)curS;
                        if (ch == 0) pr.ent[h][ne - 1].l = curl;
                    }
                    if (ne < PART_MAXE && ch == 0) pr.ent[h][ne].f = (int32_t)f;
                    ++ne;
                    curS = sv[j];
                    curl = lw[j];
                    loc = ((loc * f) >> a.g.prob_frac) + curS;
                  }
                }
            }
        }
        if (!opened) {
            Spre = curS;
            lpre = curl;
        } else if (ne - 1 < PART_MAXE) {
            over |= curS < INT32_MIN || curS > INT32_MAX;
            pr.ent[h][ne - 1].S[ch] = (int32_t)curS;
            if (ch == 0) pr.ent[h][ne - 1].l = curl;
        }
        over |= ne > PART_MAXE;
        pr.Spre[h][ch] = Spre;
        pr.Y[h][ch] = Y;
        if (ch == 0) {
            pr.lpre[h] = lpre;
            pr.nent[h] = ne < PART_MAXE ? ne : PART_MAXE;
        }
    }
    const bool bad = __syncthreads_or(over) ||
                     *reinterpret_cast<volatile int32_t *>(&a.items[item].fail) != 0;
    (void)slots;
    if (threadIdx.x == 0) {
        const volatile ItemAcc &ia = a.items[item];
        pr.fail = bad ? 1 : 0;
        pr.n_tokens = T;
        pr.resc = (int64_t)ia.resc;
        pr.sovf = (int64_t)ia.sovf;
        pr.maxs = ia.maxs;
        a.redo[item] = 0;            // a shard's item is not re-run here
    }
}

// Fold block c / GBLK of `item`; the CTA that completes the item's last block
// also folds the item and finalizes it (or writes a context shard's
// composite). A counter per item that resets itself on the last arrival
// (atomicInc) decides who is last; the last item of the launch empties the
// segment pool. Called by every thread of the CTA.
template <int H>
__device__ __forceinline__ void fold_block_and_item(const ChunkArgs &a, int item, int c, uint8_t *dyn) {
    __shared__ int flag_sm;
    __shared__ int base_sm[H];
    __shared__ long long slots[CHUNK_THREADS / 32];
    const int tid = threadIdx.x;
    const int nc = item_chunks(a, item);
    const int blk = c / GBLK, nblk = (nc + GBLK - 1) / GBLK;
    // a short item (not a context shard) is folded and finalized by the CTA of
    // its first block, in one pass over its tiles
    const bool direct = nc <= DIRECT_TILES && !a.parts;
    if (direct && blk > 0) return;
    __threadfence();
    merge_block<H>(a, item, blk, nc, base_sm, dyn, direct, slots);
    if (!direct) {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const unsigned old = atomicInc(&a.item_done[item], (unsigned)(nblk - 1));
            flag_sm = old == (unsigned)(nblk - 1);
        }
        __syncthreads();
        if (!flag_sm) return;
        __threadfence();
        const int64_t T = a.T[item / a.g.n_kv];
        if (a.parts) fold_part<H>(a, item, nblk, T, slots);
        else merge_item<H>(a, item, nblk, T, (int64_t)item * H * D, slots, dyn);
    }
    __syncthreads();
    if (tid == 0) {
        ItemAcc &ia = a.items[item];
        ia.done_blocks = 0;
        ia.resc = 0;
        ia.sovf = 0;
        ia.maxs = 0;
        ia.fail = 0;
        __threadfence();
        // the last item of the launch empties the segment pool
        if (atomicInc(a.scan_done, (unsigned)(a.n_items - 1)) == (unsigned)(a.n_items - 1)) *a.seg_top = 0;
    }
}

// Max over a warp of values in [-2^47, 2^47) or LLONG_MIN, as two 32-bit
// reductions of the offset from -2^47 - 1.
__device__ __forceinline__ long long warp_max_score(long long v) {
    const long long base = -(1ll << 47) - 1;
    const long long u = v < base ? 0 : v - base;            // < 2^48
    const int hi = (int)(u >> 20);
    const int mhi = __reduce_max_sync(FULL, hi);
    const unsigned mlo = __reduce_max_sync(FULL, hi == mhi ? (unsigned)(u & 0xFFFFF) : 0u);
    const long long m = ((long long)mhi << 20) | (long long)mlo;
    return m == 0 ? LLONG_MIN : m + base;
}

// The running maximum entering tile c of an item, for one warp: the maximum
// of the maxima of the item's tiles 0 .. c-1 (which the score launch wrote)
// and of the seed (the maximum entering a context shard, or the lowest
// score). Lane h returns head h's. The state lives in shared memory (the
// values loop has no registers to spare): a warp that walks an item's tiles
// in increasing order only reads the maxima since the tile it resolved last.
template <int H>
struct RunMax {
    long long m[H];
    int item, c;
};

template <int H>
__device__ __forceinline__ void run_max_init(RunMax<H> &r, int lane) {
    if (lane == 0) {
        r.item = -1;
        r.c = 0;
    }
    __syncwarp();
}

template <int H>
__device__ __forceinline__ long long run_max_at(RunMax<H> &r, const ChunkArgs &a, int nitem, int nc, int lane) {
    int lo = 0;
    long long m;
    if (nitem == r.item && nc >= r.c) {
        lo = r.c;
        m = lane < H ? r.m[lane] : LLONG_MIN;
    } else {
        m = DefFmt::S_LO;
        if (a.m_init && lane < H) {
            const long long sd = a.m_init[(int64_t)nitem * H + lane];
            m = sd > m ? sd : m;
        }
    }
    const long long *v = a.cmx + (int64_t)nitem * a.max_chunks * 2 * HMAX;
    // 64 tiles a step, every load of a step issued before any is used
    for (int j0 = lo; j0 < nc; j0 += 64) {
        const int ja = j0 + lane, jb = ja + 32;
        long long x[2][H];
#pragma unroll
        for (int h = 0; h < H; ++h) {
            x[0][h] = ja < nc ? ldcg(v + (int64_t)ja * 2 * HMAX + h) : LLONG_MIN;
            x[1][h] = jb < nc ? ldcg(v + (int64_t)jb * 2 * HMAX + h) : LLONG_MIN;
        }
#pragma unroll
        for (int h = 0; h < H; ++h) {
            const long long mh = warp_max_score(x[0][h] > x[1][h] ? x[0][h] : x[1][h]);
            if (lane == h && mh > m) m = mh;
        }
    }
    __syncwarp();
    if (lane < H) r.m[lane] = m;
    if (lane == 0) {
        r.item = nitem;
        r.c = nc;
    }
    __syncwarp();
    return m;
}

// The context-split merge: one CTA per item folds the shards' composites in
// causal order (the first shard holds the first tokens) and finalizes. The
// fold is the recurrence over the whole sequence provided the 32-bit clamp
// never fires; each shard proves that with |acc at its start| + Y <= 2^31 - 1.
// A shard without an exact composite (more than PART_MAXE rescales of one
// head, or a flagged item), or a failed proof, latches ST_SPLIT and leaves the
// item's outputs unwritten.
template <int H>
__global__ void __launch_bounds__(CHUNK_THREADS) k_merge_parts(Geo g, const PartRec *parts, int n_items,
                                                               int n_parts, int64_t *out, ins_stats *stats,
                                                               int32_t *status) {
    constexpr int NP = (H * D + CHUNK_THREADS - 1) / CHUNK_THREADS;
    __shared__ long long slots[CHUNK_THREADS / 32];
    const int item = blockIdx.x, tid = threadIdx.x;
    int64_t acc[NP], l[NP];
    bool bad = false;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        acc[k] = 0;
        l[k] = 0;
        const int pi = tid + k * CHUNK_THREADS;
        if (pi >= H * D) continue;
        const int h = pi / D, ch = pi % D;
        for (int r = 0; r < n_parts; ++r) {
            const PartRec &pr = parts[(int64_t)r * n_items + item];
            bad |= pr.fail != 0;
            const int64_t aa = acc[k] < 0 ? -acc[k] : acc[k];
            if (aa + pr.Y[h][ch] > INT32_MAX) bad = true;
            acc[k] += pr.Spre[h][ch];
            l[k] += pr.lpre[h];
            const int ne = pr.nent[h];
            for (int e = 0; e < ne; ++e) {
                const int64_t f = pr.ent[h][e].f;
                acc[k] = ((acc[k] * f) >> g.prob_frac) + pr.ent[h][e].S[ch];
                l[k] = ((l[k] * f) >> g.prob_frac) + pr.ent[h][e].l;
            }
        }
    }
    bad = __syncthreads_or(bad);
    if (bad) {
        if (tid == 0) atomicOr(status, ST_SPLIT);
        return;
    }
    int64_t *out_row = out + (int64_t)item * H * D;
    long long mx = 0;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        const int pi = tid + k * CHUNK_THREADS;
        if (pi >= H * D) continue;
        out_row[pi] = finalize_out(g, acc[k], l[k]);
        const long long ab = acc[k] < 0 ? -acc[k] : acc[k];
        mx = ab > mx ? ab : mx;
    }
    mx = cta_max_nonneg(mx, slots);
    if (tid == 0 && stats) {
        ins_stats st{};
        for (int r = 0; r < n_parts; ++r) {
            const PartRec &pr = parts[(int64_t)r * n_items + item];
            st.n_tokens += pr.n_tokens;
            st.rescale_events += pr.resc;
            st.score_overflows += pr.sovf;
            st.max_abs_score = pr.maxs > st.max_abs_score ? pr.maxs : st.max_abs_score;
        }
        st.acc_overflows = 0;
        st.max_abs_acc = mx;
        stats[item] = st;
    }
}

// ---------------------------------------------------------------------------
// Bulk copies into shared memory (the TMA engine, no tensor map: plain 1-D
// ranges, 16-byte aligned, sizes a multiple of 16) completing on an mbarrier.
// No multicast: every copy lands in the issuing CTA's own shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Waits for phase `parity` of the barrier to complete; gives up (false) after
// a bounded number of polls, each of which the hardware may suspend briefly.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int limit = 1 << 22) {
    const uint32_t addr = smem_addr(bar);
    for (int it = 0; it < limit; ++it) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetches into L2 the rows of the tile `td` whose page ids are `pages`: the
// K plane and norms (`which` & 1), the V plane and norms (`which` & 2), one
// lane per page. Every range starts 16-byte aligned inside its plane and is
// rounded up to 16 bytes without leaving the plane.
__device__ __forceinline__ void prefetch_rows(const ChunkArgs &a, int4 td, const int32_t *pages,
                                              int lane, int which) {
    const Geo &g = a.g;
    const int n = td.w, kvh = td.x % g.n_kv;
    if (n <= 0) return;
    const int poff = (int)(td.z % g.P);
    const int npages = (poff + n + g.P - 1) / g.P;
    auto up16 = [](int x) { return (uint32_t)((x + 15) & ~15); };
    for (int i = lane; i < npages; i += 32) {
        const uint8_t *reg = a.pool + region_off(g, pages[i], kvh);
        const int r0 = i == 0 ? poff : 0;
        const int r1 = min(g.P, poff + n - i * g.P);
        const int rows = r1 - r0;
        if (which & 1) prefetch_l2(reg + (int64_t)r0 * g.kbytes, up16(rows * g.kbytes));
        if (which & 2) prefetch_l2(reg + vplane_off(g) + (int64_t)r0 * g.vbytes, up16(rows * g.vbytes));
        prefetch_l2(reg + nplane_off(g) + (int64_t)r0 * 4, up16(rows * 4));
    }
}


// ---------------------------------------------------------------------------
// Tiles looked up two ahead of their use, for a CTA that walks its tiles
// blockIdx.x + j * gridDim.x: load() (one warp) starts the loads of local
// tile j's descriptor, row base and page ids; store(), a tile of work later,
// writes what they returned to shared memory (descriptor ring of 3, page ring
// of 2), so that no tile starts with a dependent chain of global loads. The
// item of the last lookup is kept: consecutive tiles of a CTA usually share
// it, and then only the page ids are loaded.
template <int PGMAX>
struct TileAhead {
    static constexpr int PPL = (PGMAX + 31) / 32;           // page ids per lane
    int4 *tdesc;                                             // [3]
    long long *trb;                                          // [3]
    int32_t (*pages)[PGMAX];                                 // [2][PGMAX]
    int4 run0;
    int citem = -1, cseq = 0;
    int64_t cT = 0, crb = 0;
    int4 rtd = make_int4(0, 0, 0, 0);
    long long rrb = 0;
    int32_t rpg[PPL];

    __device__ TileAhead(const ChunkArgs &a, int4 *td, long long *rb, int32_t (*pg)[PGMAX])
        : tdesc(td), trb(rb), pages(pg), run0(a.runs[0]) {}

    __device__ __forceinline__ void load(const ChunkArgs &a, int j, int lane) {
        const Geo &g = a.g;
        const int tile = (int)blockIdx.x + j * (int)gridDim.x;
        int item, c;
        if (a.n_runs == 1) {
            item = (tile - run0.y) % run0.z;
            c = run0.x + (tile - run0.y) / run0.z;
        } else {
            const int4 t = tile_at(a, tile);
            item = t.x;
            c = t.y;
        }
        if (item != citem) {
            citem = item;
            cT = a.T[item / g.n_kv];
            cseq = a.seq_ids[item / g.n_kv];
            crb = a.row_base[item];
        }
        const int64_t tt0 = (int64_t)c * a.tile_rows;
        const int64_t tn = cT - tt0 < a.tile_rows ? cT - tt0 : a.tile_rows;
        rtd = make_int4(item, c, (int)tt0, (int)(tn > 0 ? tn : 0));
        rrb = crb;
        const int poff = (int)(rtd.z % g.P);
        const int npg = rtd.w ? (poff + rtd.w + g.P - 1) / g.P : 0;
        const int32_t *pt = a.page_table + (int64_t)cseq * g.max_pages + rtd.z / g.P;
#pragma unroll
        for (int k = 0; k < PPL; ++k) {
            const int i = lane + 32 * k;
            rpg[k] = i < npg ? __ldg(pt + i) : 0;
        }
    }
    __device__ __forceinline__ void store(int j, int lane) {
#pragma unroll
        for (int k = 0; k < PPL; ++k) {
            const int i = lane + 32 * k;
            if (i < PGMAX) pages[j & 1][i] = rpg[k];
        }
        if (lane == 0) {
            tdesc[j % 3] = rtd;
            trb[j % 3] = rrb;
        }
    }
};

// Launch 1: the scores of every tile
// ---------------------------------------------------------------------------
// CompressedAttention.scores (ops/attention.py:333-359) for R rows per thread:
// the dot product of q with the rows' key centroids in FP64 (exact: integer
// operands and every partial sum below 2^53), times the key norm, floored by
// score_shift and clamped to score_width. Thread tid owns rows tid + r*NT, so
// each warp holds one 32-row block for every r. A score is stored as its offset
// below the block maximum (uint32; a larger gap flags the item for the exact
// body), the block maxima and the tile maximum as int64.
template <int H, int KB, int VB, int RS = 0>
__global__ void __launch_bounds__(CHUNK_THREADS, 2) k_scan_scores(ChunkArgs a) {
    using CF = ChunkCfg<H, KB, VB, RS>;
    constexpr int NT = CF::NT, R = CF::R, CW = CF::CW;
    // The key centroids of a channel pair, (c[k0], c[k1]) for index k0 + k1 << KB,
    // as exact doubles, in 8 replicas: lane l reads replica l & 7, so the 8
    // lanes of a 16-byte shared-memory wavefront never meet in a bank.
    extern __shared__ __align__(16) uint8_t dynA[];
    using SC = ScoreCfg<H, KB, VB, RS>;
    __shared__ __align__(16) double qd[D * H];  // [channel][head]
    double2 *ctab = reinterpret_cast<double2 *>(dynA);
    // The staging of the tiles: descriptors and page ids two tiles ahead (in
    // rings of 3 and 2), the rows one tile ahead (buffers j & 1).
    __shared__ int4 tdesc_sm[3];
    __shared__ long long trb_sm[3];
    __shared__ int32_t pages_sm[2][SC::PGMAX];
    __shared__ __align__(8) uint64_t full_bar[2];
    __shared__ long long tmax_sm[2][H];                // tile maxima of tiles j & 1

    const Geo &g = a.g;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the tile plan and the queries come from the launches before this one
    wait_prior_grid();
    for (int i = tid; i < (1 << (2 * KB)) * 8; i += NT) {
        const int e = i >> 3;
        ctab[i] = make_double2(a.tb->k_cent_f64[e & ((1 << KB) - 1)], a.tb->k_cent_f64[e >> KB]);
    }
    const double2 *myc = ctab + (lane & 7);
    constexpr int64_t s_lo = DefFmt::S_LO;
    const int G = gridDim.x;
    const int ntl = (a.n_tiles - (int)blockIdx.x + G - 1) / G;   // this CTA's tiles: blockIdx.x + j*G
    auto up16 = [](int x) { return (uint32_t)((x + 15) & ~15); };

    // Warp 1 looks tiles up two ahead; storing tile j's lookup also announces
    // the bytes of its copies on its buffer's barrier (the barrier's previous
    // phase, tile j - 2, has completed by then).
    TileAhead<SC::PGMAX> ahead(a, tdesc_sm, trb_sm, pages_sm);
    auto copy_bytes = [&](int4 td) {
        const int n = td.w, poff = (int)(td.z % g.P);
        const int npg = n ? (poff + n + g.P - 1) / g.P : 0;
        uint32_t bytes = 0;
        for (int i = 0; i < npg; ++i) {
            const int r0 = i == 0 ? poff : 0, r1 = min(g.P, poff + n - i * g.P);
            bytes += up16((r1 - r0) * KB * 8) + up16((r1 - r0) * 4);
        }
        return bytes;
    };
    auto resolve_load = [&](int j) { ahead.load(a, j, lane); };
    auto resolve_store = [&](int j) {
        ahead.store(j, lane);
        if (lane == 0) mbar_arrive_tx(&full_bar[j & 1], copy_bytes(ahead.rtd));
    };
    // The bulk copies of local tile j's K rows and norm words into buffer
    // j & 1: lane 0 of warp w issues those of pages w, w + 8, ... (the issue
    // of a bulk copy takes a while; the warps issue theirs side by side).
    // Page boundaries fall on multiples of 16 rows of a tile (tiles start at
    // multiples of C, pages hold a multiple of 16 rows), so every range starts
    // 16-byte aligned; a range rounded up to 16 bytes stays inside its plane
    // and its buffer.
    auto issue = [&](int j) {
        if (lane != 0) return;
        const int4 td = tdesc_sm[j % 3];
        const int n = td.w, kvh = td.x % g.n_kv;
        const int poff = (int)(td.z % g.P);
        const int npg = n ? (poff + n + g.P - 1) / g.P : 0;
        uint8_t *bk = dynA + SC::CTAB + (size_t)(j & 1) * SC::BUF;
        uint8_t *bn = bk + SC::KPL;
        for (int i = warp; i < npg; i += NT / 32) {
            const int r0 = i == 0 ? poff : 0, r1 = min(g.P, poff + n - i * g.P);
            const int row = i * g.P - poff + r0;              // the page's first row in the tile
            const uint8_t *reg = a.pool + region_off(g, pages_sm[j & 1][i], kvh);
            bulk_g2s(bk + (size_t)row * (KB * 8), reg + (int64_t)r0 * (KB * 8), up16((r1 - r0) * KB * 8),
                     &full_bar[j & 1]);
            bulk_g2s(bn + (size_t)row * 4, reg + nplane_off(g) + (int64_t)r0 * 4, up16((r1 - r0) * 4),
                     &full_bar[j & 1]);
        }
    };

    if (tid == 0) {
        mbar_init(&full_bar[0], 1);
        mbar_init(&full_bar[1], 1);
        mbar_fence_init();
        // the segment pool of the values launch starts empty (the folds of the
        // scan before this one empty it too; this keeps a scan that never
        // reached its folds from leaking into the next)
        if (blockIdx.x == 0) *a.seg_top = 0;
    }
    if (tid < 2 * H) tmax_sm[tid / H][tid % H] = LLONG_MIN;
    __syncthreads();
    if (warp == 1) {
        resolve_load(0);
        resolve_store(0);
        if (ntl > 1) {
            resolve_load(1);
            resolve_store(1);
        }
    }
    __syncthreads();
    if (ntl > 0) issue(0);
    int prev_item = -1;
    int4 prev_td = make_int4(0, 0, 0, 0);
    unsigned lost = 0;                           // buffers whose wait gave up
    // the maximum of tile j's scores per head, once the barrier ending tile j
    // has passed; the slot is cleared for tile j + 2
    auto tile_max_out = [&](int j, int4 td) {
        if (tid < H) {
            a.cmx[((int64_t)td.x * a.max_chunks + td.y) * 2 * HMAX + tid] = tmax_sm[j & 1][tid];
            tmax_sm[j & 1][tid] = LLONG_MIN;
        }
    };

    for (int li = 0; li < ntl; ++li) {
        const int tile = (int)blockIdx.x + li * G;
        // the value launch may take SM slots from here on (it waits for this
        // launch to finish before it reads the scores)
        if (li == ntl - 1) release_dependents();
        if (li > 0) tile_max_out(li - 1, prev_td);
        // buffer (li + 1) & 1 was released by the barrier that ended tile li - 1
        if (li + 1 < ntl) issue(li + 1);
        if (warp == 1 && li + 2 < ntl) resolve_load(li + 2);
        const int4 td = tdesc_sm[li % 3];
        const int item = td.x;
        const int64_t t0 = td.z;
        const int n = td.w;
        const int b = item / g.n_kv, kvh = item % g.n_kv;
        const int64_t qbase = ((int64_t)b * g.n_kv * H + (int64_t)kvh * H) * D;
        uint32_t *sc = a.sc + (trb_sm[li % 3] + t0) * H;

        if (item != prev_item) {                 // the same for the whole CTA
            prev_item = item;
            for (int i = tid; i < H * D; i += NT) qd[(i % D) * H + i / D] = (double)a.q_rot[qbase + i];
            __syncthreads();
            bool big = false;
            const double qlim = (double)g.q_lim;
            for (int i = tid; i < H * D; i += NT) {
                const double x = qd[i];
                big |= (x >= qlim || x <= -qlim);
            }
            // |q| >= q_lim could let an FP64 partial sum pass 2^53: the item
            // goes to the exact int64 body
            if (__syncthreads_or(big) && tid == 0) atomicExch(&a.items[item].fail, 1);
        }
        // this tile's rows, staged by the bulk copies; a wait that gives up
        // reports a timeout (the launch's results are then void) and is
        // retried, bounded, before the CTA exits
        if (!mbar_wait(&full_bar[li & 1], (uint32_t)(li >> 1) & 1u)) {
            lost |= 1u << (li & 1);
            atomicOr(a.status, ST_TIMEOUT);
        }
        prev_td = td;
        const uint8_t *bk = dynA + SC::CTAB + (size_t)(li & 1) * SC::BUF;
        const uint8_t *bn = bk + SC::KPL;
        uint32_t kw[R][KB * 2];
        int64_t knorm[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = r * NT + tid;
            const bool valid = row < n;          // a tile may be empty (a sequence of length 0)
            const uint8_t *kp = bk + (size_t)row * (KB * 8);
            if constexpr (KB == 4) {
                const uint4 x = *reinterpret_cast<const uint4 *>(kp);
                const uint4 y = *reinterpret_cast<const uint4 *>(kp + 16);
                kw[r][0] = x.x; kw[r][1] = x.y; kw[r][2] = x.z; kw[r][3] = x.w;
                kw[r][4] = y.x; kw[r][5] = y.y; kw[r][6] = y.z; kw[r][7] = y.w;
            } else {
#pragma unroll
                for (int i = 0; i < KB; ++i) {
                    const uint2 x = *reinterpret_cast<const uint2 *>(kp + 8 * i);
                    kw[r][2 * i] = x.x;
                    kw[r][2 * i + 1] = x.y;
                }
            }
#pragma unroll
            for (int i = 0; i < KB * 2; ++i) kw[r][i] = valid ? kw[r][i] : 0u;
            const uint32_t nw = *reinterpret_cast<const uint32_t *>(bn + (size_t)row * 4);
            knorm[r] = valid ? (int64_t)(int16_t)(nw & 0xffffu) : 0;
        }

        double acc[R][H];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int h = 0; h < H; ++h) acc[r][h] = 0.0;
#pragma unroll
        for (int p = 0; p < D / 2; ++p) {
            double c0[R], c1[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const double2 cc = myc[kpair<KB>(kw[r], p) * 8];
                c0[r] = cc.x;
                c1[r] = cc.y;
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = 2 * p + e;
                double qv[H];
                if constexpr (H >= 2) {
#pragma unroll
                    for (int h = 0; h < H; h += 2) {
                        const double2 q2 = *reinterpret_cast<const double2 *>(&qd[j * H + h]);
                        qv[h] = q2.x;
                        qv[h + 1] = q2.y;
                    }
                } else {
                    qv[0] = qd[j];
                }
#pragma unroll
                for (int h = 0; h < H; ++h)
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r][h] = fma(qv[h], e ? c1[r] : c0[r], acc[r][h]);
            }
            // keeps the scheduler from hoisting every lookup of the row
            if ((p & 3) == 3) asm volatile("" ::: "memory");
        }
        // scores, then the block maxima of all (r, h) as independent warp
        // reductions, then the stores
        unsigned ovf = 0, gap = 0;
        long long mx = 0;
        int64_t sv[R][H];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const bool valid = r * NT + tid < n;
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const int64_t di = __double2ll_rn(acc[r][h]);
                const int64_t prod = (int64_t)((uint64_t)di * (uint64_t)knorm[r]);
                bool hit;   // saturate (qclamp, numerics/fixed.py:161-168)
                const int64_t s0 = prod >> DefFmt::SCORE_SHIFT;
                hit = s0 < DefFmt::S_LO || s0 > DefFmt::S_HI;
                const int64_t s = s0 < DefFmt::S_LO ? DefFmt::S_LO : (s0 > DefFmt::S_HI ? DefFmt::S_HI : s0);
                ovf += hit && valid;
                const long long ab = s < 0 ? -s : s;
                mx = valid && ab > mx ? ab : mx;
                sv[r][h] = valid ? s : s_lo;
            }
        }
        // block maximum in two 32-bit reductions: |s| <= 2^47, so
        // s = hi * 2^20 + lo with hi an int and 0 <= lo < 2^20
        int mhi[R][H];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int h = 0; h < H; ++h) mhi[r][h] = __reduce_max_sync(FULL, (int)(sv[r][h] >> 20));
        int64_t hmax[H];
#pragma unroll
        for (int h = 0; h < H; ++h) hmax[h] = LLONG_MIN;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = r * NT + tid;
            uint32_t off[H];
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const bool top = (int)(sv[r][h] >> 20) == mhi[r][h];
                const unsigned mlo = __reduce_max_sync(FULL, top ? (unsigned)(sv[r][h] & 0xFFFFF) : 0u);
                const int64_t bm = (int64_t)mhi[r][h] * (1ll << 20) + (int64_t)mlo;
                hmax[h] = bm > hmax[h] ? bm : hmax[h];
                if (lane == h) a.bmg[((int64_t)tile * H + h) * CW + (row >> 5)] = bm;
                const uint64_t d = (uint64_t)(bm - sv[r][h]);
                gap |= (unsigned)(row < n && d > 0xFFFFFFFFull);
                off[h] = (uint32_t)(d > 0xFFFFFFFFull ? 0xFFFFFFFFull : d);
            }
            if (row < n) {
                uint32_t *dst = sc + (int64_t)row * H;
                if constexpr (H == 8) {
                    reinterpret_cast<uint4 *>(dst)[0] = make_uint4(off[0], off[1], off[2], off[3]);
                    reinterpret_cast<uint4 *>(dst)[1] = make_uint4(off[4], off[5], off[6], off[7]);
                } else if constexpr (H == 4) {
                    *reinterpret_cast<uint4 *>(dst) = make_uint4(off[0], off[1], off[2], off[3]);
                } else if constexpr (H == 2) {
                    *reinterpret_cast<uint2 *>(dst) = make_uint2(off[0], off[1]);
                } else {
                    dst[0] = off[0];
                }
            }
        }
        // a score more than 2^32 below its block maximum: exact body
        if (__any_sync(FULL, gap) && lane == 0) atomicExch(&a.items[item].fail, 1);
        ovf = __reduce_add_sync(FULL, ovf);
        const int xhi = __reduce_max_sync(FULL, (int)(mx >> 20));
        const unsigned xlo = __reduce_max_sync(FULL, (int)(mx >> 20) == xhi ? (unsigned)(mx & 0xFFFFF) : 0u);
        if (lane == 0) {
            ItemAcc &ia = a.items[item];
            if (ovf) atomicAdd(&ia.sovf, (unsigned long long)ovf);
            const long long wm = (long long)xhi * (1ll << 20) + (long long)xlo;
            if (wm) atomicMax(&ia.maxs, wm);
#pragma unroll
            for (int h = 0; h < H; ++h) atomicMax(&tmax_sm[li & 1][h], (long long)hmax[h]);
        }
        if (warp == 1 && li + 2 < ntl) resolve_store(li + 2);
        __syncthreads();
    }
    if (ntl > 0) tile_max_out(ntl - 1, prev_td);
    // a copy whose wait gave up must land before the CTA's shared memory goes
    for (int bb = 0; bb < 2; ++bb)
        if ((lost >> bb) & 1u) {
            const int jl = ntl - 1 - ((ntl - 1 - bb) & 1);   // the last tile that used buffer bb
            if (jl >= 0) mbar_wait(&full_bar[bb], (uint32_t)(jl >> 1) & 1u);
        }
}

// ---------------------------------------------------------------------------
// A context shard's item maxima (the exchange between ranks): one warp per
// (item, head) maxes the tile maxima the score launch wrote.
// ---------------------------------------------------------------------------
template <int H>
__global__ void __launch_bounds__(256) k_item_maxima(ChunkArgs a) {
    const int lane = threadIdx.x & 31;
    const int wi = (int)blockIdx.x * 8 + (threadIdx.x >> 5);
    wait_prior_grid();
    if (wi >= a.n_items * H) return;
    const int item = wi / H, h = wi % H;
    const int nc = item_chunks(a, item);
    const long long *v = a.cmx + (int64_t)item * a.max_chunks * 2 * HMAX + h;
    long long m = LLONG_MIN;
    for (int c = lane; c < nc; c += 32) {
        const long long x = v[(int64_t)c * 2 * HMAX];
        m = x > m ? x : m;
    }
    m = warp_max_score(m);
    if (lane == 0) a.maxima[(int64_t)item * H + h] = m > DefFmt::S_LO ? m : DefFmt::S_LO;
}

// The p-pass of a tile (4a below): p = exp(m - s) and w = v_norm * p for
// every (token, head), w written over the score offset in place; the l of
// every segment into lsum (shared atomics) and each warp's sum of |w| per head
// (the clamp-proof bound) into bnd. Thread tid owns tokens tid + r*NT, so its
// warp holds block r*NT/32 + warp for each r. All distances are loaded before
// any w is stored (the stores reuse the slots the loads read), and the
// distance arithmetic is 32-bit: the block bases are kept clamped at
// delta_max + 1 (dbase32) and each offset is clamped the same way, which
// leaves every p unchanged (any distance past delta_max gives p = 0).
template <int H, int R, int NT, int C, int CW>
__device__ __forceinline__ void p_pass(const int32_t *exp_tab, uint32_t *d_sm, const uint32_t *dbase32,
                                       const int32_t *vn_sm, const uint32_t *grew, const int32_t *gpre,
                                       unsigned int (*lsum)[SEGMAX + 1], long long (*bnd)[H], int n) {
    constexpr uint32_t DCAP = (uint32_t)DefFmt::DELTA_MAX + 1u;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t dd[R][H];
    int32_t vnt[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int t = r * NT + tid;
        vnt[r] = t < n ? vn_sm[t] : 0;
#pragma unroll
        for (int h = 0; h < H; ++h) dd[r][h] = min(d_sm[h * C + t], DCAP) + dbase32[h * CW + (t >> 5)];
    }
    uint32_t pv[R][H];
    unsigned whi[H], wlo[H];
#pragma unroll
    for (int h = 0; h < H; ++h) whi[h] = wlo[h] = 0u;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int t = r * NT + tid;
        const bool valid = t < n;
#pragma unroll
        for (int h = 0; h < H; ++h) {
            const uint32_t p = valid ? exp_lut_def(exp_tab, (int64_t)dd[r][h]) : 0u;
            const int32_t w = vnt[r] * (int32_t)p;           // |w| <= 2^30
            if (valid) d_sm[h * C + t] = (uint32_t)w;
            const uint32_t aw = (uint32_t)(w < 0 ? -w : w);
            whi[h] += aw >> 16;
            wlo[h] += aw & 0xFFFFu;
            pv[r][h] = p;
        }
    }
    // l: when the warp's R blocks are quiet for a head and share one segment
    // (the common case), one warp sum and one atomic per head
#pragma unroll
    for (int h = 0; h < H; ++h) {
        const int sg0 = gpre[h * CW + warp];
        bool uni = true;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int blk = r * (NT / 32) + warp;
            uni &= grew[h * CW + blk] == 0u && gpre[h * CW + blk] == sg0;
        }
        if (uni) {
            unsigned ps = 0;
#pragma unroll
            for (int r = 0; r < R; ++r) ps += pv[r][h];
            const unsigned sum = __reduce_add_sync(FULL, ps);   // <= R * 32 * 2^15
            if (lane == 0 && sum && sg0 <= SEGMAX) atomicAdd(&lsum[h][sg0], sum);
        } else {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int blk = r * (NT / 32) + warp;
                const uint32_t gw = grew[h * CW + blk];
                const int sg = gpre[h * CW + blk] + __popc(gw & ((2u << lane) - 1u));
                if (pv[r][h] && sg <= SEGMAX) atomicAdd(&lsum[h][sg], pv[r][h]);
            }
        }
    }
    // sum of |w| per head over the warp, exact: the high and low 16-bit parts
    // summed apart (each well inside 32 bits) and recombined
#pragma unroll
    for (int h = 0; h < H; ++h) {
        const unsigned hs = __reduce_add_sync(FULL, whi[h]);
        const unsigned ls = __reduce_add_sync(FULL, wlo[h]);
        if (lane == 0) bnd[warp][h] = ((long long)hs << 16) + (long long)ls;
    }
}

// ---------------------------------------------------------------------------
// Launch 3: the values
// ---------------------------------------------------------------------------
template <int H, int KB, int VB, int RS = 0>
__global__ void __launch_bounds__(CHUNK_THREADS, 2) k_scan_values(ChunkArgs a) {
    using CF = ChunkCfg<H, KB, VB, RS>;
    constexpr int NT = CF::NT, R = CF::R, C = CF::C, CW = CF::CW, NC = CF::NC, VW = CF::VW;
    constexpr int TPE = CF::TPE, NE = CF::NE, HG = CF::HG, HL = CF::HL, SUBT = CF::SUBT;
    constexpr int UNITS = CF::UNITS, USTR = CF::USTR, HPS = CF::HPS, TPW = CF::TPW, TWS = CF::TWS,
                  VS = CF::VS;
    constexpr int UPW = 32 / H;                 // table units per warp in the build
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ int32_t vcent[16];
    __shared__ int32_t exp_tab[256];
    __shared__ long long min_sm[3][H];                 // m_in of the tiles in the descriptor ring
    __shared__ int fail_sm;
    __shared__ int nseg_sm[H], segbase_sm[H];
    __shared__ int32_t rl_f[H][SEGMAX];
    __shared__ unsigned int lsum_sm[H][SEGMAX + 1];   // l of a tile < 2^25
    __shared__ long long bnd_sm[NT / 32][H];           // per-warp clamp-proof bounds
    __shared__ unsigned int resc_sm;
    // tiles looked up two ahead (descriptor ring of 3, page ring of 2)
    constexpr int PGMAX = C / 16 + 1;
    __shared__ int4 tdesc_sm[3];
    __shared__ long long trb_sm[3];
    __shared__ int32_t pages_sm[2][PGMAX];
    __shared__ __align__(8) uint64_t vbar;             // the staged V rows of the next tile
    __shared__ int vlost_sm;                            // a wait on them gave up

    const Geo &g = a.g;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint8_t *vbuf = dyn + CF::OFF_VB;
    const uint8_t *nbuf = dyn + CF::OFF_NB;
    // a score's offset below its block maximum, later w = v_norm * p (as int32)
    uint32_t *d_sm = reinterpret_cast<uint32_t *>(dyn + CF::OFF_S);
    uint32_t *tw = reinterpret_cast<uint32_t *>(dyn + CF::OFF_TW);
    int32_t *vn_sm = reinterpret_cast<int32_t *>(dyn + CF::OFF_VN);
    int32_t *tabs = reinterpret_cast<int32_t *>(dyn + CF::OFF_TAB);
    uint32_t *vt = reinterpret_cast<uint32_t *>(dyn + CF::OFF_TAB);      // V staging, aliases the tables
    uint32_t *grew = reinterpret_cast<uint32_t *>(dyn + CF::OFF_GREW);   // [H][CW], then any [CW]
    uint32_t *anyg = grew + H * CW;
    int32_t *gpre = reinterpret_cast<int32_t *>(dyn + CF::OFF_PRE);     // [H][CW]
    long long *bmax = reinterpret_cast<long long *>(dyn + CF::OFF_BMAX);  // [H][CW]
    long long *bcar = reinterpret_cast<long long *>(dyn + CF::OFF_BCAR);  // [H][CW]
    uint32_t *dbase = reinterpret_cast<uint32_t *>(dyn + CF::OFF_DB);     // [H][CW]: carry - block max,
                                                                           // clamped at delta_max + 1
    int32_t *s0p = reinterpret_cast<int32_t *>(dyn + CF::OFF_S0);

    for (int i = tid; i < 256; i += NT) exp_tab[i] = a.tb->exp_tab[i];
    if (tid < 16) vcent[tid] = tid < NC ? (int32_t)a.tb->v_cent[tid] : 0;
    int64_t cmax_v = 0;                       // max |V centroid|
    for (int k = 0; k < NC; ++k) {
        const int64_t ab = a.tb->v_cent[k] < 0 ? -a.tb->v_cent[k] : a.tb->v_cent[k];
        cmax_v = ab > cmax_v ? ab : cmax_v;
    }

    // Tiles are dealt round-robin (this CTA's: blockIdx.x + li * gridDim.x); no
    // tile waits on another. Warp 1 looks them up two ahead; the last warp
    // resolves the running maximum entering each one tile ahead, during the
    // control phase (whose warps are one per head).
    constexpr int WRM = NT / 32 - 1;
    const int G = gridDim.x;
    const int ntl = (a.n_tiles - (int)blockIdx.x + G - 1) / G;
    TileAhead<PGMAX> ahead(a, tdesc_sm, trb_sm, pages_sm);
    __shared__ RunMax<H> runmax;
    if (warp == WRM) run_max_init(runmax, lane);
    if (warp == 1) {
        ahead.load(a, 0, lane);
        ahead.store(0, lane);
        if (ntl > 1) {
            ahead.load(a, 1, lane);
            ahead.store(1, lane);
        }
    }
    // everything above reads only what was written before the scores launch;
    // from here on, the outputs of the launches before this one
    // The V plane and norm words of local tile j come into shared memory by
    // bulk copies (cp.async.bulk, no tensor map, no multicast) issued by one
    // thread once the tile before has taken its rows out of the buffer, so
    // they land while that tile computes. Page boundaries fall on multiples
    // of 16 rows of a tile, so every range starts 16-byte aligned; a range
    // rounded up to 16 bytes stays inside its plane and the buffer.
    auto up16 = [](int x) { return (uint32_t)((x + 15) & ~15); };
    auto stage_rows = [&](int j) {
        const int4 t = tdesc_sm[j % 3];
        const int nn = t.w, kv = t.x % g.n_kv, po = (int)(t.z % g.P);
        const int npg = nn ? (po + nn + g.P - 1) / g.P : 0;
        uint32_t bytes = 0;
        for (int i = 0; i < npg; ++i) {
            const int r0 = i == 0 ? po : 0, r1 = min(g.P, po + nn - i * g.P);
            bytes += up16((r1 - r0) * VW * 4) + up16((r1 - r0) * 4);
        }
        if ((int64_t)t.x * a.max_chunks + t.y == a.hold_rec) bytes += 16;   // the wait test
        mbar_arrive_tx(&vbar, bytes);
        for (int i = 0; i < npg; ++i) {
            const int r0 = i == 0 ? po : 0, r1 = min(g.P, po + nn - i * g.P);
            const int row = i * g.P - po + r0;
            const uint8_t *reg = a.pool + region_off(g, pages_sm[j & 1][i], kv);
            bulk_g2s(dyn + CF::OFF_VB + (size_t)row * VW * 4, reg + vplane_off(g) + (int64_t)r0 * VW * 4,
                     up16((r1 - r0) * VW * 4), &vbar);
            bulk_g2s(dyn + CF::OFF_NB + (size_t)row * 4, reg + nplane_off(g) + (int64_t)r0 * 4, up16((r1 - r0) * 4),
                     &vbar);
        }
    };
    wait_prior_grid();
    if (tid == 0) {
        mbar_init(&vbar, 1);
        mbar_fence_init();
        vlost_sm = 0;
    }
    __syncthreads();
    if (tid == 0 && ntl > 0) stage_rows(0);
    if (warp == WRM && ntl > 0) {
        const int4 t = tdesc_sm[0];
        const long long m = run_max_at(runmax, a, t.x, t.y, lane);
        if (lane < H) min_sm[0][lane] = m;
    }
    int lost_at = -1;                             // the tile whose wait gave up
    for (int li = 0; li < ntl; ++li) {
        const int tile = (int)blockIdx.x + li * G;
        if (li == ntl - 1) release_dependents();      // the fold launch may take SM slots
        const int4 td = tdesc_sm[li % 3];
        const int item = td.x, c = td.y;
        const int64_t t0 = td.z;
        const int n = td.w;
        const int rec_idx = item * a.max_chunks + c;
        const uint32_t *sc = a.sc + (trb_sm[li % 3] + t0) * H;

        // ---- 0. the tile's score offsets (each thread its own rows), setup -------
        uint32_t off[R][H];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = r * NT + tid;
            if (row < n) {
                const uint32_t *src = sc + (int64_t)row * H;
                if constexpr (H == 8) {
                    const uint4 x = __ldg(reinterpret_cast<const uint4 *>(src));
                    const uint4 y = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
                    off[r][0] = x.x; off[r][1] = x.y; off[r][2] = x.z; off[r][3] = x.w;
                    off[r][4] = y.x; off[r][5] = y.y; off[r][6] = y.z; off[r][7] = y.w;
                } else if constexpr (H == 4) {
                    const uint4 x = __ldg(reinterpret_cast<const uint4 *>(src));
                    off[r][0] = x.x; off[r][1] = x.y; off[r][2] = x.z; off[r][3] = x.w;
                } else if constexpr (H == 2) {
                    const uint2 x = __ldg(reinterpret_cast<const uint2 *>(src));
                    off[r][0] = x.x; off[r][1] = x.y;
                } else {
                    off[r][0] = __ldg(src);
                }
            }
        }
        for (int i = tid; i < H * CW; i += NT) bmax[i] = a.bmg[(int64_t)tile * H * CW + i];
        if (tid < H)
            for (int k = 0; k <= SEGMAX; ++k) lsum_sm[tid][k] = 0;
        if (tid == 0) {
            resc_sm = 0;
            fail_sm = 0;
        }
        for (int i = tid; i < (H + 1) * CW; i += NT) grew[i] = 0;
        for (int i = tid; i < H * D; i += NT) s0p[i] = 0;
        __syncthreads();

        // ---- 1. V codes, v norms and scores to shared memory ---------------------
        // (the staged rows first: a wait that gives up reports a timeout, the
        // launch's results are then void, and no copy is issued after it)
        if (!vlost_sm && !mbar_wait(&vbar, (uint32_t)li & 1u, a.poll_limit)) {
            lost_at = li;
            if (tid == 0) atomicOr(a.status, ST_TIMEOUT);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = r * NT + tid;
            if (row < n) {
                const uint32_t *vr = reinterpret_cast<const uint32_t *>(vbuf + (size_t)row * VW * 4);
                uint32_t vw[VW];
                if constexpr (VB == 2) {
                    const uint4 x = *reinterpret_cast<const uint4 *>(vr);
                    vw[0] = x.x; vw[1] = x.y; vw[2] = x.z; vw[3] = x.w;
                } else {
#pragma unroll
                    for (int i = 0; i < VW / 2; ++i) {
                        const uint2 x = reinterpret_cast<const uint2 *>(vr)[i];
                        vw[2 * i] = x.x;
                        vw[2 * i + 1] = x.y;
                    }
                }
                const uint32_t nw = *reinterpret_cast<const uint32_t *>(nbuf + (size_t)row * 4);
                vn_sm[row] = (int32_t)(int16_t)(nw >> 16);
#pragma unroll
                for (int w = 0; w < VW; ++w) vt[w * VS + row + (row >> 4)] = vw[w];
#pragma unroll
                for (int h = 0; h < H; ++h) d_sm[h * C + row] = off[r][h];
            }
        }
        if (lost_at >= 0) vlost_sm = 1;
        __syncthreads();
        // the buffer is free: the next tile's rows
        if (tid == 0 && li + 1 < ntl && !vlost_sm) stage_rows(li + 1);

        // ---- 2. V codes to channel-major words; warp 1 looks up the tile after
        //         next and prefetches the next tile's score offsets into L2 -----
        if (warp == 1) {
            if (li + 2 < ntl) ahead.load(a, li + 2, lane);
            if (li + 1 < ntl) {
                const int4 t2 = tdesc_sm[(li + 1) % 3];
                const uint32_t bytes = (uint32_t)t2.w * H * 4;
                if (lane == 0 && bytes)
                    prefetch_l2(a.sc + (trb_sm[(li + 1) % 3] + t2.z) * H, (bytes + 15) & ~15u);
            }
        }
        // word (ch, k) holds, as nibbles, the table indices of units 8k .. 8k+7
        // of channel ch
        if constexpr (VB == 2) {
            for (int task = tid; task < (C / 16) * 4; task += NT) {
                const int v = task >> 5, l = task & 31;
                const int tg = (v >> 1) * 16 + (l & 15), w = 2 * (v & 1) + (l >> 4);
                uint32_t A[16];
                const uint32_t *src = vt + w * VS + 17 * tg;   // token 16tg+i sits at 17tg+i
#pragma unroll
                for (int i = 0; i < 16; ++i) A[i] = src[i];
                transpose16x2(A);
#pragma unroll
                for (int cc = 0; cc < 16; ++cc) tw[(16 * w + cc) * TWS + tg] = A[cc];
            }
        } else {
            // 3-bit codes: task (8-token group, 8-channel group); channel ch sits
            // at bits 3ch .. 3ch+2 of the row, one nibble per token in the word.
            for (int task = tid; task < (C / 8) * 8; task += NT) {
                const int tg = task % (C / 8), cg = task / (C / 8);
                const int bit = 24 * cg, wl = bit >> 5, sh = bit & 31;
                uint32_t out[8];
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) out[cc] = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int t = 8 * tg + i, ts = t + (t >> 4);
                    uint32_t x = vt[wl * VS + ts] >> sh;
                    if (sh > 8) x |= vt[(wl + 1) * VS + ts] << (32 - sh);
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) out[cc] |= ((x >> (3 * cc)) & 7u) << (4 * i);
                }
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) tw[(8 * cg + cc) * TWS + tg] = out[cc];
            }
        }
        __syncthreads();

        // ---- 3. the online control, one warp per head at a time ------------------
        // Lane b holds 32-row block b. A prefix-max over the block maxima gives the
        // running maximum entering every block. A block whose maximum does not
        // exceed it has no rescale point: every token's p is exp(carry - s).
        // The rare blocks that can rescale are scanned token by token here:
        // rescale points (ballot bits) and factors exp(s - m_old); each of their
        // tokens' scores is rewritten to carry - (m_t - s), so that the term
        // build finds p = exp(carry - s') for it as for every other token.
        for (int h = warp; h < H; h += NT / 32) {
            const int nb = (n + 31) / 32;
            const int64_t m_in = min_sm[li % 3][h];
            int64_t x = lane < nb ? bmax[h * CW + lane] : LLONG_MIN;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int64_t y = __shfl_up_sync(FULL, x, off);
                if (lane >= off) x = y > x ? y : x;
            }
            int64_t car = __shfl_up_sync(FULL, x, 1);
            if (lane == 0) car = LLONG_MIN;
            car = car > m_in ? car : m_in;
            const bool scanb = lane < nb && bmax[h * CW + lane] > car;
            if (lane < CW) {
                bcar[h * CW + lane] = car;
                // a token's distance below the running maximum is dbase + its offset
                const int64_t db = lane < nb ? car - bmax[h * CW + lane] : 0;
                dbase[h * CW + lane] = (uint32_t)(db < DefFmt::DELTA_MAX ? db : DefFmt::DELTA_MAX + 1);
                grew[h * CW + lane] = 0u;
            }
            __syncwarp();
            uint32_t todo = __ballot_sync(FULL, scanb);
            int nres = 0;                              // rescales found in this head
            int blkres = 0;                            // this lane's block's rescales
            while (todo) {
                const int bb = __ffs(todo) - 1;
                todo &= todo - 1;
                const int t = bb * 32 + lane;
                const bool valid = t < n;
                const int64_t bmx = bmax[h * CW + bb];
                const int64_t st = valid ? bmx - (int64_t)d_sm[h * C + t] : LLONG_MIN;
                const int64_t carry = __shfl_sync(FULL, car, bb);
                int64_t y = st;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int64_t z = __shfl_up_sync(FULL, y, off);
                    if (lane >= off) y = z > y ? z : y;
                }
                const int64_t yprev = __shfl_up_sync(FULL, y, 1);
                const int64_t Mprev = lane == 0 ? carry : (yprev > carry ? yprev : carry);
                const int64_t Mt = y > carry ? y : carry;
                const bool gr = valid && st > Mprev;
                const uint32_t mask = __ballot_sync(FULL, gr);
                if (lane == 0) grew[h * CW + bb] = mask;
                // this block's tokens carry their own distance m_t - s (dbase 0);
                // one at or past 2^32 is far beyond delta_max, so clamping it
                // leaves p = 0 exact
                if (lane == 0) dbase[h * CW + bb] = 0;
                if (valid) {
                    const int64_t dn = Mt - st;
                    d_sm[h * C + t] = (uint32_t)(dn > 0xFFFFFFFFll ? 0xFFFFFFFFll : dn);
                }
                // the factor of every rescale point of this block, in order
                const int k = nres + __popc(mask & ((1u << lane) - 1u));
                if (gr && k < SEGMAX) rl_f[h][k] = (int32_t)exp_lut_def(exp_tab, st - Mprev);
                if (lane == bb) blkres = __popc(mask);
                nres += __popc(mask);
            }
            // rescales before each block
            int pre = blkres;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int z = __shfl_up_sync(FULL, pre, off);
                if (lane >= off) pre += z;
            }
            pre -= blkres;
            if (lane < CW) gpre[h * CW + lane] = pre;
            if (lane == 0) {
                nseg_sm[h] = nres;
                atomicAdd(&resc_sm, (unsigned)nres);
            }
        }
        // the running maximum entering the next tile (its descriptor is in
        // the ring; slot (li + 1) % 3 last served tile li - 2)
        if (warp == WRM && li + 1 < ntl) {
            const int4 t = tdesc_sm[(li + 1) % 3];
            const long long m = run_max_at(runmax, a, t.x, t.y, lane);
            if (lane < H) min_sm[(li + 1) % 3][lane] = m;
        }
        __syncthreads();
        for (int i = tid; i < CW; i += NT) {
            uint32_t m = 0;
#pragma unroll
            for (int h = 0; h < H; ++h) m |= grew[h * CW + i];
            anyg[i] = m;
        }
        // segment slots in the pool, zeroed for the atomic partial sums
        if (tid == 0) {
            int need = 0;
            bool ok = true;
            for (int h = 0; h < H; ++h) {
                need += nseg_sm[h];
                ok &= nseg_sm[h] <= SEGMAX;
            }
            unsigned base = 0;
            if (need && ok) {
                base = atomicAdd(a.seg_top, (unsigned)need);
                ok = base + need <= (unsigned)a.seg_cap;
            }
            if (!ok) {                   // the item is recomputed by the exact body
                fail_sm = 1;
                atomicExch(&a.items[item].fail, 1);
            }
            int acc = 0;
            for (int h = 0; h < H; ++h) {
                segbase_sm[h] = ok ? (int)base + acc : 0;
                acc += ok ? nseg_sm[h] : 0;
            }
        }
        __syncthreads();
        const bool seg_ok = !fail_sm;
        if (seg_ok) {
            for (int h = 0; h < H; ++h)
                for (int k = 0; k < nseg_sm[h]; ++k) {
                    SegEntry &e = a.segs[segbase_sm[h] + k];
                    for (int i = tid; i < D; i += NT) e.S[i] = 0;
                    if (tid == 0) e.f = rl_f[h][k];
                }
        }

        // ---- 4. V ------------------------------------------------------------------
        // 4a. p-pass: p = exp(carry - s') and w = v_norm * p for every (token,
        //     head); w replaces the score in place. The l of every segment and
        //     the clamp-proof bound are summed here.
        p_pass<H, R, NT, C, CW>(exp_tab, d_sm, dbase, vn_sm, grew, gpre, lsum_sm, bnd_sm, n);
        __syncthreads();

        // 4b. term tables per sub-tile, and the lookups
        {
            // build: task (unit u, head h) turns the unit's w into the terms
            // floor(w * c_k / 2^acc_shift) and writes its NE entries for h.
            auto build = [&](int sti, int buf) {
                const int st = sti * SUBT;
                int32_t *tab = tabs + (size_t)buf * CF::TAB_WORDS;
                for (int task = tid; task < UNITS * H; task += NT) {
                    const int l = task & 31;
                    const int u = (task >> 5) * UPW + l % UPW, h = l / UPW;
                    const int t = st + u * TPE;
                    int32_t w[TPE];                // |w| <= 2^30, |c| < 2^17: 32 x 32 -> 64-bit products
                    if constexpr (TPE == 2) {
                        const int2 w2 = *reinterpret_cast<const int2 *>(&d_sm[h * C + t]);
                        w[0] = t < n ? w2.x : 0;
                        w[1] = t + 1 < n ? w2.y : 0;
                    } else {
                        w[0] = t < n ? (int32_t)d_sm[h * C + t] : 0;
                    }
                    int32_t T[TPE][NC];
#pragma unroll
                    for (int e = 0; e < TPE; ++e)
#pragma unroll
                        for (int k = 0; k < NC; ++k)
                            T[e][k] = (int32_t)(((long long)w[e] * (long long)vcent[k]) >> DefFmt::ACC_SHIFT);
                    int32_t *dst = tab + u * USTR + (H == 1 ? 0 : (h >> 1) * HPS + (h & 1));
                    constexpr int ES = H == 1 ? 1 : 2;         // words per entry
#pragma unroll
                    for (int idx = 0; idx < NE; ++idx) {
                        int32_t v = T[0][idx & (NC - 1)];
                        if constexpr (TPE == 2) v += T[1][idx >> VB];
                        dst[idx * ES] = v;
                    }
                }
            };
            // accumulate: warp = (channel half, head group, stream); lane = channel.
            const int half = warp & 1, rest = warp >> 1;
            const int hgrp = rest % HG, stream = rest / HG;
            const int ch = half * 32 + lane;
            int32_t acc[HL];
            int cur[HL];
#pragma unroll
            for (int i = 0; i < HL; ++i) {
                acc[i] = 0;
                cur[i] = 0;
            }
            auto flush = [&](int i) {
                const int h = hgrp * HL + i;
                if (acc[i]) {
                    if (cur[i] == 0) atomicAdd(&s0p[h * D + ch], acc[i]);
                    else if (seg_ok)
                        atomicAdd((unsigned long long *)&a.segs[segbase_sm[h] + cur[i] - 1].S[ch],
                                  (unsigned long long)(long long)acc[i]);
                }
                acc[i] = 0;
            };
            // entry `nib` of the unit at `u` for this lane's heads (HL/2 head pairs)
            auto lookup = [&](const int32_t *u, uint32_t nib) {
                if constexpr (HL >= 2) {
#pragma unroll
                    for (int k = 0; k < HL / 2; ++k) {
                        const int2 x = *reinterpret_cast<const int2 *>(u + k * HPS + 2 * nib);
                        acc[2 * k] += x.x;
                        acc[2 * k + 1] += x.y;
                    }
                } else {
                    acc[0] += u[nib];
                }
            };
            // two units at once, their entries summed before the accumulators
            auto lookup2 = [&](const int32_t *u0, uint32_t n0, const int32_t *u1, uint32_t n1) {
                if constexpr (HL >= 2) {
#pragma unroll
                    for (int k = 0; k < HL / 2; ++k) {
                        const int2 x0 = *reinterpret_cast<const int2 *>(u0 + k * HPS + 2 * n0);
                        const int2 x1 = *reinterpret_cast<const int2 *>(u1 + k * HPS + 2 * n1);
                        acc[2 * k] += x0.x + x1.x;
                        acc[2 * k + 1] += x0.y + x1.y;
                    }
                } else {
                    acc[0] += u0[n0] + u1[n1];
                }
            };
            auto accumulate = [&](int sti, int buf) {
                constexpr int UPS = 32 / TPE, WPS = UPS / 8;   // units, code words per stream
                const int st = sti * SUBT, ts = st + stream * 32;
                if (ts >= n) return;
                const int blk = ts >> 5;
                const int32_t *tab = tabs + (size_t)buf * CF::TAB_WORDS +
                                     (stream * 32 / TPE) * USTR + (H == 1 ? 0 : hgrp * (HL / 2) * HPS);
                // the segment each head is in at the start of these 32 tokens
#pragma unroll
                for (int i = 0; i < HL; ++i) {
                    const int sgv = gpre[(hgrp * HL + i) * CW + blk];
                    if (sgv != cur[i]) {
                        flush(i);
                        cur[i] = sgv;
                    }
                }
                uint32_t cw[WPS];
#pragma unroll
                for (int k = 0; k < WPS; ++k) cw[k] = tw[ch * TWS + ts / TPW + k];
                const uint32_t any = anyg[blk];
                if (any == 0) {
#pragma unroll
                    for (int j = 0; j < UPS; j += 2)
                        lookup2(tab + j * USTR, (cw[j >> 3] >> (4 * (j & 7))) & 15u,
                                tab + (j + 1) * USTR, (cw[(j + 1) >> 3] >> (4 * ((j + 1) & 7))) & 15u);
                } else {
                    // rescale points inside: a token that opens a segment for a
                    // head flushes that head first; a unit whose second token
                    // opens one is added token by token from w.
                    uint32_t gb[HL];
#pragma unroll
                    for (int i = 0; i < HL; ++i) gb[i] = grew[(hgrp * HL + i) * CW + blk];
#pragma unroll
                    for (int j = 0; j < UPS; ++j) {
                        const int tt = j * TPE;
                        const uint32_t nib = (cw[j >> 3] >> (4 * (j & 7))) & 15u;
                        const uint32_t ub = (any >> tt) & ((1u << TPE) - 1u);
                        if (ub <= 1u) {
                            if (ub) {
#pragma unroll
                                for (int i = 0; i < HL; ++i)
                                    if ((gb[i] >> tt) & 1u) {
                                        flush(i);
                                        ++cur[i];
                                    }
                            }
                            lookup(tab + j * USTR, nib);
                        } else {
#pragma unroll
                            for (int e = 0; e < TPE; ++e) {
                                const int t = ts + tt + e;
                                if (t >= n) break;
                                const uint32_t code = (nib >> (VB * e)) & ((1u << VB) - 1u);
#pragma unroll
                                for (int i = 0; i < HL; ++i) {
                                    const int h = hgrp * HL + i;
                                    if ((gb[i] >> (tt + e)) & 1u) {
                                        flush(i);
                                        ++cur[i];
                                    }
                                    acc[i] += (int32_t)(((int64_t)(int32_t)d_sm[h * C + t] * (int64_t)vcent[code]) >>
                                                        DefFmt::ACC_SHIFT);
                                }
                            }
                        }
                    }
                }
            };
            const int nsub = (n + SUBT - 1) / SUBT;
            if (nsub) build(0, 0);
            __syncthreads();
            for (int i = 0; i < nsub; ++i) {
                if (i + 1 < nsub) build(i + 1, (i + 1) & 1);
                accumulate(i, i & 1);
                __syncthreads();
            }
#pragma unroll
            for (int i = 0; i < HL; ++i) flush(i);
        }
        __syncthreads();
        // l of the rescale segments, now that the p-pass has summed p
        if (seg_ok && tid < H)
            for (int k = 0; k < nseg_sm[tid]; ++k)
                a.segs[segbase_sm[tid] + k].l = (int64_t)lsum_sm[tid][k + 1];

        // ---- 5. the chunk record ------------------------------------------------
        {
            ChunkRec &rec = a.recs[rec_idx];
            for (int i = tid; i < H * D; i += NT) rec.S0[i / D][i % D] = s0p[i];
            if (tid < H) {
                const int h = tid;
                rec.l0[h] = (int64_t)lsum_sm[h][0];
                // sum_t max_k |term| <= sum_t (floor(|w_t| max|c| / 2^acc_shift) + 1)
                //                  <= floor(sum_t |w_t| * max|c| / 2^acc_shift) + n
                long long sw = 0;
                for (int w = 0; w < NT / 32; ++w) sw += bnd_sm[w][h];
                rec.B[h] = ((sw * cmax_v) >> DefFmt::ACC_SHIFT) + n;
                rec.nseg[h] = seg_ok ? nseg_sm[h] : 0;
                rec.seg_base[h] = segbase_sm[h];
            }
            if (tid == 0) {
                ItemAcc &ia = a.items[item];
                if (resc_sm) atomicAdd(&ia.resc, (unsigned long long)resc_sm);
            }
        }
        if (warp == 1 && li + 2 < ntl) ahead.store(li + 2, lane);
        __syncthreads();                 // the next tile reuses shared memory
    }
    // copies whose wait gave up must land before the CTA's shared memory goes
    if (lost_at >= 0) mbar_wait(&vbar, (uint32_t)lost_at & 1u, a.poll_limit);
}

// ---------------------------------------------------------------------------
// The fold, after every tile's record is written (the stream orders it): one
// CTA per (item, block of GBLK tiles) folds the block's records; the CTA that
// folds an item's last block folds the item's blocks and finalizes it (or
// writes a context shard's composite). The folds are a launch of their own:
// their code in the loop kernels, called or inlined, costs those loops their
// register allocation (the value loop ran at half speed).
// ---------------------------------------------------------------------------
template <int H>
__global__ void __launch_bounds__(CHUNK_THREADS, 2) k_fold(ChunkArgs a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    wait_prior_grid();
    const int item = blockIdx.x / a.max_blocks, blk = blockIdx.x % a.max_blocks;
    if (blk * GBLK >= item_chunks(a, item)) return;
    fold_block_and_item<H>(a, item, blk * GBLK, dyn);
}

// k_fold's shared memory, granted once per device and head count.
template <int H>
inline cudaError_t fold_prepare() {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    if (done[dev]) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(k_fold<H>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FoldCfg<H>::BYTES);
    done[dev] = e == cudaSuccess;
    return e;
}

// ---------------------------------------------------------------------------
// host side: the tile list, the scratch, the launches
// ---------------------------------------------------------------------------

template <int H>
inline cudaError_t launch_seq(const Geo &g, const DevTables *tb, int32_t B, const int32_t *d_seq,
                              const int64_t *d_lens, const int32_t *d_pt, const uint8_t *pool,
                              const int32_t *q_rot, int64_t *out, ins_stats *stats,
                              const int32_t *only, cudaStream_t s) {
    const size_t smem = seq_dyn_smem<H>(g);
    auto fn = (g.kb == 4 && g.vb == 2)   ? k_scan_seq<H, 4, 2>
              : (g.kb == 3 && g.vb == 3) ? k_scan_seq<H, 3, 3>
                                         : k_scan_seq<H, 0, 0>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // k_scan_seq waits for the launch before it before it reads anything
    return launch_after(fn, (unsigned)(B * g.n_kv), (unsigned)(H * 64), smem, s, g, tb, d_seq, d_lens,
                        d_pt, pool, q_rot, out, stats, only);
}


// Resident CTAs of the scores (WHICH 0) or values (WHICH 1) kernel on the
// current device: the launch grid. The dynamic-smem attribute and the
// occupancy are set and queried once per kernel and device.
template <int H, int KB, int VB, int WHICH, int RS = 0>
inline int chunk_slots() {
    auto fn = WHICH == 0 ? k_scan_scores<H, KB, VB, RS> : k_scan_values<H, KB, VB, RS>;
    const size_t dyn = WHICH == 0 ? ScoreCfg<H, KB, VB, RS>::BYTES : ChunkCfg<H, KB, VB, RS>::BYTES;
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    std::lock_guard<std::mutex> lk(mu);
    if (cached[dev] > 0) return cached[dev];
    int per_sm = 0, sms = 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, CHUNK_THREADS, dyn) != cudaSuccess)
        return -1;
    cached[dev] = (per_sm < 1 ? 1 : per_sm) * sms;
    return cached[dev];
}

// Byte layout of the scratch of one scan: `o` offsets in the order carved.
struct ScratchLayout {
    size_t top, cmx, rec, blk, seg, items, redo, desc, bmg, sc, lbw, idone, sdone, total;
    ScratchLayout(int ni, int mc, int sc_cap, int tc, int H, int CW, int64_t rows) {
        auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
        const int mb = (mc + GBLK - 1) / GBLK;
        size_t o = 0;
        top = o; o += al(8);
        // the single-launch scan's look-back words; the fold's counters
        lbw = o; o += al(sizeof(unsigned long long) * (size_t)ni * mc * H);
        idone = o; o += al(sizeof(unsigned int) * (size_t)ni);
        sdone = o; o += al(sizeof(unsigned int));
        cmx = o; o += al(sizeof(long long) * (size_t)ni * mc * 2 * HMAX);
        rec = o; o += al(sizeof(ChunkRec) * (size_t)ni * mc);
        blk = o; o += al(sizeof(BlockRec) * (size_t)ni * mb);
        seg = o; o += al(sizeof(SegEntry) * (size_t)sc_cap);
        items = o; o += al(sizeof(ItemAcc) * (size_t)ni);
        redo = o; o += al(sizeof(int32_t) * (size_t)ni);
        desc = o; o += al(TileDesc(ni, ni).total);
        // block maxima and score offsets: the separate-launch scan only
        bmg = o; o += al(sizeof(long long) * (size_t)(rows > 0 ? tc : 1) * H * CW);
        sc = o; o += al(sizeof(uint32_t) * (size_t)(rows > 0 ? rows : 1) * H);
        total = o;
    }
};

// Carve (or grow) the scratch for n_items items of up to max_nc tiles.
inline int reserve_scratch(ChunkScratch &cs, int n_items, int max_nc, int n_tiles, int H, int CW,
                           int64_t rows, cudaStream_t s) {
    const int seg_cap = 2 * (64 * n_items * H) + 4 * n_tiles;
    const int64_t sc_words = rows * H;
    if (cs.base && n_items <= cs.n_items && max_nc <= cs.max_chunks && seg_cap <= cs.seg_cap &&
        n_tiles <= cs.tile_cap && sc_words <= cs.sc_rows)
        return INS_OK;
    cudaStreamSynchronize(s);
    // grown with a quarter of slack, so a context that grows by a token per
    // step reallocates only now and then
    auto grow = [](int64_t need, int64_t have) { return need > have ? need + need / 4 : have; };
    const int ni = (int)grow(n_items, cs.n_items);
    const int mc = (int)grow(max_nc, cs.max_chunks);
    const int sc = (int)grow(seg_cap, cs.seg_cap);
    const int tc = (int)grow(n_tiles, cs.tile_cap);
    const int64_t sw = grow(sc_words, cs.sc_rows);
    cs.release();
    // sized for up to HMAX heads and 32 blocks per tile, so one scratch serves
    // every head count
    const ScratchLayout L(ni, mc, sc, tc, HMAX, 32, (sw + HMAX - 1) / HMAX);
    (void)H;
    (void)CW;
    if (cudaMalloc(&cs.base, L.total) != cudaSuccess) {
        cudaGetLastError();
        cs.base = nullptr;
        return INS_ENOMEM;
    }
    if (cudaMemset(cs.base, 0, L.total) != cudaSuccess) return INS_ECUDA;
    uint8_t *p = (uint8_t *)cs.base;
    cs.bytes = L.total;
    cs.seg_top = (unsigned int *)(p + L.top);
    cs.cmx = (long long *)(p + L.cmx);
    cs.recs = (ChunkRec *)(p + L.rec);
    cs.blks = (BlockRec *)(p + L.blk);
    cs.segs = (SegEntry *)(p + L.seg);
    cs.items = (ItemAcc *)(p + L.items);
    cs.redo = (int32_t *)(p + L.redo);
    cs.desc = p + L.desc;
    cs.bmg = (long long *)(p + L.bmg);
    cs.sc = (uint32_t *)(p + L.sc);
    cs.lbw = (unsigned long long *)(p + L.lbw);
    cs.idone = (unsigned int *)(p + L.idone);
    cs.sdone = (unsigned int *)(p + L.sdone);
    cs.lbw_words = (size_t)ni * mc * HMAX;
    cs.epoch = 0;
    cs.n_items = ni;
    cs.max_chunks = mc;
    cs.seg_cap = sc;
    cs.tile_cap = tc;
    cs.sc_rows = ((sw + HMAX - 1) / HMAX) * HMAX;
    return INS_OK;
}

// The three launches of the chunked scan (plus the exact re-run of flagged
// items) on a prepared argument block. `a` holds every pointer but the grid.
template <int H, int KB, int VB, int RS = 0>
inline int launch_chunk_kernels(ChunkArgs &a, int32_t B, const int32_t *d_seq, const int64_t *d_T,
                                cudaStream_t s) {
    const int gA = chunk_slots<H, KB, VB, 0, RS>(), gB = chunk_slots<H, KB, VB, 1, RS>();
    if (gA < 0 || gB < 0) return INS_ECUDA;
    // each launch may start while the one before finishes (it waits for it
    // before reading its results)
    const unsigned gs = (unsigned)(gA < a.n_tiles ? gA : a.n_tiles);
    const unsigned gv = (unsigned)(gB < a.n_tiles ? gB : a.n_tiles);
    if (launch_after(k_scan_scores<H, KB, VB, RS>, gs, (unsigned)CHUNK_THREADS, ScoreCfg<H, KB, VB, RS>::BYTES,
                     s, a) != cudaSuccess ||
        launch_after(k_scan_values<H, KB, VB, RS>, gv, (unsigned)CHUNK_THREADS, ChunkCfg<H, KB, VB, RS>::BYTES,
                     s, a) != cudaSuccess ||
        fold_prepare<H>() != cudaSuccess ||
        launch_after(k_fold<H>, (unsigned)(a.n_items * a.max_blocks), (unsigned)CHUNK_THREADS,
                     FoldCfg<H>::BYTES, s, a) != cudaSuccess)
        return INS_ECUDA;
    if (cudaGetLastError() != cudaSuccess) return INS_ECUDA;
    // items whose exactness the fold could not prove are recomputed in order
    (void)d_seq;
    (void)d_T;
    return launch_seq<H>(a.g, a.tb, B, a.seq_ids, a.T, a.page_table, a.pool, a.q_rot, a.out, a.stats,
                         a.redo, s) == cudaSuccess
               ? INS_OK
               : INS_ECUDA;
}

// The tile list, the scratch and the argument block of one chunked scan; no
// launch.
template <int H, int KB, int VB, int RS = 0>
inline int prepare_chunked(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                           const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                           const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                           int64_t *out, ins_stats *stats, int32_t *d_status, ChunkArgs &a,
                           cudaStream_t s, bool score_rows = true, const int32_t *h_seq = nullptr) {
    using CF = ChunkCfg<H, KB, VB, RS>;
    const int n_items = B * g.n_kv;
    TilePlan &tp = cs.plan;
    tp.build(g, B, h_T, CF::C);
    if (tp.n_tiles > INT32_MAX / 2) return INS_EBADLEN;
    const int n_tiles = (int)tp.n_tiles;
    // the separate-launch scan keeps every row's score offsets in global
    // memory; the single-launch scan keeps them in shared memory
    if (int rc = reserve_scratch(cs, n_items, tp.max_nc, n_tiles, H, CF::CW, score_rows ? tp.rows : 0, s))
        return rc;
    // no device lengths given: the host's lengths and sequence ids ride in
    // the tile plan's upload
    const bool ride = d_T == nullptr;
    const TileDesc L(n_items, ride ? B : 0);
    {
        int slot = 0;
        uint8_t *h = (uint8_t *)cs.up.take(L.total, slot);
        if (!h) return INS_ECUDA;
        tp.write(h, L);
        if (ride) {
            std::memcpy(h + L.lens, h_T, sizeof(int64_t) * (size_t)B);
            std::memcpy(h + L.seqs, h_seq, sizeof(int32_t) * (size_t)B);
            d_T = (const int64_t *)(cs.desc + L.lens);
            d_seq = (const int32_t *)(cs.desc + L.seqs);
        }
        int launched = 0;
        if (small_upload(cs.desc, h, L.total, s, &launched) != cudaSuccess || cs.up.done(slot, s))
            return INS_ECUDA;
        cs.launches += launched;
    }
    a = ChunkArgs{};
    a.g = g;
    a.tb = tb;
    a.runs = (const int4 *)(cs.desc + L.runs);
    a.n_runs = (int32_t)tp.runs.size();
    a.order = (const int32_t *)(cs.desc + L.ord);
    a.tile_rows = CF::C;
    a.n_tiles = n_tiles;
    a.max_chunks = cs.max_chunks;
    a.max_blocks = (cs.max_chunks + GBLK - 1) / GBLK;
    a.n_items = n_items;
    a.row_base = (const int64_t *)(cs.desc + L.rb);
    a.seq_ids = d_seq;
    a.T = d_T;
    a.page_table = d_pt;
    a.pool = pool;
    a.q_rot = q_rot;
    a.out = out;
    a.stats = stats;
    a.sc = cs.sc;
    a.bmg = cs.bmg;
    a.cmx = cs.cmx;
    a.recs = cs.recs;
    a.blks = cs.blks;
    a.segs = cs.segs;
    a.seg_top = cs.seg_top;
    a.seg_cap = cs.seg_cap;
    a.items = cs.items;
    a.redo = cs.redo;
    a.redo_total = cs.redo_total;
    a.status = d_status;
    a.item_done = cs.idone;
    a.scan_done = cs.sdone;
    a.poll_limit = cs.poll_limit;
    a.hold_rec = cs.hold_item < 0 || cs.hold_item >= n_items || cs.hold_chunk >= cs.max_chunks
                     ? -1
                     : (int64_t)cs.hold_item * cs.max_chunks + cs.hold_chunk;
    cs.last_items = n_items;
    return INS_OK;
}

template <int H, int KB, int VB, int RS = 0>
inline int launch_chunked(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                          const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                          const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                          int64_t *out, ins_stats *stats, int32_t *d_status, cudaStream_t s,
                          const int32_t *h_seq = nullptr) {
    ChunkArgs a;
    if (int rc = prepare_chunked<H, KB, VB, RS>(cs, g, tb, B, d_seq, d_T, h_T, d_pt, pool, q_rot, out, stats,
                                            d_status, a, s, true, h_seq))
        return rc;
    const int rc = launch_chunk_kernels<H, KB, VB, RS>(a, B, a.seq_ids, a.T, s);
    // scores, values, fold, exact re-run
    if (rc == INS_OK) cs.launches += 4;
    return rc;
}

// Context split, phase 1: the scores of this shard and each item's maximum
// (a.maxima), leaving the scores in the scratch for phase 2.
template <int H, int KB, int VB, int RS = 0>
inline int launch_split_maxima(ChunkArgs &a, cudaStream_t s) {
    const int gA = chunk_slots<H, KB, VB, 0, RS>();
    if (gA < 0) return INS_ECUDA;
    ChunkArgs m = a;
    m.m_init = nullptr;
    m.parts = nullptr;
    k_scan_scores<H, KB, VB, RS><<<gA < m.n_tiles ? gA : m.n_tiles, CHUNK_THREADS, ScoreCfg<H, KB, VB, RS>::BYTES, s>>>(m);
    k_item_maxima<H><<<(m.n_items * H + 7) / 8, 256, 0, s>>>(m);
    return cudaGetLastError() == cudaSuccess ? INS_OK : INS_ECUDA;
}

// Context split, phase 2: with the running maximum entering the shard
// (a.m_init), the values and one composite per item (a.parts).
template <int H, int KB, int VB, int RS = 0>
inline int launch_split_part(ChunkArgs &a, cudaStream_t s) {
    const int gB = chunk_slots<H, KB, VB, 1, RS>();
    if (gB < 0) return INS_ECUDA;
    ChunkArgs m = a;
    m.maxima = nullptr;
    k_scan_values<H, KB, VB, RS>
        <<<gB < m.n_tiles ? gB : m.n_tiles, CHUNK_THREADS, ChunkCfg<H, KB, VB, RS>::BYTES, s>>>(m);
    if (fold_prepare<H>() != cudaSuccess) return INS_ECUDA;
    k_fold<H><<<m.n_items * m.max_blocks, CHUNK_THREADS, FoldCfg<H>::BYTES, s>>>(m);
    return cudaGetLastError() == cudaSuccess ? INS_OK : INS_ECUDA;
}

// Tile size. Tiles of C rows (4 rows per thread where the shape allows) keep
// the per-tile work small against the rows; but a batch of short items cuts
// into few tiles and leaves SMs idle. When the default tiles would not fill
// half a wave of the values launch, tiles of half the rows are used instead
// (up to a wave, fewer and larger tiles also make the fold shorter).
enum : int32_t { TILES_AUTO = 0, TILES_LARGE = 1, TILES_SMALL = 2 };
// Online scan kernels: one persistent launch (scan_fused.cuh) or the separate
// score, prefix, value and fold launches of this file.
enum : int32_t { SCAN_FUSED = 0, SCAN_SPLIT = 1 };

template <int H, int KB, int VB>
inline bool small_tiles(const ChunkScratch &cs, const Geo &g, int32_t B, const int64_t *h_T) {
    if constexpr (ChunkCfg<H, KB, VB>::R != 4) {
        return false;
    } else {
        if (cs.tiles_mode != TILES_AUTO) return cs.tiles_mode == TILES_SMALL;
        constexpr int C = ChunkCfg<H, KB, VB>::C;
        int64_t tiles = 0;
        for (int32_t b = 0; b < B; ++b) tiles += h_T[b] ? (h_T[b] + C - 1) / C : 1;
        const int slots = chunk_slots<H, KB, VB, 1>();
        return slots > 0 && 2 * tiles * g.n_kv < (int64_t)slots;
    }
}

// Which chunked instantiation serves a cache: 0 none, else (H, KB, VB) packed.
inline int chunk_variant(const Geo &g, int H) {
    if (!is_def_fmt(g)) return 0;
    if (g.kb == 4 && g.vb == 2 && (H == 1 || H == 2 || H == 4 || H == 8)) return H * 100 + 42;
    if (g.kb == 3 && g.vb == 3 && (H == 4 || H == 8)) return H * 100 + 33;
    return 0;
}

}  // namespace ins
