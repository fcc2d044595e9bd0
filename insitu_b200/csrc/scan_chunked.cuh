// The context-parallel online scan.
//
// attend_online (ops/attention.py:451-513) is a sequential recurrence: a
// running maximum m, and at every token whose score exceeds it, a rescale
// acc = floor(acc * exp(s - m) / 2^15) before the token's own term is added.
// This kernel splits every (sequence, KV head) item into chunks of C rows and
// still returns the reference's bits:
//
//  1. Scores of a chunk are independent of everything else (exact, FP64 FMA
//     on integer operands, see row_scores_f64).
//  2. The running maximum entering chunk c is the maximum of every earlier
//     chunk's scores. Chunks publish their maximum as soon as their scores
//     exist and read their predecessors' with a decoupled look-back (bounded
//     waits; tiles are claimed in order, so every awaited tile is running).
//  3. Knowing m_in, the chunk finds the exact rescale points (tokens above
//     the running maximum), p = exp(m - s) for every token, and splits its
//     tokens into segments at the rescale points. Within a segment every term
//     is a fixed integer, so its contribution is a plain sum.
//  4. The last chunk of an item to finish folds the chunks in causal order:
//     acc = floor(acc * f / 2^15) at each rescale, + segment sums. That fold
//     equals the per-token recurrence provided the reference's 32-bit clamp
//     never fires; the fold proves it per chunk with
//     |acc at chunk start| + sum_t max_k |term(t, k)| <= 2^31 - 1, which bounds
//     every partial sum inside the chunk (a rescale never grows |acc|).
//     An item that fails the proof, overflows the segment pool, or sees a
//     bounded wait expire is recomputed by the exact sequential body in the
//     same CTA, so the result is bit-exact in every case.
#pragma once

#include <climits>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace ins {

constexpr int HMAX = 8;
constexpr int LB_SPIN_LIMIT = 1 << 22;   // ~0.4 s of polling at most
constexpr int SEGMAX = 32;               // rescales one head's chunk can hold
constexpr int GBLK = 32;                 // chunks folded per level-1 block
#ifndef INS_JGROUP
#define INS_JGROUP 8
#endif
#ifndef INS_SCORE_ROWS
#define INS_SCORE_ROWS 2
#endif

struct SegEntry {          // a rescale and the translation that follows it
    int64_t S[D];          // sum of terms after the rescale (per channel)
    int64_t l;             // sum of p over the same tokens
    int32_t f;             // factor applied to acc and l at the rescale
    int32_t pad;
};

struct ChunkRec {          // one (item, chunk)
    int32_t S0[HMAX][D];   // terms of the tokens before the chunk's first rescale
    int64_t l0[HMAX];
    int64_t B[HMAX];       // sum over tokens of max over codes of |term|
    int32_t nseg[HMAX];
    int32_t seg_base[HMAX];
};

struct BlockRec {          // GBLK consecutive chunks of one item, folded
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

struct ChunkArgs {
    Geo g;
    const DevTables *tb;
    const int4 *tiles;            // (item, chunk, t0, n)
    int32_t n_tiles;
    int32_t C;                    // rows per chunk
    int32_t max_chunks;
    int32_t max_blocks;
    int32_t n_items;
    const int32_t *item_nchunks;
    const int32_t *seq_ids;
    const int64_t *T;
    const int32_t *page_table;
    const uint8_t *pool;
    const int32_t *q_rot;
    int64_t *out;
    ins_stats *stats;
    unsigned long long *claim;
    unsigned long long claim_base;
    unsigned long long *lb_flag;  // [n_items * max_chunks]
    long long *lb_val;            // [n_items * max_chunks * 2 * HMAX]
    ChunkRec *recs;               // [n_items * max_chunks]
    BlockRec *blks;               // [n_items * max_blocks]
    unsigned int *blk_done;       // [n_items * max_blocks]
    SegEntry *segs;
    unsigned int *seg_top;
    int32_t seg_cap;
    ItemAcc *items;               // [n_items]
    int32_t *redo;                // [n_items]: 1 = recompute with the sequential body
    unsigned long long *all_done;
    int32_t *status;
    unsigned long long epoch;
};

// Device scratch of the chunked scan, owned by the cache handle and grown on
// demand. Everything in it is either rewritten each launch or reset by the
// kernel itself, so launches need no memsets.
struct ChunkScratch {
    void *base = nullptr;
    size_t bytes = 0;
    int32_t n_items = 0, max_chunks = 0, seg_cap = 0, tile_cap = 0;
    unsigned long long epoch = 0;
    unsigned long long claim_base = 0;
    unsigned long long *claim = nullptr, *lb_flag = nullptr, *all_done = nullptr;
    long long *lb_val = nullptr;
    ChunkRec *recs = nullptr;
    BlockRec *blks = nullptr;
    unsigned int *blk_done = nullptr;
    SegEntry *segs = nullptr;
    unsigned int *seg_top = nullptr;
    ItemAcc *items = nullptr;
    int32_t *redo = nullptr;
    int4 *tiles = nullptr;
    int32_t *item_nchunks = nullptr;

    void release() {
        if (base) cudaFree(base);
        base = nullptr;
        bytes = 0;
        n_items = max_chunks = seg_cap = tile_cap = 0;
    }
};

// ---------------------------------------------------------------------------
// smem layout of the chunk kernel
// ---------------------------------------------------------------------------
template <int H, int VB>
struct ChunkLayout {
    static constexpr int NC = 1 << VB;                    // V codes
    static constexpr int SUB = VB <= 2 ? 256 : 128;       // tokens per term-table sub-tile
    static constexpr int PS = SUB * H + 4;                // words per code plane (padded)
    static constexpr int VW = 2 * VB;                     // 32-bit words per V row
    int C;
    size_t off_s, off_p, off_vt, off_vn, off_tab, off_grew, off_pre, off_bmax, off_bcar, off_s0, total;
    __host__ __device__ explicit ChunkLayout(int C_) : C(C_) {
        size_t o = 0;
        off_s = o;    o += (size_t)H * C * 8;             // scores (int64)
        off_p = o;    o += (size_t)H * C * 4;             // p (int32)
        off_vt = o;   o += (size_t)VW * C * 4;            // V codes, word-major
        off_vn = o;   o += (size_t)C * 4;                 // v_norm (int32)
        off_tab = o;  o += (size_t)NC * PS * 4;           // terms [code][t][h]
        off_grew = o; o += (size_t)(H + 1) * (C / 32) * 4;  // rescale bits per head, + any
        off_pre = o;  o += (size_t)H * (C / 32) * 4;      // rescales before each bit word
        off_bmax = o; o += (size_t)H * (C / 32) * 8;      // max score of each 32-row block
        off_bcar = o; o += (size_t)H * (C / 32) * 8;      // running max entering each block
        off_s0 = o;   o += (size_t)H * D * 4;             // segment-0 partials
        total = o;
    }
};

// Scores of R rows for one thread (register-blocked over rows), exact.
// Channels are taken 32 at a time: 32 codes of KB bits are exactly KB words,
// so every code extraction below is at a compile-time position.
template <int H, int KB, int R>
__device__ __forceinline__ void score_rows(const Geo &g, const uint8_t *const *krow,
                                           const int64_t *knorm, const bool *valid,
                                           const double *__restrict__ qd,
                                           const uint32_t *__restrict__ khi, int64_t (*s)[H],
                                           int &ovf) {
    double acc[R][H];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < H; ++h) acc[r][h] = 0.0;
#pragma unroll 1
    for (int grp = 0; grp < D / 32; ++grp) {
        uint32_t w[R][KB];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(krow[r]) + grp * KB;
#pragma unroll
            for (int i = 0; i < KB; ++i) w[r][i] = valid[r] ? src[i] : 0u;
        }
        const double *qg = qd + grp * 32;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
            double c[R];
#pragma unroll
            for (int r = 0; r < R; ++r)
                c[r] = __hiloint2double((int)khi[code_at<KB>(w[r], jj, KB)], 0);
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const double qv = qg[h * D + jj];
#pragma unroll
                for (int r = 0; r < R; ++r) acc[r][h] = fma(qv, c[r], acc[r][h]);
            }
            if ((jj & (INS_JGROUP - 1)) == INS_JGROUP - 1) asm volatile("" ::: "memory");
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < H; ++h) {
            const int64_t di = __double2ll_rn(acc[r][h]);
            const int64_t prod = (int64_t)((uint64_t)di * (uint64_t)knorm[r]);
            bool hit;
            s[r][h] = qclamp(prod >> g.score_shift, g.score_width, g.saturate, hit);
            ovf += hit && valid[r];
        }
}

__device__ __forceinline__ long long ld_volatile(const long long *p) {
    return *reinterpret_cast<const volatile long long *>(p);
}
__device__ __forceinline__ unsigned long long ld_volatile(const unsigned long long *p) {
    return *reinterpret_cast<const volatile unsigned long long *>(p);
}

template <class T>
__device__ __forceinline__ T ldcg(const T *p) {
    return __ldcg(p);
}

// Level 1: fold the chunks of block `blk` of `item` into a BlockRec.
// Threads [0, H*64) own (head, channel) pairs.
template <int H>
__device__ void merge_block(const ChunkArgs &a, int item, int blk, int nchunks,
                            int *base_sm /* [H] */) {
    const int tid = threadIdx.x;
    const bool own = tid < H * D;
    const int h = own ? tid / D : 0, ch = tid % D;
    const int c0 = blk * GBLK, c1 = min(nchunks, c0 + GBLK);
    const ChunkRec *recs = a.recs + (int64_t)item * a.max_chunks;
    // entries this head needs = rescales in the block's chunks
    if (own && ch == 0) {
        int need = 0;
        for (int c = c0; c < c1; ++c) need += ldcg(&recs[c].nseg[h]);
        unsigned b = 0;
        if (need) b = atomicAdd(a.seg_top, (unsigned)need);
        if (need && b + need > (unsigned)a.seg_cap) {
            atomicExch(&a.items[item].fail, 1);
            need = 0;
        }
        base_sm[h] = need ? (int)b : -1;
    }
    __syncthreads();
    if (own) {
        const int eb = base_sm[h];
        int64_t loc = 0, Y = 0, curS = 0, curl = 0, Spre = 0, lpre = 0;
        int ne = 0;
        bool opened = false;
        for (int cb = c0; cb < c1; cb += 8) {
            int32_t S0[8], ns[8], sb[8];
            int64_t Bk[8], l0[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = cb + u;
                if (c < c1) {
                    S0[u] = ldcg(&recs[c].S0[h][ch]);
                    Bk[u] = ldcg(&recs[c].B[h]);
                    l0[u] = ldcg(&recs[c].l0[h]);
                    ns[u] = ldcg(&recs[c].nseg[h]);
                    sb[u] = ldcg(&recs[c].seg_base[h]);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (cb + u >= c1) break;
                const int64_t al = loc < 0 ? -loc : loc;
                Y = max(Y, al + Bk[u]);
                loc += S0[u];
                curS += S0[u];
                curl += l0[u];
                for (int e = 0; e < ns[u]; ++e) {
                    const SegEntry &se = a.segs[sb[u] + e];
                    const int64_t f = ldcg(&se.f);
                    const int64_t sS = ldcg(&se.S[ch]);
                    const int64_t sl = ldcg(&se.l);
                    if (eb >= 0) {
                        if (!opened) {
                            Spre = curS;
                            lpre = curl;
                            opened = true;
                        } else {
                            a.segs[eb + ne - 1].S[ch] = curS;
                            if (ch == 0) a.segs[eb + ne - 1].l = curl;
                        }
                        if (ch == 0) a.segs[eb + ne].f = (int32_t)f;
                        ++ne;
                    }
                    curS = sS;
                    curl = sl;
                    loc = ((loc * f) >> a.g.prob_frac) + sS;
                }
            }
        }
        if (!opened) {
            Spre = curS;
            lpre = curl;
        } else if (eb >= 0) {
            a.segs[eb + ne - 1].S[ch] = curS;
            if (ch == 0) a.segs[eb + ne - 1].l = curl;
        }
        BlockRec &br = a.blks[(int64_t)item * a.max_blocks + blk];
        br.Spre[h][ch] = Spre;
        br.Y[h][ch] = Y;
        if (ch == 0) {
            br.lpre[h] = lpre;
            br.nent[h] = eb >= 0 ? ne : 0;
            br.ent_base[h] = eb >= 0 ? eb : 0;
        }
    }
}

// Level 2: fold the item's blocks; finalize or mark the item for the exact
// sequential recomputation.
template <int H>
__device__ void merge_item(const ChunkArgs &a, int item, int nblocks, int64_t T,
                           int64_t qbase, long long *maxs_sm) {
    const int tid = threadIdx.x;
    const bool own = tid < H * D;
    const int h = own ? tid / D : 0, ch = tid % D;
    const BlockRec *blks = a.blks + (int64_t)item * a.max_blocks;
    int64_t acc = 0, l = 0;
    bool bad = *reinterpret_cast<volatile int32_t *>(&a.items[item].fail) != 0;
    if (own && !bad) {
        for (int bb = 0; bb < nblocks; ++bb) {
            const BlockRec &br = blks[bb];
            const int64_t Y = ldcg(&br.Y[h][ch]);
            const int64_t Sp = ldcg(&br.Spre[h][ch]);
            const int64_t lp = ldcg(&br.lpre[h]);
            const int ne = ldcg(&br.nent[h]);
            const int eb = ldcg(&br.ent_base[h]);
            const int64_t aa = acc < 0 ? -acc : acc;
            if (aa + Y > INT32_MAX) bad = true;
            acc += Sp;
            l += lp;
            for (int e = 0; e < ne; ++e) {
                const SegEntry &se = a.segs[eb + e];
                const int64_t f = ldcg(&se.f);
                acc = ((acc * f) >> a.g.prob_frac) + ldcg(&se.S[ch]);
                l = ((l * f) >> a.g.prob_frac) + ldcg(&se.l);
            }
        }
    }
    bad = __syncthreads_or(bad);
    if (tid == 0) {
        a.redo[item] = bad ? 1 : 0;
        *maxs_sm = 0;
    }
    if (bad) return;
    int64_t *out_row = a.out + qbase;
    long long mx = 0;
    if (own) {
        int64_t r;
        int shift;
        reciprocal(a.g, l, r, shift);
        out_row[h * D + ch] = (acc * r) >> shift;
        mx = acc < 0 ? -acc : acc;
    }
    __syncthreads();
    if (own) atomicMax(maxs_sm, mx);
    __syncthreads();
    if (tid == 0 && a.stats) {
        const volatile ItemAcc &ia = a.items[item];
        ins_stats st;
        st.n_tokens = T;
        st.rescale_events = (int64_t)ia.resc;
        st.score_overflows = (int64_t)ia.sovf;
        st.acc_overflows = 0;
        st.max_abs_score = ia.maxs;
        st.max_abs_acc = *maxs_sm;
        a.stats[item] = st;
    }
}

template <int H, int KB, int VB>
__global__ void __launch_bounds__(H * 64 > 256 ? H * 64 : 256, H * 64 > 256 ? 1 : 2)
    k_scan_chunk(ChunkArgs a) {
    using L = ChunkLayout<H, VB>;
    constexpr int NC = L::NC, SUB = L::SUB, VW = L::VW, PS = L::PS;
    constexpr int NT = H * 64 > 256 ? H * 64 : 256;
    constexpr int R = INS_SCORE_ROWS;                // rows per thread in the score phase
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ double qd[H * D];
    __shared__ uint32_t khi[256];
    __shared__ int32_t vcent[256];
    __shared__ int32_t exp_tab[256];
    __shared__ long long cmax[H], m_in_sm[H];
    __shared__ int tile_sm, flag_sm, fail_sm;
    __shared__ int nseg_sm[H], segbase_sm[H], base_sm[H];
    __shared__ int32_t rl_f[H][SEGMAX];
    __shared__ unsigned long long lsum_sm[H][SEGMAX + 1];
    __shared__ long long bsum_sm[H];
    __shared__ unsigned long long resc_sm;
    __shared__ unsigned int sovf_sm;
    __shared__ long long maxs_sm;
    __shared__ const uint8_t *page_sm[8];

    const Geo &g = a.g;
    const int tid = threadIdx.x;
    const L lay(a.C);
    const int CW = a.C / 32;
    int64_t *s_sm = reinterpret_cast<int64_t *>(dyn + lay.off_s);
    int32_t *p_sm = reinterpret_cast<int32_t *>(dyn + lay.off_p);
    uint32_t *vt = reinterpret_cast<uint32_t *>(dyn + lay.off_vt);
    int32_t *vn_sm = reinterpret_cast<int32_t *>(dyn + lay.off_vn);
    int32_t *tab = reinterpret_cast<int32_t *>(dyn + lay.off_tab);
    uint32_t *grew = reinterpret_cast<uint32_t *>(dyn + lay.off_grew);   // [H][CW], then any [CW]
    uint32_t *anyg = grew + H * CW;
    int32_t *gpre = reinterpret_cast<int32_t *>(dyn + lay.off_pre);     // [H][CW]
    long long *bmax = reinterpret_cast<long long *>(dyn + lay.off_bmax);  // [H][CW]
    long long *bcar = reinterpret_cast<long long *>(dyn + lay.off_bcar);  // [H][CW]
    int32_t *s0p = reinterpret_cast<int32_t *>(dyn + lay.off_s0);

    for (int i = tid; i < 256; i += NT) {
        const double c = a.tb->k_cent_f64[i];
        khi[i] = (uint32_t)__double2hiint(c);
        vcent[i] = (int32_t)a.tb->v_cent[i];
        exp_tab[i] = a.tb->exp_tab[i];
    }
    const int64_t s_lo = -(1ll << (g.score_width - 1));

    for (;;) {
        if (tid == 0) tile_sm = (int)(atomicAdd(a.claim, 1ull) - a.claim_base);
        __syncthreads();
        const int tile = tile_sm;
        if (tile >= a.n_tiles) break;
        const int4 td = a.tiles[tile];
        const int item = td.x, c = td.y;
        const int64_t t0 = td.z;
        const int n = td.w;
        const int b = item / g.n_kv, kvh = item % g.n_kv;
        const int seq = a.seq_ids[b];
        const int64_t qbase = ((int64_t)b * g.n_kv * H + (int64_t)kvh * H) * D;
        const int rec_idx = item * a.max_chunks + c;

        // ---- 0. per-tile setup -------------------------------------------------
        for (int i = tid; i < H * D; i += NT) qd[i] = (double)a.q_rot[qbase + i];
        const int npages = (n + g.P - 1) / g.P;
        if (tid < npages) {
            const int64_t page = a.page_table[(int64_t)seq * g.max_pages + (t0 / g.P) + tid];
            page_sm[tid] = a.pool + region_off(g, page, kvh);
        }
        if (tid < H) {
            cmax[tid] = LLONG_MIN;
            bsum_sm[tid] = 0;
            for (int k = 0; k <= SEGMAX; ++k) lsum_sm[tid][k] = 0;
        }
        if (tid == 0) {
            resc_sm = 0;
            sovf_sm = 0;
            maxs_sm = 0;
            fail_sm = 0;
        }
        for (int i = tid; i < (H + 1) * CW; i += NT) grew[i] = 0;
        for (int i = tid; i < H * D; i += NT) s0p[i] = 0;
        __syncthreads();
        bool big = false;
        for (int i = tid; i < H * D; i += NT) {
            const double x = qd[i];
            big |= (x >= 1073741824.0 || x <= -1073741824.0);
        }
        if (__syncthreads_or(big)) {
            // |q| >= 2^30 would let an FP64 partial sum pass 2^53; such an
            // item is left to the exact int64 sequential body.
            if (tid == 0) atomicExch(&a.items[item].fail, 1);
        }

        // ---- 1. scores, staged V codes and norms --------------------------------
        {
            int ovf = 0;
            long long mx = 0;
            int64_t hmax[H];
#pragma unroll
            for (int h = 0; h < H; ++h) hmax[h] = LLONG_MIN;
            for (int base = 0; base < n; base += NT * R) {
                const uint8_t *krow[R];
                int64_t knorm[R];
                bool valid[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = base + r * NT + tid;
                    valid[r] = row < n;
                    const int rr = valid[r] ? row : 0;
                    const uint8_t *reg = page_sm[rr / g.P];
                    const int lr = rr % g.P;
                    krow[r] = reg + (int64_t)lr * g.kbytes;
                    const int32_t nw = valid[r] ? *reinterpret_cast<const int32_t *>(
                                                      reg + nplane_off(g) + (int64_t)lr * 4)
                                                : 0;
                    knorm[r] = (int16_t)(nw & 0xffff);
                    if (valid[r]) {
                        vn_sm[row] = (int32_t)(int16_t)((uint32_t)nw >> 16);
                        const uint32_t *vrow = reinterpret_cast<const uint32_t *>(
                            reg + vplane_off(g) + (int64_t)lr * g.vbytes);
#pragma unroll
                        for (int w = 0; w < VW; ++w) vt[w * a.C + row] = vrow[w];
                    }
                }
                int64_t s[R][H];
                score_rows<H, KB, R>(g, krow, knorm, valid, qd, khi, s, ovf);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = base + r * NT + tid;
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        long long bm = valid[r] ? s[r][h] : LLONG_MIN;
                        if (valid[r]) {
                            s_sm[h * a.C + row] = s[r][h];
                            const long long ab = s[r][h] < 0 ? -s[r][h] : s[r][h];
                            mx = ab > mx ? ab : mx;
                        }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const long long w = __shfl_xor_sync(FULL, bm, o);
                            bm = w > bm ? w : bm;
                        }
                        hmax[h] = bm > hmax[h] ? bm : hmax[h];
                        if ((tid & 31) == 0 && row < a.C) bmax[h * CW + (row >> 5)] = bm;
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < H; ++h) atomicMax(&cmax[h], (long long)hmax[h]);
            if (ovf) atomicAdd(&sovf_sm, (unsigned)ovf);
            atomicMax(&maxs_sm, mx);
        }
        __syncthreads();

        // ---- 2. publish the chunk maximum, look back for the incoming one -------
        unsigned long long *flags = a.lb_flag + (int64_t)item * a.max_chunks;
        long long *vals = a.lb_val + (int64_t)item * a.max_chunks * 2 * HMAX;
        if (tid < 32) {
            const int lane = tid;
            if (lane < H) vals[(int64_t)c * 2 * HMAX + lane] = cmax[lane];
            __threadfence();
            __syncwarp();
            if (lane == 0) atomicExch(&flags[c], (a.epoch << 2) | 1ull);
            // Warp-parallel look-back: lane i inspects chunk p_hi - i. Every
            // predecessor up to the nearest one that published an inclusive
            // maximum contributes its (aggregate or inclusive) maximum.
            long long m_in[H];
#pragma unroll
            for (int h = 0; h < H; ++h) m_in[h] = s_lo;
            bool timed_out = false;
            for (int p_hi = c - 1; p_hi >= 0; p_hi -= 32) {
                const int p = p_hi - lane;
                int state = 2;                     // before chunk 0: inclusive of nothing
                if (p >= 0) {
                    unsigned long long f = 0;
                    int it = 0;
                    for (; it < LB_SPIN_LIMIT; ++it) {
                        f = ld_volatile(&flags[p]);
                        if ((f >> 2) == a.epoch && (f & 3ull)) break;
                        __nanosleep(32);
                    }
                    if (it == LB_SPIN_LIMIT) {
                        timed_out = true;
                        f = (a.epoch << 2) | 2ull;  // stop here; the item is recomputed
                    }
                    state = (int)(f & 3ull);
                }
                __threadfence();
                const uint32_t incl = __ballot_sync(FULL, state == 2);
                const int stop = incl ? __ffs(incl) - 1 : 31;
#pragma unroll
                for (int h = 0; h < H; ++h) {
                    long long v = s_lo;
                    if (p >= 0 && lane <= stop)
                        v = ld_volatile(&vals[(int64_t)p * 2 * HMAX + (state == 2 ? HMAX : 0) + h]);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const long long w = __shfl_xor_sync(FULL, v, o);
                        v = w > v ? w : v;
                    }
                    m_in[h] = v > m_in[h] ? v : m_in[h];
                }
                if (__any_sync(FULL, timed_out) || incl) break;
            }
            timed_out = __any_sync(FULL, timed_out);
            if (lane == 0) {
#pragma unroll
                for (int h = 0; h < H; ++h) {
                    m_in_sm[h] = m_in[h];
                    vals[(int64_t)c * 2 * HMAX + HMAX + h] = cmax[h] > m_in[h] ? cmax[h] : m_in[h];
                }
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                atomicExch(&flags[c], (a.epoch << 2) | 2ull);
                if (timed_out) {
                    atomicOr(a.status, ST_TIMEOUT);
                    atomicExch(&a.items[item].fail, 1);
                }
            }
        }
        __syncthreads();

        // ---- 3. the online control, one warp per head -----------------------------
        // Lane b holds 32-row block b. A prefix-max over the block maxima gives the
        // running maximum entering every block. A block whose maximum does not
        // exceed it has no rescale point and one running maximum for all its
        // tokens (p is then computed in the term build). Only the rare blocks
        // that can rescale are scanned token by token here: rescale points
        // (ballot bits), factors exp(s - m_old), p, and their l per segment.
        if (tid < H * 32) {
            const int h = tid >> 5, lane = tid & 31;
            const int nb = (n + 31) / 32;
            const int64_t m_in = m_in_sm[h];
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
                const int64_t st = valid ? s_sm[h * a.C + t] : LLONG_MIN;
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
                if (valid) p_sm[h * a.C + t] = exp_lut32(g, exp_tab, Mt - st);
                // the factor of every rescale point of this block, in order
                const int k = nres + __popc(mask & ((1u << lane) - 1u));
                if (gr && k < SEGMAX) rl_f[h][k] = exp_lut(g, exp_tab, st - Mprev);
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
                atomicAdd(&resc_sm, (unsigned long long)nres);
            }
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
            if (!ok) {
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
        __syncthreads();

        // ---- 4. V: terms per token, summed per segment ---------------------------
        {
            const int ch = tid % D, tg = tid / D;
            constexpr int TG = NT / D;
            int32_t acc[H];
            int cur[H];
            long long bnd[H];
#pragma unroll
            for (int h = 0; h < H; ++h) {
                acc[h] = 0;
                bnd[h] = 0;
            }
            const int bit0 = ch * VB, w0 = bit0 >> 5, sh0 = bit0 & 31;
            const bool straddle = sh0 + VB > 32;
            const uint32_t cmask = (1u << VB) - 1u;
            int64_t cmax_v = 0;
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const int64_t ab = vcent[k] < 0 ? -(int64_t)vcent[k] : vcent[k];
                cmax_v = ab > cmax_v ? ab : cmax_v;
            }
            const uint32_t *vw = vt + w0 * a.C;
            for (int st = 0; st < n; st += SUB) {
                const int ns = min(SUB, n - st);
                // the term table of this sub-tile: [code][t][h], one token per thread
                for (int tl0 = 0; tl0 < ns; tl0 += NT) {
                    const int tl = tl0 + tid;
                    const bool tv = tl < ns;
                    const int t = st + (tv ? tl : 0);
                    const int blkt = t >> 5;
                    const int32_t vnt = tv ? vn_sm[t] : 0;
                    int32_t term[NC][H];
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        // p: from the scan for a block that rescales, else from its
                        // single running maximum
                        const uint32_t gw = grew[h * CW + blkt];
                        const bool quiet = bmax[h * CW + blkt] <= bcar[h * CW + blkt];
                        int32_t pv = 0;
                        if (tv) pv = quiet ? exp_lut32(g, exp_tab, bcar[h * CW + blkt] - s_sm[h * a.C + t])
                                           : p_sm[h * a.C + t];
                        // l of the segment the token belongs to
                        const int seg = gpre[h * CW + blkt] + __popc(gw & ((2u << (t & 31)) - 1u));
                        const int seg0 = __shfl_sync(FULL, seg, 0);
                        if (__all_sync(FULL, seg == seg0)) {
                            unsigned sum = (unsigned)pv;
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(FULL, sum, o);
                            if ((tid & 31) == 0 && sum && seg0 <= SEGMAX)
                                atomicAdd(&lsum_sm[h][seg0], (unsigned long long)sum);
                        } else if (tv && pv && seg <= SEGMAX) {
                            atomicAdd(&lsum_sm[h][seg], (unsigned long long)pv);
                        }
                        const int32_t w = vnt * pv;                    // |w| <= 2^30
#pragma unroll
                        for (int k = 0; k < NC; ++k)
                            term[k][h] = (int32_t)(((int64_t)w * (int64_t)vcent[k]) >> g.acc_shift);
                        // |term| <= floor(|w| * max|c| / 2^acc_shift) + 1 for every code
                        const int64_t aw = w < 0 ? -(int64_t)w : (int64_t)w;
                        bnd[h] += ((aw * cmax_v) >> g.acc_shift) + 1;
                    }
#pragma unroll
                    if (tv)
#pragma unroll
                    for (int k = 0; k < NC; ++k) {
                        int32_t *dst = tab + k * PS + tl * H;
                        if constexpr (H == 4) {
                            *reinterpret_cast<int4 *>(dst) =
                                make_int4(term[k][0], term[k][1], term[k][2], term[k][3]);
                        } else if constexpr (H == 8) {
                            reinterpret_cast<int4 *>(dst)[0] =
                                make_int4(term[k][0], term[k][1], term[k][2], term[k][3]);
                            reinterpret_cast<int4 *>(dst)[1] =
                                make_int4(term[k][4], term[k][5], term[k][6], term[k][7]);
                        } else {
#pragma unroll
                            for (int h = 0; h < H; ++h) dst[h] = term[k][h];
                        }
                    }
                }
                __syncthreads();
                const int per = (ns + TG - 1) / TG;
                const int ta = st + tg * per, tb = min(st + ns, ta + per);
                if (ta < tb) {
#pragma unroll
                    for (int h = 0; h < H; ++h)
                        cur[h] = gpre[h * CW + (ta >> 5)] +
                                 __popc(grew[h * CW + (ta >> 5)] & ((1u << (ta & 31)) - 1u));
                    const int32_t *tab_t = tab - st * H;   // index with t directly
                    int t = ta;
                    while (t < tb) {
                        int nxt = tb;
                        for (int wd = t >> 5; wd <= ((tb - 1) >> 5); ++wd) {
                            uint32_t m = anyg[wd];
                            if (wd == (t >> 5)) m &= ~((1u << (t & 31)) - 1u);
                            if (m) {
                                nxt = min(tb, wd * 32 + __ffs(m) - 1);
                                break;
                            }
                        }
                        auto one = [&](int tt) {
                            uint32_t wv = vw[tt] >> sh0;
                            if (straddle) wv |= vw[a.C + tt] << (32 - sh0);
                            const int32_t *e = tab_t + (int)(wv & cmask) * PS + tt * H;
                            if constexpr (H == 4) {
                                const int4 v4 = *reinterpret_cast<const int4 *>(e);
                                acc[0] += v4.x;
                                acc[1] += v4.y;
                                acc[2] += v4.z;
                                acc[3] += v4.w;
                            } else {
#pragma unroll
                                for (int h = 0; h < H; ++h) acc[h] += e[h];
                            }
                        };
                        for (; t < nxt && (t & 3); ++t) one(t);
                        if constexpr (H == 4 && !(VB == 3)) {
                            for (; t + 4 <= nxt; t += 4) {
                                const uint4 w4 = *reinterpret_cast<const uint4 *>(vw + t);
                                const int32_t *e0 = tab_t + (int)((w4.x >> sh0) & cmask) * PS + t * H;
                                const int32_t *e1 = tab_t + (int)((w4.y >> sh0) & cmask) * PS + (t + 1) * H;
                                const int32_t *e2 = tab_t + (int)((w4.z >> sh0) & cmask) * PS + (t + 2) * H;
                                const int32_t *e3 = tab_t + (int)((w4.w >> sh0) & cmask) * PS + (t + 3) * H;
                                const int4 a0 = *reinterpret_cast<const int4 *>(e0);
                                const int4 a1 = *reinterpret_cast<const int4 *>(e1);
                                const int4 a2 = *reinterpret_cast<const int4 *>(e2);
                                const int4 a3 = *reinterpret_cast<const int4 *>(e3);
                                acc[0] += a0.x + a1.x;
                                acc[1] += a0.y + a1.y;
                                acc[2] += a0.z + a1.z;
                                acc[3] += a0.w + a1.w;
                                acc[0] += a2.x + a3.x;
                                acc[1] += a2.y + a3.y;
                                acc[2] += a2.z + a3.z;
                                acc[3] += a2.w + a3.w;
                            }
                        }
                        for (; t < nxt; ++t) one(t);
                        if (t < tb) {
                            // token t opens a new segment for the heads that grew
#pragma unroll
                            for (int h = 0; h < H; ++h) {
                                if ((grew[h * CW + (t >> 5)] >> (t & 31)) & 1u) {
                                    if (cur[h] == 0) atomicAdd(&s0p[h * D + ch], acc[h]);
                                    else if (seg_ok)
                                        atomicAdd((unsigned long long *)&a.segs[segbase_sm[h] + cur[h] - 1].S[ch],
                                                  (unsigned long long)(long long)acc[h]);
                                    acc[h] = 0;
                                    ++cur[h];
                                }
                            }
                            one(t);
                            ++t;
                        }
                    }
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        if (acc[h]) {
                            if (cur[h] == 0) atomicAdd(&s0p[h * D + ch], acc[h]);
                            else if (seg_ok)
                                atomicAdd((unsigned long long *)&a.segs[segbase_sm[h] + cur[h] - 1].S[ch],
                                          (unsigned long long)(long long)acc[h]);
                        }
                        acc[h] = 0;
                    }
                }
                __syncthreads();
            }
#pragma unroll
            for (int h = 0; h < H; ++h) {
                unsigned long long v = (unsigned long long)bnd[h];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
                if ((tid & 31) == 0 && v) atomicAdd((unsigned long long *)&bsum_sm[h], v);
            }
        }
        __syncthreads();
        // l of the rescale segments, now that the build has summed p
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
                rec.B[h] = bsum_sm[h];
                rec.nseg[h] = seg_ok ? nseg_sm[h] : 0;
                rec.seg_base[h] = segbase_sm[h];
            }
            if (tid == 0) {
                ItemAcc &ia = a.items[item];
                atomicAdd(&ia.resc, resc_sm);
                atomicAdd(&ia.sovf, (unsigned long long)sovf_sm);
                atomicMax(&ia.maxs, maxs_sm);
            }
        }
        __threadfence();
        __syncthreads();

        // ---- 6. fold: the last chunk of a block folds the block, the last block
        //         of an item folds the item ---------------------------------------
        const int nc = a.item_nchunks[item];
        const int blk = c / GBLK;
        const int nblk = (nc + GBLK - 1) / GBLK;
        const int in_blk = min(nc, blk * GBLK + GBLK) - blk * GBLK;
        if (tid == 0) {
            const unsigned old = atomicAdd(&a.blk_done[(int64_t)item * a.max_blocks + blk], 1u);
            flag_sm = old + 1 == (unsigned)in_blk;
        }
        __syncthreads();
        if (flag_sm) {
            __threadfence();
            merge_block<H>(a, item, blk, nc, base_sm);
            __threadfence();
            __syncthreads();
            if (tid == 0) {
                a.blk_done[(int64_t)item * a.max_blocks + blk] = 0;
                const unsigned long long old = atomicAdd(&a.items[item].done_blocks, 1ull);
                flag_sm = old + 1 == (unsigned long long)nblk;
            }
            __syncthreads();
            if (flag_sm) {
                __threadfence();
                merge_item<H>(a, item, nblk, a.T[b], qbase, &maxs_sm);
                __syncthreads();
                if (tid == 0) {
                    ItemAcc &ia = a.items[item];
                    ia.done_blocks = 0;
                    ia.resc = 0;
                    ia.sovf = 0;
                    ia.maxs = 0;
                    ia.fail = 0;
                }
            }
        }
        // ---- 7. the last tile of the launch resets the pool ----------------------
        if (tid == 0) {
            __threadfence();
            const unsigned long long d = atomicAdd(a.all_done, 1ull);
            if (d + 1 == (unsigned long long)a.n_tiles) {
                *a.seg_top = 0;
                *a.all_done = 0;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// host side: the tile list, the scratch, the launch
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
    fn<<<B * g.n_kv, H * 64, smem, s>>>(g, tb, d_seq, d_lens, d_pt, pool, q_rot, out, stats, only);
    return cudaGetLastError();
}

// Rows per chunk: as many whole pages as fit the layout's smem budget, at most 1024.
template <int H, int VB>
inline int chunk_rows(const Geo &g, size_t smem_cap) {
    int pages = 1024 / g.P;
    if (pages < 1) pages = 1;
    while (pages > 1 && ChunkLayout<H, VB>(pages * g.P).total > smem_cap) --pages;
    return pages * g.P;
}

// The tile list: every item's chunks, in (chunk, item) order so a chunk is
// always claimed after all of its predecessors.
inline void build_tiles(const Geo &g, int32_t B, const int64_t *h_T, int C, std::vector<int4> &tiles,
                        std::vector<int32_t> &nc, int &max_nc) {
    const int n_items = B * g.n_kv;
    nc.assign(n_items, 1);
    max_nc = 1;
    for (int it = 0; it < n_items; ++it) {
        const int64_t T = h_T[it / g.n_kv];
        nc[it] = T ? (int)((T + C - 1) / C) : 1;
        max_nc = nc[it] > max_nc ? nc[it] : max_nc;
    }
    tiles.clear();
    for (int cidx = 0; cidx < max_nc; ++cidx)
        for (int it = 0; it < n_items; ++it)
            if (cidx < nc[it]) {
                const int64_t T = h_T[it / g.n_kv];
                const int64_t t0 = (int64_t)cidx * C;
                tiles.push_back(make_int4(it, cidx, (int)t0, (int)(T - t0 < C ? T - t0 : C)));
            }
}

// Carve (or grow) the scratch for n_items items of up to max_nc chunks.
inline int reserve_scratch(ChunkScratch &cs, int n_items, int max_nc, int n_tiles, int H,
                           cudaStream_t s) {
    const int seg_cap = 2 * (64 * n_items * H) + 4 * n_tiles;
    if (cs.base && n_items <= cs.n_items && max_nc <= cs.max_chunks && seg_cap <= cs.seg_cap &&
        n_tiles <= cs.tile_cap)
        return INS_OK;
    cudaStreamSynchronize(s);
    const int ni = n_items > cs.n_items ? n_items : cs.n_items;
    const int mc = max_nc > cs.max_chunks ? max_nc : cs.max_chunks;
    const int sc = seg_cap > cs.seg_cap ? seg_cap : cs.seg_cap;
    const int tc = n_tiles > cs.tile_cap ? n_tiles : cs.tile_cap;
    const int mb = (mc + GBLK - 1) / GBLK;
    cs.release();
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o = 0;
    const size_t o_claim = o; o += al(8);
    const size_t o_all = o; o += al(8);
    const size_t o_top = o; o += al(8);
    const size_t o_flag = o; o += al(sizeof(unsigned long long) * (size_t)ni * mc);
    const size_t o_val = o; o += al(sizeof(long long) * (size_t)ni * mc * 2 * HMAX);
    const size_t o_rec = o; o += al(sizeof(ChunkRec) * (size_t)ni * mc);
    const size_t o_blk = o; o += al(sizeof(BlockRec) * (size_t)ni * mb);
    const size_t o_bd = o; o += al(sizeof(unsigned int) * (size_t)ni * mb);
    const size_t o_seg = o; o += al(sizeof(SegEntry) * (size_t)sc);
    const size_t o_items = o; o += al(sizeof(ItemAcc) * (size_t)ni);
    const size_t o_redo = o; o += al(sizeof(int32_t) * (size_t)ni);
    const size_t o_tiles = o; o += al(sizeof(int4) * (size_t)tc);
    const size_t o_nc = o; o += al(sizeof(int32_t) * (size_t)ni);
    if (cudaMalloc(&cs.base, o) != cudaSuccess) {
        cudaGetLastError();
        cs.base = nullptr;
        return INS_ENOMEM;
    }
    if (cudaMemset(cs.base, 0, o) != cudaSuccess) return INS_ECUDA;
    uint8_t *p = (uint8_t *)cs.base;
    cs.bytes = o;
    cs.claim = (unsigned long long *)(p + o_claim);
    cs.all_done = (unsigned long long *)(p + o_all);
    cs.seg_top = (unsigned int *)(p + o_top);
    cs.lb_flag = (unsigned long long *)(p + o_flag);
    cs.lb_val = (long long *)(p + o_val);
    cs.recs = (ChunkRec *)(p + o_rec);
    cs.blks = (BlockRec *)(p + o_blk);
    cs.blk_done = (unsigned int *)(p + o_bd);
    cs.segs = (SegEntry *)(p + o_seg);
    cs.items = (ItemAcc *)(p + o_items);
    cs.redo = (int32_t *)(p + o_redo);
    cs.tiles = (int4 *)(p + o_tiles);
    cs.item_nchunks = (int32_t *)(p + o_nc);
    cs.n_items = ni;
    cs.max_chunks = mc;
    cs.seg_cap = sc;
    cs.tile_cap = tc;
    cs.claim_base = 0;
    return INS_OK;
}

template <int H, int KB, int VB>
inline int launch_chunked(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                          const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                          const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                          int64_t *out, ins_stats *stats, int32_t *d_status, cudaStream_t s) {
    const int n_items = B * g.n_kv;
    const int C = chunk_rows<H, VB>(g, 100 * 1024);
    const ChunkLayout<H, VB> lay(C);
    std::vector<int4> tiles;
    std::vector<int32_t> nc;
    int max_nc = 1;
    build_tiles(g, B, h_T, C, tiles, nc, max_nc);
    const int n_tiles = (int)tiles.size();
    if (int rc = reserve_scratch(cs, n_items, max_nc, n_tiles, H, s)) return rc;
    if (cudaMemcpyAsync(cs.tiles, tiles.data(), sizeof(int4) * tiles.size(), cudaMemcpyHostToDevice,
                        s) != cudaSuccess ||
        cudaMemcpyAsync(cs.item_nchunks, nc.data(), sizeof(int32_t) * nc.size(),
                        cudaMemcpyHostToDevice, s) != cudaSuccess)
        return INS_ECUDA;
    auto fn = k_scan_chunk<H, KB, VB>;
    const size_t dyn = lay.total;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess)
        return INS_ECUDA;
    constexpr int NT = H * 64 > 256 ? H * 64 : 256;
    int per_sm = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, NT, dyn);
    if (per_sm < 1) per_sm = 1;
    int grid = per_sm * sms;
    if (grid > n_tiles) grid = n_tiles;
    ChunkArgs a{};
    a.g = g;
    a.tb = tb;
    a.tiles = cs.tiles;
    a.n_tiles = n_tiles;
    a.C = C;
    a.max_chunks = cs.max_chunks;
    a.max_blocks = (cs.max_chunks + GBLK - 1) / GBLK;
    a.n_items = n_items;
    a.item_nchunks = cs.item_nchunks;
    a.seq_ids = d_seq;
    a.T = d_T;
    a.page_table = d_pt;
    a.pool = pool;
    a.q_rot = q_rot;
    a.out = out;
    a.stats = stats;
    a.claim = cs.claim;
    a.claim_base = cs.claim_base;
    a.lb_flag = cs.lb_flag;
    a.lb_val = cs.lb_val;
    a.recs = cs.recs;
    a.blks = cs.blks;
    a.blk_done = cs.blk_done;
    a.segs = cs.segs;
    a.seg_top = cs.seg_top;
    a.seg_cap = cs.seg_cap;
    a.items = cs.items;
    a.redo = cs.redo;
    a.all_done = cs.all_done;
    a.status = d_status;
    a.epoch = ++cs.epoch;
    fn<<<grid, NT, dyn, s>>>(a);
    // every tile claim and every CTA's final failing claim bump the counter once
    cs.claim_base += (unsigned long long)n_tiles + (unsigned long long)grid;
    if (cudaGetLastError() != cudaSuccess) return INS_ECUDA;
    // items whose exactness the fold could not prove are recomputed in order
    return launch_seq<H>(g, tb, B, d_seq, d_T, d_pt, pool, q_rot, out, stats, cs.redo, s) ==
                   cudaSuccess
               ? INS_OK
               : INS_ECUDA;
}

inline int launch_online(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                         const int32_t *d_seq, const int64_t *d_lens, const int64_t *h_lens,
                         const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                         int64_t *out, ins_stats *stats, int32_t *d_status, int H,
                         cudaStream_t s) {
#define INS_CH(HH, KK, VV)                                                                 \
    return launch_chunked<HH, KK, VV>(cs, g, tb, B, d_seq, d_lens, h_lens, d_pt, pool, q_rot, \
                                      out, stats, d_status, s)
    if (g.kb == 4 && g.vb == 2) {
        switch (H) {
            case 1: INS_CH(1, 4, 2);
            case 2: INS_CH(2, 4, 2);
            case 4: INS_CH(4, 4, 2);
            case 8: INS_CH(8, 4, 2);
        }
    }
    if (g.kb == 3 && g.vb == 3) {
        switch (H) {
            case 4: INS_CH(4, 3, 3);
            case 8: INS_CH(8, 3, 3);
        }
    }
#undef INS_CH
    cudaError_t e = cudaErrorInvalidValue;
    switch (H) {
        case 1: e = launch_seq<1>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 2: e = launch_seq<2>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 4: e = launch_seq<4>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 8: e = launch_seq<8>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
    }
    return e == cudaSuccess ? INS_OK : INS_ECUDA;
}

}  // namespace ins
