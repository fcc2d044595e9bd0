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
constexpr int SEGMAX = 32;               // rescales of one head one chunk can hold

struct SegEntry {          // one rescale segment of one head in one chunk
    int32_t S[D];          // sum of terms from the rescale token to the segment end
    int64_t l;             // sum of p over the same tokens
    int32_t f;             // the factor applied to acc and l before this segment
    int32_t tok;
};

struct ChunkRec {          // one (item, chunk)
    int32_t S0[HMAX][D];   // terms of the tokens before the chunk's first rescale
    int64_t l0[HMAX];
    int64_t B[HMAX];       // sum over tokens of max over codes of |term|
    int32_t nseg[HMAX];
    int32_t seg_base[HMAX];
};

struct ItemAcc {
    unsigned long long done;
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
    SegEntry *segs;
    unsigned int *seg_top;
    int32_t seg_cap;
    ItemAcc *items;               // [n_items]
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
    int32_t n_items = 0, max_chunks = 0, seg_cap = 0;
    unsigned long long epoch = 0;
    unsigned long long claim_base = 0;
    // carved views
    unsigned long long *claim = nullptr, *lb_flag = nullptr, *all_done = nullptr;
    long long *lb_val = nullptr;
    ChunkRec *recs = nullptr;
    SegEntry *segs = nullptr;
    unsigned int *seg_top = nullptr;
    ItemAcc *items = nullptr;
    int4 *tiles = nullptr;
    int32_t *item_nchunks = nullptr;
    int32_t tile_cap = 0;

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
    static constexpr int VW = 2 * VB;                     // 32-bit words per V row
    int C;
    size_t off_s, off_p, off_vt, off_vn, off_tab, off_grew, off_any, off_s0, total;
    __host__ __device__ explicit ChunkLayout(int C_) : C(C_) {
        size_t o = 0;
        off_s = o;    o += (size_t)H * C * 8;             // scores (int64)
        off_p = o;    o += (size_t)H * C * 4;             // p (int32)
        off_vt = o;   o += (size_t)VW * C * 4;            // V codes, word-major
        off_vn = o;   o += (size_t)C * 4;                 // v_norm (int32)
        off_tab = o;  o += (size_t)SUB * NC * H * 4;      // terms [t][code][h]
        off_grew = o; o += (size_t)H * (C / 32) * 4;      // rescale bitmask per head
        off_any = o;  o += (size_t)(C / 32) * 4;          // any head
        off_s0 = o;   o += (size_t)H * D * 4;             // segment-0 partials
        total = o;
    }
};

// Scores of R rows for one thread (register-blocked over rows), exact.
template <int H, int KB, int R>
__device__ __forceinline__ void score_rows(const Geo &g, const uint8_t *const *krow,
                                           const int64_t *knorm, const bool *valid,
                                           const double *__restrict__ qd,
                                           const uint32_t *__restrict__ khi, int64_t (*s)[H],
                                           int &ovf) {
    constexpr int NW = 2 * KB;                 // 32-bit words of K codes per row
    uint32_t w[R][NW];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint2 *src = reinterpret_cast<const uint2 *>(krow[r]);
#pragma unroll
        for (int i = 0; i < KB; ++i) {
            uint2 x = valid[r] ? src[i] : make_uint2(0u, 0u);
            w[r][2 * i] = x.x;
            w[r][2 * i + 1] = x.y;
        }
    }
    double acc[R][H];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int h = 0; h < H; ++h) acc[r][h] = 0.0;
#pragma unroll
    for (int j = 0; j < D; ++j) {
        double c[R];
#pragma unroll
        for (int r = 0; r < R; ++r) c[r] = __hiloint2double((int)khi[code_at<KB>(w[r], j, KB)], 0);
#pragma unroll
        for (int h = 0; h < H; ++h) {
            const double qv = qd[h * D + j];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][h] = fma(qv, c[r], acc[r][h]);
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

__device__ __forceinline__ int64_t ld_volatile(const long long *p) {
    return *reinterpret_cast<const volatile long long *>(p);
}
__device__ __forceinline__ unsigned long long ld_volatile(const unsigned long long *p) {
    return *reinterpret_cast<const volatile unsigned long long *>(p);
}

template <int H, int KB, int VB>
__global__ void __launch_bounds__(H * 64 > 256 ? H * 64 : 256, H * 64 > 256 ? 1 : 2)
    k_scan_chunk(ChunkArgs a) {
    using L = ChunkLayout<H, VB>;
    constexpr int NC = L::NC, SUB = L::SUB, VW = L::VW;
    constexpr int NT = H * 64 > 256 ? H * 64 : 256;
    constexpr int R = 4;                             // rows per thread in the score phase
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ SeqSmem<H> seqsm;                     // the fallback's own state
    __shared__ double qd[H * D];
    __shared__ uint32_t khi[256];
    __shared__ int32_t vcent[256];
    __shared__ int32_t exp_tab[256];
    __shared__ long long cmax[H], m_in_sm[H];
    __shared__ int tile_sm, merge_sm, fail_sm;
    __shared__ int nseg_sm[H], segbase_sm[H];
    __shared__ unsigned long long lsum_sm[H][SEGMAX + 1];
    __shared__ long long bsum_sm[H];
    __shared__ unsigned long long resc_sm;
    __shared__ unsigned int sovf_sm;
    __shared__ long long maxs_sm;
    __shared__ const uint8_t *page_sm[8];

    const Geo &g = a.g;
    const int tid = threadIdx.x;
    const L lay(a.C);
    int64_t *s_sm = reinterpret_cast<int64_t *>(dyn + lay.off_s);
    int32_t *p_sm = reinterpret_cast<int32_t *>(dyn + lay.off_p);
    uint32_t *vt = reinterpret_cast<uint32_t *>(dyn + lay.off_vt);
    int32_t *vn_sm = reinterpret_cast<int32_t *>(dyn + lay.off_vn);
    int32_t *tab = reinterpret_cast<int32_t *>(dyn + lay.off_tab);
    uint32_t *grew = reinterpret_cast<uint32_t *>(dyn + lay.off_grew);
    uint32_t *anyg = reinterpret_cast<uint32_t *>(dyn + lay.off_any);
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
        for (int i = tid; i < H * (a.C / 32); i += NT) grew[i] = 0;
        for (int i = tid; i < a.C / 32; i += NT) anyg[i] = 0;
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
                    if (!valid[r]) continue;
                    const int row = base + r * NT + tid;
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        s_sm[h * a.C + row] = s[r][h];
                        hmax[h] = s[r][h] > hmax[h] ? s[r][h] : hmax[h];
                        const long long ab = s[r][h] < 0 ? -s[r][h] : s[r][h];
                        mx = ab > mx ? ab : mx;
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
            long long m_in = s_lo;
            bool timed_out = false;
            for (int p = c - 1; p >= 0; --p) {
                unsigned long long f = 0;
                int it = 0;
                for (; it < LB_SPIN_LIMIT; ++it) {
                    f = ld_volatile(&flags[p]);
                    if ((f >> 2) == a.epoch && (f & 3ull)) break;
                    __nanosleep(64);
                }
                if (it == LB_SPIN_LIMIT) {
                    timed_out = true;
                    break;
                }
                __threadfence();
                const bool incl = (f & 3ull) == 2ull;
                if (lane < H) {
                    const long long v = ld_volatile(&vals[(int64_t)p * 2 * HMAX + (incl ? HMAX : 0) + lane]);
                    m_in = v > m_in ? v : m_in;
                }
                if (incl) break;
            }
            if (lane < H) {
                m_in_sm[lane] = m_in;
                const long long inc = cmax[lane] > m_in ? cmax[lane] : m_in;
                vals[(int64_t)c * 2 * HMAX + HMAX + lane] = inc;
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

        // ---- 3. the online control: running max, rescale points, p ---------------
        if (tid < H * 32) {
            const int h = tid >> 5, lane = tid & 31;
            const int64_t *s = s_sm + h * a.C;
            const int per = (n + 31) / 32;
            const int ta = lane * per, tb = min(n, ta + per);
            int64_t lmax = LLONG_MIN;
            for (int t = ta; t < tb; ++t) lmax = s[t] > lmax ? s[t] : lmax;
            int64_t incl = lmax;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int64_t o = __shfl_up_sync(FULL, incl, off);
                if (lane >= off) incl = o > incl ? o : incl;
            }
            int64_t excl = __shfl_up_sync(FULL, incl, 1);
            const int64_t m_in = m_in_sm[h];
            if (lane == 0) excl = LLONG_MIN;
            int64_t run = excl > m_in ? excl : m_in;
            int cnt = 0;
            unsigned long long lpart = 0;
            for (int t = ta; t < tb; ++t) {
                const int64_t st = s[t];
                if (st > run) {
                    run = st;
                    ++cnt;
                    atomicOr(&grew[h * (a.C / 32) + (t >> 5)], 1u << (t & 31));
                    atomicOr(&anyg[t >> 5], 1u << (t & 31));
                }
                const int32_t pv = exp_lut(g, exp_tab, run - st);
                p_sm[h * a.C + t] = pv;
                lpart += (unsigned long long)pv;
            }
            // segment index of this lane's first token = rescales before it
            int before = cnt;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(FULL, before, off);
                if (lane >= off) before += o;
            }
            before -= cnt;
            const int total = __shfl_sync(FULL, before + cnt, 31);
            __syncwarp();
            if (cnt == 0) {
                if (lpart && before <= SEGMAX) atomicAdd(&lsum_sm[h][before], lpart);
            } else {
                // a lane whose range holds a rescale splits its sum per segment
                int seg = before;
                int64_t rr = run;  // recompute the walk to split at rescale points
                rr = excl > m_in ? excl : m_in;
                unsigned long long acc = 0;
                for (int t = ta; t < tb; ++t) {
                    if (s[t] > rr) {
                        if (seg <= SEGMAX && acc) atomicAdd(&lsum_sm[h][seg], acc);
                        acc = 0;
                        ++seg;
                        rr = s[t];
                    }
                    acc += (unsigned long long)p_sm[h * a.C + t];
                }
                if (seg <= SEGMAX && acc) atomicAdd(&lsum_sm[h][seg], acc);
            }
            if (lane == 0) {
                nseg_sm[h] = total;
                atomicAdd(&resc_sm, (unsigned long long)total);
            }
        }
        __syncthreads();

        // segment slots in the pool, zeroed for the atomic partial sums
        if (tid == 0) {
            int need = 0;
            for (int h = 0; h < H; ++h) need += nseg_sm[h];
            bool ok = true;
            for (int h = 0; h < H; ++h) ok &= nseg_sm[h] <= SEGMAX;
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
                acc += nseg_sm[h];
            }
        }
        __syncthreads();
        const bool seg_ok = !fail_sm;
        if (seg_ok) {
            for (int h = 0; h < H; ++h)
                for (int k = 0; k < nseg_sm[h]; ++k) {
                    SegEntry &e = a.segs[segbase_sm[h] + k];
                    for (int i = tid; i < D; i += NT) e.S[i] = 0;
                }
        }
        __syncthreads();

        // ---- 4. V: terms per token, summed per segment ---------------------------
        {
            const int ch = tid % D, tg = tid / D;
            constexpr int TG = NT / D;
            int32_t acc[H];
            int cur[H];
#pragma unroll
            for (int h = 0; h < H; ++h) acc[h] = 0;
            long long bnd[H];
#pragma unroll
            for (int h = 0; h < H; ++h) bnd[h] = 0;
            // where this thread's channel sits in a V row
            const int bit0 = ch * VB, w0 = bit0 >> 5, sh0 = bit0 & 31;
            const bool straddle = sh0 + VB > 32;
            for (int st = 0; st < n; st += SUB) {
                const int ns = min(SUB, n - st);
                // build the term table of this sub-tile: [t][code][h]
                for (int tl = tid; tl < ns; tl += NT) {
                    const int t = st + tl;
                    const int64_t vnt = vn_sm[t];
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        const int64_t w = vnt * (int64_t)p_sm[h * a.C + t];
                        int64_t mxk = 0;
#pragma unroll
                        for (int k = 0; k < NC; ++k) {
                            const int64_t term = (w * (int64_t)vcent[k]) >> g.acc_shift;
                            tab[(tl * NC + k) * H + h] = (int32_t)term;
                            const int64_t ab = term < 0 ? -term : term;
                            mxk = ab > mxk ? ab : mxk;
                        }
                        bnd[h] += mxk;
                    }
                }
                __syncthreads();
                // this thread's tokens of the sub-tile
                const int per = (ns + TG - 1) / TG;
                const int ta = st + tg * per, tb = min(st + ns, ta + per);
                if (ta < tb) {
                    // segment of each head at ta
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        int k = 0;
                        for (int wd = 0; wd < (ta >> 5); ++wd) k += __popc(grew[h * (a.C / 32) + wd]);
                        k += __popc(grew[h * (a.C / 32) + (ta >> 5)] & ((1u << (ta & 31)) - 1u));
                        cur[h] = k;
                    }
                    int t = ta;
                    while (t < tb) {
                        // next token in [t, tb) where some head rescales
                        int nxt = tb;
                        for (int wd = t >> 5; wd <= ((tb - 1) >> 5); ++wd) {
                            uint32_t m = anyg[wd];
                            if (wd == (t >> 5)) m &= ~((1u << (t & 31)) - 1u);
                            if (m) {
                                nxt = min(tb, wd * 32 + __ffs(m) - 1);
                                break;
                            }
                        }
                        for (; t < nxt; ++t) {
                            uint32_t wv = vt[w0 * a.C + t] >> sh0;
                            if (straddle) wv |= vt[(w0 + 1) * a.C + t] << (32 - sh0);
                            const int code = (int)(wv & ((1u << VB) - 1u));
                            const int32_t *tt = tab + ((t - st) * NC + code) * H;
                            if constexpr (H == 4) {
                                const int4 v4 = *reinterpret_cast<const int4 *>(tt);
                                acc[0] += v4.x;
                                acc[1] += v4.y;
                                acc[2] += v4.z;
                                acc[3] += v4.w;
                            } else {
#pragma unroll
                                for (int h = 0; h < H; ++h) acc[h] += tt[h];
                            }
                        }
                        if (t < tb) {
                            // token t starts a new segment for the heads that grew
#pragma unroll
                            for (int h = 0; h < H; ++h) {
                                if ((grew[h * (a.C / 32) + (t >> 5)] >> (t & 31)) & 1u) {
                                    if (cur[h] == 0) atomicAdd(&s0p[h * D + ch], acc[h]);
                                    else if (seg_ok)
                                        atomicAdd(&a.segs[segbase_sm[h] + cur[h] - 1].S[ch], acc[h]);
                                    acc[h] = 0;
                                    ++cur[h];
                                }
                            }
                            uint32_t wv = vt[w0 * a.C + t] >> sh0;
                            if (straddle) wv |= vt[(w0 + 1) * a.C + t] << (32 - sh0);
                            const int code = (int)(wv & ((1u << VB) - 1u));
                            const int32_t *tt = tab + ((t - st) * NC + code) * H;
#pragma unroll
                            for (int h = 0; h < H; ++h) acc[h] += tt[h];
                            ++t;
                        }
                    }
                    // flush to the segment each head ended the range in
#pragma unroll
                    for (int h = 0; h < H; ++h) {
                        if (acc[h]) {
                            if (cur[h] == 0) atomicAdd(&s0p[h * D + ch], acc[h]);
                            else if (seg_ok)
                                atomicAdd(&a.segs[segbase_sm[h] + cur[h] - 1].S[ch], acc[h]);
                        }
                        acc[h] = 0;
                    }
                }
                __syncthreads();
            }
#pragma unroll
            for (int h = 0; h < H; ++h)
                if (bnd[h]) atomicAdd((unsigned long long *)&bsum_sm[h], (unsigned long long)bnd[h]);
        }
        __syncthreads();

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
                if (seg_ok) {
                    // factors and l sums of the rescale segments
                    const int64_t *s = s_sm + h * a.C;
                    int64_t prev = m_in_sm[h];
                    int k = 0;
                    for (int wd = 0; wd < (n + 31) / 32 && k < nseg_sm[h]; ++wd) {
                        uint32_t m = grew[h * (a.C / 32) + wd];
                        while (m) {
                            const int t = wd * 32 + __ffs(m) - 1;
                            m &= m - 1;
                            SegEntry &e = a.segs[segbase_sm[h] + k];
                            e.f = exp_lut(g, exp_tab, s[t] - prev);
                            e.tok = t;
                            e.l = (int64_t)lsum_sm[h][k + 1];
                            prev = s[t];
                            ++k;
                        }
                    }
                }
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

        // ---- 6. the last chunk of an item folds the item --------------------------
        if (tid == 0) {
            const unsigned long long old = atomicAdd(&a.items[item].done, 1ull);
            merge_sm = old + 1 == (unsigned long long)a.item_nchunks[item];
        }
        __syncthreads();
        if (merge_sm) {
            __threadfence();
            const int nc = a.item_nchunks[item];
            const int64_t T = a.T[b];
            bool bad = *reinterpret_cast<volatile int32_t *>(&a.items[item].fail) != 0;
            int64_t acc_k[(H * D + NT - 1) / NT];
            int64_t l_k[(H * D + NT - 1) / NT];
            constexpr int KK = (H * D + NT - 1) / NT;
#pragma unroll
            for (int k = 0; k < KK; ++k) acc_k[k] = l_k[k] = 0;
            if (!bad) {
                const ChunkRec *recs = a.recs + (int64_t)item * a.max_chunks;
                for (int cc = 0; cc < nc; ++cc) {
                    const ChunkRec &rec = recs[cc];
#pragma unroll
                    for (int k = 0; k < KK; ++k) {
                        const int i = tid + k * NT;
                        if (i >= H * D) continue;
                        const int h = i / D, ch = i % D;
                        const int64_t ab = acc_k[k] < 0 ? -acc_k[k] : acc_k[k];
                        if (ab + *reinterpret_cast<const volatile int64_t *>(&rec.B[h]) > INT32_MAX) bad = true;
                        acc_k[k] += *reinterpret_cast<const volatile int32_t *>(&rec.S0[h][ch]);
                        l_k[k] += *reinterpret_cast<const volatile int64_t *>(&rec.l0[h]);
                        const int ns = *reinterpret_cast<const volatile int32_t *>(&rec.nseg[h]);
                        const int sb = *reinterpret_cast<const volatile int32_t *>(&rec.seg_base[h]);
                        for (int e = 0; e < ns; ++e) {
                            const SegEntry &se = a.segs[sb + e];
                            const int64_t f = *reinterpret_cast<const volatile int32_t *>(&se.f);
                            acc_k[k] = (acc_k[k] * f) >> g.prob_frac;
                            l_k[k] = (l_k[k] * f) >> g.prob_frac;
                            acc_k[k] += *reinterpret_cast<const volatile int32_t *>(&se.S[ch]);
                            l_k[k] += *reinterpret_cast<const volatile int64_t *>(&se.l);
                        }
                    }
                }
            }
            bad = __syncthreads_or(bad);
            int64_t *out_row = a.out + qbase;
            ins_stats *st_out = a.stats ? a.stats + item : nullptr;
            if (bad) {
                seq_scan_item<H, KB, VB>(g, a.tb, seq, T, kvh, a.page_table, a.pool,
                                         a.q_rot + qbase, out_row, st_out, seqsm, dyn);
            } else {
                long long mx = 0;
#pragma unroll
                for (int k = 0; k < KK; ++k) {
                    const int i = tid + k * NT;
                    if (i >= H * D) continue;
                    int64_t r;
                    int shift;
                    reciprocal(g, l_k[k], r, shift);
                    out_row[i] = (acc_k[k] * r) >> shift;
                    const long long ab = acc_k[k] < 0 ? -acc_k[k] : acc_k[k];
                    mx = ab > mx ? ab : mx;
                }
                if (tid == 0) maxs_sm = 0;
                __syncthreads();
                atomicMax(&maxs_sm, mx);
                __syncthreads();
                if (tid == 0 && st_out) {
                    const volatile ItemAcc &ia = a.items[item];
                    ins_stats st;
                    st.n_tokens = T;
                    st.rescale_events = (int64_t)ia.resc;
                    st.score_overflows = (int64_t)ia.sovf;
                    st.acc_overflows = 0;
                    st.max_abs_score = ia.maxs;
                    st.max_abs_acc = maxs_sm;
                    *st_out = st;
                }
            }
            __syncthreads();
            if (tid == 0) {
                ItemAcc &ia = a.items[item];
                ia.done = 0;
                ia.resc = 0;
                ia.sovf = 0;
                ia.maxs = 0;
                ia.fail = 0;
            }
        }
        // ---- 7. the last tile of the launch resets the shared counters ------------
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

template <int H, int KB, int VB>
inline int launch_chunked(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                          const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                          const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                          int64_t *out, ins_stats *stats, int32_t *d_status, cudaStream_t s) {
    const int n_items = B * g.n_kv;
    const size_t smem_cap = 100 * 1024;
    const int C = chunk_rows<H, VB>(g, smem_cap);
    const ChunkLayout<H, VB> lay(C);
    size_t dyn = lay.total;
    const size_t seqdyn = seq_dyn_smem<H>(g);
    if (seqdyn > dyn) dyn = seqdyn;
    // tiles in (chunk, item) order, so a chunk is always claimed after its predecessors
    int max_nc = 1;
    std::vector<int> nc(n_items);
    for (int it = 0; it < n_items; ++it) {
        const int64_t T = h_T[it / g.n_kv];
        nc[it] = T ? (int)((T + C - 1) / C) : 1;
        max_nc = nc[it] > max_nc ? nc[it] : max_nc;
    }
    std::vector<int4> tiles;
    tiles.reserve((size_t)n_items * 2);
    for (int cidx = 0; cidx < max_nc; ++cidx)
        for (int it = 0; it < n_items; ++it)
            if (cidx < nc[it]) {
                const int64_t T = h_T[it / g.n_kv];
                const int64_t t0 = (int64_t)cidx * C;
                tiles.push_back(make_int4(it, cidx, (int)t0, (int)(T - t0 < C ? T - t0 : C)));
            }
    const int n_tiles = (int)tiles.size();
    // scratch
    const int seg_cap = 64 * n_items * H + 4 * n_tiles;
    const bool grow = !cs.base || n_items > cs.n_items || max_nc > cs.max_chunks ||
                      seg_cap > cs.seg_cap || n_tiles > cs.tile_cap;
    if (grow) {
        cudaStreamSynchronize(s);
        const int ni = n_items > cs.n_items ? n_items : cs.n_items;
        const int mc = max_nc > cs.max_chunks ? max_nc : cs.max_chunks;
        const int sc = seg_cap > cs.seg_cap ? seg_cap : cs.seg_cap;
        const int tc = n_tiles > cs.tile_cap ? n_tiles : cs.tile_cap;
        cs.release();
        auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
        size_t o = 0;
        const size_t o_claim = o; o += al(8);
        const size_t o_all = o; o += al(8);
        const size_t o_top = o; o += al(8);
        const size_t o_flag = o; o += al(sizeof(unsigned long long) * (size_t)ni * mc);
        const size_t o_val = o; o += al(sizeof(long long) * (size_t)ni * mc * 2 * HMAX);
        const size_t o_rec = o; o += al(sizeof(ChunkRec) * (size_t)ni * mc);
        const size_t o_seg = o; o += al(sizeof(SegEntry) * (size_t)sc);
        const size_t o_items = o; o += al(sizeof(ItemAcc) * (size_t)ni);
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
        cs.segs = (SegEntry *)(p + o_seg);
        cs.items = (ItemAcc *)(p + o_items);
        cs.tiles = (int4 *)(p + o_tiles);
        cs.item_nchunks = (int32_t *)(p + o_nc);
        cs.n_items = ni;
        cs.max_chunks = mc;
        cs.seg_cap = sc;
        cs.tile_cap = tc;
        cs.claim_base = 0;
    }
    if (cudaMemcpyAsync(cs.tiles, tiles.data(), sizeof(int4) * tiles.size(), cudaMemcpyHostToDevice,
                        s) != cudaSuccess ||
        cudaMemcpyAsync(cs.item_nchunks, nc.data(), sizeof(int32_t) * nc.size(),
                        cudaMemcpyHostToDevice, s) != cudaSuccess)
        return INS_ECUDA;
    auto fn = k_scan_chunk<H, KB, VB>;
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
    a.segs = cs.segs;
    a.seg_top = cs.seg_top;
    a.seg_cap = cs.seg_cap;
    a.items = cs.items;
    a.all_done = cs.all_done;
    a.status = d_status;
    a.epoch = ++cs.epoch;
    fn<<<grid, NT, dyn, s>>>(a);
    // every tile claim and every CTA's final failing claim bump the counter once
    cs.claim_base += (unsigned long long)n_tiles + (unsigned long long)grid;
    return cudaGetLastError() == cudaSuccess ? INS_OK : INS_ECUDA;
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
