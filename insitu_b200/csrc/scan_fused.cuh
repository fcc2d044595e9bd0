// The online scan in one launch.
//
// The context-parallel scan of scan_chunked.cuh as a single persistent kernel.
// Every CTA walks its tiles (tile blockIdx.x + li * gridDim.x, chunk-major as
// before) and, for each li, runs two phases:
//
//   values(li - 1)  the V side of the tile it scored one step earlier: V rows,
//                   the running maximum entering the tile (below), rescale
//                   points, p = exp(m - s), term tables, segment sums and
//                   the tile record;
//   scores(li)      the exact FP64 scores of the next tile, kept in shared
//                   memory as offsets below their 32-row block maxima (no
//                   round trip through HBM), and the tile's maximum published.
//
// Two CTAs share an SM and drift out of phase, so one's FP64 score work runs
// beside the other's integer and shared-memory value work.
//
// The running maximum entering tile c of an item is the maximum of the tile
// maxima of chunks 0 .. c-1 (and, for a context shard, the maximum entering
// the shard). Each tile publishes one 64-bit word per query head: its own
// maximum as soon as it is scored (an aggregate), replaced by the inclusive
// running maximum once its values phase knows what enters it (a prefix). A
// tile looks back over its predecessors' words, a warp per head and 32
// chunks per step, maxing aggregates until it meets a prefix. Words carry the
// scan's epoch, so words left by an earlier scan are never read as ready.
//
// Every wait is on a tile with a smaller global index, whose CTA never waits
// on this one (its own waits go further down), and the grid is exactly the
// resident CTAs, so the waits always end; each is also bounded, and one that
// gives up sets ST_TIMEOUT, takes what it has, and lets the launch finish
// (its results are then void; ins_cache_status reports INS_ETIMEOUT).
//
// The records are folded by k_fold, the launch after this one (the fold's
// code inside this kernel cost its loop most of its speed), and items whose
// exactness the folds cannot prove are recomputed by k_scan_seq.
#pragma once

#include "scan_chunked.cuh"

namespace ins {

// Look-back words: bits 0..49 the value + 2^47 (a score maximum, 48-bit
// signed), bits 50..51 the kind, bits 52..63 the scan's epoch (never 0).
enum : int { LB_NONE = 0, LB_AGG = 1, LB_PRE = 2 };
constexpr int LB_EPOCH_BITS = 12;

__device__ __forceinline__ unsigned long long lb_word(long long v, int kind, unsigned epoch) {
    return ((unsigned long long)epoch << 52) | ((unsigned long long)kind << 50) |
           (unsigned long long)(v + (1ll << 47));
}
__device__ __forceinline__ long long lb_value(unsigned long long w) {
    return (long long)(w & ((1ull << 50) - 1)) - (1ll << 47);
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// The scratch the fused launch needs beyond the chunked scan's records.
struct FusedExtra {
    unsigned long long *lbw;      // [n_items][max_chunks][H] look-back words
    unsigned int epoch;           // 1 .. 2^12 - 1
    int32_t poll_limit;           // polls before a look-back wait gives up
    int64_t hold_word;            // a word index never published (test of the bounded wait), or -1
};

// Shared memory of the fused kernel: the replicated centroid-pair table of
// the scores, then the tile's scores and block maxima (written by scores(li),
// read by values(li) one step later), then the values phase's working set
// (the layout of ChunkCfg without its score-offset and block-max areas).
template <int H, int KB, int VB, int RS = 0>
struct FusedCfg {
    using CF = ChunkCfg<H, KB, VB, RS>;
    static constexpr int C = CF::C, CW = CF::CW;
    static constexpr size_t CTAB = (size_t)(1 << (2 * KB)) * 8 * 16;
    static constexpr size_t OFF_S = CTAB;                                          // u32 [H][C]
    static constexpr size_t OFF_BMAX = OFF_S + (size_t)H * C * 4;                  // int64 [H][CW]
    static constexpr size_t OFF_TW = OFF_BMAX + (size_t)H * CW * 8;                // u32 [64][TWS]
    static constexpr size_t OFF_VN = OFF_TW + (size_t)64 * CF::TWS * 4;            // int32 [C]
    static constexpr size_t OFF_TAB = (OFF_VN + (size_t)C * 4 + 15) & ~(size_t)15;
    static constexpr size_t OFF_GREW = OFF_TAB + CF::TABS_BYTES;                   // u32 [H+1][CW]
    static constexpr size_t OFF_PRE = OFF_GREW + (size_t)(H + 1) * CW * 4;         // int32 [H][CW]
    static constexpr size_t OFF_DB = (OFF_PRE + (size_t)H * CW * 4 + 7) & ~(size_t)7;  // int64 [H][CW]
    static constexpr size_t OFF_S0 = OFF_DB + (size_t)H * CW * 8;                  // int32 [H][64]
    static constexpr size_t BYTES = OFF_S0 + (size_t)H * D * 4;
    static_assert(CTAB % 16 == 0 && OFF_S % 16 == 0, "alignment");
};

// The running maximum entering chunk c of `item` for head h: one warp, lane j
// reading chunk c-1-j's word (32 chunks a step, nearest first).
template <int H>
__device__ __forceinline__ long long look_back(const ChunkArgs &a, const FusedExtra &x, int item, int c, int h,
                               long long seed, bool &gave_up) {
    const int lane = threadIdx.x & 31;
    const unsigned long long *words = x.lbw + (int64_t)item * a.max_chunks * H + h;
    long long m = seed;
    for (int hi = c; hi > 0; hi -= 32) {
        const int j = hi - 1 - lane;
        unsigned long long w = 0;
        int kind = LB_NONE;
        bool late = false;
        if (j >= 0) {
            const unsigned long long *p = words + (int64_t)j * H;
            for (int it = 0;; ++it) {
                w = ld_relaxed_gpu(p);
                kind = (int)((w >> 50) & 3);
                if (kind != LB_NONE && (unsigned)(w >> 52) == x.epoch) break;
                if (it >= x.poll_limit) {
                    late = true;
                    break;
                }
                __nanosleep(it < 16 ? 32 : 256);
            }
        }
        if (__any_sync(FULL, late)) {
            gave_up = true;
            break;
        }
        const unsigned pm = __ballot_sync(FULL, j >= 0 && kind == LB_PRE);
        const int first = pm ? __ffs(pm) - 1 : 31;
        const long long v = (j >= 0 && lane <= first) ? lb_value(w) : LLONG_MIN;
        const long long mx = warp_max_score(v);
        m = mx > m ? mx : m;
        if (pm) break;
    }
    return m;
}

template <int H, int KB, int VB, int RS = 0>
__global__ void __launch_bounds__(CHUNK_THREADS, 2) k_scan_fused(ChunkArgs a, FusedExtra x) {
    using CF = ChunkCfg<H, KB, VB, RS>;
    using FC = FusedCfg<H, KB, VB, RS>;
    constexpr int NT = CF::NT, R = CF::R, C = CF::C, CW = CF::CW, NC = CF::NC, VW = CF::VW;
    constexpr int TPE = CF::TPE, NE = CF::NE, HG = CF::HG, HL = CF::HL, SUBT = CF::SUBT;
    constexpr int UNITS = CF::UNITS, USTR = CF::USTR, HPS = CF::HPS, TPW = CF::TPW, TWS = CF::TWS,
                  VS = CF::VS;
    constexpr int UPW = 32 / H;                 // table units per warp in the build
    constexpr int PGMAX = C / 16 + 1;           // pages a tile touches (P >= 16)
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ __align__(16) double qd[D * H];   // [channel][head] of the item being scored
    __shared__ int32_t vcent[16];
    __shared__ int32_t exp_tab[256];
    __shared__ long long m_in_sm[H];
    __shared__ long long tmax_sm[H];
    __shared__ int fail_sm;
    __shared__ int nseg_sm[H], segbase_sm[H];
    __shared__ int32_t rl_f[H][SEGMAX];
    __shared__ unsigned int lsum_sm[H][SEGMAX + 1];    // l of a tile < 2^25
    __shared__ long long bnd_sm[NT / 32][H];           // per-warp clamp-proof bounds
    __shared__ unsigned int resc_sm;
    __shared__ int4 tdesc_sm[4];                       // tiles li-1 .. li+2 (ring of 4)
    __shared__ int32_t pages_sm[4][PGMAX];
    __shared__ int prev_item_sm, gave_up_sm;

    const double2 *ctab = reinterpret_cast<const double2 *>(dyn);
    uint32_t *d_sm = reinterpret_cast<uint32_t *>(dyn + FC::OFF_S);
    long long *bmax = reinterpret_cast<long long *>(dyn + FC::OFF_BMAX);
    uint32_t *tw = reinterpret_cast<uint32_t *>(dyn + FC::OFF_TW);
    int32_t *vn_sm = reinterpret_cast<int32_t *>(dyn + FC::OFF_VN);
    int32_t *tabs = reinterpret_cast<int32_t *>(dyn + FC::OFF_TAB);
    uint32_t *vt = reinterpret_cast<uint32_t *>(dyn + FC::OFF_TAB);       // V staging, aliases the tables
    uint32_t *grew = reinterpret_cast<uint32_t *>(dyn + FC::OFF_GREW);
    uint32_t *anyg = grew + H * CW;
    int32_t *gpre = reinterpret_cast<int32_t *>(dyn + FC::OFF_PRE);
    uint32_t *dbase = reinterpret_cast<uint32_t *>(dyn + FC::OFF_DB);   // clamped at delta_max + 1
    int32_t *s0p = reinterpret_cast<int32_t *>(dyn + FC::OFF_S0);

    const Geo &g = a.g;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        double2 *ct = reinterpret_cast<double2 *>(dyn);
        for (int i = tid; i < (1 << (2 * KB)) * 8; i += NT) {
            const int e = i >> 3;
            ct[i] = make_double2(a.tb->k_cent_f64[e & ((1 << KB) - 1)], a.tb->k_cent_f64[e >> KB]);
        }
        for (int i = tid; i < 256; i += NT) exp_tab[i] = a.tb->exp_tab[i];
        if (tid < 16) vcent[tid] = tid < NC ? (int32_t)a.tb->v_cent[tid] : 0;
        if (tid == 0) {
            prev_item_sm = -1;
            gave_up_sm = 0;
        }
    }
    const int G = gridDim.x;
    const int ntl = (a.n_tiles - (int)blockIdx.x + G - 1) / G;
    constexpr long long s_lo = DefFmt::S_LO;

    // everything below reads what the launches before this one wrote
    wait_prior_grid();

    // Tile j's descriptor and page ids into ring slot j % 4, by one warp:
    // loaded and stored at once, so that nothing of it stays in registers.
    auto look = [&](int j) {
        const int tile = (int)blockIdx.x + j * G;
        int item, c;
        if (a.n_runs == 1) {
            const int4 r0 = a.runs[0];
            item = (tile - r0.y) % r0.z;
            c = r0.x + (tile - r0.y) / r0.z;
        } else {
            const int4 t = tile_at(a, tile);
            item = t.x;
            c = t.y;
        }
        const int64_t T = a.T[item / g.n_kv];
        const int seq = a.seq_ids[item / g.n_kv];
        const int64_t tt0 = (int64_t)c * a.tile_rows;
        const int64_t tn = T - tt0 < a.tile_rows ? T - tt0 : a.tile_rows;
        const int4 td = make_int4(item, c, (int)tt0, (int)(tn > 0 ? tn : 0));
        const int poff = (int)(td.z % g.P);
        const int npg = td.w ? (poff + td.w + g.P - 1) / g.P : 0;
        const int32_t *pt = a.page_table + (int64_t)seq * g.max_pages + td.z / g.P;
        for (int i = lane; i < PGMAX; i += 32) pages_sm[j & 3][i] = i < npg ? __ldg(pt + i) : 0;
        if (lane == 0) tdesc_sm[j & 3] = td;
    };
    constexpr int LOOK_WARP = NT / 32 - 1;
    if (warp == LOOK_WARP) {
        if (ntl > 0) look(0);
        if (ntl > 1) look(1);
        __syncwarp();
        if (ntl > 0) prefetch_rows(a, tdesc_sm[0], pages_sm[0], lane, 3);
    }
    __syncthreads();

    for (int li = 0; li <= ntl; ++li) {
        // tile li + 2 is looked up while this step runs (its ring slot is free)
        if (warp == LOOK_WARP && li + 2 < ntl) look(li + 2);

        // =====================================================================
        // values(li - 1)
        // =====================================================================
        if (li >= 1) {
            const int vj = li - 1;
            const int4 td = tdesc_sm[vj & 3];
            const int item = td.x, c = td.y;
            const int64_t t0 = td.z;
            const int n = td.w;
            const int kvh = item % g.n_kv;
            const int rec_idx = item * a.max_chunks + c;
            const int poff = (int)(t0 % g.P);
            const int32_t *ptab = pages_sm[vj & 3];

            // ---- 0. the tile's V rows (each thread its own) ------------------
            uint32_t vw[R][VW], nw[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r * NT + tid;
                if (row < n) {
                    int pi, lr;
                    page_row(g, poff + row, pi, lr);
                    load_vrow<VB>(g, a.pool + region_off(g, ptab[pi], kvh), lr, vw[r], nw[r]);
                }
            }
            if (tid == 0) {
                resc_sm = 0;
                fail_sm = 0;
            }
            if (tid < H)
                for (int k = 0; k <= SEGMAX; ++k) lsum_sm[tid][k] = 0;
            for (int i = tid; i < (H + 1) * CW; i += NT) grew[i] = 0;
            for (int i = tid; i < H * D; i += NT) s0p[i] = 0;

            // ---- 1. the running maximum entering the tile: warp h, head h -----
            if (warp < H) {
                long long seed = s_lo;
                if (a.m_init) {
                    const long long mi = a.m_init[(int64_t)item * H + warp];
                    seed = mi > s_lo ? mi : s_lo;
                }
                bool late = false;
                const long long m_in = look_back<H>(a, x, item, c, warp, seed, late);
                // the tile's own maximum, from its block maxima
                const int nb = (n + 31) / 32;
                const long long bm = lane < nb ? bmax[warp * CW + lane] : LLONG_MIN;
                const long long tm = warp_max_score(bm);
                if (lane == 0) {
                    m_in_sm[warp] = m_in;
                    if (late) gave_up_sm = 1;
                    const int64_t wi = ((int64_t)item * a.max_chunks + c) * H + warp;
                    if (wi != x.hold_word)
                        st_relaxed_gpu(x.lbw + wi, lb_word(tm > m_in ? tm : m_in, LB_PRE, x.epoch));
                }
            }
            // ---- 2. V codes and v norms to shared memory ----------------------
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r * NT + tid;
                if (row < n) {
                    vn_sm[row] = (int32_t)(int16_t)(nw[r] >> 16);
#pragma unroll
                    for (int w = 0; w < VW; ++w) vt[w * VS + row + (row >> 4)] = vw[r][w];
                }
            }
            __syncthreads();

            // ---- 3. V codes to channel-major words ----------------------------
            if constexpr (VB == 2) {
                for (int task = tid; task < (C / 16) * 4; task += NT) {
                    const int v = task >> 5, l = task & 31;
                    const int tg = (v >> 1) * 16 + (l & 15), w = 2 * (v & 1) + (l >> 4);
                    uint32_t A[16];
                    const uint32_t *src = vt + w * VS + 17 * tg;
#pragma unroll
                    for (int i = 0; i < 16; ++i) A[i] = src[i];
                    transpose16x2(A);
#pragma unroll
                    for (int cc = 0; cc < 16; ++cc) tw[(16 * w + cc) * TWS + tg] = A[cc];
                }
            } else {
                for (int task = tid; task < (C / 8) * 8; task += NT) {
                    const int tg = task % (C / 8), cg = task / (C / 8);
                    const int bit = 24 * cg, wl = bit >> 5, sh = bit & 31;
                    uint32_t out[8];
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) out[cc] = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int t = 8 * tg + i, ts = t + (t >> 4);
                        uint32_t xw = vt[wl * VS + ts] >> sh;
                        if (sh > 8) xw |= vt[(wl + 1) * VS + ts] << (32 - sh);
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) out[cc] |= ((xw >> (3 * cc)) & 7u) << (4 * i);
                    }
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) tw[(8 * cg + cc) * TWS + tg] = out[cc];
                }
            }
            __syncthreads();

            // ---- 4. the online control, one warp per head ---------------------
            for (int h = warp; h < H; h += NT / 32) {
                const int nb = (n + 31) / 32;
                const int64_t m_in = m_in_sm[h];
                int64_t xm = lane < nb ? bmax[h * CW + lane] : LLONG_MIN;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int64_t y = __shfl_up_sync(FULL, xm, off);
                    if (lane >= off) xm = y > xm ? y : xm;
                }
                int64_t car = __shfl_up_sync(FULL, xm, 1);
                if (lane == 0) car = LLONG_MIN;
                car = car > m_in ? car : m_in;
                const bool scanb = lane < nb && bmax[h * CW + lane] > car;
                if (lane < CW) {
                    const int64_t db = lane < nb ? car - bmax[h * CW + lane] : 0;
                    dbase[h * CW + lane] = (uint32_t)(db < DefFmt::DELTA_MAX ? db : DefFmt::DELTA_MAX + 1);
                    grew[h * CW + lane] = 0u;
                }
                __syncwarp();
                uint32_t todo = __ballot_sync(FULL, scanb);
                int nres = 0, blkres = 0;
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
                    if (lane == 0) dbase[h * CW + bb] = 0;
                    if (valid) {
                        const int64_t dn = Mt - st;
                        d_sm[h * C + t] = (uint32_t)(dn > 0xFFFFFFFFll ? 0xFFFFFFFFll : dn);
                    }
                    const int k = nres + __popc(mask & ((1u << lane) - 1u));
                    if (gr && k < SEGMAX) rl_f[h][k] = (int32_t)exp_lut_def(exp_tab, st - Mprev);
                    if (lane == bb) blkres = __popc(mask);
                    nres += __popc(mask);
                }
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
            __syncthreads();
            for (int i = tid; i < CW; i += NT) {
                uint32_t m = 0;
#pragma unroll
                for (int h = 0; h < H; ++h) m |= grew[h * CW + i];
                anyg[i] = m;
            }
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

            // ---- 5a. p-pass: p = exp(carry - s'), w = v_norm * p in place --------
            p_pass<H, R, NT, C, CW>(exp_tab, d_sm, dbase, vn_sm, grew, gpre, lsum_sm, bnd_sm, n);
            __syncthreads();

            // ---- 5b. term tables per sub-tile, and the lookups ------------------
            {
                auto build = [&](int sti, int buf) {
                    const int st = sti * SUBT;
                    int32_t *tab = tabs + (size_t)buf * CF::TAB_WORDS;
                    for (int task = tid; task < UNITS * H; task += NT) {
                        const int l = task & 31;
                        const int u = (task >> 5) * UPW + l % UPW, h = l / UPW;
                        const int t = st + u * TPE;
                        int32_t w[TPE];            // |w| <= 2^30, |c| < 2^17: 32 x 32 -> 64-bit products
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
                        constexpr int ES = H == 1 ? 1 : 2;
#pragma unroll
                        for (int idx = 0; idx < NE; ++idx) {
                            int32_t v = T[0][idx & (NC - 1)];
                            if constexpr (TPE == 2) v += T[1][idx >> VB];
                            dst[idx * ES] = v;
                        }
                    }
                };
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
                auto lookup = [&](const int32_t *u, uint32_t nib) {
                    if constexpr (HL >= 2) {
#pragma unroll
                        for (int k = 0; k < HL / 2; ++k) {
                            const int2 xv = *reinterpret_cast<const int2 *>(u + k * HPS + 2 * nib);
                            acc[2 * k] += xv.x;
                            acc[2 * k + 1] += xv.y;
                        }
                    } else {
                        acc[0] += u[nib];
                    }
                };
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
                    constexpr int UPS = 32 / TPE, WPS = UPS / 8;
                    const int st = sti * SUBT, ts = st + stream * 32;
                    if (ts >= n) return;
                    const int blk = ts >> 5;
                    const int32_t *tab = tabs + (size_t)buf * CF::TAB_WORDS + (stream * 32 / TPE) * USTR +
                                         (H == 1 ? 0 : hgrp * (HL / 2) * HPS);
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
                            lookup2(tab + j * USTR, (cw[j >> 3] >> (4 * (j & 7))) & 15u, tab + (j + 1) * USTR,
                                    (cw[(j + 1) >> 3] >> (4 * ((j + 1) & 7))) & 15u);
                    } else {
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
                                        acc[i] += (int32_t)(((int64_t)(int32_t)d_sm[h * C + t] *
                                                             (int64_t)vcent[code]) >>
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
            if (seg_ok && tid < H)
                for (int k = 0; k < nseg_sm[tid]; ++k)
                    a.segs[segbase_sm[tid] + k].l = (int64_t)lsum_sm[tid][k + 1];

            // ---- 6. the tile record --------------------------------------------
            {
                ChunkRec &rec = a.recs[rec_idx];
                for (int i = tid; i < H * D; i += NT) rec.S0[i / D][i % D] = s0p[i];
                if (tid < H) {
                    const int h = tid;
                    rec.l0[h] = (int64_t)lsum_sm[h][0];
                    long long sw = 0;
                    for (int w = 0; w < NT / 32; ++w) sw += bnd_sm[w][h];
                    int64_t cmax_v = 0;                  // max |V centroid|
                    for (int k = 0; k < NC; ++k) {
                        const int64_t ab = vcent[k] < 0 ? -(int64_t)vcent[k] : (int64_t)vcent[k];
                        cmax_v = ab > cmax_v ? ab : cmax_v;
                    }
                    rec.B[h] = ((sw * cmax_v) >> DefFmt::ACC_SHIFT) + n;
                    rec.nseg[h] = seg_ok ? nseg_sm[h] : 0;
                    rec.seg_base[h] = segbase_sm[h];
                }
                if (tid == 0 && resc_sm) atomicAdd(&a.items[item].resc, (unsigned long long)resc_sm);
            }

            __syncthreads();                 // the tile's shared memory is reused below
        }

        // =====================================================================
        // scores(li)
        // =====================================================================
        if (li < ntl) {
            const int4 td = tdesc_sm[li & 3];
            const int item = td.x, c = td.y;
            const int64_t t0 = td.z;
            const int n = td.w;
            const int b = item / g.n_kv, kvh = item % g.n_kv;
            const int64_t qbase = ((int64_t)b * g.n_kv * H + (int64_t)kvh * H) * D;
            const int poff = (int)(t0 % g.P);
            const int32_t *ptab = pages_sm[li & 3];

            // the rows first, so their loads overlap the query setup
            uint32_t kw[R][KB * 2];
            int64_t knorm[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r * NT + tid;
                uint32_t nwr = 0;
                if (row < n) {
                    int pi, lr;
                    page_row(g, poff + row, pi, lr);
                    load_krow<KB>(g, a.pool + region_off(g, ptab[pi], kvh), lr, kw[r], nwr);
                } else {
#pragma unroll
                    for (int i = 0; i < KB * 2; ++i) kw[r][i] = 0u;
                }
                knorm[r] = row < n ? (int64_t)(int16_t)(nwr & 0xffffu) : 0;
            }
            // the next tile's rows into L2 while this one computes
            if (warp == 1 && li + 1 < ntl) prefetch_rows(a, tdesc_sm[(li + 1) & 3], pages_sm[(li + 1) & 3], lane, 3);
            if (tid < H) tmax_sm[tid] = LLONG_MIN;
            if (item != prev_item_sm) {
                __syncthreads();                 // every thread has read prev_item_sm
                if (tid == 0) prev_item_sm = item;
                for (int i = tid; i < H * D; i += NT) qd[(i % D) * H + i / D] = (double)a.q_rot[qbase + i];
                __syncthreads();
                bool big = false;
                const double qlim = (double)g.q_lim;
                for (int i = tid; i < H * D; i += NT) {
                    const double xq = qd[i];
                    big |= (xq >= qlim || xq <= -qlim);
                }
                // |q| >= q_lim could let an FP64 partial sum pass 2^53: the
                // item goes to the exact int64 body
                if (__syncthreads_or(big) && tid == 0) atomicExch(&a.items[item].fail, 1);
            } else {
                __syncthreads();
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
                    const double2 cc = ctab[(lane & 7) + kpair<KB>(kw[r], p) * 8];
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
                if ((p & 3) == 3) asm volatile("" ::: "memory");
            }
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
                    const int64_t s0 = prod >> DefFmt::SCORE_SHIFT;
                    const bool hit = s0 < DefFmt::S_LO || s0 > DefFmt::S_HI;
                    const int64_t s = s0 < DefFmt::S_LO ? DefFmt::S_LO : (s0 > DefFmt::S_HI ? DefFmt::S_HI : s0);
                    ovf += hit && valid;
                    const long long ab = s < 0 ? -s : s;
                    mx = valid && ab > mx ? ab : mx;
                    sv[r][h] = valid ? s : s_lo;
                }
            }
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
#pragma unroll
                for (int h = 0; h < H; ++h) {
                    const bool top = (int)(sv[r][h] >> 20) == mhi[r][h];
                    const unsigned mlo = __reduce_max_sync(FULL, top ? (unsigned)(sv[r][h] & 0xFFFFF) : 0u);
                    const int64_t bm = (int64_t)mhi[r][h] * (1ll << 20) + (int64_t)mlo;
                    hmax[h] = bm > hmax[h] ? bm : hmax[h];
                    if (lane == h) bmax[h * CW + (row >> 5)] = bm;
                    const uint64_t dd = (uint64_t)(bm - sv[r][h]);
                    gap |= (unsigned)(row < n && dd > 0xFFFFFFFFull);
                    d_sm[h * C + row] = (uint32_t)(dd > 0xFFFFFFFFull ? 0xFFFFFFFFull : dd);
                }
            }
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
                for (int h = 0; h < H; ++h) atomicMax(&tmax_sm[h], (long long)hmax[h]);
            }
            __syncthreads();
            // the tile's maximum, for the tiles after it
            if (tid < H) {
                const int64_t wi = ((int64_t)item * a.max_chunks + c) * H + tid;
                if (wi != x.hold_word) st_relaxed_gpu(x.lbw + wi, lb_word(tmax_sm[tid], LB_AGG, x.epoch));
            }
        }
        __syncthreads();
    }
    if (tid == 0 && gave_up_sm) atomicOr(a.status, ST_TIMEOUT);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// Resident CTAs of the fused kernel on the current device: its grid (every
// CTA must be resident for the look-back waits to end).
template <int H, int KB, int VB, int RS = 0>
inline int fused_slots() {
    auto fn = k_scan_fused<H, KB, VB, RS>;
    const size_t dyn = FusedCfg<H, KB, VB, RS>::BYTES;
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    std::lock_guard<std::mutex> lk(mu);
    if (cached[dev] > 0) return cached[dev];
    int per_sm = 0, sms = 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, CHUNK_THREADS, dyn) != cudaSuccess ||
        per_sm < 1)
        return -1;
    cached[dev] = per_sm * sms;
    return cached[dev];
}

// The next epoch of a scratch's look-back words; the words are cleared when
// the 12-bit epoch wraps, so a word from 4095 scans ago is never read as
// this scan's.
inline int next_epoch(ChunkScratch &cs, cudaStream_t s) {
    cs.epoch = cs.epoch % ((1u << LB_EPOCH_BITS) - 1) + 1;
    if (cs.epoch == 1 &&
        cudaMemsetAsync(cs.lbw, 0, cs.lbw_words * sizeof(unsigned long long), s) != cudaSuccess)
        return INS_ECUDA;
    return INS_OK;
}

// The single launch of the scan, then the exact re-run of flagged items.
template <int H, int KB, int VB, int RS = 0>
inline int launch_fused_kernels(ChunkArgs &a, const FusedExtra &x, int32_t B, const int32_t *d_seq,
                                const int64_t *d_T, cudaStream_t s) {
    const int G = fused_slots<H, KB, VB, RS>();
    if (G < 0) return INS_ECUDA;
    const unsigned grid = (unsigned)(G < a.n_tiles ? G : a.n_tiles);
    if (launch_after(k_scan_fused<H, KB, VB, RS>, grid, (unsigned)CHUNK_THREADS,
                     FusedCfg<H, KB, VB, RS>::BYTES, s, a, x) != cudaSuccess ||
        fold_prepare<H>() != cudaSuccess ||
        launch_after(k_fold<H>, (unsigned)(a.n_items * a.max_blocks), (unsigned)CHUNK_THREADS,
                     FoldCfg<H>::BYTES, s, a) != cudaSuccess)
        return INS_ECUDA;
    (void)d_seq;
    (void)d_T;
    return launch_seq<H>(a.g, a.tb, B, a.seq_ids, a.T, a.page_table, a.pool, a.q_rot, a.out, a.stats,
                         a.redo, s) == cudaSuccess
               ? INS_OK
               : INS_ECUDA;
}

template <int H, int KB, int VB, int RS = 0>
inline int launch_online_tiles(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                               const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                               const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                               int64_t *out, ins_stats *stats, int32_t *d_status, cudaStream_t s,
                               const int32_t *h_seq) {
    if (cs.scan_kernel == SCAN_SPLIT)
        return launch_chunked<H, KB, VB, RS>(cs, g, tb, B, d_seq, d_T, h_T, d_pt, pool, q_rot, out, stats,
                                             d_status, s, h_seq);
    ChunkArgs a;
    if (int rc = prepare_chunked<H, KB, VB, RS>(cs, g, tb, B, d_seq, d_T, h_T, d_pt, pool, q_rot, out, stats,
                                                d_status, a, s, false, h_seq))
        return rc;
    if (int rc = next_epoch(cs, s)) return rc;
    FusedExtra x;
    x.lbw = cs.lbw;
    x.epoch = cs.epoch;
    x.poll_limit = cs.poll_limit;
    x.hold_word = cs.hold_item < 0 || cs.hold_item >= a.n_items || cs.hold_chunk >= a.max_chunks
                      ? -1
                      : ((int64_t)cs.hold_item * a.max_chunks + cs.hold_chunk) * H + cs.hold_head;
    const int rc = launch_fused_kernels<H, KB, VB, RS>(a, x, B, a.seq_ids, a.T, s);
    if (rc == INS_OK) cs.launches += 3;          // the scan, the fold, the exact re-run
    return rc;
}

template <int H, int KB, int VB>
inline int launch_chunked_auto(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                               const int32_t *d_seq, const int64_t *d_T, const int64_t *h_T,
                               const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                               int64_t *out, ins_stats *stats, int32_t *d_status, cudaStream_t s,
                               const int32_t *h_seq) {
    if constexpr (ChunkCfg<H, KB, VB>::R == 4)
        if (small_tiles<H, KB, VB>(cs, g, B, h_T))
            return launch_online_tiles<H, KB, VB, 2>(cs, g, tb, B, d_seq, d_T, h_T, d_pt, pool, q_rot, out,
                                                     stats, d_status, s, h_seq);
    return launch_online_tiles<H, KB, VB>(cs, g, tb, B, d_seq, d_T, h_T, d_pt, pool, q_rot, out, stats,
                                          d_status, s, h_seq);
}

inline int launch_online(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                         const int32_t *d_seq, const int64_t *d_lens, const int64_t *h_lens,
                         const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                         int64_t *out, ins_stats *stats, int32_t *d_status, int H,
                         cudaStream_t s, const int32_t *h_seq = nullptr) {
#define INS_CH(HH, KK, VV)                                                                      \
    return launch_chunked_auto<HH, KK, VV>(cs, g, tb, B, d_seq, d_lens, h_lens, d_pt, pool, q_rot, \
                                           out, stats, d_status, s, h_seq)
    if (is_def_fmt(g) && g.kb == 4 && g.vb == 2) {
        switch (H) {
            case 1: INS_CH(1, 4, 2);
            case 2: INS_CH(2, 4, 2);
            case 4: INS_CH(4, 4, 2);
            case 8: INS_CH(8, 4, 2);
        }
    }
    if (is_def_fmt(g) && g.kb == 3 && g.vb == 3) {
        switch (H) {
            case 4: INS_CH(4, 3, 3);
            case 8: INS_CH(8, 3, 3);
        }
    }
#undef INS_CH
    cs.last_items = 0;
    cudaError_t e = cudaErrorInvalidValue;
    switch (H) {
        case 1: e = launch_seq<1>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 2: e = launch_seq<2>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 4: e = launch_seq<4>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
        case 8: e = launch_seq<8>(g, tb, B, d_seq, d_lens, d_pt, pool, q_rot, out, stats, nullptr, s); break;
    }
    if (e == cudaSuccess) cs.launches += 1;
    return e == cudaSuccess ? INS_OK : INS_ECUDA;
}


}  // namespace ins
