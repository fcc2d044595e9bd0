/*
 * CPU restatement of INSITU's compressed-KV decode attention.
 *
 * TEST INFRASTRUCTURE: the checker for the CUDA path and the timed CPU
 * reference arm. Never linked into the product library. See oracle.h.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define MAX_D 256

/* Q.clamp for a signed `width`-bit format with saturation
 * (numerics/fixed.py:161-168). Wrap when saturate is off. */
static int64_t clamp_w(int64_t a, int32_t width, int32_t saturate, int64_t *ovf) {
    const int64_t lo = -((int64_t)1 << (width - 1));
    const int64_t hi = ((int64_t)1 << (width - 1)) - 1;
    if (a >= lo && a <= hi) return a;
    if (ovf) (*ovf)++;
    if (saturate) return a < lo ? lo : hi;
    uint64_t span = (uint64_t)1 << width;
    uint64_t u = ((uint64_t)a + ((uint64_t)1 << (width - 1))) & (span - 1);
    return (int64_t)u - ((int64_t)1 << (width - 1));
}

/* rshift with floor / half-even rounding (numerics/fixed.py:49-89). */
static int64_t rshift_floor(int64_t a, int32_t n) { return n == 0 ? a : (a >> n); }

static int64_t rshift_even(int64_t a, int32_t n) {
    if (n == 0) return a;
    const int64_t half = (int64_t)1 << (n - 1);
    int64_t q = (a + half) >> n;
    if ((a & (((int64_t)1 << n) - 1)) == half) q &= ~(int64_t)1;
    return q;
}

static int64_t lshift(int64_t a, int32_t n) { return (int64_t)((uint64_t)a << n); }

int or_check_cfg(const or_cfg *c) {
    if (!c || c->d <= 0 || c->d > MAX_D || (c->d & (c->d - 1))) return OR_EINVAL;
    if (c->key_bits < 1 || c->key_bits > 8 || c->value_bits < 1 || c->value_bits > 8)
        return OR_EINVAL;
    if (c->norm_bits % 8 || c->norm_frac >= c->norm_bits) return OR_EINVAL;
    if (c->rounds < 0 || (c->rounds && !c->signs)) return OR_EINVAL;
    if (!c->k_centroids || !c->k_bounds || !c->v_centroids || !c->v_bounds || !c->exp_table)
        return OR_EINVAL;
    /* KVQuantizer.__init__ refuses a comparison that would truncate x
     * (ops/quantize.py:150-156). */
    if (c->centroid_frac + c->norm_frac < c->qk_frac) return OR_EINVAL;
    return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* rotation                                                                */
/* ---------------------------------------------------------------------- */

/* Unnormalised Walsh-Hadamard, stages h = 1, 2, 4, ... (numerics/fixed.py:202-226). */
void or_fwht(int64_t *a, int32_t n) {
    for (int32_t h = 1; h < n; h <<= 1)
        for (int32_t blk = 0; blk < n; blk += 2 * h)
            for (int32_t j = 0; j < h; j++) {
                int64_t lo = a[blk + j], hi = a[blk + h + j];
                a[blk + j] = lo + hi;
                a[blk + h + j] = lo - hi;
            }
}

/* Rotation.apply (ops/rotate.py:170-197): per round, flip signs, transform,
 * then scale by 1/sqrt(d) as a floor shift (or a Q15 multiply and shift). */
int or_rotate(const or_cfg *c, const int64_t *x, int64_t *y, int64_t n) {
    if (or_check_cfg(c)) return OR_EINVAL;
    const int32_t d = c->d;
    int64_t buf[MAX_D];
    for (int64_t i = 0; i < n; i++) {
        memcpy(buf, x + i * d, sizeof(int64_t) * d);
        for (int32_t r = 0; r < c->rounds; r++) {
            for (int32_t j = 0; j < d; j++) buf[j] *= c->signs[r * d + j];
            or_fwht(buf, d);
            for (int32_t j = 0; j < d; j++)
                buf[j] = c->rot_shift >= 0 ? rshift_floor(buf[j], c->rot_shift)
                                           : rshift_floor(buf[j] * c->rot_inv_sqrt_q15, 15);
        }
        memcpy(y + i * d, buf, sizeof(int64_t) * d);
    }
    return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* quantizer                                                               */
/* ---------------------------------------------------------------------- */

/* Exact integer square root (ops/quantize.py:42-60): a float seed, then
 * corrected until r*r <= a < (r+1)^2. */
int64_t or_isqrt(int64_t a) {
    if (a < 0) return -1;
    int64_t r = (int64_t)sqrt((double)a);
    if (r > 0) r -= 1;
    while ((__int128)(r + 1) * (r + 1) <= a) r++;
    while ((__int128)r * r > a) r--;
    return r;
}

/* RMS at wire precision (ops/quantize.py:164-181): floor(sum x^2 / d), exact
 * isqrt, then Q.requantize from qk_frac to norm_frac rounding half to even
 * (numerics/fixed.py:189-196) and the Q(norm_bits, norm_frac) clamp. */
int or_norm_wire(const or_cfg *c, const int64_t *x, int64_t *norm, int64_t n) {
    if (or_check_cfg(c)) return OR_EINVAL;
    const int32_t d = c->d;
    for (int64_t i = 0; i < n; i++) {
        int64_t sq = 0;
        for (int32_t j = 0; j < d; j++) sq += x[i * d + j] * x[i * d + j];
        int64_t ms = sq / d; /* sq >= 0, so truncation is floor */
        int64_t r = or_isqrt(ms);
        int32_t shift = c->qk_frac - c->norm_frac;
        if (shift > 0) r = rshift_even(r, shift);
        else if (shift < 0) r = lshift(r, -shift);
        norm[i] = clamp_w(r, c->norm_bits, 1, NULL);
    }
    return OR_OK;
}

/* Threshold encoder (ops/quantize.py:183-196): code = #{ x<<s > norm*b }. */
int or_encode_plane(const or_cfg *c, const int64_t *x, const int64_t *norm, int32_t plane,
                    uint8_t *idx, int64_t n) {
    if (or_check_cfg(c)) return OR_EINVAL;
    const int32_t d = c->d;
    const int32_t bits = plane ? c->value_bits : c->key_bits;
    const int64_t *b = plane ? c->v_bounds : c->k_bounds;
    const int32_t nb = (1 << bits) - 1;
    const int32_t s = c->centroid_frac + c->norm_frac - c->qk_frac;
    for (int64_t i = 0; i < n; i++) {
        int64_t thr[255];
        for (int32_t k = 0; k < nb; k++) thr[k] = norm[i] * b[k];
        for (int32_t j = 0; j < d; j++) {
            int64_t xs = lshift(x[i * d + j], s);
            int32_t cnt = 0;
            for (int32_t k = 0; k < nb; k++) cnt += xs > thr[k];
            idx[i * d + j] = (uint8_t)cnt;
        }
    }
    return OR_OK;
}

int32_t or_bytes_per_token(const or_cfg *c) {
    int32_t bits = c->d * (c->key_bits + c->value_bits);
    if (bits % 8 || (c->d * c->key_bits) % 8 || (c->d * c->value_bits) % 8) return -1;
    return bits / 8 + 2 * (c->norm_bits / 8);
}

/* LSB-first bit packing of `d` codes (ops/quantize.py:271-275). */
static void pack_codes(const uint8_t *idx, int32_t d, int32_t bits, uint8_t *out) {
    memset(out, 0, (size_t)(d * bits / 8));
    for (int32_t j = 0; j < d; j++)
        for (int32_t k = 0; k < bits; k++)
            if ((idx[j] >> k) & 1) {
                int32_t pos = j * bits + k;
                out[pos >> 3] |= (uint8_t)(1u << (pos & 7));
            }
}

static void unpack_codes(const uint8_t *buf, int32_t d, int32_t bits, uint8_t *idx) {
    for (int32_t j = 0; j < d; j++) {
        uint32_t v = 0;
        for (int32_t k = 0; k < bits; k++) {
            int32_t pos = j * bits + k;
            v |= (uint32_t)((buf[pos >> 3] >> (pos & 7)) & 1) << k;
        }
        idx[j] = (uint8_t)v;
    }
}

int or_pack(const or_cfg *c, const uint8_t *k_idx, const int64_t *k_norm,
            const uint8_t *v_idx, const int64_t *v_norm, uint8_t *rows, int64_t n) {
    const int32_t row = or_bytes_per_token(c);
    if (row < 0) return OR_EINVAL;
    const int32_t d = c->d, kb = d * c->key_bits / 8, vb = d * c->value_bits / 8;
    const int32_t nb = c->norm_bits / 8;
    for (int64_t i = 0; i < n; i++) {
        uint8_t *r = rows + i * row;
        pack_codes(k_idx + i * d, d, c->key_bits, r);
        pack_codes(v_idx + i * d, d, c->value_bits, r + kb);
        /* _pack_word: little-endian two's complement (ops/quantize.py:286-289) */
        for (int32_t k = 0; k < nb; k++) {
            r[kb + vb + k] = (uint8_t)(((uint64_t)k_norm[i] >> (8 * k)) & 0xFF);
            r[kb + vb + nb + k] = (uint8_t)(((uint64_t)v_norm[i] >> (8 * k)) & 0xFF);
        }
    }
    return OR_OK;
}

static int64_t unpack_word(const uint8_t *b, int32_t bits) {
    uint64_t v = 0;
    for (int32_t k = 0; k < bits / 8; k++) v |= (uint64_t)b[k] << (8 * k);
    const int64_t sign = (int64_t)1 << (bits - 1);
    return ((int64_t)v ^ sign) - sign; /* sign-extend (ops/quantize.py:292-296) */
}

int or_unpack(const or_cfg *c, const uint8_t *rows, uint8_t *k_idx, int64_t *k_norm,
              uint8_t *v_idx, int64_t *v_norm, int64_t n) {
    const int32_t row = or_bytes_per_token(c);
    if (row < 0) return OR_EINVAL;
    const int32_t d = c->d, kb = d * c->key_bits / 8, vb = d * c->value_bits / 8;
    const int32_t nb = c->norm_bits / 8;
    for (int64_t i = 0; i < n; i++) {
        const uint8_t *r = rows + i * row;
        unpack_codes(r, d, c->key_bits, k_idx + i * d);
        unpack_codes(r + kb, d, c->value_bits, v_idx + i * d);
        k_norm[i] = unpack_word(r + kb + vb, c->norm_bits);
        v_norm[i] = unpack_word(r + kb + vb + nb, c->norm_bits);
    }
    return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* softmax pieces                                                          */
/* ---------------------------------------------------------------------- */

static int32_t exp_shift(const or_cfg *c) { return c->acc_frac - c->exp_lut_bits; }
static int64_t exp_max_int(const or_cfg *c) { return c->prob_frac + 1; }
static int64_t exp_span(const or_cfg *c) { return (exp_max_int(c) + 1) << c->exp_lut_bits; }

int64_t or_exp_delta_max(const or_cfg *c) {
    /* ceil(((span << shift) << acc_frac) / log2e) (ops/attention.py:145-146) */
    __int128 num = (__int128)exp_span(c) << exp_shift(c);
    num <<= c->acc_frac;
    __int128 q = num / c->log2e;
    if (q * c->log2e != num) q += 1;
    return (int64_t)q;
}

/* The flat gather (ops/attention.py:147-159), evaluated without the table:
 * u = min(t >> shift, span); zero past the last integer part. */
int64_t or_exp(const or_cfg *c, int64_t delta) {
    if (delta < 0) return -1;
    const int64_t dmax = or_exp_delta_max(c);
    int64_t d = delta < dmax ? delta : dmax;
    int64_t t = rshift_floor(d * c->log2e, c->acc_frac);
    int64_t u = t >> exp_shift(c);
    const int64_t span = exp_span(c);
    if (u >= span) return 0;
    int64_t ip = u >> c->exp_lut_bits;
    if (ip > exp_max_int(c)) return 0;
    return c->exp_table[u & ((1 << c->exp_lut_bits) - 1)] >> ip;
}

/* ExpLut.two_step (ops/attention.py:161-169). */
int64_t or_exp_two_step(const or_cfg *c, int64_t delta) {
    const int64_t dmax = or_exp_delta_max(c);
    int64_t d = delta < dmax ? delta : dmax;
    int64_t t = rshift_floor(d * c->log2e, c->acc_frac);
    int64_t i = rshift_floor(t, c->acc_frac);
    int64_t f = t & (((int64_t)1 << c->acc_frac) - 1);
    int64_t addr = rshift_floor(f, c->acc_frac - c->exp_lut_bits);
    int64_t mi = exp_max_int(c);
    int64_t p = c->exp_table[addr] >> (i < mi ? i : mi);
    return i > mi ? 0 : p;
}

#define L_WIDTH 48
#define RECIP_NORM_BITS 32
#define RECIP_NUM_SHIFT (2 * RECIP_NORM_BITS - 2)

/* Leading-one position, capped the way `_lead` caps it
 * (ops/attention.py:177-183): the largest b in [1, L_WIDTH) with l >= 2^b. */
static int64_t lead(int64_t l) {
    int64_t n = 0;
    for (int32_t b = 1; b < L_WIDTH; b++)
        if (l >= ((int64_t)1 << b)) n = b;
    return n;
}

/* Normalised reciprocal (ops/attention.py:197-250). */
void or_reciprocal(const or_cfg *c, int64_t l, int64_t *r, int64_t *shift) {
    int64_t s = lead(l);
    int64_t k = s - (RECIP_NORM_BITS - 1);
    int64_t ln = k >= 0 ? (l >> k) : lshift(l, (int32_t)-k);
    const int64_t num = (int64_t)1 << RECIP_NUM_SHIFT;
    *r = l > 0 ? num / (ln > 1 ? ln : 1) : 0;
    *shift = RECIP_NUM_SHIFT - c->prob_frac + k;
}

void or_finalize(const or_cfg *c, const int64_t *acc, int64_t l, int64_t *out) {
    int64_t r, sh;
    or_reciprocal(c, l, &r, &sh);
    for (int32_t j = 0; j < c->d; j++) out[j] = rshift_floor(acc[j] * r, (int32_t)sh);
}

/* ---------------------------------------------------------------------- */
/* scores and the two softmaxes                                            */
/* ---------------------------------------------------------------------- */

static int32_t score_shift(const or_cfg *c) {
    return c->qk_frac + c->centroid_frac + c->norm_frac - c->acc_frac; /* config.py:249-250 */
}
static int32_t acc_shift(const or_cfg *c) {
    return c->centroid_frac + c->norm_frac + c->prob_frac - c->acc_frac; /* config.py:252-254 */
}

/* One fused score (ops/attention.py:349-353): the planes are summed, then one
 * multiply by the norm and one floor shift. The product wraps at 64 bits
 * exactly as numpy's int64 does. */
static int64_t score_one(const or_cfg *c, const int64_t *q, const uint8_t *codes, int64_t norm) {
    int64_t dot = 0;
    for (int32_t j = 0; j < c->d; j++) dot += q[j] * c->k_centroids[codes[j]];
    int64_t prod = (int64_t)((uint64_t)dot * (uint64_t)norm);
    return rshift_floor(prod, score_shift(c));
}

int64_t or_scores(const or_cfg *c, const int64_t *q, int32_t H, const uint8_t *k_idx,
                  const int64_t *k_norm, int64_t T, int64_t *s) {
    int64_t ovf = 0;
    for (int32_t h = 0; h < H; h++)
        for (int64_t t = 0; t < T; t++)
            s[h * T + t] = clamp_w(score_one(c, q + h * c->d, k_idx + t * c->d, k_norm[t]),
                                   c->score_width, c->saturate, &ovf);
    return ovf;
}

static int64_t iabs64(int64_t a) { return a < 0 ? -a : a; }

/* The per-token recurrence of attend_online (ops/attention.py:480-503), for
 * one token against H heads. State m, l, acc is carried by the caller. */
static void online_token(const or_cfg *c, int32_t H, const int64_t *st, const uint8_t *vcodes,
                         int64_t v_norm, int64_t *m, int64_t *l, int64_t *acc, or_stats *stats,
                         const or_trace *tr, int64_t t) {
    const int32_t d = c->d;
    const int64_t unity = (int64_t)1 << c->prob_frac;
    int any = 0;
    for (int32_t h = 0; h < H; h++) any |= st[h] > m[h];
    int64_t factor[64];
    int64_t grew[64];
    for (int32_t h = 0; h < H; h++) {
        grew[h] = st[h] > m[h];
        factor[h] = unity;
    }
    if (any) {
        for (int32_t h = 0; h < H; h++) {
            if (grew[h]) factor[h] = or_exp(c, st[h] - m[h]);
            for (int32_t j = 0; j < d; j++)
                acc[h * d + j] = rshift_floor(acc[h * d + j] * factor[h], c->prob_frac);
            l[h] = rshift_floor(l[h] * factor[h], c->prob_frac);
            if (grew[h]) {
                m[h] = st[h];
                stats->rescale_events++;
            }
        }
    }
    for (int32_t h = 0; h < H; h++) {
        int64_t p = or_exp(c, m[h] - st[h]);
        l[h] += p;
        int64_t w = v_norm * p;
        for (int32_t j = 0; j < d; j++) {
            int64_t term = rshift_floor(w * c->v_centroids[vcodes[j]], acc_shift(c));
            acc[h * d + j] = clamp_w(acc[h * d + j] + term, c->acc_width, c->saturate,
                                     &stats->acc_overflows);
        }
        if (tr) {
            if (tr->s) tr->s[t * H + h] = st[h];
            if (tr->m) tr->m[t * H + h] = m[h];
            if (tr->p) tr->p[t * H + h] = p;
            if (tr->l) tr->l[t * H + h] = l[h];
            if (tr->grew) tr->grew[t * H + h] = grew[h];
            if (tr->factor) tr->factor[t * H + h] = factor[h];
            if (tr->acc) memcpy(tr->acc + (t * H + h) * d, acc + h * d, sizeof(int64_t) * d);
        }
    }
}

static void online_finish(const or_cfg *c, int32_t H, const int64_t *acc, const int64_t *l,
                          int64_t *out, or_stats *st) {
    int64_t mx = 0;
    for (int32_t i = 0; i < H * c->d; i++) {
        int64_t a = iabs64(acc[i]);
        if (a > mx) mx = a;
    }
    st->max_abs_acc = mx;
    for (int32_t h = 0; h < H; h++) or_finalize(c, acc + h * c->d, l[h], out + h * c->d);
}

int or_attend_online(const or_cfg *c, const int64_t *q, int32_t H, const uint8_t *k_idx,
                     const int64_t *k_norm, const uint8_t *v_idx, const int64_t *v_norm,
                     int64_t T, int64_t *out, or_stats *st, const or_trace *tr) {
    if (or_check_cfg(c) || H < 1 || H > 64) return OR_EINVAL;
    const int32_t d = c->d;
    memset(st, 0, sizeof(*st));
    st->n_tokens = T;
    int64_t *acc = calloc((size_t)H * d, sizeof(int64_t));
    int64_t l[64], m[64], s[64];
    for (int32_t h = 0; h < H; h++) {
        l[h] = 0;
        m[h] = -((int64_t)1 << (c->score_width - 1));
    }
    for (int64_t t = 0; t < T; t++) {
        for (int32_t h = 0; h < H; h++) {
            s[h] = clamp_w(score_one(c, q + h * d, k_idx + t * d, k_norm[t]), c->score_width,
                           c->saturate, &st->score_overflows);
            int64_t a = iabs64(s[h]);
            if (a > st->max_abs_score) st->max_abs_score = a;
        }
        online_token(c, H, s, v_idx + t * d, v_norm[t], m, l, acc, st, tr, t);
    }
    online_finish(c, H, acc, l, out, st);
    free(acc);
    return OR_OK;
}

int or_attend_online_rows(const or_cfg *c, const int64_t *q, int32_t H, const uint8_t *rows,
                          int64_t row_stride, int64_t T, int64_t *out, or_stats *st) {
    if (or_check_cfg(c) || H < 1 || H > 64 || or_bytes_per_token(c) < 0) return OR_EINVAL;
    const int32_t d = c->d;
    memset(st, 0, sizeof(*st));
    st->n_tokens = T;
    int64_t *acc = calloc((size_t)H * d, sizeof(int64_t));
    int64_t l[64], m[64], s[64];
    uint8_t kc[MAX_D], vc[MAX_D];
    for (int32_t h = 0; h < H; h++) {
        l[h] = 0;
        m[h] = -((int64_t)1 << (c->score_width - 1));
    }
    for (int64_t t = 0; t < T; t++) {
        int64_t kn, vn;
        or_unpack(c, rows + t * row_stride, kc, &kn, vc, &vn, 1);
        for (int32_t h = 0; h < H; h++) {
            s[h] = clamp_w(score_one(c, q + h * d, kc, kn), c->score_width, c->saturate,
                           &st->score_overflows);
            int64_t a = iabs64(s[h]);
            if (a > st->max_abs_score) st->max_abs_score = a;
        }
        online_token(c, H, s, vc, vn, m, l, acc, st, NULL, t);
    }
    online_finish(c, H, acc, l, out, st);
    free(acc);
    return OR_OK;
}

int or_attend_two_pass(const or_cfg *c, const int64_t *q, int32_t H, const uint8_t *k_idx,
                       const int64_t *k_norm, const uint8_t *v_idx, const int64_t *v_norm,
                       int64_t T, int64_t *out, or_stats *st) {
    if (or_check_cfg(c) || H < 1 || H > 64) return OR_EINVAL;
    const int32_t d = c->d;
    memset(st, 0, sizeof(*st));
    st->n_tokens = T;
    int64_t *s = malloc(sizeof(int64_t) * (size_t)(H * (T ? T : 1)));
    st->score_overflows = or_scores(c, q, H, k_idx, k_norm, T, s);
    for (int64_t i = 0; i < (int64_t)H * T; i++) {
        int64_t a = iabs64(s[i]);
        if (a > st->max_abs_score) st->max_abs_score = a;
    }
    int64_t *acc = calloc((size_t)H * d, sizeof(int64_t));
    for (int32_t h = 0; h < H; h++) {
        /* m = s.max(axis=-1); an empty cache has no maximum. */
        int64_t m = T ? s[h * T] : 0, l = 0;
        for (int64_t t = 1; t < T; t++) m = s[h * T + t] > m ? s[h * T + t] : m;
        for (int64_t t = 0; t < T; t++) {
            int64_t p = or_exp(c, m - s[h * T + t]);
            l += p;
            int64_t w = v_norm[t] * p;
            for (int32_t j = 0; j < d; j++)
                acc[h * d + j] += rshift_floor(w * c->v_centroids[v_idx[t * d + j]],
                                               acc_shift(c));
        }
        for (int32_t j = 0; j < d; j++)
            acc[h * d + j] = clamp_w(acc[h * d + j], c->acc_width, c->saturate,
                                     &st->acc_overflows);
        or_finalize(c, acc + h * d, l, out + h * d);
    }
    int64_t mx = 0;
    for (int32_t i = 0; i < H * d; i++) mx = iabs64(acc[i]) > mx ? iabs64(acc[i]) : mx;
    st->max_abs_acc = mx;
    free(acc);
    free(s);
    return OR_OK;
}

int or_decode_layer(const or_cfg *c, int32_t B, int32_t n_kv, int32_t H,
                    const uint8_t *const *rows, const int64_t *T, const int64_t *q,
                    int64_t *out, or_stats *stats, int32_t threads) {
    if (or_check_cfg(c) || or_bytes_per_token(c) < 0) return OR_EINVAL;
    const int64_t row = or_bytes_per_token(c);
    const int64_t items = (int64_t)B * n_kv;
    int rc = OR_OK;
#ifdef _OPENMP
    if (threads < 1) threads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
    for (int64_t it = 0; it < items; it++) {
        const int64_t b = it / n_kv, g = it % n_kv;
        const int64_t off = (b * n_kv + g) * (int64_t)H * c->d;
        int r = or_attend_online_rows(c, q + off, H, rows[b] + g * row, row * n_kv, T[b],
                                      out + off, stats + it);
        if (r) rc = r;
    }
    return rc;
}

int or_ingress_rows(const or_cfg *c, const int64_t *k, const int64_t *v, uint8_t *rows,
                    int64_t n, int32_t threads) {
    if (or_check_cfg(c) || or_bytes_per_token(c) < 0) return OR_EINVAL;
    const int32_t d = c->d, row = or_bytes_per_token(c);
#ifdef _OPENMP
    if (threads < 1) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int64_t i = 0; i < n; i++) {
        int64_t kr[MAX_D], vr[MAX_D], kn, vn;
        uint8_t kc[MAX_D], vc[MAX_D];
        or_rotate(c, k + i * d, kr, 1);
        or_rotate(c, v + i * d, vr, 1);
        or_norm_wire(c, kr, &kn, 1);
        or_norm_wire(c, vr, &vn, 1);
        or_encode_plane(c, kr, &kn, 0, kc, 1);
        or_encode_plane(c, vr, &vn, 1, vc, 1);
        or_pack(c, kc, &kn, vc, &vn, rows + i * row, 1);
    }
    return OR_OK;
}
