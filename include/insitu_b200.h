/*
 * insitu_b200 -- the C ABI of the B200 compressed-KV decode attention path.
 *
 * This is the drop-in boundary. Everything below it is hand-written CUDA for
 * sm_100a; everything above it (the Python package `insitu_b200`, or any
 * other host language through its FFI) mirrors the reference's operator
 * interfaces and calls only these functions. No torch types cross: plain
 * pointers, sizes and a cudaStream_t passed as `void *`.
 *
 * Citations are path:line inside the INSITU reference repository.
 *
 * Ownership. The handle owns the paged cache pool and its page tables, which
 * it allocates at creation and never grows (capacity is fixed at
 * construction, cache/base.py:30-36 and 67-73). Every other device buffer --
 * q/k/v in, rotated q and outputs out, stats -- is owned by the caller.
 *
 * Ordering. Device work is enqueued on the caller's stream and returns
 * without synchronising, except where a function says it blocks (the export,
 * import and status readers, which move data to or from host memory).
 *
 * Errors. Every function returns an ins_status. Argument and capacity
 * errors are detected on the host before anything is enqueued and leave the
 * cache unchanged, the way the reference raises ValueError. Conditions only
 * the device can see (a value outside the 24-bit wire range, a bounded wait
 * that expired) are latched in a device status word that
 * ins_cache_status() reads and clears.
 */
#ifndef INSITU_B200_H
#define INSITU_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The board protocol's numbering (host/attn_proto.h:47-55) is
 * kept for the codes that have a meaning here. */
typedef enum {
    INS_OK = 0,
    INS_EBADLEN = 4,   /* capacity exceeded, or a length/shape mismatch  */
    INS_ETIMEOUT = 5,  /* a bounded device-side wait gave up              */
    INS_ERANGE = 7,    /* a value escaped its fixed-point format          */
    INS_EINVAL = 8,    /* bad argument or unsupported configuration       */
    INS_ENOMEM = 9,    /* device or pinned allocation failed              */
    INS_ECUDA = 10     /* a CUDA runtime call failed                      */
} ins_status;

/* The fixed-point contract, field for field from QuantConfig and FixedFormat
 * (config.py:132-254), plus the cache geometry. */
typedef struct {
    int32_t head_dim;         /* d; this build supports 64                    */
    int32_t n_kv_heads;       /* KV heads per layer                           */
    int32_t kv_groups;        /* query heads per KV head: 1, 2, 4 or 8        */
    int32_t key_bits;         /* 1..8                                         */
    int32_t value_bits;       /* 1..8                                         */
    int32_t norm_bits;        /* 16                                           */
    int32_t norm_frac;        /* 9                                            */
    int32_t qk_frac;          /* 16                                           */
    int32_t centroid_frac;    /* 15                                           */
    int32_t acc_frac;         /* 16                                           */
    int32_t acc_width;        /* 32                                           */
    int32_t score_width;      /* 48                                           */
    int32_t prob_frac;        /* 15                                           */
    int32_t exp_lut_bits;     /* 8                                            */
    int32_t saturate;         /* 1                                            */
    int32_t rot_rounds;       /* QuantConfig.rot_rounds                       */
    int32_t rot_shift;        /* sqrt_shift(d), -1 when d is an odd power     */
    int32_t rot_inv_sqrt_q15; /* round(2^15/sqrt(d)), used when rot_shift < 0 */
    int32_t page_tokens;      /* tokens per cache page, a multiple of 16      */
    int32_t max_seqs;         /* sequences the page table can hold            */
    int32_t max_pages_per_seq;/* per-sequence capacity = this * page_tokens   */
    int32_t reserved0;
    int64_t n_pages;          /* pages in the pool                            */
} ins_config;

/* The integer tables (host pointers, copied at creation). They are format
 * artefacts the host builds once: the PCG64 sign diagonal
 * (ops/rotate.py:144-155), the Lloyd-Max codebooks (ops/codebook.py:67-120)
 * and the exp table with its constants (ops/attention.py:104-151). */
typedef struct {
    const int64_t *signs;        /* rot_rounds * head_dim entries of +-1     */
    const int64_t *k_centroids;  /* 2^key_bits                               */
    const int64_t *k_bounds;     /* 2^key_bits - 1                           */
    const int64_t *v_centroids;  /* 2^value_bits                             */
    const int64_t *v_bounds;     /* 2^value_bits - 1                         */
    const int64_t *exp_table;    /* 2^exp_lut_bits                           */
    int64_t log2e;               /* round(log2(e) * 2^acc_frac)              */
    int64_t delta_max;           /* ExpLut._delta_max                        */
} ins_tables;

/* AttentionStats (ops/attention.py:257-274), one per (sequence, KV head). */
typedef struct {
    int64_t n_tokens;
    int64_t rescale_events;
    int64_t score_overflows;
    int64_t acc_overflows;
    int64_t max_abs_score;
    int64_t max_abs_acc;
} ins_stats;

typedef struct ins_cache ins_cache;

/* Softmax forms of CompressedAttention (ops/attention.py:429-513). */
typedef enum { INS_SOFTMAX_ONLINE = 0, INS_SOFTMAX_TWO_PASS = 1 } ins_softmax;

/* Version of this ABI; bumped on any incompatible change. */
int32_t ins_abi_version(void);

/* Bytes of one compressed token of one KV head: QuantConfig.bytes_per_token
 * (config.py:192-207). -1 for an invalid configuration. */
int32_t ins_bytes_per_token(const ins_config *cfg);

/* Create a paged compressed cache on `device`: the GPU form of
 * CompressedCache.__init__ (cache/compressed.py:42-52) for max_seqs
 * sequences at once. */
int ins_cache_create(const ins_config *cfg, const ins_tables *tables, int32_t device,
                     ins_cache **out);

/* Free the pool, the page tables and the handle. NULL is a no-op. */
int ins_cache_destroy(ins_cache *cache);

/* KVCache.reset (cache/base.py:64-65) for one sequence (seq >= 0) or for all
 * (seq < 0). Its pages return to the pool. Host-side only; ordered after
 * work already enqueued by the caller's next synchronisation. */
int ins_cache_reset(ins_cache *cache, int32_t seq);

/* Tile size of the context-parallel online scan (no reference counterpart:
 * a tuning knob of this implementation; results are identical in every mode).
 * AUTO (the default) takes tiles of 4 rows per thread for long contexts and
 * of 2 when the default tiles would leave SMs idle; LARGE and SMALL force one
 * of them (shapes whose default is already 2 rows per thread ignore it). */
enum { INS_TILES_AUTO = 0, INS_TILES_LARGE = 1, INS_TILES_SMALL = 2 };
int ins_cache_set_tiles(ins_cache *cache, int32_t mode);

/* Which kernels run the context-parallel online scan (no reference
 * counterpart; results are identical either way). SPLIT, the default: a
 * score launch, then a value launch, with the scores kept in global memory
 * between them (the context split always uses these).
 * FUSED: one persistent launch that scores each tile, finds the running
 * maximum entering it from the tiles before (a bounded look-back on words the
 * other CTAs publish) and accumulates V; no per-row scratch (ins_scan_noalloc
 * always uses it). Either way a fold launch and the exact re-run of items the
 * fold could not prove follow. */
enum { INS_SCAN_FUSED = 0, INS_SCAN_SPLIT = 1 };
int ins_cache_set_scan_kernel(ins_cache *cache, int32_t mode);

/* A test of the scans' failure path, with no reference counterpart and no
 * use outside tests: every bounded wait of the online scan's look-back (fused
 * kernel) and of its value pass's staged rows (separate launches) gives up
 * after `poll_limit` polls (default 2^22, about a second), and tile `chunk`
 * of item `item` (sequence b, KV head h: item b * n_kv + h, in the order of
 * the scan's seq_ids) is held back: with the fused kernel the word it
 * publishes for query head `head` is withheld, so the tiles after it wait
 * for a word nothing writes; with the separate launches the bytes of its
 * staged rows are announced 16 larger than the copies that land, so its own
 * wait cannot complete. The waits give up, the launch still finishes, and
 * ins_cache_status returns INS_ETIMEOUT; no GPU fault is involved. item < 0
 * holds nothing back. */
int ins_cache_set_wait_test(ins_cache *cache, int32_t poll_limit, int32_t item, int32_t chunk,
                            int32_t head);

/* Tokens currently held for `seq` (KVCache.length), or -1. */
int64_t ins_cache_length(const ins_cache *cache, int32_t seq);

/* Tokens one sequence can hold (KVCache.capacity). */
int64_t ins_cache_capacity(const ins_cache *cache);

/* Kernels this cache has launched so far through ins_ingress,
 * ins_ingress_lanes, ins_seam, ins_seam_device_positions and ins_scan (a
 * running count, for a caller that reports what ran). The online scan is 4
 * launches with the separate kernels (scores, values, fold, exact re-run)
 * and 3 with the fused kernel (the scan, the fold, the exact re-run), plus
 * one for its small host->device upload (a kernel whose parameter carries
 * the bytes); an ingress is 2 (its upload, the ingress). No reference
 * counterpart. -1 for NULL. */
int64_t ins_cache_launches(const ins_cache *cache);

/* Flags of ins_ingress. */
enum {
    /* k and v (and q) are already rotated, as CompressedCache.append_rotated
     * takes them (cache/compressed.py:64-86): skip the rotation and the 24-bit
     * wire-range check. */
    INS_INGRESS_PREROTATED = 1
};

/* The ingress: rotate q, k and v (Rotation.apply, ops/rotate.py:170-197),
 * quantise k and v (KVQuantizer.encode, ops/quantize.py:164-212), bit-pack
 * them (KVQuantizer.pack, ops/quantize.py:237-252) and append each token at
 * its sequence's current length (CompressedCache.append_rotated,
 * cache/compressed.py:64-86), in the kernel.py:271-284 order.
 *
 * n tokens; seq_ids (host, n) names each token's sequence, and tokens of one
 * sequence are appended in the order given. q (device, [n, n_kv*groups, d]
 * int32) may be NULL; when given, its rotation is written to q_rot (device,
 * same shape). k and v are device [n, n_kv, d] int32, Q(qk_frac) in 24-bit
 * lanes. EBADLEN, with nothing appended, if a sequence would exceed its
 * capacity or the pool runs out of pages. */
int ins_ingress(ins_cache *cache, int32_t n, const int32_t *seq_ids,
                const int32_t *q, const int32_t *k, const int32_t *v, int32_t *q_rot,
                uint32_t flags, void *stream);

/* The seam on the GPU: the host half of kernel.py:211-249 after the
 * projections. q, k, v are the projections' float32 outputs (device; q [n,
 * n_kv*groups, d], k and v [n, n_kv, d]); per vector: QK-norm of q and k when
 * gains are given (rms_norm, ops/norm.py:35-49), q times attn_scale, then
 * RoPE in float64 and the round-half-even saturating cast to Q(qk_frac) in
 * 24-bit lanes (cast_after_rope, the reference's default; ops/rope.py:181-198,
 * ops/convert.py:44-57), or the cast and RoPE in fixed point
 * (ops/rope.py:150-179). Writes the wire q, k, v (device int32, same shapes;
 * ins_ingress takes them as they are) and adds to conv (device int64 [3]:
 * values cast, values saturated, and the largest |float| as the bits of a
 * double -- ConversionStats, ops/convert.py:25-41; zero it to start).
 * positions: host int64 [n], each below max_position (else EINVAL, the
 * reference's ValueError). The RoPE tables are RoPE.build's (ops/rope.py:
 * 131-148), on the device. */
typedef struct {
    const float *q_norm, *k_norm;     /* device [head_dim] QK-norm gains, or NULL */
    float norm_eps;
    int32_t cast_after_rope;
    double attn_scale;                /* 1 / sqrt(head_dim) in the reference */
    const int64_t *rope_cos, *rope_sin;  /* device [max_position][head_dim / 2], Q(rope_frac) */
    int32_t rope_frac, max_position;
} ins_seam_cfg;
int ins_seam(ins_cache *cache, int32_t n, const float *q, const float *k, const float *v,
             const int64_t *positions, const ins_seam_cfg *cfg, int32_t *wq, int32_t *wk,
             int32_t *wv, int64_t *conv, void *stream);

/* ins_seam with positions already on the device (int64 [n]), e.g. a model's
 * position_ids tensor, so that the call needs no device-to-host read. The
 * kernel checks each position against max_position instead of the host: a
 * token outside the table gets zero lanes and the next ins_cache_status
 * returns EINVAL (the reference raises ValueError at the call,
 * ops/rope.py:159). */
int ins_seam_device_positions(ins_cache *cache, int32_t n, const float *q, const float *k,
                              const float *v, const int64_t *positions, const ins_seam_cfg *cfg,
                              int32_t *wq, int32_t *wk, int32_t *wv, int64_t *conv, void *stream);

/* ins_ingress fed the board's ingress stream instead of int32 arrays: the
 * byte stream VectorSet.ingress_bytes builds (hw/vectors.py:178-196) -- per
 * token, per KV head h, the vectors k_h, v_h, q_{h*groups} .. q_{h*groups +
 * groups - 1}, each head_dim signed 24-bit lanes packed LSB first
 * (pack_lanes, hw/vectors.py:72-104); 9,216 bytes per token at 8 KV heads
 * with 4 query heads each (ins_lanes_bytes_per_token). lanes: device, n tokens back to back,
 * 2-byte aligned; q_rot: device [n, n_kv*groups, d] int32, required. The lanes
 * are sign-extended on the GPU; everything after is ins_ingress. */
int ins_ingress_lanes(ins_cache *cache, int32_t n, const int32_t *seq_ids, const uint8_t *lanes,
                      int32_t *q_rot, void *stream);
int64_t ins_lanes_bytes_per_token(const ins_cache *cache);

/* Rotation.apply (ops/rotate.py:170-197) alone: n vectors of head_dim int32
 * on the device, x -> y (may alias). Same Q in and out, not clamped; a result
 * that does not fit int32 latches INS_ERANGE. */
int ins_rotate(ins_cache *cache, int64_t n, const int32_t *x, int32_t *y, void *stream);

/* CompressedAttention.scores, fused mode (ops/attention.py:333-359): the
 * kv_groups query heads q_rot (device, [groups, d] int32) against rows
 * [t0, t0+n) of one sequence and KV head. s (device, [groups, n] int64,
 * Q(acc_frac), clamped to score_width); ovf (device, one int64, may be NULL)
 * receives the number of scores the clamp changed. */
int ins_scores(ins_cache *cache, int32_t seq, int32_t kv_head, int64_t t0, int64_t n,
               const int32_t *q_rot, int64_t *s, int64_t *ovf, void *stream);

/* The projections of the host half (matvec, numerics/fp.py:25-62, used by
 * kernel.py:197-210 and the output projection, ops/output.py:80-84) as a
 * kernel of this library: y[t][o] = sum_i w16[o][i] * fp16(x[t][i]) (+ bias[o])
 * with exact fp32 products and fp32 sums, in another order than numpy's (the
 * results agree to float32 rounding). w16: device fp16 [out_dim][in_dim]
 * (raw 16-bit words; the fp16-rounded weights of Weights.prepare,
 * weights.py:70-109), 16-byte aligned; x: device fp32 [n][in_dim]; bias:
 * device fp32 [out_dim] or NULL; y: device fp32 [n][out_dim]. in_dim a
 * multiple of 8 in [8, 8192]. No cache is involved; runs on the device of
 * the current context, stream-ordered. */
int ins_project(int32_t n, int32_t in_dim, int32_t out_dim, const uint16_t *w16, const float *x,
                const float *bias, float *y, void *stream);

/* The scan's finalize on its own: _finalize (ops/attention.py:873-880) with
 * the normalised reciprocal (reciprocal, ops/attention.py:177-250) for n
 * (acc, l) pairs, through the very device function every scan epilogue calls,
 * so the finalize edge cases can be driven directly (the reference treats
 * them as finalize.sv's contract, tests/test_vectors.py:557-634).
 * acc: device int64 [n][head_dim]; l: device int64 [n]; out: device int64
 * [n][head_dim]; recip, shift: device int64 [n] (the reciprocal and the total
 * shift), each may be NULL. Stream-ordered. */
int ins_finalize(ins_cache *cache, int64_t n, const int64_t *acc, const int64_t *l, int64_t *out,
                 int64_t *recip, int64_t *shift, void *stream);

/* ExpLut.__call__ (ops/attention.py:153-159) on the device for n distances
 * (device int64 [n], each >= 0) through the scan kernels' three forms of the
 * lookup: p (device int32 [3][n]) row 0 the general form of the sequential
 * and two-pass scans, row 1 its 32-bit form, row 2 the context-parallel
 * scan's form (zero unless the cache uses the default fixed-point format).
 * A negative distance -- the reference's ValueError (ops/attention.py:
 * 156-157) -- gives -1 and latches INS_ERANGE for ins_cache_status. */
int ins_exp_lut(ins_cache *cache, int64_t n, const int64_t *delta, int32_t *p, void *stream);

/* The code-domain scan: one decode step of attention for B sequences, every
 * KV head, every query head of its group (kernel.py:338-346, with
 * CompressedAttention.attend_online at ops/attention.py:451-513, or
 * attend_two_pass at 429-449).
 *
 * seq_ids (host, B); lengths (host, B, may be NULL): how many leading tokens
 * of each sequence to attend -- the causal prefix kv.select(slice(0, ctx))
 * of kernel.py:387 -- or the whole current length when NULL; q_rot (device,
 * [B, n_kv*groups, d] int32, already rotated and scaled); out (device,
 * [B, n_kv*groups, d] int64, Q(acc_frac) in merge_heads order,
 * ops/project.py:67-74); stats (device, [B, n_kv] ins_stats, may be NULL). */
int ins_scan(ins_cache *cache, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
             const int32_t *q_rot, int64_t *out, ins_stats *stats, ins_softmax mode,
             void *stream);

/* The online scan of ins_scan, allocating no device memory. This entry point
 * has no counterpart in the reference; it exists for callers that cannot
 * allocate device memory once they are running -- an engine that has handed
 * all of HBM to its own pool at start-up, a runtime whose allocator may not be
 * entered from the decode thread, host code that must never block on an
 * allocation mid-step. ins_scan grows its scratch with cudaMalloc when a larger
 * batch or context first arrives; this call instead carves the scratch of the
 * single-launch scan (INS_SCAN_FUSED, whatever ins_cache_set_scan_kernel
 * says) out of one static device array of 192 MiB that every GPU loading this
 * library holds until the process exits.
 *
 * Arguments and results are those of ins_scan with mode INS_SOFTMAX_ONLINE,
 * bit for bit. Limits: at most 4096 sequences, and a scratch layout that fits
 * 192 MiB -- about 2.4 KB per (sequence, KV head, 1,024-token tile) plus
 * about 8.5 KB per (sequence, KV head): some 9M tokens of one sequence at 8
 * KV heads, or about 1,200 sequences of 4K; a call beyond them returns
 * INS_EBADLEN before enqueuing anything. The pool of rescale segments gets
 * what the rest of the layout leaves (at 256 sequences of 4K, room for about
 * 310,000 segments
 * against the 150,000 or so such a batch needs with random keys); an item
 * whose segments do not fit is recomputed by the sequential kernel -- still
 * exact, only slower (ins_scan_recomputed_total counts such items). The first
 * call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current, so make it before any
 * stream capture. Every call clears the parts of the array that must start
 * at zero, but all calls share the one array: calls whose GPU work overlaps
 * (other streams, other threads, other caches on the same device) race on
 * it, so order them. */
int ins_scan_noalloc(ins_cache *cache, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                     const int32_t *q_rot, int64_t *out, ins_stats *stats, void *stream);

/* Export rows [t0, t0+n) of one sequence and KV head in the reference's
 * packed row format (KVQuantizer.pack, ops/quantize.py:237-252), the bytes
 * CompressedCache.buf[t0:t0+n, kv_head] holds (cache/compressed.py:42-52).
 * rows: host, n * bytes_per_token. Blocks until the copy is done. */
int ins_cache_export(ins_cache *cache, int32_t seq, int32_t kv_head, int64_t t0, int64_t n,
                     uint8_t *rows);

/* Append n tokens given as packed rows (host, [n, n_kv, bytes_per_token],
 * the layout of CompressedCache.buf) -- loading a cache image the way the
 * board's CMD_LOAD does (host/attn_proto.h:36). Blocks. */
int ins_cache_import(ins_cache *cache, int32_t seq, int64_t n, const uint8_t *rows);

/* The board's DDR image of one sequence's cache (DdrLayout.image,
 * hw/ddr_layout.py:227-245): the packed rows split at their fields and into
 * 16-byte beats, each plane padded to a 4 KB-aligned span of `capacity`
 * tokens of the widest plane, head-major (plane_span / plane_base,
 * hw/ddr_layout.py:181-212). img: device, ins_ddr_image_bytes(cache,
 * capacity) bytes; stream-ordered. EBADLEN when the sequence holds more than
 * `capacity` tokens (the reference's ValueError). */
int64_t ins_ddr_image_bytes(const ins_cache *cache, int64_t capacity);
int ins_cache_ddr_image(ins_cache *cache, int32_t seq, int64_t capacity, uint8_t *img, void *stream);

/* Read and clear the device status word latched by earlier kernels. Blocks
 * on the stream. INS_OK when nothing went wrong. */
int ins_cache_status(ins_cache *cache, void *stream);

/* How many (sequence, KV head) items of the last online ins_scan on this
 * cache the context-parallel scan handed to the exact sequential kernel (its
 * proof of exactness failed, or a value lay outside the formats it assumes);
 * results are bit-exact either way. A diagnostic with no counterpart in the
 * reference. Blocks on the stream; -1 on error (see ins_last_error). */
int64_t ins_scan_recomputed(ins_cache *cache, void *stream);

/* The running count, since the cache was created, of items that the exact
 * sequential kernel recomputed after the context-parallel online scan could
 * not prove them exact (ins_scan_recomputed counts the last scan only), so
 * that a caller timing many scans can report whether any took the slow path.
 * No reference counterpart. Blocks on the stream; -1 on error. */
int64_t ins_scan_recomputed_total(ins_cache *cache, void *stream);

/* Context split (one sequence's cached tokens held by several shards -- GPUs
 * or caches -- each a causal range). No reference function does this; the reference scans one sequence in one
 * process (ops/attention.py:451-513), and the merged result is that scan's
 * output bit for bit whenever the merge can prove the 32-bit accumulator
 * clamp never fires (otherwise it latches INS_ERANGE, read by
 * ins_cache_status). Online softmax only; needs the context-parallel scan
 * (4b/2b or 3b/3b codes, the default fixed-point format).
 *
 * 1. ins_scan_maxima: scores this shard's items and writes each item's
 *    maximum score per query head to `maxima` (device int64
 *    [B][n_kv][kv_groups]). Keeps the scores for step 2.
 * 2. The caller exchanges the maxima; shard r's m_in is the maximum over
 *    shards before it (-2^47 for the first), same layout.
 * 3. ins_scan_part, with the arguments of step 1: writes one composite per
 *    item to `part` (device, ins_part_bytes(B) bytes).
 * 4. The caller gathers the shards' parts, in causal order, into one device
 *    buffer; ins_merge_parts folds them and writes `out` and `stats` as
 *    ins_scan would for the whole sequences. */
int64_t ins_part_bytes(ins_cache *cache, int32_t B);
int ins_scan_maxima(ins_cache *cache, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                    const int32_t *q_rot, int64_t *maxima, void *stream);
int ins_scan_part(ins_cache *cache, int32_t B, const int32_t *seq_ids, const int64_t *lengths,
                  const int32_t *q_rot, const int64_t *m_in, void *part, void *stream);
int ins_merge_parts(ins_cache *cache, int32_t B, int32_t n_parts, const void *parts, int64_t *out,
                    ins_stats *stats, void *stream);

/* The last error message recorded on this thread ("" if none). */
const char *ins_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
