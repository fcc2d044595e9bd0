// Shared device-side definitions of the B200 compressed-KV attention path.
//
// Integer semantics follow the reference numpy model (INSITU, cited as
// path:line): int64 everywhere a value can grow, arithmetic right shifts that
// floor, and narrowing only at the named clamps.
#pragma once

#include <cstring>
#include <utility>

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/insitu_b200.h"

namespace ins {

constexpr int D = 64;                // head_dim this build supports
constexpr int MAX_ROUNDS = 8;        // rotation rounds carried in the sign masks
constexpr uint32_t FULL = 0xffffffffu;

// Device status bits, latched by kernels and read by ins_cache_status().
enum : int32_t { ST_RANGE = 1, ST_TIMEOUT = 2, ST_INTERNAL = 4, ST_SPLIT = 8, ST_POSITION = 16 };

// Tables, one copy per cache in device global memory.
struct DevTables {
    int64_t k_cent[256];
    int64_t k_bound[256];
    int64_t v_cent[256];
    int64_t v_bound[256];
    double k_cent_f64[256];          // the same key centroids as exact doubles
    int32_t exp_tab[256];
    uint64_t sign_mask[MAX_ROUNDS];  // bit j set: round negates channel j
};

// Geometry and the fixed-point contract, passed to kernels by value.
struct Geo {
    int32_t n_kv, H, kb, vb;
    int32_t kbytes, vbytes, row_bytes;
    int32_t P;                       // tokens per page
    int32_t p_log2;                  // log2(P) when P is a power of two, else -1
    int32_t max_pages;               // page-table row length
    int32_t norm_bits, norm_frac, qk_frac, centroid_frac, acc_frac, acc_width;
    int32_t score_width, prob_frac, exp_lut_bits, saturate;
    int32_t rounds, rot_shift, rot_inv;
    int32_t score_shift, acc_shift, enc_shift;
    int64_t head_bytes, page_bytes;
    int64_t log2e, delta_max;
    // |q| below q_lim keeps every FP64 partial sum of a dot product under
    // 2^53: min(2^30, floor(2^47 / max |key centroid|)), so that 64 products
    // of at most 2^47 each sum exactly; larger queries take the int64 path
    int64_t q_lim;
};

// Byte offsets of one (page, head) region's three planes: K codes (P rows of
// kbytes), V codes (P rows of vbytes), norms (P rows of 4 bytes: k_norm then
// v_norm, little-endian int16).
__host__ __device__ inline int64_t region_off(const Geo &g, int64_t page, int32_t head) {
    return page * g.page_bytes + (int64_t)head * g.head_bytes;
}
__host__ __device__ inline int64_t vplane_off(const Geo &g) { return (int64_t)g.P * g.kbytes; }
__host__ __device__ inline int64_t nplane_off(const Geo &g) {
    return (int64_t)g.P * (g.kbytes + g.vbytes);
}

// A kernel launched with programmatic stream serialization may start while
// the kernel before it on the stream is finishing; this waits until that
// kernel has completed and its memory is visible (a no-op for a kernel
// launched the ordinary way).
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the launch after this one (if launched with programmatic stream
// serialization) be scheduled once every CTA of this grid has called this
// or exited; that launch still waits (wait_prior_grid) before it reads what
// this one writes.
__device__ __forceinline__ void release_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kernel` so that it may start while the previous kernel on the
// stream finishes (programmatic stream serialization); the kernel calls
// wait_prior_grid() before it reads that kernel's results.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_after(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                                cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// A small host->device upload carried as a kernel parameter. Between two
// kernels on a stream a copy-engine transfer of a few bytes left the device
// idle ≈10 µs on either side (measured with CUPTI on B200); a launch in the
// stream's queue costs a few. The parameter is read in place
// (__grid_constant__): up to PARAM_UPLOAD_MAX bytes, the destination 4-byte
// aligned with room for the bytes rounded up to 4.
constexpr int PARAM_UPLOAD_MAX = 3840;
template <int N>
struct ParamBlob {
    uint32_t words;
    uint32_t pad;
    uint32_t w[N / 4];
};

template <int N>
__global__ void __launch_bounds__(256) k_upload(uint32_t *__restrict__ dst, const __grid_constant__ ParamBlob<N> b) {
    wait_prior_grid();                   // the kernel before may still read dst
    for (uint32_t i = threadIdx.x; i < b.words; i += blockDim.x) dst[i] = b.w[i];
}

template <int N>
inline cudaError_t param_upload(void *dst, const void *src, size_t bytes, cudaStream_t s) {
    ParamBlob<N> b;
    b.words = (uint32_t)((bytes + 3) / 4);
    b.pad = 0;
    b.w[b.words - 1] = 0;
    std::memcpy(b.w, src, bytes);
    return launch_after(k_upload<N>, 1u, 256u, 0, s, reinterpret_cast<uint32_t *>(dst), b);
}

// Upload `bytes` from host memory to `dst` on `s`: as k_upload's parameter
// when it fits (*launched = 1; a parameter of 256 bytes or of the maximum,
// whichever holds it), else by a copy from `src` (which must then stay
// unchanged until the copy has run).
inline cudaError_t small_upload(void *dst, const void *src, size_t bytes, cudaStream_t s, int *launched) {
    *launched = 0;
    if (bytes == 0) return cudaSuccess;
    if (bytes <= (size_t)PARAM_UPLOAD_MAX) {
        *launched = 1;
        return bytes <= 256 ? param_upload<256>(dst, src, bytes, s) : param_upload<PARAM_UPLOAD_MAX>(dst, src, bytes, s);
    }
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
}

__device__ __forceinline__ int64_t shfl_xor64(int64_t v, int m) {
    return __shfl_xor_sync(FULL, v, m);
}

// Exact integer square root, digit by digit (two result bits per step), the
// textbook method the reference's isqrt is checked against
// (ops/quantize.py:42-60).
__device__ __forceinline__ uint64_t isqrt_u64(uint64_t a) {
    uint64_t r = 0, bit = 1ull << 62;
    while (bit > a) bit >>= 2;
    while (bit) {
        if (a >= r + bit) {
            a -= r + bit;
            r = (r >> 1) + bit;
        } else {
            r >>= 1;
        }
        bit >>= 2;
    }
    return r;
}

// Round-half-to-even right shift (numerics/fixed.py:83-88).
__device__ __forceinline__ int64_t rshift_even(int64_t a, int n) {
    if (n == 0) return a;
    const int64_t half = 1ll << (n - 1);
    int64_t q = (a + half) >> n;
    if ((a & ((1ll << n) - 1)) == half) q &= ~1ll;
    return q;
}

__device__ __forceinline__ int64_t clamp_bits(int64_t a, int width, bool &hit) {
    const int64_t lo = -(1ll << (width - 1)), hi = (1ll << (width - 1)) - 1;
    hit = a < lo || a > hi;
    return a < lo ? lo : (a > hi ? hi : a);
}

// Q.clamp with the wrap mode kept for completeness (numerics/fixed.py:161-168).
__device__ __forceinline__ int64_t qclamp(int64_t a, int width, int saturate, bool &hit) {
    const int64_t lo = -(1ll << (width - 1)), hi = (1ll << (width - 1)) - 1;
    hit = a < lo || a > hi;
    if (!hit) return a;
    if (saturate) return a < lo ? lo : hi;
    const uint64_t span = 1ull << width;
    const uint64_t u = ((uint64_t)a + (1ull << (width - 1))) & (span - 1);
    return (int64_t)u - (1ll << (width - 1));
}

// ExpLut.__call__ (ops/attention.py:153-159) for delta >= 0: clamp at
// delta_max, t = floor(delta * log2e / 2^acc_frac), then
// table[(t >> shift) & mask] >> integer part, zero past the last one.
__device__ __forceinline__ int32_t exp_lut(const Geo &g, const int32_t *tab, int64_t delta) {
    const int64_t d = delta < g.delta_max ? delta : g.delta_max;
    const int64_t t = (d * g.log2e) >> g.acc_frac;
    const int64_t u = t >> (g.acc_frac - g.exp_lut_bits);
    const int64_t span = (int64_t)(g.prob_frac + 2) << g.exp_lut_bits;
    if (u >= span) return 0;
    return tab[u & ((1 << g.exp_lut_bits) - 1)] >> (int)(u >> g.exp_lut_bits);
}

// exp_lut for a distance known to be non-negative, in 32-bit arithmetic:
// after the clamp d <= delta_max < 2^32, and u = floor(d * log2e / 2^(2*acc_frac
// - exp_lut_bits)) is the same nested floor exp_lut takes in two steps.
__device__ __forceinline__ int32_t exp_lut32(const Geo &g, const int32_t *tab, int64_t delta) {
    const uint32_t d = (uint32_t)(delta < g.delta_max ? delta : g.delta_max);
    const uint64_t prod = (uint64_t)d * (uint64_t)(uint32_t)g.log2e;
    const uint32_t u = (uint32_t)(prod >> (2 * g.acc_frac - g.exp_lut_bits));
    const uint32_t span = (uint32_t)(g.prob_frac + 2) << g.exp_lut_bits;
    return u >= span ? 0 : (tab[u & ((1u << g.exp_lut_bits) - 1u)] >> (u >> g.exp_lut_bits));
}

// 2^62 / den by restoring division, 64 quotient bits.
__device__ __forceinline__ uint64_t div_pow62(uint64_t den) {
    uint64_t q = 0, rem = 0;
    for (int i = 63; i >= 0; --i) {
        rem = (rem << 1) | (i == 62 ? 1ull : 0ull);
        if (rem >= den) {
            rem -= den;
            q |= 1ull << i;
        }
    }
    return q;
}

// The normalised reciprocal (ops/attention.py:177-250): leading one capped
// at L_WIDTH-1 = 47, l shifted into a 32-bit window, r = 2^62 // l_n, and the
// total shift 62 - prob_frac + k.
__device__ __forceinline__ void reciprocal(const Geo &g, int64_t l, int64_t &r, int &shift) {
    int lead = 0;
    if (l >= 2) {
        lead = 63 - __clzll((unsigned long long)l);
        if (lead > 47) lead = 47;
    }
    const int k = lead - 31;
    const int64_t ln = k >= 0 ? (l >> k) : (int64_t)((uint64_t)l << (-k));
    r = l > 0 ? (int64_t)div_pow62((uint64_t)(ln > 1 ? ln : 1)) : 0;
    shift = 62 - g.prob_frac + k;
}

// _finalize (ops/attention.py:873-880) of one channel: acc times the
// normalised reciprocal of l, floored by the total shift; no clamp. Every
// scan's epilogue and ins_finalize go through this one function.
__device__ __forceinline__ int64_t finalize_out(const Geo &g, int64_t acc, int64_t l) {
    int64_t r;
    int shift;
    reciprocal(g, l, r, shift);
    return (acc * r) >> shift;
}

// Code `j` of a row held as 32-bit words, `kb` bits per code, LSB first
// (ops/quantize.py:271-275).
template <int KB>
__device__ __forceinline__ uint32_t code_at(const uint32_t *w, int j, int kb_rt) {
    const int kb = KB ? KB : kb_rt;
    const int pos = j * kb, wi = pos >> 5, sh = pos & 31;
    uint32_t val = w[wi] >> sh;
    if (sh + kb > 32) val |= w[wi + 1] << (32 - sh);
    return val & ((1u << kb) - 1u);
}

// Code `j` of a packed field starting at byte pointer `p`.
__device__ __forceinline__ uint32_t code_at_bytes(const uint8_t *p, int j, int bits,
                                                  int field_bytes) {
    const int pos = j * bits, b = pos >> 3, sh = pos & 7;
    uint32_t v = p[b];
    if (b + 1 < field_bytes) v |= (uint32_t)p[b + 1] << 8;
    return (v >> sh) & ((1u << bits) - 1u);
}

}  // namespace ins
