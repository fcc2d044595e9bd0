// Launch selection for the online scan.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace ins {

// Device scratch owned by the cache handle for the context-parallel scan.
struct ChunkScratch {
    void release() {}
};

template <int H>
inline cudaError_t launch_seq(const Geo &g, const DevTables *tb, int32_t B, const int32_t *d_seq,
                              const int64_t *d_lens, const int32_t *d_pt, const uint8_t *pool,
                              const int32_t *q_rot, int64_t *out, ins_stats *stats,
                              const int32_t *only, cudaStream_t s) {
    const size_t smem = (size_t)H * g.P * (8 + 4 + 4 + 1) + (size_t)g.P * g.vbytes +
                        (size_t)g.P * 4;
    auto fn = (g.kb == 4 && g.vb == 2)   ? k_scan_seq<H, 4, 2>
              : (g.kb == 3 && g.vb == 3) ? k_scan_seq<H, 3, 3>
                                         : k_scan_seq<H, 0, 0>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    fn<<<B * g.n_kv, H * 64, smem, s>>>(g, tb, d_seq, d_lens, d_pt, pool, q_rot, out, stats, only);
    return cudaGetLastError();
}

inline int launch_online(ChunkScratch &cs, const Geo &g, const DevTables *tb, int32_t B,
                         const int32_t *d_seq, const int64_t *d_lens, const int64_t *h_lens,
                         const int32_t *d_pt, const uint8_t *pool, const int32_t *q_rot,
                         int64_t *out, ins_stats *stats, int32_t *d_status, int H,
                         cudaStream_t s) {
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
