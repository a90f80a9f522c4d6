// The reference backend's per-matrix op (colizig_cuda.cu:45-76 mm_fp8_kernel,
// fp8.zig:162-188 matmulFp8Keyed):
//   y[S,O] = x[S,I] @ (e4m3(w[O,I]) * scales[o/128, i/128])^T
// Two output rows per warp, four tokens per pass.  When I is a multiple of 16
// (every model projection) lanes read 16-byte chunks (coalesced), decode them
// with the hardware E4M3->f16 conversion and fold the block scale once per
// chunk; any other I takes a byte-wise path.  f32 accumulation throughout, in
// the same order for every row whatever the rows per warp.
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {

constexpr int kMmWarps = 8;
constexpr int kMmChunks = 4;  // 16-byte chunks of a row in flight per lane
constexpr int kMmRows = 2;    // output rows per warp (their chunks in flight together, one read of x for both)

__global__ void __launch_bounds__(kMmWarps * 32) fp8_matmul_kernel(float* __restrict__ y, const float* __restrict__ x,
                                                                  const uint8_t* __restrict__ w,
                                                                  const float* __restrict__ scales, int S, int I,
                                                                  int O) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int o0 = (blockIdx.x * kMmWarps + warp) * kMmRows;
    if (o0 >= O) return;
    const int nr = min(kMmRows, O - o0);
    const int nbi = cz_nblk(I);
    if ((I % 16) != 0) {
        // byte-wise path (shapes that are not whole 16-byte chunks), one row at a time
        for (int r = 0; r < nr; ++r) {
            const uint8_t* wr = w + (size_t)(o0 + r) * I;
            const float* sr = scales + (size_t)((o0 + r) >> 7) * nbi;
            for (int s0 = 0; s0 < S; s0 += 4) {
                const int ns = min(4, S - s0);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                for (int i = lane; i < I; i += 32) {
                    const float wv = e4m3x2_to_f32x2((uint16_t)__ldg(wr + i)).x * __ldg(sr + (i >> 7));
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (q < ns) acc[q] = __fmaf_rn(__ldg(x + (size_t)(s0 + q) * I + i), wv, acc[q]);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float v = warp_sum(acc[q]);
                    if (lane == 0 && q < ns) y[(size_t)(s0 + q) * O + o0 + r] = v;
                }
            }
        }
        return;
    }
    // lanes read 16-byte chunks (coalesced), decode them with the hardware E4M3 -> f16
    // conversion and fold the block scale once per chunk; kMmChunks chunks of each of
    // the warp's rows are in flight before any is used (a decode-sized call is one
    // pass: the loads, not the arithmetic, set its time)
    const uint8_t* wr[kMmRows];
    const float* sr[kMmRows];
#pragma unroll
    for (int r = 0; r < kMmRows; ++r) {
        const int o = r < nr ? o0 + r : o0;
        wr[r] = w + (size_t)o * I;
        sr[r] = scales + (size_t)(o >> 7) * nbi;
    }
    const int nch = I >> 4;
    for (int s0 = 0; s0 < S; s0 += 4) {
        const int ns = min(4, S - s0);
        float acc[kMmRows][4] = {};
        for (int c0 = lane; c0 < nch; c0 += 32 * kMmChunks) {
            uint4 wv[kMmRows][kMmChunks];
#pragma unroll
            for (int r = 0; r < kMmRows; ++r)
#pragma unroll
                for (int u = 0; u < kMmChunks; ++u)
                    wv[r][u] = (r < nr && c0 + 32 * u < nch)
                                   ? __ldg(reinterpret_cast<const uint4*>(wr[r]) + c0 + 32 * u)
                                   : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int u = 0; u < kMmChunks; ++u) {
                const int ch = c0 + 32 * u;
                if (ch >= nch) break;
                float f[kMmRows][16];
                float sc[kMmRows];
#pragma unroll
                for (int r = 0; r < kMmRows; ++r) {
                    decode16(wv[r][u], f[r]);
                    sc[r] = __ldg(sr[r] + (ch >> 3));
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (q < ns) {
                        const float4* xp = reinterpret_cast<const float4*>(x + (size_t)(s0 + q) * I) + ch * 4;
                        float4 xv[4];
#pragma unroll
                        for (int v = 0; v < 4; ++v) xv[v] = __ldg(xp + v);
#pragma unroll
                        for (int r = 0; r < kMmRows; ++r) {
                            float d0 = 0.f, d1 = 0.f;
#pragma unroll
                            for (int v = 0; v < 4; ++v) {
                                d0 = __fmaf_rn(xv[v].x, f[r][4 * v + 0], d0);
                                d1 = __fmaf_rn(xv[v].y, f[r][4 * v + 1], d1);
                                d0 = __fmaf_rn(xv[v].z, f[r][4 * v + 2], d0);
                                d1 = __fmaf_rn(xv[v].w, f[r][4 * v + 3], d1);
                            }
                            acc[r][q] = __fmaf_rn(sc[r], d0 + d1, acc[r][q]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kMmRows; ++r)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float v = warp_sum(acc[r][q]);
                if (lane == 0 && q < ns && r < nr) y[(size_t)(s0 + q) * O + o0 + r] = v;
            }
    }
}

int fp8_matmul_launch(float* y, const float* x, const uint8_t* w, const float* scales, int S, int I, int O,
                      cudaStream_t stream) {
    if (S < 1 || I < 1 || O < 1) return CZ_EARGS;
    const int blocks = (O + kMmWarps * kMmRows - 1) / (kMmWarps * kMmRows);
    fp8_matmul_kernel<<<blocks, kMmWarps * 32, 0, stream>>>(y, x, w, scales, S, I, O);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

__global__ void debug_expf_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = cz_expf(x[i]);
}

int debug_expf_launch(const float* x, float* y, size_t n, cudaStream_t stream) {
    if (n == 0) return CZ_OK;
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    debug_expf_kernel<<<blocks, 256, 0, stream>>>(x, y, n);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

}  // namespace cz
