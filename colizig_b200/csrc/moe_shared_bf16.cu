// BF16 shared expert (addSharedExpert, src/qwen38/moe.zig:467-479, on the
// reference's BF16 NativeMatrix weights, moe.zig:297-338 / tensors.zig:65-120):
//   sh  = silu(x . Wg^T) * (x . Wu^T)          Wg, Wu bf16 [SI][H]
//   out += sigmoid(x . sh_gate) * (sh . Wd^T)   Wd bf16 [H][SI]
// Real Qwen4-Exp checkpoints keep this expert in BF16 (no block scales), so it
// runs beside the block-FP8 routed path as two kernels:
//   shb_gu_kernel   before the routed kernels: gate/up rows and the sigmoid gate
//                   from the layer input (rms-normalised in stack mode), into scratch;
//   shb_down_kernel after them (and after the ranks' combine): out += gate * down.
// Both are HBM-bound GEMVs over bf16 rows: a warp per weight row, 16-byte loads
// (8 bf16) per lane, bf16 widened exactly (bits << 16), f32 FMA sums, tokens
// staged in shared memory in groups of TG (larger batches re-read the rows from L2).
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {
namespace {

constexpr int SHB_WARPS = 8;
constexpr int SHB_THREADS = SHB_WARPS * 32;
constexpr int SHB_UNROLL = 4;  // 256-column chunks in flight per lane and matrix

__device__ __forceinline__ void widen8(const uint4 v, float (&f)[8]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
    f[4] = __uint_as_float(v.z << 16);
    f[5] = __uint_as_float(v.z & 0xffff0000u);
    f[6] = __uint_as_float(v.w << 16);
    f[7] = __uint_as_float(v.w & 0xffff0000u);
}

__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// acc[t] += sum over the row of w[k] * xs[t][k] for the TG staged tokens (K
// columns, a multiple of 8); each lane takes 8-column pieces lane, lane + 32, ...
template <int TG, int NM>
__device__ __forceinline__ void row_dots(const uint16_t* const (&w)[NM], const float* __restrict__ xs, int K, int xstride,
                                         int nt, float (&acc)[NM][TG]) {
    const int lane = threadIdx.x & 31;
    const int npc = K >> 3;  // 8-column pieces
    for (int c0 = 0; c0 < npc; c0 += 32 * SHB_UNROLL) {
        uint4 v[NM][SHB_UNROLL];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int u = 0; u < SHB_UNROLL; ++u) {
                const int pc = c0 + u * 32 + lane;
                v[m][u] = pc < npc ? ld_stream(w[m] + (size_t)pc * 8) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
        for (int u = 0; u < SHB_UNROLL; ++u) {
            const int pc = c0 + u * 32 + lane;
            if (pc >= npc) break;
            float wf[NM][8];
#pragma unroll
            for (int m = 0; m < NM; ++m) widen8(v[m][u], wf[m]);
#pragma unroll
            for (int t = 0; t < TG; ++t) {
                if (t >= nt) break;
                const float4 a = *reinterpret_cast<const float4*>(xs + (size_t)t * xstride + pc * 8);
                const float4 b = *reinterpret_cast<const float4*>(xs + (size_t)t * xstride + pc * 8 + 4);
#pragma unroll
                for (int m = 0; m < NM; ++m) {
                    float s = acc[m][t];
                    s = __fmaf_rn(a.x, wf[m][0], s);
                    s = __fmaf_rn(a.y, wf[m][1], s);
                    s = __fmaf_rn(a.z, wf[m][2], s);
                    s = __fmaf_rn(a.w, wf[m][3], s);
                    s = __fmaf_rn(b.x, wf[m][4], s);
                    s = __fmaf_rn(b.y, wf[m][5], s);
                    s = __fmaf_rn(b.z, wf[m][6], s);
                    s = __fmaf_rn(b.w, wf[m][7], s);
                    acc[m][t] = s;
                }
            }
        }
    }
}

// Tokens [t0, t0 + nt) of x (f32 or bf16 [T][H]) into xs [TG][H] f32; with rms_w,
// rms-normalised as the per-layer caller does (rmsnorm.zig:32-40: f64 sum of
// squares, mean rounded to f32, r = 1/sqrt(mean + eps), v * r * w).
template <int TG>
__device__ void stage_tokens(float* __restrict__ xs, const ShbParams& p, int t0, int nt) {
    const int H = p.H;
    for (int k = threadIdx.x; k < nt * H; k += SHB_THREADS) {
        const int t = k / H, i = k - t * H;
        const size_t g = (size_t)(t0 + t) * H + i;
        xs[(size_t)t * H + i] = p.x_bf16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p.x)[g] << 16)
                                         : reinterpret_cast<const float*>(p.x)[g];
    }
    __syncthreads();
    if (!p.rms_w) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float rs[TG];
    for (int t = warp; t < nt; t += SHB_WARPS) {
        double ss = 0.0;
        for (int i = lane; i < H; i += 32) {
            const double v = (double)xs[(size_t)t * H + i];
            ss = __fma_rn(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) {
            const float mean = __double2float_rn(__ddiv_rn(ss, (double)H));
            rs[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < nt * H; k += SHB_THREADS) {
        const int t = k / H, i = k - t * H;
        xs[k] = __fmul_rn(__fmul_rn(xs[k], rs[t]), p.rms_w[i]);
    }
    __syncthreads();
}

// Gate/up rows (CTAs [0, SI/8)) and the sigmoid gate (the last CTA).
template <int TG>
__global__ void __launch_bounds__(SHB_THREADS) shb_gu_kernel(const ShbParams p) {
    extern __shared__ __align__(16) float xs[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, SI = p.SI;
    const int nrb = SI / SHB_WARPS;
    const bool gate_cta = (int)blockIdx.x == nrb;
    const int j = blockIdx.x * SHB_WARPS + warp;  // this warp's row
    for (int t0 = 0; t0 < p.T; t0 += TG) {
        const int nt = p.T - t0 < TG ? p.T - t0 : TG;
        stage_tokens<TG>(xs, p, t0, nt);
        if (!gate_cta) {
            float acc[2][TG];
#pragma unroll
            for (int t = 0; t < TG; ++t) acc[0][t] = acc[1][t] = 0.f;
            const uint16_t* const w[2] = {p.wg + (size_t)j * H, p.wu + (size_t)j * H};
            row_dots<TG, 2>(w, xs, H, H, nt, acc);
#pragma unroll
            for (int t = 0; t < TG; ++t) {
                if (t >= nt) break;
                const float g = warp_sum(acc[0][t]), u = warp_sum(acc[1][t]);
                if (lane == 0) p.hsh[(size_t)(t0 + t) * SI + j] = __fmul_rn(cz_silu(g), u);
            }
        } else {
            // sgate = sigmoid(sum x[d] * sh_gate[d]) (moe.zig:476-478)
            for (int t = warp; t < nt; t += SHB_WARPS) {
                float s = 0.f;
                for (int i = lane; i < H; i += 32) s = __fmaf_rn(xs[(size_t)t * H + i], p.sh_gate[i], s);
                s = warp_sum(s);
                if (lane == 0) p.sg[t0 + t] = cz_sigmoid(s);
            }
        }
        __syncthreads();
    }
}

// Down rows: out[t][o] += sg[t] * (hsh[t] . Wd[o]).
template <int TG>
__global__ void __launch_bounds__(SHB_THREADS) shb_down_kernel(const ShbParams p) {
    extern __shared__ __align__(16) float hs[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, SI = p.SI;
    const int o = blockIdx.x * SHB_WARPS + warp;
    for (int t0 = 0; t0 < p.T; t0 += TG) {
        const int nt = p.T - t0 < TG ? p.T - t0 : TG;
        for (int k = threadIdx.x; k < nt * SI; k += SHB_THREADS) hs[k] = p.hsh[(size_t)t0 * SI + k];
        __syncthreads();
        if (o < H) {
            float acc[1][TG];
#pragma unroll
            for (int t = 0; t < TG; ++t) acc[0][t] = 0.f;
            const uint16_t* const w[1] = {p.wd + (size_t)o * SI};
            row_dots<TG, 1>(w, hs, SI, SI, nt, acc);
#pragma unroll
            for (int t = 0; t < TG; ++t) {
                if (t >= nt) break;
                const float d = warp_sum(acc[0][t]);
                if (lane == 0) {
                    float* dst = p.out + (size_t)(t0 + t) * H + o;
                    *dst = __fadd_rn(*dst, __fmul_rn(p.sg[t0 + t], d));
                }
            }
        }
        __syncthreads();
    }
}

template <int TG>
int launch_tg(const ShbParams& p, bool gu, cudaStream_t st) {
    if (gu) {
        const size_t smem = (size_t)TG * p.H * 4;
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(shb_gu_kernel<TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
            return CZ_ELAUNCH;
        shb_gu_kernel<TG><<<p.SI / SHB_WARPS + 1, SHB_THREADS, smem, st>>>(p);
    } else {
        const size_t smem = (size_t)TG * p.SI * 4;
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(shb_down_kernel<TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
            return CZ_ELAUNCH;
        shb_down_kernel<TG><<<(p.H + SHB_WARPS - 1) / SHB_WARPS, SHB_THREADS, smem, st>>>(p);
    }
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

}  // namespace

bool shb_supported(int H, int SI) {
    // whole 8-column pieces (16-byte rows), warp-sized row blocks, tokens staged in shared memory
    return H > 0 && SI > 0 && H % 8 == 0 && SI % SHB_WARPS == 0 && SI % 8 == 0 && (size_t)8 * H * 4 <= 200 * 1024 &&
           (size_t)8 * SI * 4 <= 200 * 1024;
}

size_t shb_scratch_bytes(int T, int SI) { return ((size_t)T * SI * 4 + 255) / 256 * 256 + (size_t)T * 4; }

int shb_launch(const ShbParams& p, bool gate_up, cudaStream_t st) {
    if (p.T <= 0) return CZ_OK;
    if (!shb_supported(p.H, p.SI)) return CZ_ESHAPE;
    if (p.T == 1) return launch_tg<1>(p, gate_up, st);
    if (p.T <= 4) return launch_tg<4>(p, gate_up, st);
    return launch_tg<8>(p, gate_up, st);
}

}  // namespace cz
