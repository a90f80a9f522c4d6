// Expert parallelism with sharded tokens: the device halves of the exchange.
//
// Each rank routes its own tokens, sends every token row once to each rank
// that holds one of its experts (with the token's full top-k ids and gates),
// runs the grouped expert pipeline on the rows it receives (pairs of experts it
// does not hold are skipped), sends each row's partial sum back, and adds the
// partials of its tokens in ascending rank order, i.e. ascending expert ranges
// (moe.zig forwardGrouped, 597-665, split over ranks).  The host side (counts,
// NCCL send/recv) is in api.cu.
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {
namespace {

constexpr int kMaxWorld = 32;

// Rank holding expert e: the last r with r*E/W <= e (the partition of
// colizig_cuda_moe_register_layer with COLIZIG_EP).
__device__ __forceinline__ int expert_owner(int e, int E, int W) {
    int r = (int)(((long long)e * W) / E);
    while (r + 1 < W && (long long)(r + 1) * E / W <= e) ++r;
    while (r > 0 && (long long)r * E / W > e) --r;
    return r;
}

__global__ void ep_mask_kernel(const uint32_t* idx, int T, int K, int E, int W, int* mask) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    uint32_t m = 0;
    for (int z = 0; z < K; ++z) {
        const int e = (int)idx[(size_t)t * K + z];
        if (e >= 0 && e < E) m |= 1u << expert_owner(e, E, W);
    }
    mask[t] = (int)m;
}

// One block of 1024 threads: thread i owns tokens [i*per, (i+1)*per).  For
// destination d (in order), the tokens that go to d get consecutive slots in
// token order, after all of destination d-1's.
__global__ void __launch_bounds__(1024) ep_slot_kernel(const int* mask, int T, int W, int* slot, int* counts) {
    __shared__ int wsum[32];
    __shared__ int dbase;
    const int per = (T + blockDim.x - 1) / blockDim.x;
    const int t0 = threadIdx.x * per, t1 = min(T, t0 + per);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (threadIdx.x == 0) dbase = 0;
    __syncthreads();
    for (int d = 0; d < W; ++d) {
        int c = 0;
        for (int t = t0; t < t1; ++t) c += (mask[t] >> d) & 1;
        // exclusive scan of c over the block
        int x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int v = lane < nw ? wsum[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            if (lane < nw) wsum[lane] = v;
        }
        __syncthreads();
        int run = dbase + x - c + (warp ? wsum[warp - 1] : 0);
        for (int t = t0; t < t1; ++t) {
            const bool go = (mask[t] >> d) & 1;
            slot[(size_t)t * W + d] = go ? run : -1;
            run += go;
        }
        const int tot = wsum[nw - 1];
        __syncthreads();
        if (threadIdx.x == 0) {
            counts[d] = tot;
            dbase += tot;
        }
        __syncthreads();
    }
}

// One block per token: its row to every destination slot.
__global__ void ep_pack_kernel(const uint8_t* x, size_t xrow, const uint32_t* idx, const float* gates, int K, int W,
                               const int* slot, uint8_t* send, size_t rs) {
    const int t = blockIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * xrow);
    const int n16 = (int)(xrow / 16);
    for (int d = 0; d < W; ++d) {
        const int sl = slot[(size_t)t * W + d];
        if (sl < 0) continue;
        uint8_t* row = send + (size_t)sl * rs;
        uint4* dst = reinterpret_cast<uint4*>(row);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
        uint32_t* ri = reinterpret_cast<uint32_t*>(row + xrow);
        float* rg = reinterpret_cast<float*>(row + xrow + (size_t)K * 4);
        for (int z = threadIdx.x; z < K; z += blockDim.x) {
            ri[z] = idx[(size_t)t * K + z];
            rg[z] = gates[(size_t)t * K + z];
        }
    }
}

__global__ void ep_unpack_kernel(const uint8_t* recv, size_t rs, size_t xrow, int K, uint8_t* x, uint32_t* idx,
                                 float* gates) {
    const int r = blockIdx.x;
    const uint8_t* row = recv + (size_t)r * rs;
    const uint4* src = reinterpret_cast<const uint4*>(row);
    uint4* dst = reinterpret_cast<uint4*>(x + (size_t)r * xrow);
    const int n16 = (int)(xrow / 16);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    const uint32_t* ri = reinterpret_cast<const uint32_t*>(row + xrow);
    const float* rg = reinterpret_cast<const float*>(row + xrow + (size_t)K * 4);
    for (int z = threadIdx.x; z < K; z += blockDim.x) {
        idx[(size_t)r * K + z] = ri[z];
        gates[(size_t)r * K + z] = rg[z];
    }
}

__global__ void ep_combine_kernel(const float* back, const int* slot, int T, int W, int H, const float* residual,
                                  float* out) {
    const int per = H / 4;
    const long long gi = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int t = (int)(gi / per), o4 = (int)(gi - (long long)t * per);
    if (t >= T) return;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    bool first = true;
    for (int d = 0; d < W; ++d) {
        const int sl = slot[(size_t)t * W + d];
        if (sl < 0) continue;
        const float4 v = *reinterpret_cast<const float4*>(back + (size_t)sl * H + (size_t)o4 * 4);
        if (first) {
            s = v;
            first = false;
        } else {
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
    }
    if (residual) {
        const float4 r = *reinterpret_cast<const float4*>(residual + (size_t)t * H + (size_t)o4 * 4);
        s.x = __fadd_rn(r.x, s.x);
        s.y = __fadd_rn(r.y, s.y);
        s.z = __fadd_rn(r.z, s.z);
        s.w = __fadd_rn(r.w, s.w);
    }
    *reinterpret_cast<float4*>(out + (size_t)t * H + (size_t)o4 * 4) = s;
}

}  // namespace

int ep_plan(const uint32_t* idx, int T, int K, int E, int W, int* slot, int* counts, void* tmp, size_t tmp_bytes,
            cudaStream_t st) {
    if (W < 1 || W > kMaxWorld || T < 0 || (size_t)T * 4 > tmp_bytes) return CZ_EARGS;
    if (T == 0) return cudaMemsetAsync(counts, 0, (size_t)W * 4, st) == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
    int* mask = reinterpret_cast<int*>(tmp);
    ep_mask_kernel<<<(T + 255) / 256, 256, 0, st>>>(idx, T, K, E, W, mask);
    ep_slot_kernel<<<1, 1024, 0, st>>>(mask, T, W, slot, counts);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

int ep_pack(const void* x, size_t xrow_bytes, const uint32_t* idx, const float* gates, int T, int K, int W,
            const int* slot, uint8_t* send, size_t rs, cudaStream_t st) {
    if (T == 0) return CZ_OK;
    if (xrow_bytes % 16 || rs % 16) return CZ_EARGS;
    ep_pack_kernel<<<T, 128, 0, st>>>(reinterpret_cast<const uint8_t*>(x), xrow_bytes, idx, gates, K, W, slot, send,
                                      rs);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

int ep_unpack(const uint8_t* recv, size_t rs, int R, size_t xrow_bytes, int K, void* x, uint32_t* idx, float* gates,
              cudaStream_t st) {
    if (R == 0) return CZ_OK;
    ep_unpack_kernel<<<R, 128, 0, st>>>(recv, rs, xrow_bytes, K, reinterpret_cast<uint8_t*>(x), idx, gates);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

int ep_combine(const float* back, const int* slot, int T, int W, int H, const float* residual, float* out,
               cudaStream_t st) {
    if (T == 0) return CZ_OK;
    const long long n = (long long)T * (H / 4);
    ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(back, slot, T, W, H, residual, out);
    return cudaGetLastError() == cudaSuccess ? CZ_OK : CZ_ELAUNCH;
}

}  // namespace cz
