// Decode-regime MoE layer (up to 4 tokens per launch) as ONE persistent
// cooperative kernel.
//
// Reference path (src/qwen38/moe.zig): route (435-463) -> per expert gate/up
// (fp8.zig:165-257) -> silu(g)*u (activation.zig:8-20) -> down -> out += gate*eo,
// plus the always-on shared expert (467-479).
//
// Grid = one CTA per SM: 8 consumer warps + 1 producer warp.  The weights go
// HBM -> shared memory through a ring of bulk-copy (TMA) stages filled by one
// producer thread; no global memory is read inside a compute loop.
//
//   R  router logits.  CTA c owns router rows [c*E'/G, (c+1)*E'/G) (E' = E, +1
//      for the shared expert's gate vector).  Rows and tokens are bulk-copied
//      into shared memory; every logit is formed in the reference's exact f32
//      order (dotF32, matmul.zig:60-82: 32 FMA chains = one per lane, then the
//      lane-ordered combine), so the top-k below is bit-identical to it.  In
//      stack mode the tokens are rms-normalised in place first.  The tokens are
//      then split into E4M3 terms (below).  A grid-wide arrive counter closes
//      the phase.
//   K  top-k.  Every CTA bulk-copies the logits, computes softmax/top-k for all
//      tokens (identically) and groups the (token, slot) pairs by expert
//      (ascending id, shared expert last).  Under expert parallelism a GPU
//      holds experts [e_lo, e_hi) only; the other groups get no chunks here and
//      the GPUs' outputs are summed by one all-reduce after the launch.
//   C  chunks.  Each group's intermediate rows are cut into chunks of 16; the
//      flattened chunk list is split evenly over the CTAs (split-K: a chunk's
//      gate, up AND down work stays on one SM, so h never leaves it).  Pass 1
//      streams, per chunk, gate rows [r0, r0+16) x 2048-column slabs of H (one
//      bulk copy per row) and the same for up; the consumer warps split the
//      K blocks, reduce, and keep h = silu(gate)*up of every chunk in shared
//      memory.  Pass 2 streams, per slab of output rows, the down columns
//      [r0, r0+16) of every chunk of the CTA (2D TMA boxes of 16 x 256); each
//      warp owns 16-row output tiles and accumulates all of the CTA's chunks
//      into registers, then writes its rows of the CTA's partial [T][H] to
//      global scratch once.  The weight copies carry an L2 evict-first hint:
//      streamed once, they should not push the kernel's code, the router rows
//      or the scratch out of L2.
//
// Arithmetic: mma.sync m16n8k32 E4M3 x E4M3 -> f32, which forms and sums the
// exact products (checked on B200 to round like f32).  The weights enter as
// their stored bytes.  The other operand is split exactly into E4M3 terms: a
// token x (scaled by 2^s so that max|x| lies in [128, 256)) = t1 + t2 (+ t3),
// every term a column of the MMA; a bf16 token is exact in 2 terms, an f32
// token is kept to 12 bits in 3; h (per chunk and pair, scaled the same way)
// to 16 bits in 4 terms.  Each 128-column block's sum is multiplied by its
// 128x128 scale in f32.  Down sums accumulate in registers (every output row
// owned by one warp, chunks in a fixed order); each CTA writes its partial
// [T][H] once, and after a grid-wide arrive counter CTA c adds the G partial
// rows of its slice of out in a fixed order: deterministic, no float atomics.
//
// Every wait is bounded; a CTA that gives up sets a bit in the device error
// word, stops issuing work (draining its in-flight copies) and the host
// returns -7.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {

constexpr int NCW = 8;                    // consumer warps (2 per SM sub-partition)
constexpr int PW = NCW;                   // producer warp
constexpr int HW = NCW + 1;               // h warp
constexpr int NWARPS = NCW + 2;
constexpr int NTHREADS = NWARPS * 32;
constexpr int CR = 16;                    // intermediate (h) rows per chunk
constexpr int KS = 2048;                  // columns of a gate/up stage slab
constexpr int OS = 2048;                  // output rows of a down stage
constexpr int GU_BYTES = CR * KS;         // a gate/up stage: [K block][16 rows][128 B], 128-byte swizzled
constexpr int SC_BYTES = 2048;            // block scales carried with every stage
constexpr int SLOT_BYTES = 34 * 1024;     // >= GU_BYTES + SC_BYTES; a down stage uses OS * 16
constexpr int NSLOT = 4;                  // ring slots at least (more when shared memory allows)
constexpr int MAXSLOT = 6;
constexpr int RING_BYTES = NSLOT * SLOT_BYTES;  // the smallest ring (also stages phase R)
constexpr int BOX_ROWS = 256;             // down-weight TMA box: 16 bytes x 256 rows
constexpr int JH = 4;                     // E4M3 terms of h
constexpr int MAXCH = 32;                 // chunks per CTA (h terms of all of them stay in shared memory)
constexpr int MAXT = kDecodeMaxTokens;    // 4
constexpr int MAXK = kMaxTopk;            // 16
constexpr int MAXE = kMaxExperts;         // 512
constexpr int MAXP = MAXT * (MAXK + 1);   // (token, slot) pairs incl. shared-expert pairs: 68
constexpr int MAXG = MAXP;                // groups <= pairs
constexpr int SMEM_LIMIT = 227 * 1024;

static_assert(GU_BYTES + SC_BYTES <= SLOT_BYTES, "slot");
static_assert(OS * 16 <= GU_BYTES, "down stage");
static_assert(SLOT_BYTES % 1024 == 0, "TMA destinations stay 1024-aligned");

// Small shared state (after the large regions).
struct __align__(16) DecodeMisc {
    uint64_t full[MAXSLOT];
    uint64_t empty[MAXSLOT];
    uint64_t rbar;
    uint64_t lbar;
    int abort;
    int U, P, NC;
    uint32_t xmax[MAXT];  // max |x_t| (f32 bits)
    int xexp[MAXT];       // s per token (terms hold x_t * 2^s)
    float xscale[MAXT];   // 2^-s per token
    float sdcol[2][64];   // down scales of a chunk's column block, one per 128 output rows (chunk parity)
    float hmax[MAXT][64]; // max over chunks of |gate * h * down scale| per (token, 128-row block)
    int hexp[MAXT][64];   // its power-of-two prescale
    int pe[MAXP];         // expert of pair p = t*K + z (shared: p = T*K + t -> E)
    float pg[MAXP];       // gate of pair p
    int order[MAXP];      // pairs sorted by (expert, pair)
    int g_expert[MAXG];
    int g_pair0[MAXG];
    int g_npairs[MAXG];
    int g_chunk0[MAXG + 1];
};

// Shared-memory map of one launch: [ring][x terms][red][h of every chunk][misc].
struct Carve {
    int JX, CS;  // E4M3 terms per token; byte stride of one term column
    int ns;      // ring slots
    uint32_t xterm, red, hterm, misc, total;
};

__host__ __device__ inline Carve carve(int T, int H, int x_bf16) {
    Carve c;
    c.JX = x_bf16 ? 2 : 3;
    c.CS = ((H + 127) & ~127) + 64;  // column stride = 64 mod 128: lanes of 2 columns hit disjoint banks
    // the rest of the map decides how many slots fit
    const uint32_t rest = (((uint32_t)(T * c.JX * c.CS) + 127u) & ~127u) + 2 * NCW * 2 * 16 * 16 * 4 +
                          MAXCH * 16 * MAXT * 4 + (((uint32_t)sizeof(DecodeMisc) + 127u) & ~127u);
    const int fit = ((int)SMEM_LIMIT - 1024 - (int)rest) / SLOT_BYTES;
    c.ns = fit < NSLOT ? NSLOT : (fit > MAXSLOT ? MAXSLOT : fit);
    uint32_t off = (uint32_t)c.ns * SLOT_BYTES;
    c.xterm = off;
    off += ((uint32_t)(T * c.JX * c.CS) + 127u) & ~127u;
    c.red = off;
    off += 2 * NCW * 2 * 16 * 16 * 4;  // two chunks in flight: [chunk parity][warp][gate/up][16 x 16]
    c.hterm = off;
    off += MAXCH * 16 * MAXT * 4;  // h of every chunk: [chunk][16 rows][MAXT tokens] f32
    c.misc = off;
    off += ((uint32_t)sizeof(DecodeMisc) + 127u) & ~127u;
    c.total = off;
    return c;
}

// ---- sync words ------------------------------------------------------------
// sync[0] = launch sequence number, sync[1] = error word, then two regions of
// kSyncRegionWords: [0] router arrivals, [1] CTAs done, [2] partial sums
// written.  A launch uses region seq&1 and zeroes the other one, so a launch
// that stopped early leaves nothing behind.
__device__ __forceinline__ uint32_t* region(uint32_t* sync, int par) { return sync + 2 + par * kSyncRegionWords; }

struct GroupW {
    const uint8_t *gw, *uw;
    const float *gs, *us, *ds;
    int inter;
    int down_row0;                // first row of this expert in its down tensor map
    int gu_row0;                  // first row of this expert in its gate/up tensor maps
    int dgrp;                     // down boxes: groups of 256 rows per box (0 = 2D boxes)
    const CUtensorMap *dmap, *gmap, *umap;
};

__device__ __forceinline__ GroupW group_w(const DecodeParams& p, int e) {
    GroupW g;
    if (e == p.E) {
        g.inter = p.SI;
        g.gw = p.sh_gate_w;
        g.uw = p.sh_up_w;
        g.gs = p.sh_gate_s;
        g.us = p.sh_up_s;
        g.ds = p.sh_down_s;
        g.down_row0 = 0;
        g.gu_row0 = 0;
        g.dgrp = p.sh_dn_grp;
        g.dmap = &p.sh_down_map;
        g.gmap = &p.sh_gate_map;
        g.umap = &p.sh_up_map;
    } else {
        g.inter = p.I;
        e -= p.e_lo;  // experts are stacked from the first one held here
        const size_t wsz = (size_t)p.I * p.H;
        g.gw = p.gate_w + (size_t)e * wsz;
        g.uw = p.up_w + (size_t)e * wsz;
        const size_t ssz = (size_t)cz_nblk(p.I) * cz_nbp(p.H);
        g.gs = p.gate_s + (size_t)e * ssz;
        g.us = p.up_s + (size_t)e * ssz;
        g.ds = p.down_s + (size_t)e * cz_nblk(p.H) * cz_nbp(p.I);
        g.down_row0 = e * p.H;
        g.gu_row0 = e * p.I;
        g.dgrp = p.dn_grp;
        g.dmap = &p.down_map;
        g.gmap = &p.gate_map;
        g.umap = &p.up_map;
    }
    return g;
}

__device__ void set_error(uint32_t* err, DecodeMisc& s, uint32_t bit) {
    atomicOr(err, bit);
    s.abort = 1;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Bulk copy global -> shared with an L2 cache-policy hint (streamed weights).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// One 2D TMA box (16 x 256 bytes) of a u8 tensor map -> shared memory (no multicast).
__device__ __forceinline__ void tma_box_g2s(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// One 3D TMA box of a u8 tensor map -> shared memory (no multicast).
__device__ __forceinline__ void tma_box3_g2s(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                             uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void mma_e4m3(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Power-of-two exponent s with max * 2^s in [128, 256) (0 for max == 0 or
// non-finite), so that the leading E4M3 term never saturates (max 448); read
// off the exponent bits (mx in [2^(be-127), 2^(be-126)) for a normal mx), and
// clamped to [-100, 100] so that 2^s and 2^-s are normal floats.
__device__ __forceinline__ int prescale_exp(float mx) {
    const int be = (int)(__float_as_uint(mx) >> 23);
    if (!(mx > 0.0f) || be >= 255) return 0;
    return max(-100, min(134 - be, 100));
}

// v * 2^e for e in [-126, 127] (exact while the product is a normal float).
__device__ __forceinline__ float scale2(float v, int e) { return v * __int_as_float((127 + e) << 23); }

// silu with the fast exponential (relative error ~1e-6, far inside the
// layer-output tolerance).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Two values -> their next E4M3 terms (round to nearest even; bytes lo = a,
// hi = b) and the residuals a - term(a), b - term(b), which are exact.
__device__ __forceinline__ uint16_t e4m3_term2(float& a, float& b) {
    uint16_t d;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(b), "f"(a));
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(d));
    const __half2 hv = *reinterpret_cast<__half2*>(&h2);
    a = __fsub_rn(a, __low2float(hv));
    b = __fsub_rn(b, __high2float(hv));
    return d;
}

// Router dot of one row with one token, in dotF32's exact order (lane l holds
// chain l: elements l, l+32, ...; then the lane-ordered combine and the FMA
// tail).  wrow / xs are shared memory.  Returns the logit in every lane.  Kept
// rolled and out of line: it runs once per launch, fetched cold.
template <bool BF16>
__device__ __noinline__ float router_dot(const float* __restrict__ wrow, const uint8_t* __restrict__ xs, int H,
                                         int lane) {
    auto xv = [&](int i) -> float {
        return BF16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(xs)[i] << 16)
                    : reinterpret_cast<const float*>(xs)[i];
    };
    float acc = 0.0f;
    int i = 0;
    // batches of 16 elements per lane: the loads go out together, the FMAs keep the chain order
#pragma unroll 1
    for (; i + 512 <= H; i += 512) {
        float xb[16], wb[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            xb[j] = xv(i + 32 * j + lane);
            wb[j] = wrow[i + 32 * j + lane];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = __fmaf_rn(xb[j], wb[j], acc);
    }
#pragma unroll 1
    for (; i + 32 <= H; i += 32) acc = __fmaf_rn(xv(i + lane), wrow[i + lane], acc);
#pragma unroll 1
    for (; i + 8 <= H; i += 8)  // a final 8-wide block: lanes 0..7 only
        if (lane < 8) acc = __fmaf_rn(xv(i + lane), wrow[i + lane], acc);
    // total[l] = (((0 + acc0[l]) + acc1[l]) + acc2[l]) + acc3[l]; chain k = lanes 8k..8k+7
    const float a8 = __shfl_down_sync(0xffffffffu, acc, 8);
    const float a16 = __shfl_down_sync(0xffffffffu, acc, 16);
    const float a24 = __shfl_down_sync(0xffffffffu, acc, 24);
    const float tl = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, acc), a8), a16), a24);
    float sum = __shfl_sync(0xffffffffu, tl, 0);
#pragma unroll 1
    for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, tl, l));
#pragma unroll 1
    for (; i < H; ++i) sum = __fmaf_rn(xv(i), wrow[i], sum);
    return sum;
}

// Top-k of one token (moe.zig:435-463) by one warp; lg = the token's logits in
// shared memory, key = E words of shared scratch.  Lane l owns experts l, l+32,
// ...  Keys are the f32 bits of exp(v - max) + 1 (non-negative floats order like
// their bits; 0 = not a candidate: chosen, NaN or beyond E).  Each round takes
// the largest key and, among equal keys, the smallest id — the reference's
// strict-greater scan from e = 0 with bv = -1.  A round without a candidate
// yields id 0, as in the reference.  The loops are kept rolled: this code runs
// once per launch, so its size (fetched cold) matters more than its trip count.
__device__ __noinline__ void route_token(const float* __restrict__ lg, uint32_t* __restrict__ key, int E, int K,
                                         int norm_topk, int has_shared, int T, int t, int lane, DecodeMisc& s,
                                         uint32_t* topk_idx, float* topk_gates, bool write_out) {
    float mx = __int_as_float(0xffc00000);  // NaN: fmaxf ignores it
#pragma unroll 1
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
    mx = warp_max(mx);
    double all = 0.0;
    float ex0 = 0.0f;
    // four experts per lane at a time: their exp chains run side by side
#pragma unroll 1
    for (int e0 = lane; e0 < E; e0 += 128) {
        float ex[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ex[j] = e0 + 32 * j < E ? cz_expf_inline(__fsub_rn(lg[e0 + 32 * j], mx)) : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + 32 * j;
            if (e < E) {
                all += (double)ex[j];
                key[e] = ex[j] > -1.0f ? __float_as_uint(ex[j]) + 1u : 0u;
                if (e == 0) ex0 = ex[j];
            }
        }
    }
    all = warp_sum_d(all);
    const float ex_e0 = __shfl_sync(0xffffffffu, ex0, 0);
    __syncwarp();
    double top = 0.0;
#pragma unroll 1
    for (int z = 0; z < K; ++z) {
        uint32_t lbest = 0u;
        int lid = 0x7fffffff;
#pragma unroll 1
        for (int e0 = lane; e0 < E; e0 += 128) {
            uint32_t kk[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) kk[j] = e0 + 32 * j < E ? key[e0 + 32 * j] : 0u;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (kk[j] > lbest) {
                    lbest = kk[j];
                    lid = e0 + 32 * j;
                }
        }
        const uint32_t kmax = redux_max_u32(lbest);
        int best;
        float bv;
        if (kmax == 0u) {
            best = 0;
            bv = ex_e0;
        } else {
            best = (int)redux_min_u32(lbest == kmax ? (uint32_t)lid : 0xffffffffu);
            bv = __uint_as_float(kmax - 1u);
        }
        __syncwarp();
        if (lane == 0) {
            if (kmax != 0u) key[best] = 0u;
            s.pe[t * K + z] = best;
            s.pg[t * K + z] = bv;  // exp value for now; the gate is formed below
        }
        __syncwarp();
        top = __dadd_rn(top, (double)bv);
    }
    const double den = norm_topk ? top : all;
    if (lane < K) {
        const float g = __double2float_rn(__ddiv_rn((double)s.pg[t * K + lane], den));
        s.pg[t * K + lane] = g;
        if (write_out) {
            if (topk_idx) topk_idx[(size_t)t * K + lane] = (uint32_t)s.pe[t * K + lane];
            if (topk_gates) topk_gates[(size_t)t * K + lane] = g;
        }
    }
    if (lane == 0 && has_shared) {
        s.pe[T * K + t] = E;
        s.pg[T * K + t] = cz_sigmoid(lg[E]);
    }
    __syncwarp();
}

__device__ __forceinline__ int pair_token(int pr, int T, int K) { return pr < T * K ? pr / K : pr - T * K; }

// Bounded wait of all lanes on an mbarrier phase; warp-uniform result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, DecodeMisc& s) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, &s.abort));
}

// Named barriers between the consumer warps and the h warp (288 threads each):
// RED_FULL(b): the consumers' partial gate/up sums of a chunk of parity b are in
// red[b]; RED_FREE(b): the h warp has read them; H_DONE: h, its maxima and
// exponents of every chunk are in shared memory.
constexpr int BAR_RED_FULL = 2, BAR_RED_FREE = 4, BAR_H_DONE = 6;
__device__ __forceinline__ void bar_sync_n(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"((NCW + 1) * 32) : "memory"); }
__device__ __forceinline__ void bar_arrive_n(int id) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "n"((NCW + 1) * 32) : "memory"); }

// One instance per token count: loop trip counts, fragment shapes and slab sizes
// become constants, so each launch runs a short, branch-free path.
template <int TT>
__global__ void __launch_bounds__(NTHREADS, 1) moe_decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-aligned base as an offset into the __shared__ array itself, so every
    // pointer below stays in the shared address space (plain LDS/STS, not
    // generic accesses)
    uint8_t* const sb = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    constexpr int T = TT;
    const int H = p.H, E = p.E, K = p.K;
    const int SI = p.SI, Ir = p.I;
    const int Er = E + (SI ? 1 : 0);
    const int LS = logit_stride(E);
    const bool xbf = p.x_bf16 != 0;
    const Carve cv = carve(T, H, p.x_bf16);
    DecodeMisc& s = *reinterpret_cast<DecodeMisc*>(sb + cv.misc);
    uint8_t* const ring = sb;
    uint8_t* const xterm = sb + cv.xterm;
    float* const red = reinterpret_cast<float*>(sb + cv.red);
    uint8_t* const hterm = sb + cv.hterm;
    uint32_t* const err = p.sync + 1;

    const uint32_t seq = ld_relaxed_gpu(p.sync);
    uint32_t* reg = region(p.sync, seq & 1);
    if (c == 0 && tid < kSyncRegionWords) region(p.sync, (seq & 1) ^ 1)[tid] = 0u;
    if (tid == 0) {
        for (int i = 0; i < cv.ns; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], NCW);
        }
        mbar_init(&s.rbar, 1);
        mbar_init(&s.lbar, 1);
        s.abort = 0;
        fence_mbarrier_init();
    }
    if (tid < MAXT) s.xmax[tid] = 0u;
    for (int i = tid; i < MAXT * 64; i += NTHREADS) (&s.hmax[0][0])[i] = 0.0f;
    __syncthreads();

    // ---------------- phase R: router logits ----------------
    const int row_lo = (int)((long long)c * Er / G), row_hi = (int)((long long)(c + 1) * Er / G);
    const int nrows = row_hi - row_lo;
    const uint32_t xbytes = (uint32_t)T * H * (xbf ? 2u : 4u);
    const uint32_t rbytes = (uint32_t)nrows * H * 4u;
    // ring during phase R: [router rows][tokens][rms weight]
    float* rows = reinterpret_cast<float*>(ring);
    uint8_t* xs = ring + rbytes;
    float* wnorm = reinterpret_cast<float*>(ring + rbytes + xbytes);
    if (tid == 0) {
        const uint32_t wbytes = p.rms_w ? (uint32_t)H * 4u : 0u;
        mbar_arrive_expect_tx(&s.rbar, xbytes + rbytes + wbytes);
        bulk_g2s(xs, p.x, xbytes, &s.rbar);
        if (wbytes) bulk_g2s(wnorm, p.rms_w, wbytes, &s.rbar);
        for (int r = 0; r < nrows; ++r) {
            const int e = row_lo + r;
            bulk_g2s(rows + (size_t)r * H, (e < E) ? p.router + (size_t)e * H : p.sh_gate, (uint32_t)H * 4u, &s.rbar);
        }
    }
    if (!mbar_wait_bounded(&s.rbar, 0, &s.abort) && lane == 0) set_error(err, s, CZ_DERR_FULL_WAIT);
    __syncthreads();

    if (p.rms_w && !s.abort) {
        // stack mode: x = rms(h, w) in place (rmsnorm.zig:32-40): f64 sum of
        // squares, mean rounded to f32, r = 1/sqrt(mean + eps), v*r*w.
        float* xf = reinterpret_cast<float*>(xs);
        for (int t = warp; t < T; t += NWARPS) {
            double ss = 0.0;
            for (int i = lane; i < H; i += 32) {
                const double v = (double)xf[(size_t)t * H + i];
                ss = __fma_rn(v, v, ss);
            }
            ss = warp_sum_d(ss);
            if (lane == 0) {
                const float mean = __double2float_rn(__ddiv_rn(ss, (double)H));
                s.xscale[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));  // r, for now
            }
        }
        __syncthreads();
        for (int k = tid; k < T * H; k += NTHREADS) {
            const int t = k / H, i = k - t * H;
            xf[k] = __fmul_rn(__fmul_rn(xf[k], s.xscale[t]), wnorm[i]);
        }
        __syncthreads();
    }

    auto xval = [&](int k) -> float {
        return xbf ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(xs)[k] << 16)
                   : reinterpret_cast<const float*>(xs)[k];
    };
    if (!s.abort) {
        for (int it = warp; it < nrows * T; it += NWARPS) {
            const int r = it / T, t = it - r * T;
            const float* wr = rows + (size_t)r * H;
            const float v = xbf ? router_dot<true>(wr, xs + (size_t)t * H * 2, H, lane)
                                : router_dot<false>(wr, xs + (size_t)t * H * 4, H, lane);
            if (lane == 0) p.logits[(size_t)t * LS + row_lo + r] = v;
        }
        // max |x_t| for the per-token power-of-two prescale (one atomic per warp)
        for (int t = 0; t < T; ++t) {
            float m = 0.0f;
            for (int i = tid; i < H; i += NTHREADS) {
                const float a = fabsf(xval(t * H + i));
                if (a < 3.0e38f) m = fmaxf(m, a);
            }
            m = warp_max(m);
            if (lane == 0 && m > 0.0f) atomicMax(&s.xmax[t], __float_as_uint(m));
        }
    }
    __syncthreads();
    if (tid < T) {
        const int e = prescale_exp(__uint_as_float(s.xmax[tid]));
        s.xexp[tid] = e;
        s.xscale[tid] = scale2(1.0f, -e);
    }
    __syncthreads();
    // Tokens as MMA columns: x_t * 2^s_t = term 0 + term 1 (+ term 2), E4M3.
    // Column (t, j) holds term j of token t, H bytes at xterm + (t*JX + j)*CS.
    if (!s.abort) {
        for (int t = 0; t < T; ++t) {
            const int sx = s.xexp[t];
            uint8_t* col = xterm + (size_t)(t * cv.JX) * cv.CS;
            for (int i = 2 * tid; i < H; i += 2 * NTHREADS) {
                float a = scale2(xval(t * H + i), sx), b = scale2(xval(t * H + i + 1), sx);
                for (int j = 0; j < cv.JX; ++j) {
                    const uint16_t d = e4m3_term2(a, b);
                    *reinterpret_cast<uint16_t*>(col + (size_t)j * cv.CS + i) = d;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        red_release_add_gpu(&reg[0], 1u);
        if (!wait_geq_bounded(&reg[0], (uint32_t)G, err)) set_error(err, s, CZ_DERR_ROUTER_BARRIER);
        if (!s.abort) {
            // all logits -> shared memory (ring offset 0; the weight stream starts later)
            fence_proxy_async_smem();
            asm volatile("fence.proxy.async.global;" ::: "memory");
            const uint32_t lbytes = (uint32_t)T * LS * 4u;
            mbar_arrive_expect_tx(&s.lbar, lbytes);
            bulk_g2s(ring, p.logits, lbytes, &s.lbar);
        }
    }
    __syncthreads();

    // ---------------- phase K: top-k + grouping (every CTA) ----------------
    if (!s.abort && !mbar_wait_bounded(&s.lbar, 0, &s.abort) && lane == 0) set_error(err, s, CZ_DERR_FULL_WAIT);
    __syncthreads();
    if (!s.abort) {
        for (int t = warp; t < T; t += NWARPS) {
            const float* lg = reinterpret_cast<const float*>(ring) + (size_t)t * LS;
            // keys of token t: shared scratch after the logits (the ring is idle until phase C)
            uint32_t* key = reinterpret_cast<uint32_t*>(ring) + (size_t)MAXT * LS + (size_t)t * LS;
            route_token(lg, key, E, K, p.norm_topk, SI != 0, T, t, lane, s, p.topk_idx, p.topk_gates, c == 0);
        }
    }
    __syncthreads();
    if (!s.abort) {
        const int P = T * K + (SI ? T : 0);
        // sort pairs by (expert, pair) with ranks: P <= 68
        for (int i = tid; i < P; i += NTHREADS) {
            const int e = s.pe[i];
            int r = 0;
            for (int j = 0; j < P; ++j) {
                const int ej = s.pe[j];
                r += (ej < e) || (ej == e && j < i);
            }
            s.order[r] = i;
        }
    }
    __syncthreads();
    if (warp == 0) {
        if (!s.abort) {
            const int P = T * K + (SI ? T : 0);
            // group starts: positions where the expert changes
            int base = 0;
            for (int r0 = 0; r0 < P; r0 += 32) {
                const int r = r0 + lane;
                const bool start = r < P && (r == 0 || s.pe[s.order[r]] != s.pe[s.order[r - 1]]);
                const uint32_t m = __ballot_sync(0xffffffffu, start);
                if (start) {
                    const int u = base + __popc(m & ((1u << lane) - 1u));
                    s.g_expert[u] = s.pe[s.order[r]];
                    s.g_pair0[u] = r;
                }
                base += __popc(m);
            }
            __syncwarp();
            for (int u = lane; u < base; u += 32) {
                const int end = (u + 1 < base) ? s.g_pair0[u + 1] : P;
                s.g_npairs[u] = end - s.g_pair0[u];
            }
            __syncwarp();
            if (lane == 0) {
                int nc = 0;
                for (int u = 0; u < base; ++u) {
                    // groups of experts held elsewhere (expert parallelism) get no chunks
                    const int eu = s.g_expert[u];
                    const bool here = eu == E ? p.shared_here != 0 : (eu >= p.e_lo && eu < p.e_hi);
                    s.g_chunk0[u] = nc;
                    if (here) nc += (eu == E ? SI : Ir) / CR;
                }
                s.g_chunk0[base] = nc;
                s.U = base;
                s.P = P;
                s.NC = nc;
            }
        } else if (lane == 0) {
            s.U = 0;
            s.NC = 0;
        }
    }
    __syncthreads();

    // ---------------- phase C: this CTA's chunks ----------------
    {
        const int NC = s.NC;
        const int NS = cv.ns;
        const int ch_lo = (int)((long long)c * NC / G), ch_hi = (int)((long long)(c + 1) * NC / G);
        const int nks = (H + KS - 1) / KS;     // gate (and up) stages per chunk
        const int nbpH = cz_nbp(H);
        const int nkbH = cz_nblk(H);           // 128-column blocks of H
        // down: tiles per warp (each warp's accumulators live in registers across
        // all chunks) and the output rows of one slab
        // column groups of 8 (token, term) columns, and 16-row tiles per warp (NMD x TPW = 16 accumulators)
        constexpr int NMD = T * JH <= 8 ? 1 : (T * JH <= 16 ? 2 : 4);
        constexpr int TPW = 16 / NMD;
        const int OSr = TPW * 16 * NCW;

        if (warp == PW) {
            // ---------------- producer (one thread) ----------------
            if (lane == 0) {
                fence_proxy_async_smem();  // generic reads of the ring (logits) precede the async writes
                const uint64_t pol = l2_evict_first_policy();
                int si = 0;
                // wait until slot si % NS is free again (bounded); false = stop
                auto acquire_slot = [&](int slot, int round) -> bool {
                    if (round == 0) return true;
                    bool ok = false;
                    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok && !s.abort; ++it) {
                        ok = mbar_try_wait(&s.empty[slot], (round - 1) & 1);
                        if (!ok && it > 64) __nanosleep(64);
                    }
                    if (!ok && !s.abort) set_error(err, s, CZ_DERR_EMPTY_WAIT);
                    return ok;
                };
                // pass 1: gate/up slabs of every chunk
                {
                    int u = 0;
                    for (int ch = ch_lo; ch < ch_hi && !s.abort; ++ch) {
                        while (s.g_chunk0[u + 1] <= ch) ++u;
                        const GroupW gw = group_w(p, s.g_expert[u]);
                        const int r0 = (ch - s.g_chunk0[u]) * CR;
                        const int nbpI = cz_nbp(gw.inter);
                        for (int st = 0; st < 2 * nks && !s.abort; ++st, ++si) {
                            const int slot = si % NS;
                            if (!acquire_slot(slot, si / NS)) break;
                            uint8_t* dst = ring + (size_t)slot * SLOT_BYTES;
                            float* sdst = reinterpret_cast<float*>(dst + GU_BYTES);
                            // slab st/2: gate (st even) or up (st odd) rows [r0, r0+16), column
                            // blocks [kb0, kb0 + nkbs) as [block][row][128 B] (128-byte swizzle)
                            const bool up = st & 1;
                            const int kb0 = (st >> 1) * (KS / 128), nkbs = min(KS / 128, nkbH - kb0);
                            const CUtensorMap* map = up ? gw.umap : gw.gmap;
                            const float* ssrc = (up ? gw.us : gw.gs) + (size_t)(r0 >> 7) * nbpH;
                            // the first up slab also carries the expert's down-scale table
                            const uint32_t dsb = st == 1 ? (uint32_t)(cz_nblk(H) * nbpI * 4) : 0u;
                            const uint32_t wb = (uint32_t)(CR * 128) * (uint32_t)(p.gu3d ? p.gu_kb : nkbs);
                            mbar_arrive_expect_tx(&s.full[slot], wb + (uint32_t)(nbpH * 4) + dsb);
                            if (p.gu3d) {
                                tma_box3_g2s(dst, map, 0, gw.gu_row0 + r0, kb0, &s.full[slot], pol);
                            } else {
                                for (int kb = 0; kb < nkbs; ++kb)
                                    tma_box_g2s(dst + (size_t)kb * CR * 128, map, (kb0 + kb) * 128, gw.gu_row0 + r0,
                                                &s.full[slot], pol);
                            }
                            bulk_g2s(sdst, ssrc, (uint32_t)nbpH * 4u, &s.full[slot]);
                            if (dsb) bulk_g2s(sdst + nbpH, gw.ds, dsb, &s.full[slot]);
                        }
                    }
                }
                // pass 2: for every slab of OSr output rows, the down columns of every chunk
                for (int o0 = 0; o0 < H && !s.abort; o0 += OSr) {
                    const int OSl = min(OSr, H - o0);
                    const int nbox = (OSl + BOX_ROWS - 1) / BOX_ROWS;
                    const int ob0 = o0 >> 7, nob = (OSl + 127) >> 7;
                    int u = 0;
                    for (int ch = ch_lo; ch < ch_hi && !s.abort; ++ch, ++si) {
                        while (s.g_chunk0[u + 1] <= ch) ++u;
                        const GroupW gw = group_w(p, s.g_expert[u]);
                        const int r0 = (ch - s.g_chunk0[u]) * CR;
                        const int nbpI = cz_nbp(gw.inter);
                        const int slot = si % NS;
                        if (!acquire_slot(slot, si / NS)) break;
                        uint8_t* dst = ring + (size_t)slot * SLOT_BYTES;
                        float* sdst = reinterpret_cast<float*>(dst + GU_BYTES);
                        if (gw.dgrp) {
                            // boxes of dgrp x 256 rows (3D map: [group][256 rows][cols])
                            const int rows_b = BOX_ROWS * gw.dgrp, nb3 = (OSl + rows_b - 1) / rows_b;
                            mbar_arrive_expect_tx(&s.full[slot], (uint32_t)(nb3 * rows_b * 16 + nob * nbpI * 4));
                            for (int b = 0; b < nb3; ++b)
                                tma_box3_g2s(dst + (size_t)b * rows_b * 16, gw.dmap, r0, 0,
                                             (gw.down_row0 + o0) / BOX_ROWS + b * gw.dgrp, &s.full[slot], pol);
                        } else {
                            mbar_arrive_expect_tx(&s.full[slot], (uint32_t)(nbox * BOX_ROWS * 16 + nob * nbpI * 4));
                            for (int b = 0; b < nbox; ++b)
                                tma_box_g2s(dst + (size_t)b * BOX_ROWS * 16, gw.dmap, r0,
                                            gw.down_row0 + o0 + b * BOX_ROWS, &s.full[slot], pol);
                        }
                        bulk_g2s(sdst, gw.ds + (size_t)ob0 * nbpI, (uint32_t)(nob * nbpI * 4), &s.full[slot]);
                    }
                }
                // drain: no copy may land after this CTA exits (waiting on a phase
                // that already completed returns at once)
                for (int k = max(0, si - NS); k < si; ++k) {
                    bool ok = false;
                    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok; ++it) {
                        ok = mbar_try_wait(&s.full[k % NS], (k / NS) & 1);
                        if (!ok) __nanosleep(64);
                    }
                    if (!ok) atomicOr(err, CZ_DERR_DRAIN_WAIT);
                }
            }
            __syncwarp();
        } else if (warp == HW) {
            // ---------------- h warp ----------------
            // Per chunk, once the consumers' partial gate/up sums are in red[b]:
            // hw = gate * silu(g) * u per (row r, token tk) (0 for tokens not routed
            // to the chunk's expert) and the running max of |hw * down scale| per
            // (token, 128-row output block).  Runs beside the next chunk's MMAs.
            const int nch = ch_hi - ch_lo;
            int u = 0;
            for (int ch = ch_lo; ch < ch_hi; ++ch) {
                while (s.g_chunk0[u + 1] <= ch) ++u;
                const int ci = ch - ch_lo, b = ci & 1;
                const int np = s.g_npairs[u];
                const int* pairs = s.order + s.g_pair0[u];
                bar_sync_n(BAR_RED_FULL + b);
                const float* rb = red + b * (NCW * 2 * 256);
#pragma unroll 1
                for (int half = 0; half < (T + 1) / 2; ++half) {
                    const int tk = 2 * half + (lane >> 4), r = lane & 15;
                    int q = -1;
                    for (int qq = 0; qq < np; ++qq)
                        if (pair_token(pairs[qq], T, K) == tk) q = qq;
                    float hw = 0.0f;
                    if (q >= 0 && !s.abort) {
                        float gs = 0.0f, us = 0.0f;
                        const float* rg = rb + r * 16 + q * cv.JX;
                        float gv[NCW][3], uv[NCW][3];
#pragma unroll
                        for (int w = 0; w < NCW; ++w)
#pragma unroll
                            for (int j = 0; j < 3; ++j) {
                                gv[w][j] = j < cv.JX ? rg[w * 512 + j] : 0.0f;
                                uv[w][j] = j < cv.JX ? rg[w * 512 + 256 + j] : 0.0f;
                            }
#pragma unroll
                        for (int w = 0; w < NCW; ++w)
#pragma unroll
                            for (int j = 0; j < 3; ++j)
                                if (j < cv.JX) {
                                    gs += gv[w][j];
                                    us += uv[w][j];
                                }
                        const float xsc = s.xscale[tk];
                        hw = s.pg[pairs[q]] * (silu_fast(gs * xsc) * (us * xsc));
                    }
                    reinterpret_cast<float*>(hterm)[(ci * 16 + r) * MAXT + tk] = hw;
                    float mh = fabsf(hw);
                    if (!(mh < 3.0e38f)) mh = 0.0f;
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
                    if (q >= 0)
                        for (int ob = r; ob < cz_nblk(H); ob += 16)
                            s.hmax[tk][ob] = fmaxf(s.hmax[tk][ob], mh * fabsf(s.sdcol[b][ob]));
                }
                __threadfence_block();
                if (ci + 2 < nch) bar_arrive_n(BAR_RED_FREE + b);
            }
            // one power-of-two scale per (token, 128-row output block) for every chunk
            __syncwarp();
            for (int i = lane; i < MAXT * 64; i += 32) (&s.hexp[0][0])[i] = prescale_exp((&s.hmax[0][0])[i]);
            __threadfence_block();
            bar_arrive_n(BAR_H_DONE);
        } else {
            // ---------------- consumers ----------------
            const int g = lane >> 2, t = lane & 3;  // MMA fragment coordinates
            // MMA rows g, g + 8 hold chunk rows rho, rho + 8: the two rows a quarter-warp
            // reads then sit 4 apart in the swizzle pattern, so their chunks use disjoint banks
            const int rho = (g >> 1) + 4 * (g & 1);
            int si = 0;
            int u = 0;
            // ==== pass 1: gate/up of every chunk (h is formed by the h warp) ====
            for (int ch = ch_lo; ch < ch_hi; ++ch) {
                while (s.g_chunk0[u + 1] <= ch) ++u;
                const int ci = ch - ch_lo, b = ci & 1;
                // red[b] and sdcol[b] are reused: the h warp must be done with chunk ci-2
                if (ci >= 2) bar_sync_n(BAR_RED_FREE + b);
                const int np = s.g_npairs[u];
                const int* pairs = s.order + s.g_pair0[u];
                const int ib = ((ch - s.g_chunk0[u]) * CR) >> 7;  // the chunk's 128-column block of down
                const int nbpI = cz_nbp(s.g_expert[u] == E ? SI : Ir);
                // columns of the gate/up MMAs: c = q*JX + j (pair q, term j); lane's column g of MMA m
                const int ncolA = np * cv.JX, nmA = (ncolA + 7) >> 3;
                const uint8_t* xcol[2];
                bool xok[2];
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const int cc = 8 * m + g;
                    xok[m] = cc < ncolA;
                    const int q = xok[m] ? cc / cv.JX : 0, j = cc - q * cv.JX;
                    const int tok = pair_token(pairs[q], T, K);
                    xcol[m] = xterm + (size_t)(tok * cv.JX + (xok[m] ? j : 0)) * cv.CS;
                }
                float accg[2][4], accu[2][4];
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int i = 0; i < 4; ++i) accg[m][i] = accu[m][i] = 0.0f;

                // ---- gate / up: slab k is the stage pair (gate, up); both tiles in one pass ----
                for (int kq = 0; kq < nks; ++kq, si += 2) {
                    const int slg = si % NS, slu = (si + 1) % NS;
                    bool ok = !s.abort && warp_wait(&s.full[slg], (si / NS) & 1, s);
                    ok = ok && warp_wait(&s.full[slu], ((si + 1) / NS) & 1, s);
                    if (!ok) {
                        if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_FULL_WAIT);
                        continue;
                    }
                    const uint8_t* stg = ring + (size_t)slg * SLOT_BYTES;
                    const uint8_t* stu = ring + (size_t)slu * SLOT_BYTES;
                    const float* tg = reinterpret_cast<const float*>(stg + GU_BYTES);
                    const float* tu = reinterpret_cast<const float*>(stu + GU_BYTES);
                    const int k0 = kq * KS, L = min(KS, H - k0);
                    const int nkb = (L + 127) >> 7;
                    const int kb_lo = warp * nkb / NCW, kb_hi = (warp + 1) * nkb / NCW;
                    float ag[2][4] = {}, au[2][4] = {};
#pragma unroll 1
                    for (int kb = kb_lo; kb < kb_hi; ++kb) {
                        float cg[2][4] = {}, cu[2][4] = {};
#pragma unroll
                        for (int sg = 0; sg < 2; ++sg) {
                            const int base = kb * 128 + sg * 64;
                            if (base >= L) break;  // warp-uniform
                            const int kk = base + 16 * t;
                            const bool kin = kk < L;
                            uint4 ga = make_uint4(0, 0, 0, 0), gb = ga, ua = ga, ub = ga, xb0 = ga, xb1 = ga;
                            if (kin) {
                                // rows rho and rho + 8 of block kb; 16-byte chunk (kk/16)%8 is
                                // stored at chunk ((kk/16)%8) ^ (rho%8)
                                const uint32_t wo = (uint32_t)(kb * (CR * 128) + rho * 128) +
                                                    (((uint32_t)(kk >> 4) & 7u) ^ (uint32_t)(rho & 7)) * 16u;
                                ga = *reinterpret_cast<const uint4*>(stg + wo);
                                gb = *reinterpret_cast<const uint4*>(stg + wo + 8 * 128);
                                ua = *reinterpret_cast<const uint4*>(stu + wo);
                                ub = *reinterpret_cast<const uint4*>(stu + wo + 8 * 128);
                                if (xok[0]) xb0 = *reinterpret_cast<const uint4*>(xcol[0] + k0 + kk);
                                if (nmA > 1 && xok[1]) xb1 = *reinterpret_cast<const uint4*>(xcol[1] + k0 + kk);
                            }
                            mma_e4m3(cg[0], ga.x, gb.x, ga.y, gb.y, xb0.x, xb0.y);
                            mma_e4m3(cu[0], ua.x, ub.x, ua.y, ub.y, xb0.x, xb0.y);
                            mma_e4m3(cg[0], ga.z, gb.z, ga.w, gb.w, xb0.z, xb0.w);
                            mma_e4m3(cu[0], ua.z, ub.z, ua.w, ub.w, xb0.z, xb0.w);
                            if (nmA > 1) {  // warp-uniform
                                mma_e4m3(cg[1], ga.x, gb.x, ga.y, gb.y, xb1.x, xb1.y);
                                mma_e4m3(cu[1], ua.x, ub.x, ua.y, ub.y, xb1.x, xb1.y);
                                mma_e4m3(cg[1], ga.z, gb.z, ga.w, gb.w, xb1.z, xb1.w);
                                mma_e4m3(cu[1], ua.z, ub.z, ua.w, ub.w, xb1.z, xb1.w);
                            }
                        }
                        const float scg = tg[(k0 >> 7) + kb], scu = tu[(k0 >> 7) + kb];
#pragma unroll
                        for (int m = 0; m < 2; ++m)
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                ag[m][i] = __fmaf_rn(scg, cg[m][i], ag[m][i]);
                                au[m][i] = __fmaf_rn(scu, cu[m][i], au[m][i]);
                            }
                    }
#pragma unroll
                    for (int m = 0; m < 2; ++m)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            accg[m][i] += ag[m][i];
                            accu[m][i] += au[m][i];
                        }
                    if (kq == 0 && warp == 0) {  // down scales of column block ib, from the up slab
                        const float* dtab = tu + nbpH;
                        for (int ob = lane; ob < cz_nblk(H); ob += 32) s.sdcol[b][ob] = dtab[ob * nbpI + ib];
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&s.empty[slg]);
                        mbar_arrive(&s.empty[slu]);
                    }
                }

                // ---- this warp's partial gate/up sums of the chunk -> red[b] (h warp) ----
                {
                    float* rg = red + (b * NCW * 2 + warp * 2 + 0) * 256;
                    float* ru = rg + 256;
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const int col = 8 * m + 2 * t;
                        rg[rho * 16 + col] = accg[m][0];
                        rg[rho * 16 + col + 1] = accg[m][1];
                        rg[(rho + 8) * 16 + col] = accg[m][2];
                        rg[(rho + 8) * 16 + col + 1] = accg[m][3];
                        ru[rho * 16 + col] = accu[m][0];
                        ru[rho * 16 + col + 1] = accu[m][1];
                        ru[(rho + 8) * 16 + col] = accu[m][2];
                        ru[(rho + 8) * 16 + col + 1] = accu[m][3];
                    }
                }
                __threadfence_block();
                bar_arrive_n(BAR_RED_FULL + b);
            }
            // h, its maxima and the exponents of every chunk are ready
            bar_sync_n(BAR_H_DONE);

            // ==== pass 2: per slab of OSr output rows, down of every chunk ====
            // Warp w owns tiles [w*TPW, (w+1)*TPW) of the slab; its accumulators stay in
            // registers across the chunks (columns = (token, term) for every chunk).  The
            // B operand of a chunk and 128-row block: the E4M3 terms of
            // hw * down scale * 2^s(token, block).
            for (int o0 = 0; o0 < H; o0 += OSr) {
                const int OSl = min(OSr, H - o0);
                const int ntile = OSl >> 4;
                float accd[16][4];
#pragma unroll
                for (int i = 0; i < 16; ++i)
#pragma unroll
                    for (int k = 0; k < 4; ++k) accd[i][k] = 0.0f;
                const int tw0 = warp * TPW;  // first tile of this warp in the slab
                const int obw = (o0 >> 7) + ((tw0 * 16) >> 7);  // first 128-row block of those tiles
                // chunks in pairs: chunk A's 16 columns are the MMA's K values 0-15, chunk
                // B's (the next stage) K values 16-31, so one MMA serves both
                u = 0;
                for (int ch = ch_lo; ch < ch_hi; ch += 2) {
                    const int nh = ch + 1 < ch_hi ? 2 : 1;
                    const uint8_t* stA = nullptr;
                    const uint8_t* stB = nullptr;
                    uint32_t bfA[2][NMD] = {}, bfB[2][NMD] = {};
                    bool ok = !s.abort;
#pragma unroll 1
                    for (int hh = 0; hh < nh && ok; ++hh) {
                        const int chh = ch + hh, sidx = si + hh;
                        while (s.g_chunk0[u + 1] <= chh) ++u;
                        const int ci = chh - ch_lo;
                        const int ib = ((chh - s.g_chunk0[u]) * CR) >> 7;
                        const int nbpI = cz_nbp(s.g_expert[u] == E ? SI : Ir);
                        const int slot = sidx % NS;
                        ok = warp_wait(&s.full[slot], (sidx / NS) & 1, s);
                        if (!ok) break;
                        const uint8_t* stage = ring + (size_t)slot * SLOT_BYTES;
                        const float* stab = reinterpret_cast<const float*>(stage + GU_BYTES);
                        // B fragments: lane column c = 8m + g = (token c/4, term c%4), rows 4t..4t+3
                        uint32_t bw[2][NMD];
#pragma unroll
                        for (int ol = 0; ol < 2; ++ol)
#pragma unroll
                            for (int m = 0; m < NMD; ++m) {
                                const int cc = 8 * m + g, tk = cc >> 2, jt = cc & 3;
                                const int ob = obw + ol;
                                uint32_t word = 0u;
                                if (tk < T && (ob << 7) < o0 + OSl) {
                                    const float f = stab[(ob - (o0 >> 7)) * nbpI + ib];
                                    const float sc = scale2(f, s.hexp[tk][ob]);
                                    const float* hv = reinterpret_cast<const float*>(hterm) + (ci * 16 + 4 * t) * MAXT + tk;
                                    float a0 = hv[0] * sc, b0 = hv[MAXT] * sc, a1 = hv[2 * MAXT] * sc, b1 = hv[3 * MAXT] * sc;
#pragma unroll
                                    for (int j = 0; j < JH; ++j) {
                                        const uint32_t d0 = e4m3_term2(a0, b0), d1 = e4m3_term2(a1, b1);
                                        if (j == jt) word = d0 | (d1 << 16);
                                    }
                                }
                                bw[ol][m] = word;
                            }
                        if (hh == 0) {
                            stA = stage;
#pragma unroll
                            for (int ol = 0; ol < 2; ++ol)
#pragma unroll
                                for (int m = 0; m < NMD; ++m) bfA[ol][m] = bw[ol][m];
                        } else {
                            stB = stage;
#pragma unroll
                            for (int ol = 0; ol < 2; ++ol)
#pragma unroll
                                for (int m = 0; m < NMD; ++m) bfB[ol][m] = bw[ol][m];
                        }
                    }
                    if (ok) {
#pragma unroll
                        for (int it = 0; it < TPW; ++it) {
                            if (tw0 + it < ntile) {
                                const size_t ra = (size_t)((tw0 + it) * 16 + g) * 16 + 4 * t;
                                const uint32_t a0 = *reinterpret_cast<const uint32_t*>(stA + ra);
                                const uint32_t a1 = *reinterpret_cast<const uint32_t*>(stA + ra + 8 * 16);
                                uint32_t a2 = 0u, a3 = 0u;
                                if (nh == 2) {
                                    a2 = *reinterpret_cast<const uint32_t*>(stB + ra);
                                    a3 = *reinterpret_cast<const uint32_t*>(stB + ra + 8 * 16);
                                }
                                const int obl = (it * 16) >> 7;
#pragma unroll
                                for (int m = 0; m < NMD; ++m)
                                    mma_e4m3(accd[it * NMD + m], a0, a1, a2, a3, bfA[obl][m], bfB[obl][m]);
                            }
                        }
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&s.empty[si % NS]);
                            if (nh == 2) mbar_arrive(&s.empty[(si + 1) % NS]);
                        }
                    } else if (lane == 0 && !s.abort) {
                        set_error(err, s, CZ_DERR_FULL_WAIT);
                    }
                    si += nh;
                }
                // slab done: combine the 4 terms of each token, undo the scale, write the
                // CTA's partial rows (every (token, row) of the slab is written, zeros included)
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int tile = i / NMD, m = i % NMD;
                    {
                        float v0 = accd[i][0] + accd[i][1], v1 = accd[i][2] + accd[i][3];
                        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
                        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
                        const int tk = 2 * m + (t >> 1);
                        if (tw0 + tile < ntile && (t & 1) == 0 && tk < T) {
                            const int o = o0 + (tw0 + tile) * 16 + g;
                            const float us = scale2(1.0f, -s.hexp[tk][o >> 7]);
                            float* dst = p.partial + ((size_t)c * T + tk) * H + o;
                            dst[0] = v0 * us;
                            dst[8] = v1 * us;
                        }
                    }
                }
            }
        }
    }

    // ---------------- this CTA's slice of out: the G partial rows in a fixed order ----------------
    // the block barrier orders every thread's partial rows before thread 0's
    // fence and release; the other CTAs acquire them through the counter
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        red_release_add_gpu(&reg[2], 1u);
        if (!wait_geq_bounded(&reg[2], (uint32_t)G, err)) set_error(err, s, CZ_DERR_READY_WAIT);
    }
    __syncthreads();
    if (!s.abort) {
        // CTA c owns output rows [c*RPC, (c+1)*RPC) (RPC a multiple of 4): items
        // (t, 4 rows); thread (item, part) sums partials part, part+NP, ... in
        // order, then the parts are added in order.
        const int RPC = (((H + G - 1) / G) + 3) & ~3;
        const int o_lo = c * RPC, o_hi = min(H, o_lo + RPC);
        const int nq4 = o_hi > o_lo ? (o_hi - o_lo) >> 2 : 0;
        const int nitem = T * nq4;
        float4* part = reinterpret_cast<float4*>(red);  // [item][NPART]
        const int NPART = nitem > 0 ? max(1, min(32, NTHREADS / nitem)) : 1;
        const int it = tid / NPART, pt = tid - it * NPART;
        if (nitem > 0 && it < nitem) {
            const int tk = it / nq4, o = o_lo + 4 * (it - tk * nq4);
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            // batches of up to 8 loads in flight, added in order
            for (int cc0 = pt; cc0 < G; cc0 += 8 * NPART) {
                float4 v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int cc = cc0 + k * NPART;
                    v[k] = cc < G ? __ldcg(reinterpret_cast<const float4*>(p.partial + ((size_t)cc * T + tk) * H + o))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (cc0 + k * NPART < G) {
                        sum.x += v[k].x;
                        sum.y += v[k].y;
                        sum.z += v[k].z;
                        sum.w += v[k].w;
                    }
            }
            part[it * NPART + pt] = sum;
        }
        __syncthreads();
        if (nitem > 0 && tid < nitem) {
            const int tk = tid / nq4, o = o_lo + 4 * (tid - tk * nq4);
            float4 sum = part[tid * NPART];
            for (int k = 1; k < NPART; ++k) {
                const float4 v = part[tid * NPART + k];
                sum.x += v.x;
                sum.y += v.y;
                sum.z += v.z;
                sum.w += v.w;
            }
            if (p.residual) {
                const float4 r = *reinterpret_cast<const float4*>(p.residual + (size_t)tk * H + o);
                sum.x = __fadd_rn(r.x, sum.x);
                sum.y = __fadd_rn(r.y, sum.y);
                sum.z = __fadd_rn(r.z, sum.z);
                sum.w = __fadd_rn(r.w, sum.w);
            }
            *reinterpret_cast<float4*>(p.out + (size_t)tk * H + o) = sum;
        }
    }

    // ---------------- completion: advance the launch sequence ----------------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&reg[1], 1u);
        if (old == (uint32_t)G - 1u) atomicExch(p.sync, seq + 1u);
    }
}

// ---- host side --------------------------------------------------------------

static bool g_attr_set = false;

size_t decode_smem_bytes(int T, int H, int x_bf16) { return carve(T, H, x_bf16).total + 1024; }

int decode_max_tokens(int H, int E, int K, int I, int SI, int x_bf16, int num_sms) {
    if (K < 1 || K > MAXK || E < K || E > MAXE || H % 16 || I % 16 || SI % 16 || H < 16 || I < 16) return 0;
    if (num_sms > kMaxGrid) return 0;
    const int IM = I > SI ? I : SI;
    if (cz_nblk(H) > 64) return 0;  // per-(token, 128-row block) scale tables
    // scales carried with a stage: gate/up row block + (first up slab) the expert's down table;
    // a down stage: its 128-row blocks of the down table
    if ((size_t)(cz_nbp(H) + cz_nblk(H) * cz_nbp(IM)) * 4 > (size_t)SC_BYTES) return 0;
    if ((size_t)(OS / 128) * cz_nbp(IM) * 4 > (size_t)SC_BYTES) return 0;
    const int max_rows = (E + (SI ? 1 : 0) + num_sms - 1) / num_sms;  // router rows staged per CTA
    const int IM16 = (I > SI ? I : SI) / CR;  // chunks of the largest group
    int t = MAXT;
    while (t > 0) {
        // gate/up MMA columns: a group holds at most t pairs, each as JX E4M3 term columns (<= 16)
        if (t * (x_bf16 ? 2 : 3) > 16) {
            --t;
            continue;
        }
        const int worst_chunks = (t * K + (SI ? t : 0)) * IM16;  // every pair its own group
        if ((worst_chunks + num_sms - 1) / num_sms > MAXCH) {
            --t;
            continue;
        }
        const size_t stage_r = (size_t)max_rows * H * 4 + (size_t)t * H * (x_bf16 ? 2 : 4) + (size_t)H * 4;
        const size_t lg = (size_t)t * logit_stride(E) * 4;
        if (stage_r <= (size_t)RING_BYTES && lg <= (size_t)RING_BYTES && decode_smem_bytes(t, H, x_bf16) <= SMEM_LIMIT)
            break;
        --t;
    }
    return t;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f)
            return nullptr;
        fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

bool make_down_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t cols, int H, int* grp) {
    const EncodeTiledFn fn = encode_fn();
    if (!fn || cols % 16 || rows == 0 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint32_t estr[3] = {1, 1, 1};
    if (H % BOX_ROWS == 0 && rows % BOX_ROWS == 0) {
        // [rows / 256][256][cols]: one box = 16 columns of up to 4 groups of 256 rows
        const uint64_t ng = rows / BOX_ROWS;
        const int g = (int)(ng < 4 ? ng : 4);
        const cuuint64_t dims[3] = {cols, (cuuint64_t)BOX_ROWS, ng};
        const cuuint64_t strides[2] = {cols, cols * BOX_ROWS};
        const cuuint32_t box[3] = {16, (cuuint32_t)BOX_ROWS, (cuuint32_t)g};
        if (fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            *grp = g;
            return true;
        }
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols};
    const cuuint32_t box[2] = {16, (cuuint32_t)BOX_ROWS};
    *grp = 0;
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_gu_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t H, int* kb) {
    const EncodeTiledFn fn = encode_fn();
    if (!fn || H % 16 || rows == 0 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint32_t estr[3] = {1, 1, 1};
    if (H % 128 == 0) {
        // [H / 128 blocks][rows][128 bytes]: one box = 16 rows x up to 16 column blocks,
        // laid out [block][row][128 B] in shared memory
        const uint64_t nkb = H / 128;
        const int d = (int)(nkb < (uint64_t)(KS / 128) ? nkb : (uint64_t)(KS / 128));
        const cuuint64_t dims[3] = {128, rows, nkb};
        const cuuint64_t strides[2] = {H, 128};
        const cuuint32_t box[3] = {128, (cuuint32_t)CR, (cuuint32_t)d};
        if (fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            *kb = d;
            return true;
        }
    }
    const cuuint64_t dims[2] = {H, rows};
    const cuuint64_t strides[1] = {H};
    const cuuint32_t box[2] = {128, (cuuint32_t)CR};
    *kb = 0;
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int decode_launch(const DecodeParams& prm, int num_sms, cudaStream_t stream) {
    const int tmax = decode_max_tokens(prm.H, prm.E, prm.K, prm.I, prm.SI, prm.x_bf16, num_sms);
    if (prm.T < 1 || prm.T > tmax) return CZ_ESHAPE;
    if (prm.rms_w && prm.x_bf16) return CZ_EARGS;
    static_assert(MAXT == 4, "one kernel instance per token count");
    static void (*const kern[MAXT])(DecodeParams) = {moe_decode_kernel<1>, moe_decode_kernel<2>, moe_decode_kernel<3>,
                                                      moe_decode_kernel<4>};
    if (!g_attr_set) {
        for (int i = 0; i < MAXT; ++i)
            if (cudaFuncSetAttribute(kern[i], cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT) != cudaSuccess)
                return CZ_ELAUNCH;
        g_attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = decode_smem_bytes(prm.T, prm.H, prm.x_bf16);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern[prm.T - 1], prm) != cudaSuccess) return CZ_ELAUNCH;
    return CZ_OK;
}

}  // namespace cz
