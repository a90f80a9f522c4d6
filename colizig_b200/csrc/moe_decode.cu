// Decode-regime MoE layer (up to 4 tokens per launch) as ONE persistent
// cooperative kernel.
//
// Reference path (src/qwen38/moe.zig): route (435-463) -> per expert gate/up
// (fp8.zig:165-257) -> silu(g)*u (activation.zig:8-20) -> down -> out += gate*eo,
// plus the always-on shared expert (467-479).
//
// Grid = one CTA per SM: 5 consumer warps + 1 producer warp.  The weight stream
// goes HBM -> shared memory through a ring of bulk-copy (TMA) stages, one slot
// per consumer warp and one bulk copy per weight row into a padded row stride
// (no bank conflicts when the rows of an MMA fragment are read together).  A
// warp owns every stage it computes: no barrier or cross-warp reduction per
// stage.  No global memory is read inside a compute loop: while HBM is
// saturated by the weight stream, any other load would wait behind it.
//
//   R  router logits.  CTA c owns router rows [c*E'/G, (c+1)*E'/G) (E' = E, +1
//      for the shared expert's gate vector).  Rows and tokens are bulk-copied
//      into shared memory; every logit is formed in the reference's exact f32
//      order (dotF32, matmul.zig:60-82: 32 FMA chains = one per lane, then the
//      lane-ordered combine), so the top-k below is bit-identical to it.  In
//      stack mode the tokens are rms-normalised in place first.  The tokens are
//      then re-encoded for the MMA (below).  A grid-wide arrive counter closes
//      the phase.
//   K  top-k.  Every CTA bulk-copies the logits, computes softmax/top-k for all
//      tokens (identically) and groups the (token, slot) pairs by expert
//      (ascending id, shared expert last).  The producer then bulk-copies the
//      block scales this CTA needs.
//   A  gate/up.  The flattened (group, row) list is split evenly over CTAs.  A
//      stage holds up to 8 gate rows (MMA tile rows 0-7) and the same up rows
//      (tile rows 8-15) of mma.sync m16n8k16 (f16 x f16 -> f32): E4M3 bytes
//      become f16 exactly in registers (cvt.rn.f16x2.e4m3x2) and feed the A
//      fragments directly.  The tokens are the B columns: each token, scaled by
//      a power of two, is split into f16 hi + lo parts (columns t and t+4), so
//      products keep ~22 bits.  Each 128-column block's partial is multiplied by
//      its 128x128 scale.  h = silu(g)*u (f32) goes to HBM with the per-pair
//      max |h|.
//   B  down + combine.  CTA c owns output rows [c*H/G, (c+1)*H/G) of every
//      group, as 16-row tiles; a down stage is one tile and up to 4 of the
//      group's pairs.  The producer streams the down-weight rows as slots free
//      up (they do not depend on h); once every CTA has finished phase A it adds
//      the stage's h rows (one bulk copy per pair) on a second barrier of the
//      slot.  The consumer splits them into per-pair 2^s-scaled f16 hi/lo in
//      place and runs the tile with the pairs as columns; each warp adds
//      gate * dot(h, w) into per-(row, token) registers, and the warps' sums are
//      combined in a fixed order at the end (deterministic, no atomics).
//
// Every wait is bounded; a CTA that gives up sets a bit in the device error
// word, stops early (draining its in-flight copies) and the host returns -7.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {

constexpr int NCW = 5;                    // consumer warps (one ring slot each)
constexpr int NTHREADS = (NCW + 1) * 32;  // + 1 producer warp
constexpr int STAGE_BYTES = 33 * 1024;    // 8 gate + 8 up rows of 2048 (+16 pad); 16 down rows + their h
constexpr int NSTAGES = NCW;
constexpr int RING_BYTES = STAGE_BYTES * NSTAGES;
constexpr int XH_BYTES = 33 * 1024;       // tokens as f16 hi/lo columns (phase A)
constexpr int MAXT = kDecodeMaxTokens;    // 4
constexpr int MAXK = kMaxTopk;            // 16
constexpr int MAXE = kMaxExperts;         // 512
constexpr int MAXP = MAXT * (MAXK + 1);   // (token, slot) pairs incl. shared-expert pairs: 68
constexpr int MAXG = MAXP;                // groups <= pairs
constexpr int MAXM = MAXE / 32;           // router values per lane
constexpr int SA_FLOATS = 1024;           // cached gate/up scale tables (phase A)
constexpr int SB_FLOATS = 512;            // cached down scale rows (phase B)
constexpr int MAXAG = 8;                  // groups cached for phase A
constexpr int MAXBT = 4;                  // 16-row output tiles per CTA in phase B (rows per CTA <= 64)
constexpr int RED_FLOATS = NCW * MAXBT * 16 * 4 * 2;
constexpr int WPAD = 16;                  // bytes of padding after every staged weight row
constexpr int HPAD = 32;                  // bytes of padding after every staged h row (down stages)

struct __align__(128) DecodeSmem {
    uint8_t ring[RING_BYTES];
    uint8_t xh[XH_BYTES];
    float sA[SA_FLOATS];
    float sB[SB_FLOATS];
    float red[RED_FLOATS];
    uint64_t full[NSTAGES];   // a stage's weight rows landed
    uint64_t hfull[NSTAGES];  // a down stage's h rows landed
    uint64_t empty[NSTAGES];
    uint64_t rbar;
    uint64_t lbar;
    uint64_t sbar;
    int abort;
    int U, P;
    int sA_ok, sB_ok, a_u0, a_u1;
    int sA_off[MAXAG + 1];
    uint32_t xmax[MAXT];  // max |x_t| (f32 bits)
    int xexp[MAXT];       // s per token (tokens are stored * 2^s)
    float xscale[MAXT];   // 2^-s per token
    int pe[MAXP];         // expert of pair p = t*K + z (shared: p = T*K + t -> E)
    float pg[MAXP];       // gate of pair p
    int order[MAXP];      // pairs sorted by (expert, pair)
    int g_expert[MAXG];
    int g_pair0[MAXG];
    int g_npairs[MAXG];
    int g_rowA[MAXG + 1];
};

static_assert(sizeof(DecodeSmem) + 1024 <= 227 * 1024, "decode smem too large");

// ---- sync words ------------------------------------------------------------
// sync[0] = launch sequence number, sync[1] = error word, then two regions of
// kSyncRegionWords: [0] router arrivals, [1] CTAs done, [2] CTAs done with
// phase A, [8 + p] max |h| of pair p (f32 bits).  A launch uses region seq&1 and
// zeroes the other one, so a launch that stopped early leaves nothing behind.
__device__ __forceinline__ uint32_t* region(uint32_t* sync, int par) { return sync + 2 + par * kSyncRegionWords; }

struct Stage {
    int phase;  // 0 = A (gate/up), 1 = B (down)
    int u;      // group
    int r0;     // A: first row within the group; B: first absolute output row (a 16-row tile)
    int n;      // rows
    int q0, nq; // B: the group's pairs q0 .. q0+nq-1 (at most 4: their h rides in the stage)
};

// Deterministic stage schedule shared by the producer and the consumers:
// gate/up stages of this CTA's row range, then for every group (ascending),
// every 16-row tile of this CTA's output rows, every batch of 4 pairs.
struct StageIter {
    int phase, u, a, a_hi, b_lo, b_hi, brow, bq, U, RA;
    const int* rowA;
    const int* npairs;

    __device__ void init(const DecodeSmem& s, int a_lo, int a_hi_, int b_lo_, int b_hi_, int ra) {
        phase = 0;
        U = s.U;
        rowA = s.g_rowA;
        npairs = s.g_npairs;
        a = a_lo;
        a_hi = a_hi_;
        b_lo = b_lo_;
        b_hi = b_hi_;
        brow = b_lo_;
        bq = 0;
        RA = ra;
        u = 0;
        while (u < U && rowA[u + 1] <= a) ++u;
    }
    __device__ bool next(Stage& st) {
        if (phase == 0) {
            if (a < a_hi) {
                while (rowA[u + 1] <= a) ++u;
                const int n = min(RA, min(rowA[u + 1] - a, a_hi - a));
                st.phase = 0;
                st.u = u;
                st.r0 = a - rowA[u];
                st.n = n;
                st.q0 = 0;
                st.nq = 0;
                a += n;
                return true;
            }
            phase = 1;
            u = 0;
            brow = b_lo;
            bq = 0;
        }
        if (b_lo >= b_hi || u >= U) return false;
        st.phase = 1;
        st.u = u;
        st.r0 = brow;
        st.n = min(16, b_hi - brow);
        st.q0 = bq;
        st.nq = min(4, npairs[u] - bq);
        bq += 4;
        if (bq >= npairs[u]) {
            bq = 0;
            brow += st.n;
            if (brow >= b_hi) {
                brow = b_lo;
                ++u;
            }
        }
        return true;
    }
};

struct GroupW {
    const uint8_t *gw, *uw, *dw;
    const float *gs, *us, *ds;
    int inter;
};

__device__ __forceinline__ GroupW group_w(const DecodeParams& p, int e) {
    GroupW g;
    if (e == p.E) {
        g.inter = p.SI;
        g.gw = p.sh_gate_w;
        g.uw = p.sh_up_w;
        g.dw = p.sh_down_w;
        g.gs = p.sh_gate_s;
        g.us = p.sh_up_s;
        g.ds = p.sh_down_s;
    } else {
        g.inter = p.I;
        const size_t wsz = (size_t)p.I * p.H;
        g.gw = p.gate_w + (size_t)e * wsz;
        g.uw = p.up_w + (size_t)e * wsz;
        g.dw = p.down_w + (size_t)e * wsz;
        const size_t ssz = (size_t)cz_nblk(p.I) * cz_nbp(p.H);
        g.gs = p.gate_s + (size_t)e * ssz;
        g.us = p.up_s + (size_t)e * ssz;
        g.ds = p.down_s + (size_t)e * cz_nblk(p.H) * cz_nbp(p.I);
    }
    return g;
}

__device__ void set_error(uint32_t* err, DecodeSmem& s, uint32_t bit) {
    atomicOr(err, bit);
    s.abort = 1;
}

// 4 E4M3 bytes -> two f16x2 (bytes 0,1 and bytes 2,3), exact.
__device__ __forceinline__ void cvt4(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Power-of-two exponent s with max * 2^s in [2^13, 2^14) (0 for max == 0 or
// non-finite): keeps the f16 hi/lo parts of every value inside f16's range.
__device__ __forceinline__ int prescale_exp(float mx) {
    if (!(mx > 0.0f) || !(mx < 3.0e38f)) return 0;
    int e;
    frexpf(mx, &e);
    return max(-100, min(14 - e, 100));
}

// 2^e as a float, e in [-126, 127] (exact).
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// v * 2^e split into f16 hi + lo (the multiply by a power of two is exact
// unless it leaves the f32 range; e is chosen so that it does not).
__device__ __forceinline__ void split_f16(float v, int e, __half& hi, __half& lo) {
    const float sv = e >= -126 && e <= 127 ? v * pow2f(e) : ldexpf(v, e);
    hi = __float2half_rn(sv);
    lo = __float2half_rn(sv - __half2float(hi));
}

// One 16-row x 8-column MMA tile over K (full K, one warp).  Lane (g, tq):
// A rows g (top) and g+8 (bottom) start at `top` / `bot` in shared memory;
// its B column starts at `bcol` (16-element chunks of 64 bytes: 16 hi halves
// then 16 lo halves; `bcol` already points at the hi or lo half).  Each
// 128-column block's partial is multiplied by stab[kb] / sbot[kb].
// acc: C[g][2tq], C[g][2tq+1], C[g+8][2tq], C[g+8][2tq+1].
__device__ __forceinline__ void tile_mma(const uint8_t* top, const uint8_t* bot, bool oktop, bool okbot,
                                         const uint8_t* bcol, bool bok, int K, int tq, const float* stop,
                                         const float* sbot, float* acc) {
    const int nb = cz_nblk(K);
    for (int kb = 0; kb < nb; ++kb) {
        float cb[2][4] = {};
#pragma unroll
        for (int sb = 0; sb < 2; ++sb) {
            const int kbase = kb * 128 + sb * 64;
            if (kbase >= K) break;  // warp-uniform
            const int k0 = kbase + 16 * tq;
            const bool kin = k0 < K;  // lanes past the end feed zeros to the MMA
            uint4 wa = make_uint4(0, 0, 0, 0), wb = wa, x0 = wa, x1 = wa;
            if (oktop && kin) wa = *reinterpret_cast<const uint4*>(top + k0);
            if (okbot && kin) wb = *reinterpret_cast<const uint4*>(bot + k0);
            if (bok && kin) {
                const uint4* xp = reinterpret_cast<const uint4*>(bcol + (size_t)(k0 >> 4) * 64);
                x0 = xp[0];
                x1 = xp[1];
            }
            const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w}, B[4] = {wb.x, wb.y, wb.z, wb.w};
            const uint32_t X[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t a0, a2, a1, a3;
                cvt4(A[j], a0, a2);
                cvt4(B[j], a1, a3);
                mma16816(cb[j & 1], a0, a1, a2, a3, X[2 * j], X[2 * j + 1]);
            }
        }
        const float st = oktop ? stop[kb] : 0.f, sbt = okbot ? sbot[kb] : 0.f;
        acc[0] = __fmaf_rn(st, cb[0][0] + cb[1][0], acc[0]);
        acc[1] = __fmaf_rn(st, cb[0][1] + cb[1][1], acc[1]);
        acc[2] = __fmaf_rn(sbt, cb[0][2] + cb[1][2], acc[2]);
        acc[3] = __fmaf_rn(sbt, cb[0][3] + cb[1][3], acc[3]);
    }
}

// Router dot of one row with up to 4 tokens, in dotF32's exact order.
// wrow / xs are shared memory.  Writes logits (lane 0).
template <bool BF16>
__device__ __forceinline__ void router_item(const float* __restrict__ wrow, const uint8_t* __restrict__ xs, int H,
                                            int t0, int nt, int lane, float* __restrict__ logits, int lstride,
                                            int col) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t* xb = reinterpret_cast<const uint16_t*>(xs);
    const float* xf = reinterpret_cast<const float*>(xs);
    auto xv = [&](int t, int i) -> float {
        if (BF16) return __uint_as_float((uint32_t)xb[(size_t)t * H + i] << 16);
        return xf[(size_t)t * H + i];
    };
    int i = 0;
    for (; i + 32 <= H; i += 32) {
        const float w = wrow[i + lane];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (q < nt) acc[q] = __fmaf_rn(xv(t0 + q, i + lane), w, acc[q]);
    }
    for (; i + 8 <= H; i += 8) {
        if (lane < 8) {
            const float w = wrow[i + lane];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (q < nt) acc[q] = __fmaf_rn(xv(t0 + q, i + lane), w, acc[q]);
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        // total[l] = (((0 + acc0[l]) + acc1[l]) + acc2[l]) + acc3[l]; chain k = lanes 8k..8k+7
        const float a = acc[q];
        const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
        const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
        const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
        const float tl = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a), a8), a16), a24);
        float sum = __shfl_sync(0xffffffffu, tl, 0);
#pragma unroll
        for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, tl, l));
        if (q < nt) {
            for (int ii = i; ii < H; ++ii) sum = __fmaf_rn(xv(t0 + q, ii), wrow[ii], sum);
            if (lane == 0) logits[(size_t)(t0 + q) * lstride + col] = sum;
        }
    }
}

// Top-k of one token (moe.zig:435-463) by one warp; lg = the token's logits in
// shared memory.  Lane l holds experts l, l+32, ...  Keys are the f32 bits of
// exp(v - max) + 1 (non-negative floats order like their bits; 0 = not a
// candidate: chosen, NaN or beyond E).  Each round takes the largest key and,
// among equal keys, the smallest id — the reference's strict-greater scan from
// e = 0 with bv = -1.  A round without a candidate yields id 0, as in the
// reference.
__device__ void route_token(const float* __restrict__ lg, int E, int K, int norm_topk, int has_shared, int T, int t,
                            int lane, DecodeSmem& s, uint32_t* topk_idx, float* topk_gates, bool write_out) {
    float v[MAXM];
    float mx = __int_as_float(0xffc00000);  // NaN: fmaxf ignores it
    const int nm = (E + 31) >> 5;
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        const int e = lane + 32 * m;
        v[m] = (m < nm && e < E) ? lg[e] : __int_as_float(0xffc00000);
        mx = fmaxf(mx, v[m]);
    }
    mx = warp_max(mx);
    uint32_t key[MAXM];
    double all = 0.0;
    float ex0 = 0.0f;
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        const int e = lane + 32 * m;
        key[m] = 0u;
        if (m < nm && e < E) {
            const float ex = cz_expf(__fsub_rn(v[m], mx));
            all += (double)ex;
            if (ex > -1.0f) key[m] = __float_as_uint(ex) + 1u;
            if (m == 0) ex0 = ex;
        }
    }
    all = warp_sum_d(all);
    const float ex_e0 = __shfl_sync(0xffffffffu, ex0, 0);
    double top = 0.0;
    for (int z = 0; z < K; ++z) {
        uint32_t lbest = 0u;
        int lid = 0x7fffffff;
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            if (key[m] > lbest) {
                lbest = key[m];
                lid = lane + 32 * m;
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
#pragma unroll
            for (int m = 0; m < MAXM; ++m)
                if (lane + 32 * m == best) key[m] = 0u;
        }
        top = __dadd_rn(top, (double)bv);
        if (lane == 0) {
            s.pe[t * K + z] = best;
            s.pg[t * K + z] = bv;  // exp value for now; the gate is formed below
        }
    }
    __syncwarp();
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
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, DecodeSmem& s) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, &s.abort));
}

__global__ void __launch_bounds__(NTHREADS, 1) moe_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    DecodeSmem& s = *reinterpret_cast<DecodeSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int T = p.T, H = p.H, E = p.E, K = p.K;
    const int SI = p.SI, Ir = p.I;
    const int Er = E + (SI ? 1 : 0);
    const int LS = logit_stride(E);
    const bool xbf = p.x_bf16 != 0;
    uint32_t* const err = p.sync + 1;

    const uint32_t seq = ld_relaxed_gpu(p.sync);
    uint32_t* reg = region(p.sync, seq & 1);
    if (c == 0 && tid < kSyncRegionWords) region(p.sync, (seq & 1) ^ 1)[tid] = 0u;
    if (tid == 0) {
        for (int i = 0; i < NSTAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.hfull[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.rbar, 1);
        mbar_init(&s.lbar, 1);
        mbar_init(&s.sbar, 1);
        s.abort = 0;
        fence_mbarrier_init();
    }
    if (tid < MAXT) s.xmax[tid] = 0u;
    __syncthreads();

    // ---------------- phase R: router logits ----------------
    const int row_lo = (int)((long long)c * Er / G), row_hi = (int)((long long)(c + 1) * Er / G);
    const int nrows = row_hi - row_lo;
    const uint32_t xbytes = (uint32_t)T * H * (xbf ? 2u : 4u);
    const uint32_t rbytes = (uint32_t)nrows * H * 4u;
    // ring during phase R: [router rows][tokens][rms weight]
    float* rows = reinterpret_cast<float*>(s.ring);
    uint8_t* xs = s.ring + rbytes;
    float* wnorm = reinterpret_cast<float*>(s.ring + rbytes + xbytes);
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
        for (int t = warp; t < T; t += NCW + 1) {
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
        const int ntg = (T + 3) / 4;
        for (int it = warp; it < nrows * ntg; it += NCW + 1) {
            const int r = it / ntg, t0 = (it % ntg) * 4;
            if (xbf)
                router_item<true>(rows + (size_t)r * H, xs, H, t0, min(4, T - t0), lane, p.logits, LS, row_lo + r);
            else
                router_item<false>(rows + (size_t)r * H, xs, H, t0, min(4, T - t0), lane, p.logits, LS, row_lo + r);
        }
        // max |x_t| for the per-token power-of-two prescale (register max, one atomic per warp)
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
        s.xscale[tid] = ldexpf(1.0f, -e);
    }
    __syncthreads();
    // Tokens as MMA B columns: x_t * 2^s_t split into f16 hi/lo.  xh holds token
    // rows of stride XQS bytes; 16-element chunk c of a row is 16 hi halves then
    // 16 lo halves (64 bytes).  One thread per 2 elements (an f16x2 of each part).
    const int XQS = H * 4 + 32;
    if (!s.abort) {
        for (int k = tid; k < (T * H) >> 1; k += NTHREADS) {
            const int e2 = 2 * k, t = e2 / H, i = e2 - t * H;
            __half h0, l0, h1, l1;
            split_f16(xval(e2), s.xexp[t], h0, l0);
            split_f16(xval(e2 + 1), s.xexp[t], h1, l1);
            uint8_t* row = s.xh + (size_t)t * XQS + (size_t)(i >> 4) * 64 + (i & 15) * 2;
            *reinterpret_cast<__half2*>(row) = __halves2half2(h0, h1);
            *reinterpret_cast<__half2*>(row + 32) = __halves2half2(l0, l1);
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
            bulk_g2s(s.ring, p.logits, lbytes, &s.lbar);
        }
    }
    __syncthreads();

    // ---------------- phase K: top-k + grouping (every CTA) ----------------
    if (s.abort) goto finish;  // uniform: settled before the barrier above
    if (!mbar_wait_bounded(&s.lbar, 0, &s.abort) && lane == 0) set_error(err, s, CZ_DERR_FULL_WAIT);
    __syncthreads();
    if (s.abort) goto finish;
    for (int t = warp; t < T; t += NCW + 1)
        route_token(reinterpret_cast<const float*>(s.ring) + (size_t)t * LS, E, K, p.norm_topk, SI != 0, T, t, lane,
                    s, p.topk_idx, p.topk_gates, c == 0);
    __syncthreads();
    {
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
        __syncthreads();
        if (warp == 0) {
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
            for (int u = lane; u <= base; u += 32) s.g_rowA[u] = u * Ir;  // routed groups: I rows each
            __syncwarp();
            if (lane == 0) {
                if (base > 0 && s.g_expert[base - 1] == E) s.g_rowA[base] = (base - 1) * Ir + SI;  // shared: last
                s.U = base;
                s.P = P;
            }
        }
        __syncthreads();
    }

    // ---------------- phases A and B ----------------
    {
        const int U = s.U;
        const int NA = s.g_rowA[U];
        const int a_lo = (int)((long long)c * NA / G), a_hi = (int)((long long)(c + 1) * NA / G);
        const int b_lo = (int)((long long)c * H / G), b_hi = (int)((long long)(c + 1) * H / G);
        const int WS = H + WPAD;
        const int RA = min(8, STAGE_BYTES / (2 * WS));
        const int HS = max(Ir, SI);
        const int nbHp = cz_nbp(H), nbIrp = cz_nbp(Ir);
        uint32_t* const adone = reg + 2;
        uint32_t* const hmax = reg + 8;
        const bool has_b = (b_lo < b_hi) && U > 0;
        const int bb0 = b_lo >> 7, nbb = has_b ? ((b_hi - 1) >> 7) - bb0 + 1 : 0;

        // block-scale tables this CTA needs (bulk-copied by the producer)
        if (tid == 0) {
            int u0 = 0;
            while (u0 < U && s.g_rowA[u0 + 1] <= a_lo) ++u0;
            int u1 = u0, need = 0;
            s.sA_off[0] = 0;
            while (u1 < U && s.g_rowA[u1] < a_hi && u1 - u0 < MAXAG) {
                const int inter = s.g_expert[u1] == E ? SI : Ir;
                need += 2 * cz_nblk(inter) * nbHp;
                ++u1;
                s.sA_off[u1 - u0] = need;
            }
            s.a_u0 = u0;
            s.a_u1 = u1;
            s.sA_ok = (need <= SA_FLOATS) && (u1 >= U || s.g_rowA[u1] >= a_hi);
            const int nbSp = cz_nbp(SI ? SI : Ir);
            const int needB = U > 0 ? (U - 1) * nbb * nbIrp + nbb * (s.g_expert[U - 1] == E ? nbSp : nbIrp) : 0;
            s.sB_ok = needB <= SB_FLOATS;
        }
        __syncthreads();

        if (warp == NCW) {
            // ---------------- producer (one thread) ----------------
            if (lane == 0) {
                fence_proxy_async_smem();  // generic reads of the ring (logits) precede the async writes
                uint32_t sbytes = 0;
                if (s.sA_ok)
                    for (int u = s.a_u0; u < s.a_u1; ++u)
                        sbytes += 2u * (uint32_t)cz_nblk(s.g_expert[u] == E ? SI : Ir) * nbHp * 4u;
                if (s.sB_ok && has_b)
                    for (int u = 0; u < U; ++u) sbytes += (uint32_t)nbb * cz_nbp(s.g_expert[u] == E ? SI : Ir) * 4u;
                mbar_arrive_expect_tx(&s.sbar, sbytes);
                if (s.sA_ok) {
                    for (int u = s.a_u0; u < s.a_u1; ++u) {
                        const GroupW gwt = group_w(p, s.g_expert[u]);
                        const uint32_t tb = (uint32_t)cz_nblk(gwt.inter) * nbHp * 4u;
                        float* dst = s.sA + s.sA_off[u - s.a_u0];
                        bulk_g2s(dst, gwt.gs, tb, &s.sbar);
                        bulk_g2s(reinterpret_cast<uint8_t*>(dst) + tb, gwt.us, tb, &s.sbar);
                    }
                }
                if (s.sB_ok && has_b) {
                    for (int u = 0; u < U; ++u) {
                        const GroupW gwt = group_w(p, s.g_expert[u]);
                        const int nbIp = cz_nbp(gwt.inter);
                        bulk_g2s(s.sB + u * nbb * nbIrp, gwt.ds + (size_t)bb0 * nbIp, (uint32_t)nbb * nbIp * 4u,
                                 &s.sbar);
                    }
                }
                StageIter itr;
                itr.init(s, a_lo, a_hi, b_lo, b_hi, RA);
                Stage st;
                int si = 0;
                bool adone_seen = false;
                // down stages whose h rows wait for every CTA to finish phase A
                int pend_u[NSTAGES], pend_q0[NSTAGES], pend_nq[NSTAGES];
#pragma unroll
                for (int i = 0; i < NSTAGES; ++i) pend_nq[i] = 0;
                auto issue_h = [&](int slot, int u, int q0, int nq) {
                    const GroupW gwt = group_w(p, s.g_expert[u]);
                    const int* pairs = s.order + s.g_pair0[u];
                    uint8_t* hdst = s.ring + (size_t)slot * STAGE_BYTES + 16 * (gwt.inter + WPAD);
                    mbar_arrive_expect_tx(&s.hfull[slot], (uint32_t)nq * gwt.inter * 4u);
                    for (int q = 0; q < nq; ++q)
                        bulk_g2s(hdst + (size_t)q * (gwt.inter * 4 + HPAD), p.hbuf + (size_t)pairs[q0 + q] * HS,
                                 (uint32_t)gwt.inter * 4u, &s.hfull[slot]);
                };
                auto poll_adone = [&]() {
                    if (adone_seen || !has_b || ld_acquire_gpu(adone) < (uint32_t)G) return;
                    adone_seen = true;
                    asm volatile("fence.proxy.async.global;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < NSTAGES; ++i)
                        if (pend_nq[i]) {
                            issue_h(i, pend_u[i], pend_q0[i], pend_nq[i]);
                            pend_nq[i] = 0;
                        }
                };
                while (!s.abort && itr.next(st)) {
                    const int slot = si % NSTAGES, round = si / NSTAGES;
                    if (round > 0) {
                        bool ok = false;
                        for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok && !s.abort; ++it) {
                            ok = mbar_try_wait(&s.empty[slot], (round - 1) & 1);
                            if (!ok) {
                                poll_adone();
                                if (it > 64) __nanosleep(64);
                            }
                        }
                        if (!ok) {
                            if (!s.abort) set_error(err, s, CZ_DERR_EMPTY_WAIT);
                            break;
                        }
                    }
                    const GroupW gwt = group_w(p, s.g_expert[st.u]);
                    uint8_t* dst = s.ring + (size_t)slot * STAGE_BYTES;
                    if (st.phase == 0) {
                        // gate rows -> dst rows 0..n-1, up rows -> dst rows n..2n-1 (stride WS)
                        mbar_arrive_expect_tx(&s.full[slot], 2u * st.n * H);
                        for (int r = 0; r < st.n; ++r) {
                            bulk_g2s(dst + (size_t)r * WS, gwt.gw + (size_t)(st.r0 + r) * H, (uint32_t)H, &s.full[slot]);
                            bulk_g2s(dst + (size_t)(st.n + r) * WS, gwt.uw + (size_t)(st.r0 + r) * H, (uint32_t)H,
                                     &s.full[slot]);
                        }
                    } else {
                        const int IS = gwt.inter + WPAD;
                        mbar_arrive_expect_tx(&s.full[slot], (uint32_t)st.n * gwt.inter);
                        for (int r = 0; r < st.n; ++r)
                            bulk_g2s(dst + (size_t)r * IS, gwt.dw + (size_t)(st.r0 + r) * gwt.inter, (uint32_t)gwt.inter,
                                     &s.full[slot]);
                        poll_adone();
                        if (adone_seen) {
                            issue_h(slot, st.u, st.q0, st.nq);
                        } else {
#pragma unroll
                            for (int i = 0; i < NSTAGES; ++i)
                                if (i == slot) {
                                    pend_u[i] = st.u;
                                    pend_q0[i] = st.q0;
                                    pend_nq[i] = st.nq;
                                }
                        }
                    }
                    ++si;
                }
                bool pending = false;
#pragma unroll
                for (int i = 0; i < NSTAGES; ++i) pending |= pend_nq[i] != 0;
                for (uint32_t it = 0; pending && !adone_seen && !s.abort && it < CZ_SPIN_LIMIT; ++it) {
                    poll_adone();
                    if (!adone_seen && it > 16) __nanosleep(128);
                }
                if (pending && !adone_seen && !s.abort) set_error(err, s, CZ_DERR_READY_WAIT);
                // drain: no copy may land after this CTA exits (waiting on a phase
                // that already completed returns at once)
                for (int k = max(0, si - NSTAGES); k < si; ++k) {
                    bool ok = false;
                    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok; ++it) {
                        ok = mbar_try_wait(&s.full[k % NSTAGES], (k / NSTAGES) & 1);
                        if (!ok) __nanosleep(64);
                    }
                    if (!ok) atomicOr(err, CZ_DERR_DRAIN_WAIT);
                }
                bool ok = false;
                for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok; ++it) {
                    ok = mbar_try_wait(&s.sbar, 0);
                    if (!ok) __nanosleep(64);
                }
                if (!ok) atomicOr(err, CZ_DERR_DRAIN_WAIT);
                // h copies: if one is still in flight, the consumer of that slot
                // is waiting for it; the consumers drain them (below) before exit.
            }
            __syncwarp();
        } else {
            // ---------------- consumers: warp w computes stages w, w+NCW, ... ----------------
            const int g = lane >> 2, tq = lane & 3;  // MMA fragment coordinates
            float bacc[MAXBT][2][4];                // phase B: [tile][row g / g+8][token]
#pragma unroll
            for (int a = 0; a < MAXBT; ++a)
#pragma unroll
                for (int b = 0; b < 2; ++b)
#pragma unroll
                    for (int q = 0; q < 4; ++q) bacc[a][b][q] = 0.0f;
            StageIter itr;
            itr.init(s, a_lo, a_hi, b_lo, b_hi, RA);
            Stage st;
            int si = 0, hcnt = 0;
            bool switched = false, hmax_seen = false;
            // Every consumer warp runs this once, at the first down stage of the
            // schedule (or at the end): all of this CTA's h rows and max |h| are
            // stored, so the CTA counts itself done with phase A.
            auto transition = [&]() {
                switched = true;
                asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
                if (tid == 0) {
                    __threadfence();
                    red_release_add_gpu(adone, 1u);
                }
            };
            if (!warp_wait(&s.sbar, 0, s) && lane == 0 && !s.abort) set_error(err, s, CZ_DERR_FULL_WAIT);
            while (!s.abort && itr.next(st)) {
                if (st.phase == 1 && !switched) transition();
                if ((si % NCW) != warp) {
                    ++si;
                    continue;
                }
                const int slot = si % NSTAGES;
                if (!warp_wait(&s.full[slot], (si / NSTAGES) & 1, s)) {
                    if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_FULL_WAIT);
                    break;
                }
                uint8_t* stage = s.ring + (size_t)slot * STAGE_BYTES;
                const int u = st.u;
                const int np = s.g_npairs[u];
                const int* pairs = s.order + s.g_pair0[u];
                const GroupW gwt = group_w(p, s.g_expert[u]);
                if (st.phase == 0) {
                    // ---- gate/up: tile rows 0..7 = gate rows r0..r0+n-1, rows 8..15 = up rows ----
                    const int n = st.n;
                    const int nbI = cz_nblk(gwt.inter);
                    const float* gtab = s.sA_ok ? s.sA + s.sA_off[u - s.a_u0] : gwt.gs;
                    const float* utab = s.sA_ok ? gtab + nbI * nbHp : gwt.us;
                    const bool rowok = g < n;
                    const int rowblk = (st.r0 + min(g, n - 1)) >> 7;
                    for (int q0 = 0; q0 < np; q0 += 4) {
                        const int nq = min(4, np - q0);
                        const int col_tok = (g & 3) < nq ? pair_token(pairs[q0 + (g & 3)], T, K) : -1;
                        const uint8_t* xcol = s.xh + (size_t)max(col_tok, 0) * XQS + ((g >> 2) ? 32 : 0);
                        float acc[4] = {0.f, 0.f, 0.f, 0.f};
                        tile_mma(stage + (size_t)g * WS, stage + (size_t)(n + g) * WS, rowok, rowok, xcol, col_tok >= 0,
                                 H, tq, gtab + (size_t)rowblk * nbHp, utab + (size_t)rowblk * nbHp, acc);
                        // hi (cols 0..3) + lo (cols 4..7, two lanes over)
                        const float lo0 = __shfl_down_sync(0xffffffffu, acc[0], 2);
                        const float lo1 = __shfl_down_sync(0xffffffffu, acc[1], 2);
                        const float lo2 = __shfl_down_sync(0xffffffffu, acc[2], 2);
                        const float lo3 = __shfl_down_sync(0xffffffffu, acc[3], 2);
                        float mh[2] = {0.f, 0.f};
                        if (tq < 2 && rowok) {
                            const float gv[2] = {acc[0] + lo0, acc[1] + lo1};
                            const float uv[2] = {acc[2] + lo2, acc[3] + lo3};
#pragma unroll
                            for (int d = 0; d < 2; ++d) {
                                const int q = 2 * tq + d;
                                if (q < nq) {
                                    const int pr = pairs[q0 + q];
                                    const float xsc = s.xscale[pair_token(pr, T, K)];
                                    const float hv = cz_silu(gv[d] * xsc) * (uv[d] * xsc);
                                    p.hbuf[(size_t)pr * HS + st.r0 + g] = hv;
                                    mh[d] = fabsf(hv);
                                }
                            }
                        }
                        // max |h| per pair over the tile rows (lanes g*4 + tq, same tq)
#pragma unroll
                        for (int d = 0; d < 2; ++d) {
                            float m = mh[d];
                            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
                            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                            const int q = 2 * tq + d;
                            if (g == 0 && tq < 2 && q < nq && m > 0.0f && m < 3.0e38f)
                                atomicMax(hmax + pairs[q0 + q], __float_as_uint(m));
                        }
                    }
                } else {
                    // ---- down: tile = 16 of this CTA's output rows, columns = pairs q0.. of the group ----
                    const int inter = gwt.inter;
                    const int IS = inter + WPAD;
                    const int nbIp = cz_nbp(inter);
                    const int tile = (st.r0 - b_lo) >> 4;
                    const int nq = st.nq;
                    bool ok = warp_wait(&s.hfull[slot], hcnt & 1, s);
                    if (ok) ++hcnt;
                    if (ok && !hmax_seen) {  // every CTA's max |h| is visible once the count is (acquire)
                        bool seen = true;
                        if (lane == 0) seen = wait_geq_bounded(adone, (uint32_t)G, err);
                        ok = __shfl_sync(0xffffffffu, seen, 0);
                        hmax_seen = ok;
                        __syncwarp();
                    }
                    if (!ok) {
                        if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_READY_WAIT);
                        break;
                    }
                    // this stage's h rows: f32 -> per-pair 2^s scaled f16 hi/lo chunks, in place
                    uint8_t* hrows = stage + 16 * IS;
                    const int HRS = inter * 4 + HPAD;
                    int hexp[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        hexp[q] = q < nq ? prescale_exp(__uint_as_float(ld_relaxed_gpu(hmax + pairs[st.q0 + q]))) : 0;
                    const int nch = inter >> 4;
                    for (int k = lane; k < nq * nch; k += 32) {
                        const int q = k / nch, ch = k - q * nch;
                        int e = hexp[0];
#pragma unroll
                        for (int qq = 1; qq < 4; ++qq)
                            if (qq == q) e = hexp[qq];
                        float4* cp = reinterpret_cast<float4*>(hrows + (size_t)q * HRS + ch * 64);
                        float v[16];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 f = cp[j];
                            v[4 * j] = f.x;
                            v[4 * j + 1] = f.y;
                            v[4 * j + 2] = f.z;
                            v[4 * j + 3] = f.w;
                        }
                        __align__(16) __half hv[32];
#pragma unroll
                        for (int j = 0; j < 16; ++j) split_f16(v[j], e, hv[j], hv[16 + j]);
                        const uint4* src = reinterpret_cast<const uint4*>(hv);
                        uint4* dst = reinterpret_cast<uint4*>(cp);
#pragma unroll
                        for (int j = 0; j < 4; ++j) dst[j] = src[j];
                    }
                    __syncwarp();
                    const bool oka = g < st.n, okb = g + 8 < st.n;
                    const int oa = st.r0 + min(g, st.n - 1), ob = st.r0 + min(g + 8, st.n - 1);
                    const float* dtab = s.sB_ok ? s.sB + u * nbb * nbIrp : nullptr;
                    const float* sa = dtab ? dtab + ((oa >> 7) - bb0) * nbIp : gwt.ds + (size_t)(oa >> 7) * nbIp;
                    const float* sbr = dtab ? dtab + ((ob >> 7) - bb0) * nbIp : gwt.ds + (size_t)(ob >> 7) * nbIp;
                    const int cq = g & 3;
                    const uint8_t* hcol = hrows + (size_t)min(cq, max(nq - 1, 0)) * HRS + ((g >> 2) ? 32 : 0);
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
                    tile_mma(stage + (size_t)g * IS, stage + (size_t)(g + 8) * IS, oka, okb, hcol, cq < nq, inter, tq,
                             sa, sbr, acc);
                    const float lo0 = __shfl_down_sync(0xffffffffu, acc[0], 2);
                    const float lo1 = __shfl_down_sync(0xffffffffu, acc[1], 2);
                    const float lo2 = __shfl_down_sync(0xffffffffu, acc[2], 2);
                    const float lo3 = __shfl_down_sync(0xffffffffu, acc[3], 2);
                    if (tq < 2) {
                        const float va[2] = {acc[0] + lo0, acc[1] + lo1};
                        const float vb[2] = {acc[2] + lo2, acc[3] + lo3};
#pragma unroll
                        for (int d = 0; d < 2; ++d) {
                            const int q = 2 * tq + d;
                            if (q < nq) {
                                const int pr = pairs[st.q0 + q];
                                const int tk = pair_token(pr, T, K);
                                int e = hexp[0];
#pragma unroll
                                for (int qq = 1; qq < 4; ++qq)
                                    if (qq == q) e = hexp[qq];
                                const float w = s.pg[pr] * ldexpf(1.0f, -e);
#pragma unroll
                                for (int tt = 0; tt < MAXBT; ++tt) {
                                    if (tt != tile) continue;
#pragma unroll
                                    for (int t4 = 0; t4 < 4; ++t4) {
                                        if (t4 != tk) continue;
                                        bacc[tt][0][t4] = __fmaf_rn(w, va[d], bacc[tt][0][t4]);
                                        bacc[tt][1][t4] = __fmaf_rn(w, vb[d], bacc[tt][1][t4]);
                                    }
                                }
                            }
                        }
                    }
                    // the in-place h writes precede the next bulk copy into this slot
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.empty[slot]);
                ++si;
            }
            if (!switched) transition();
            // an h copy into this warp's slot may still be in flight after an early
            // stop: wait (bounded) for every one the producer could have issued
            if (s.abort) {
                for (uint32_t it = 0; it < CZ_SPIN_LIMIT; ++it) {
                    if (mbar_try_wait(&s.hfull[warp], hcnt & 1)) break;
                    if (it > 16) __nanosleep(64);
                    if (it > 4096) break;
                }
            }
            // combine the warps' down sums in a fixed order and write the rows once
            if (tq < 2) {
#pragma unroll
                for (int tt = 0; tt < MAXBT; ++tt)
#pragma unroll
                    for (int b = 0; b < 2; ++b)
#pragma unroll
                        for (int t4 = 0; t4 < 4; ++t4)
                            s.red[((((warp * MAXBT + tt) * 16 + g + 8 * b) * 4 + t4) * 2) + tq] = bacc[tt][b][t4];
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
            if (!s.abort) {
                for (int k = tid; k < (b_hi - b_lo) * 4; k += NCW * 32) {
                    const int ol = k >> 2, tk = k & 3;
                    if (tk >= T) continue;
                    const int tt = ol >> 4, row = ol & 15;
                    float v = 0.0f;
                    for (int w = 0; w < NCW; ++w)
                        for (int h2 = 0; h2 < 2; ++h2) v += s.red[((((w * MAXBT + tt) * 16 + row) * 4 + tk) * 2) + h2];
                    const int o = b_lo + ol;
                    if (p.residual) v = __fadd_rn(p.residual[(size_t)tk * H + o], v);
                    p.out[(size_t)tk * H + o] = v;
                }
            }
        }
    }

    // ---------------- completion: advance the launch sequence ----------------
finish:
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&reg[1], 1u);
        if (old == (uint32_t)G - 1u) atomicExch(p.sync, seq + 1u);
    }
}

// ---- host side --------------------------------------------------------------

static bool g_attr_set = false;

size_t decode_smem_bytes() { return sizeof(DecodeSmem) + 1024; }

int decode_max_tokens(int H, int E, int K, int I, int SI, int x_bf16, int num_sms) {
    if (K < 1 || K > MAXK || E < K || E > MAXE || H % 16 || I % 16 || SI % 16 || H < 16 || I < 16) return 0;
    const int rows_b = (H + num_sms - 1) / num_sms;  // output rows per CTA
    if (rows_b > 16 * MAXBT) return 0;
    if (2 * (H + WPAD) > STAGE_BYTES) return 0;  // >= 1 gate + 1 up row per stage
    // a down stage: a 16-row tile + the h rows of 4 pairs
    if (16 * (I + WPAD) + 4 * (4 * I + HPAD) > STAGE_BYTES || 16 * (SI + WPAD) + 4 * (4 * SI + HPAD) > STAGE_BYTES)
        return 0;
    const int max_rows = (E + (SI ? 1 : 0) + num_sms - 1) / num_sms;  // router rows staged per CTA
    int t = MAXT;
    while (t > 0) {
        const size_t ring = (size_t)max_rows * H * 4 + (size_t)t * H * (x_bf16 ? 2 : 4) + (size_t)H * 4;
        const size_t lg = (size_t)t * logit_stride(E) * 4;
        const size_t xq = (size_t)t * (H * 4 + 32);
        if (ring <= (size_t)RING_BYTES && lg <= (size_t)RING_BYTES && xq <= (size_t)XH_BYTES) break;
        --t;
    }
    return t;
}

int decode_launch(const DecodeParams& prm, int num_sms, cudaStream_t stream) {
    const int tmax = decode_max_tokens(prm.H, prm.E, prm.K, prm.I, prm.SI, prm.x_bf16, num_sms);
    if (prm.T < 1 || prm.T > tmax) return CZ_ESHAPE;
    if (prm.rms_w && prm.x_bf16) return CZ_EARGS;
    const size_t smem = decode_smem_bytes();
    if (!g_attr_set) {
        if (cudaFuncSetAttribute(moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return CZ_ELAUNCH;
        g_attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, moe_decode_kernel, prm) != cudaSuccess) return CZ_ELAUNCH;
    return CZ_OK;
}

}  // namespace cz
