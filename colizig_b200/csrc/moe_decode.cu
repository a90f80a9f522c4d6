// Decode-regime MoE layer (a few tokens) as ONE persistent cooperative kernel.
//
// Reference path (src/qwen38/moe.zig): route (435-463) -> per expert gate/up
// (fp8.zig:165-257) -> silu(g)*u (activation.zig:8-20) -> down -> out += gate*eo,
// plus the always-on shared expert (467-479).
//
// Grid = one CTA per SM: 8 consumer warps + 1 producer warp.  Shared memory:
// a ring of bulk-copy (TMA) stages, a token/h staging area and the routing
// tables.  No global memory is read inside an inner loop: while HBM is
// saturated by the weight stream, any other load waits behind it.
//
//   R  router logits.  CTA c owns router rows [c*E'/G, (c+1)*E'/G) (E' = E, +1
//      for the shared expert's gate vector).  Rows and tokens are bulk-copied
//      into shared memory; every logit is formed in the reference's exact f32
//      order (dotF32, matmul.zig:60-82: 32 FMA chains = one per lane, then the
//      lane-ordered combine), so the top-k below is bit-identical to it.  In
//      stack mode the tokens are rms-normalised in place first.  A grid-wide
//      arrive counter closes the phase.
//   K  top-k.  Every CTA computes softmax/top-k for all tokens (identically),
//      groups the (token, slot) pairs by expert (ascending id, shared expert
//      last) and preloads the block scales it will need into shared memory.
//   A  gate/up.  The flattened (group, row) list is split evenly over CTAs.  The
//      producer streams gate+up rows through the ring; consumers decode E4M3 in
//      registers, fold the 128x128 block scale once per 16-column chunk, reduce
//      with warp shuffles and store h = silu(g)*u (f32) to HBM.
//   B  down + combine.  CTA c owns output rows [c*H/G, (c+1)*H/G) of every
//      group.  The producer streams these down-weight rows as soon as ring slots
//      free up (they do not depend on h); once every CTA has finished phase A
//      it bulk-copies all of h into shared memory.  Each (token, row) sums
//      gate * dot(h, w) over the groups in ascending expert order in registers
//      (fixed order, no atomics) and is written exactly once.
//
// Every wait is bounded; a CTA that gives up sets a bit in the device error
// word, stops early (draining its in-flight copies) and the host returns -7.
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {

constexpr int NCW = 8;                    // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;  // + 1 producer warp
constexpr int STAGE_BYTES = 32 * 1024;
constexpr int NSTAGES = 3;
constexpr int RING_BYTES = STAGE_BYTES * NSTAGES;
constexpr int XH_BYTES = 96 * 1024;       // tokens (phases R, A), then h (phase B)
constexpr int MAXT = kDecodeMaxTokens;    // 32: one lane per token in phase B
constexpr int MAXK = kMaxTopk;            // 16
constexpr int MAXE = kMaxExperts;         // 512
constexpr int MAXG = MAXE + 1;            // routed experts + shared
constexpr int MAXP = MAXT * (MAXK + 1);   // (token, slot) pairs incl. shared-expert pairs
constexpr int MAXBK = 8;                  // phase-B rows per warp (rows per CTA <= 64)
constexpr int MAXM = MAXE / 32;           // router values per lane
constexpr int SA_FLOATS = 1024;           // cached gate/up scale tables (phase A)
constexpr int SB_FLOATS = 512;            // cached down scale rows (phase B)
constexpr int MAXAG = 8;                  // groups cached for phase A
constexpr int RED_FLOATS = NCW * NCW * 4 * 2;

struct __align__(128) DecodeSmem {
    uint8_t ring[RING_BYTES];
    uint8_t xh[XH_BYTES];
    float sA[SA_FLOATS];
    float sB[SB_FLOATS];
    float red[RED_FLOATS];
    uint64_t full[NSTAGES];
    uint64_t empty[NSTAGES];
    uint64_t rbar;
    uint64_t hbar;
    int abort;
    int U;
    int sA_ok, sB_ok, a_u0, a_u1;
    int sA_off[MAXAG + 1];
    float rsc[MAXT];
    int pe[MAXP];
    float pg[MAXP];
    int cnt[MAXG + 1];
    int goff[MAXG + 1];
    int gidx[MAXG + 1];
    int g_expert[MAXG];
    int g_pair0[MAXG];
    int g_npairs[MAXG];
    int g_rowA[MAXG + 1];
    int sorted_pairs[MAXP];
};

static_assert(sizeof(DecodeSmem) + 1024 <= 227 * 1024, "decode smem too large");

// ---- sync words ------------------------------------------------------------
// sync[0] = launch sequence number, sync[1] = error word, then two regions of
// kSyncRegionWords: [0] router arrivals, [1] CTAs done, [2] CTAs done with
// phase A.  A launch uses region seq&1 and zeroes the other one, so a launch
// that stopped early leaves nothing behind for the next.
__device__ __forceinline__ uint32_t* region(uint32_t* sync, int par) { return sync + 2 + par * kSyncRegionWords; }

struct Stage {
    int phase;  // 0 = A (gate/up), 1 = B (down)
    int u;      // group
    int r0;     // A: first row within the group; B: first absolute output row
    int n;      // rows
};

// Deterministic stage schedule shared by the producer and the consumers.
struct StageIter {
    int phase, u, a, a_hi, b_lo, b_hi, brow, U, RA, E, I, SI;
    const int* rowA;
    const int* g_expert;

    __device__ void init(const DecodeSmem& s, int a_lo, int a_hi_, int b_lo_, int b_hi_, int ra, int E_, int I_,
                         int SI_) {
        phase = 0;
        U = s.U;
        rowA = s.g_rowA;
        g_expert = s.g_expert;
        a = a_lo;
        a_hi = a_hi_;
        b_lo = b_lo_;
        b_hi = b_hi_;
        brow = b_lo_;
        RA = ra;
        E = E_;
        I = I_;
        SI = SI_;
        u = 0;
        while (u < U && rowA[u + 1] <= a) ++u;
    }
    __device__ int inter_of(int g) const { return g_expert[g] == E ? SI : I; }
    __device__ bool next(Stage& st) {
        if (phase == 0) {
            if (a < a_hi) {
                while (rowA[u + 1] <= a) ++u;
                const int n = min(RA, min(rowA[u + 1] - a, a_hi - a));
                st.phase = 0;
                st.u = u;
                st.r0 = a - rowA[u];
                st.n = n;
                a += n;
                return true;
            }
            phase = 1;
            u = 0;
            brow = b_lo;
        }
        if (b_lo >= b_hi || u >= U) return false;
        const int rb = max(1, STAGE_BYTES / inter_of(u));
        const int n = min(rb, b_hi - brow);
        st.phase = 1;
        st.u = u;
        st.r0 = brow;
        st.n = n;
        brow += n;
        if (brow >= b_hi) {
            ++u;
            brow = b_lo;
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
        const size_t ssz = (size_t)cz_nblk(p.I) * cz_nblk(p.H);
        g.gs = p.gate_s + (size_t)e * ssz;
        g.us = p.up_s + (size_t)e * ssz;
        g.ds = p.down_s + (size_t)e * ssz;
    }
    return g;
}

__device__ void set_error(uint32_t* err, DecodeSmem& s, uint32_t bit) {
    atomicOr(err, bit);
    s.abort = 1;
}

// Exclusive scan of n ints by one warp (flags: scan (in[i] > 0) instead).
__device__ int warp_exclusive_scan(const int* in, int* out, int n, int lane, bool flags) {
    const int per = (n + 31) / 32;
    const int lo = min(n, lane * per), hi = min(n, lo + per);
    int local = 0;
    for (int i = lo; i < hi; ++i) local += flags ? (in[i] > 0) : in[i];
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int i = lo; i < hi; ++i) {
        out[i] = run;
        run += flags ? (in[i] > 0) : in[i];
    }
    return __shfl_sync(0xffffffffu, incl, 31);
}

// 16 consecutive token values (f32) from the staged tokens.
__device__ __forceinline__ void load_x16(const uint8_t* xs, bool bf16, int H, int t, int col, float* x) {
    if (bf16) {
        const uint4* p = reinterpret_cast<const uint4*>(xs + ((size_t)t * H + col) * 2);
        const uint4 a = p[0], b = p[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            x[2 * k] = __uint_as_float(w[k] << 16);
            x[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
        }
    } else {
        const float4* p = reinterpret_cast<const float4*>(xs + ((size_t)t * H + col) * 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float4 v = p[k];
            x[4 * k] = v.x;
            x[4 * k + 1] = v.y;
            x[4 * k + 2] = v.z;
            x[4 * k + 3] = v.w;
        }
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

// Top-k of one token (moe.zig:435-463) by one warp.  Lane l holds experts
// l, l+32, ...  Keys are the f32 bits of exp(v - max) + 1 (non-negative floats
// order like their bits; 0 = not a candidate: chosen, NaN or beyond E).  Each
// round takes the largest key and, among equal keys, the smallest id — the
// reference's strict-greater scan from e = 0 with bv = -1.  A round without a
// candidate yields id 0, as in the reference.
__device__ void route_token(const float* __restrict__ lg, int E, int K, int norm_topk, int has_shared, int T, int t,
                            int lane, DecodeSmem& s, uint32_t* topk_idx, float* topk_gates, bool write_out) {
    float v[MAXM];
    float mx = __int_as_float(0xffc00000);  // NaN: fmaxf ignores it
    const int nm = (E + 31) >> 5;
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        const int e = lane + 32 * m;
        v[m] = (m < nm && e < E) ? __ldcg(lg + e) : __int_as_float(0xffc00000);
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
        s.pg[T * K + t] = cz_sigmoid(__ldcg(lg + E));
    }
    __syncwarp();
}

__global__ void __launch_bounds__(NTHREADS, 1) moe_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    DecodeSmem& s = *reinterpret_cast<DecodeSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int T = p.T, H = p.H, E = p.E, K = p.K;
    const int SI = p.SI, Ir = p.I;
    const int Er = E + (SI ? 1 : 0);
    const bool xbf = p.x_bf16 != 0;
    uint32_t* const err = p.sync + 1;

    const uint32_t seq = ld_relaxed_gpu(p.sync);
    uint32_t* reg = region(p.sync, seq & 1);
    if (c == 0 && tid < kSyncRegionWords) region(p.sync, (seq & 1) ^ 1)[tid] = 0u;
    if (tid == 0) {
        for (int i = 0; i < NSTAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], NCW);
        }
        mbar_init(&s.rbar, 1);
        mbar_init(&s.hbar, 1);
        s.abort = 0;
        fence_mbarrier_init();
    }
    __syncthreads();

    // ---------------- phase R: router logits ----------------
    const int row_lo = (int)((long long)c * Er / G), row_hi = (int)((long long)(c + 1) * Er / G);
    const int nrows = row_hi - row_lo;
    const uint32_t xbytes = (uint32_t)T * H * (xbf ? 2u : 4u);
    const uint32_t rbytes = (uint32_t)nrows * H * 4u;
    float* rows = reinterpret_cast<float*>(s.ring);
    float* wnorm = reinterpret_cast<float*>(s.ring + rbytes);  // stack mode: rms weight
    uint8_t* xs = s.xh;
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
                s.rsc[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            }
        }
        __syncthreads();
        for (int k = tid; k < T * H; k += NTHREADS) {
            const int t = k / H, i = k - t * H;
            xf[k] = __fmul_rn(__fmul_rn(xf[k], s.rsc[t]), wnorm[i]);
        }
        __syncthreads();
    }

    if (!s.abort) {
        const int ntg = (T + 3) / 4;
        for (int it = warp; it < nrows * ntg; it += NCW + 1) {
            const int r = it / ntg, t0 = (it % ntg) * 4;
            if (xbf)
                router_item<true>(rows + (size_t)r * H, xs, H, t0, min(4, T - t0), lane, p.logits, E + 1, row_lo + r);
            else
                router_item<false>(rows + (size_t)r * H, xs, H, t0, min(4, T - t0), lane, p.logits, E + 1, row_lo + r);
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        red_release_add_gpu(&reg[0], 1u);
        if (!wait_geq_bounded(&reg[0], (uint32_t)G, err)) set_error(err, s, CZ_DERR_ROUTER_BARRIER);
    }
    __syncthreads();

    // ---------------- phase K: top-k + grouping (every CTA) ----------------
    if (s.abort) goto finish;  // uniform: settled before the barrier above
    for (int t = warp; t < T; t += NCW + 1)
        route_token(p.logits + (size_t)t * (E + 1), E, K, p.norm_topk, SI != 0, T, t, lane, s, p.topk_idx,
                    p.topk_gates, c == 0);
    {
        const int P = T * K + (SI ? T : 0);
        for (int i = tid; i <= Er; i += NTHREADS) s.cnt[i] = 0;
        __syncthreads();
        for (int i = tid; i < P; i += NTHREADS) atomicAdd(&s.cnt[s.pe[i]], 1);
        __syncthreads();
        if (warp == 0) {
            warp_exclusive_scan(s.cnt, s.goff, Er, lane, false);
        } else if (warp == 1) {
            const int U = warp_exclusive_scan(s.cnt, s.gidx, Er, lane, true);
            if (lane == 0) s.U = U;
        }
        __syncthreads();
        const int U = s.U;
        for (int e = tid; e < Er; e += NTHREADS) {
            if (s.cnt[e] > 0) {
                const int u = s.gidx[e];
                s.g_expert[u] = e;
                s.g_pair0[u] = s.goff[e];
                s.g_npairs[u] = s.cnt[e];
            }
        }
        for (int u = tid; u <= U; u += NTHREADS) s.g_rowA[u] = u * Ir;  // routed groups: I rows each
        __syncthreads();
        if (tid == 0 && U > 0 && s.g_expert[U - 1] == E) s.g_rowA[U] = (U - 1) * Ir + SI;  // shared: last
        for (int i = tid; i < P; i += NTHREADS) {
            const int e = s.pe[i];
            int pos = s.goff[e];
            for (int q = 0; q < i; ++q) pos += (s.pe[q] == e);
            s.sorted_pairs[pos] = i;
        }
        __syncthreads();
    }

    // ---------------- phases A and B ----------------
    {
        const int U = s.U;
        const int NA = s.g_rowA[U];
        const int a_lo = (int)((long long)c * NA / G), a_hi = (int)((long long)(c + 1) * NA / G);
        const int b_lo = (int)((long long)c * H / G), b_hi = (int)((long long)(c + 1) * H / G);
        const int RA = max(1, STAGE_BYTES / (2 * H));
        const int HS = max(Ir, SI);
        const int nbH = cz_nblk(H);
        const int P = T * K + (SI ? T : 0);
        const uint32_t hbytes = (uint32_t)P * HS * 4u;
        uint32_t* const adone = reg + 2;
        const bool has_b = (b_lo < b_hi) && U > 0;
        const int bb0 = b_lo >> 7, nbb = has_b ? ((b_hi - 1) >> 7) - bb0 + 1 : 0;
        const int nbIr = cz_nblk(Ir);

        // Preload the block scales this CTA needs (plain loads, one latency).
        if (tid == 0) {
            int u0 = 0;
            while (u0 < U && s.g_rowA[u0 + 1] <= a_lo) ++u0;
            int u1 = u0, need = 0;
            s.sA_off[0] = 0;
            while (u1 < U && s.g_rowA[u1] < a_hi && u1 - u0 < MAXAG) {
                const int inter = s.g_expert[u1] == E ? SI : Ir;
                need += 2 * cz_nblk(inter) * nbH;
                ++u1;
                s.sA_off[u1 - u0] = need;
            }
            s.a_u0 = u0;
            s.a_u1 = u1;
            s.sA_ok = (need <= SA_FLOATS) && (u1 >= U || s.g_rowA[u1] >= a_hi);
            const int needB =
                U > 0 ? (U - 1) * nbb * nbIr + nbb * cz_nblk(s.g_expert[U - 1] == E ? SI : Ir) : 0;
            s.sB_ok = needB <= SB_FLOATS;
        }
        __syncthreads();
        if (s.sA_ok) {
            for (int u = s.a_u0; u < s.a_u1; ++u) {
                const GroupW gwt = group_w(p, s.g_expert[u]);
                const int n1 = cz_nblk(gwt.inter) * nbH;
                float* dst = s.sA + s.sA_off[u - s.a_u0];
                for (int i = tid; i < n1; i += NTHREADS) {
                    dst[i] = __ldg(gwt.gs + i);
                    dst[n1 + i] = __ldg(gwt.us + i);
                }
            }
        }
        if (s.sB_ok && has_b) {
            // group u's cached rows start at u * nbb * nb(I) (the shared group is last)
            for (int u = 0; u < U; ++u) {
                const GroupW gwt = group_w(p, s.g_expert[u]);
                const int nbI = cz_nblk(gwt.inter);
                for (int k = tid; k < nbb * nbI; k += NTHREADS)
                    s.sB[u * nbb * nbIr + k] = __ldg(gwt.ds + (size_t)bb0 * nbI + k);
            }
        }
        __syncthreads();

        if (warp == NCW) {
            // ---------------- producer (one thread) ----------------
            if (lane == 0) {
                fence_proxy_async_smem();
                StageIter itr;
                itr.init(s, a_lo, a_hi, b_lo, b_hi, RA, E, Ir, SI);
                Stage st;
                int si = 0;
                bool h_issued = false;
                auto try_issue_h = [&]() {
                    if (!h_issued && has_b && ld_acquire_gpu(adone) >= (uint32_t)G) {
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        mbar_arrive_expect_tx(&s.hbar, hbytes);
                        bulk_g2s(s.xh, p.hbuf, hbytes, &s.hbar);
                        h_issued = true;
                    }
                };
                while (!s.abort && itr.next(st)) {
                    const int slot = si % NSTAGES, round = si / NSTAGES;
                    if (round > 0) {
                        bool ok = false;
                        for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok && !s.abort; ++it) {
                            ok = mbar_try_wait(&s.empty[slot], (round - 1) & 1);
                            if (!ok) {
                                try_issue_h();
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
                        const uint32_t bytes = (uint32_t)st.n * H;
                        mbar_arrive_expect_tx(&s.full[slot], 2 * bytes);
                        bulk_g2s(dst, gwt.gw + (size_t)st.r0 * H, bytes, &s.full[slot]);
                        bulk_g2s(dst + bytes, gwt.uw + (size_t)st.r0 * H, bytes, &s.full[slot]);
                    } else {
                        const uint32_t bytes = (uint32_t)st.n * gwt.inter;
                        mbar_arrive_expect_tx(&s.full[slot], bytes);
                        bulk_g2s(dst, gwt.dw + (size_t)st.r0 * gwt.inter, bytes, &s.full[slot]);
                    }
                    ++si;
                }
                for (uint32_t it = 0; has_b && !h_issued && !s.abort && it < CZ_SPIN_LIMIT; ++it) {
                    try_issue_h();
                    if (!h_issued && it > 16) __nanosleep(128);
                }
                if (has_b && !h_issued && !s.abort) set_error(err, s, CZ_DERR_READY_WAIT);
                // drain: no copy may land after this CTA exits
                for (int k = max(0, si - NSTAGES); k < si; ++k) {
                    bool ok = false;
                    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok; ++it) {
                        ok = mbar_try_wait(&s.full[k % NSTAGES], (k / NSTAGES) & 1);
                        if (!ok) __nanosleep(64);
                    }
                    if (!ok) atomicOr(err, CZ_DERR_DRAIN_WAIT);
                }
                if (h_issued) {
                    bool ok = false;
                    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok; ++it) {
                        ok = mbar_try_wait(&s.hbar, 0);
                        if (!ok) __nanosleep(64);
                    }
                    if (!ok) atomicOr(err, CZ_DERR_DRAIN_WAIT);
                }
            }
            __syncwarp();
        } else {
            // ---------------- consumers ----------------
            float bacc[MAXBK];
#pragma unroll
            for (int k = 0; k < MAXBK; ++k) bacc[k] = 0.0f;
            StageIter itr;
            itr.init(s, a_lo, a_hi, b_lo, b_hi, RA, E, Ir, SI);
            Stage st;
            int si = 0;
            bool signalled = false, h_ready = false;
            const int nch = H >> 4;
            auto signal_phase_a = [&]() {
                fence_proxy_async_smem();  // our reads of the tokens precede the async write of h
                asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
                if (tid == 0) {
                    __threadfence();
                    red_release_add_gpu(adone, 1u);
                }
                signalled = true;
            };
            while (!s.abort && itr.next(st)) {
                if (st.phase == 1 && !signalled) signal_phase_a();
                if (st.phase == 1 && !h_ready) {
                    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s.hbar, 0, &s.abort))) {
                        if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_READY_WAIT);
                        break;
                    }
                    h_ready = true;
                }
                const int slot = si % NSTAGES;
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s.full[slot], (si / NSTAGES) & 1, &s.abort))) {
                    if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_FULL_WAIT);
                    break;
                }
                const uint8_t* stage = s.ring + (size_t)slot * STAGE_BYTES;
                const int u = st.u;
                const int e = s.g_expert[u];
                const int np = s.g_npairs[u];
                const int* pairs = s.sorted_pairs + s.g_pair0[u];
                const GroupW gwt = group_w(p, e);
                if (st.phase == 0) {
                    // gate/up rows st.r0 .. st.r0+n of group u; wpr warps share a row when n < NCW
                    const int n = st.n;
                    const int wpr = n >= NCW ? 1 : NCW / n;
                    const int nbI = cz_nblk(gwt.inter);
                    const float* gtab = s.sA_ok ? s.sA + s.sA_off[u - s.a_u0] : gwt.gs;
                    const float* utab = s.sA_ok ? gtab + nbI * nbH : gwt.us;
                    for (int q0 = 0; q0 < np; q0 += 4) {
                        const int nq = min(4, np - q0);
                        int tok[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int pr = pairs[q0 + min(q, nq - 1)];
                            tok[q] = pr < T * K ? pr / K : pr - T * K;
                        }
                        const int sub = wpr == 1 ? 0 : warp % wpr;
                        for (int rr = (wpr == 1 ? warp : warp / wpr); rr < n && warp < n * wpr;
                             rr += (wpr == 1 ? NCW : n)) {
                            const int j = st.r0 + rr;
                            const uint8_t* wg = stage + (size_t)rr * H;
                            const uint8_t* wu = stage + (size_t)n * H + (size_t)rr * H;
                            const float* sgr = gtab + (size_t)(j >> 7) * nbH;
                            const float* sur = utab + (size_t)(j >> 7) * nbH;
                            float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
                            for (int ch = sub * 32 + lane; ch < nch; ch += 32 * wpr) {
                                float fg[16], fu[16];
                                decode16(*reinterpret_cast<const uint4*>(wg + ch * 16), fg);
                                decode16(*reinterpret_cast<const uint4*>(wu + ch * 16), fu);
                                const float scg = sgr[ch >> 3], scu = sur[ch >> 3];
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    if (q < nq) {
                                        float xv[16];
                                        load_x16(xs, xbf, H, tok[q], ch * 16, xv);
                                        float pg0 = 0.f, pg1 = 0.f, pu0 = 0.f, pu1 = 0.f;
#pragma unroll
                                        for (int k = 0; k < 16; k += 2) {
                                            pg0 = __fmaf_rn(xv[k], fg[k], pg0);
                                            pg1 = __fmaf_rn(xv[k + 1], fg[k + 1], pg1);
                                            pu0 = __fmaf_rn(xv[k], fu[k], pu0);
                                            pu1 = __fmaf_rn(xv[k + 1], fu[k + 1], pu1);
                                        }
                                        ag[q] = __fmaf_rn(scg, pg0 + pg1, ag[q]);
                                        au[q] = __fmaf_rn(scu, pu0 + pu1, au[q]);
                                    }
                                }
                            }
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float gq = warp_sum(ag[q]);
                                const float uq = warp_sum(au[q]);
                                if (wpr == 1) {
                                    if (lane == q && q < nq) p.hbuf[(size_t)pairs[q0 + q] * HS + j] = cz_silu(gq) * uq;
                                } else if (lane == 0) {
                                    s.red[((rr * wpr + sub) * 4 + q) * 2 + 0] = gq;
                                    s.red[((rr * wpr + sub) * 4 + q) * 2 + 1] = uq;
                                }
                            }
                        }
                        if (wpr > 1) {
                            // combine the row's partial sums in a fixed order (sub 0..wpr-1)
                            asm volatile("bar.sync 2, %0;" ::"n"(NCW * 32) : "memory");
                            const int k = tid;  // one consumer thread per (row, token)
                            if (k < n * nq) {
                                const int rr = k / nq, q = k % nq;
                                float gq = 0.f, uq = 0.f;
                                for (int sb = 0; sb < wpr; ++sb) {
                                    gq += s.red[((rr * wpr + sb) * 4 + q) * 2 + 0];
                                    uq += s.red[((rr * wpr + sb) * 4 + q) * 2 + 1];
                                }
                                p.hbuf[(size_t)pairs[q0 + q] * HS + st.r0 + rr] = cz_silu(gq) * uq;
                            }
                            asm volatile("bar.sync 2, %0;" ::"n"(NCW * 32) : "memory");
                        }
                    }
                } else {
                    // down rows st.r0 .. st.r0+n (absolute) of group u; h from shared memory
                    const int inter = gwt.inter;
                    const int nbI = cz_nblk(inter);
                    const int nchI = inter >> 4;
                    const float* hs = reinterpret_cast<const float*>(s.xh);
                    const float* dtab = s.sB_ok ? s.sB + u * nbb * nbIr : nullptr;
#pragma unroll
                    for (int k = 0; k < MAXBK; ++k) {
                        const int o = b_lo + warp + NCW * k;
                        if (o < b_hi && o >= st.r0 && o < st.r0 + st.n) {
                            const uint8_t* wr = stage + (size_t)(o - st.r0) * inter;
                            const float* sr = dtab ? dtab + ((o >> 7) - bb0) * nbI : gwt.ds + (size_t)(o >> 7) * nbI;
                            for (int q0 = 0; q0 < np; q0 += 4) {
                                const int nq = min(4, np - q0);
                                int pr[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q) pr[q] = pairs[q0 + min(q, nq - 1)];
                                float a4[4] = {0.f, 0.f, 0.f, 0.f};
                                for (int ch = lane; ch < nchI; ch += 32) {
                                    float f[16];
                                    decode16(*reinterpret_cast<const uint4*>(wr + ch * 16), f);
                                    const float sc = sr[ch >> 3];
#pragma unroll
                                    for (int q = 0; q < 4; ++q) {
                                        if (q < nq) {
                                            const float4* hp =
                                                reinterpret_cast<const float4*>(hs + (size_t)pr[q] * HS + ch * 16);
                                            float d0 = 0.f, d1 = 0.f;
#pragma unroll
                                            for (int v4 = 0; v4 < 4; ++v4) {
                                                const float4 hv = hp[v4];
                                                d0 = __fmaf_rn(hv.x, f[4 * v4 + 0], d0);
                                                d1 = __fmaf_rn(hv.y, f[4 * v4 + 1], d1);
                                                d0 = __fmaf_rn(hv.z, f[4 * v4 + 2], d0);
                                                d1 = __fmaf_rn(hv.w, f[4 * v4 + 3], d1);
                                            }
                                            a4[q] = __fmaf_rn(sc, d0 + d1, a4[q]);
                                        }
                                    }
                                }
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const float tot = warp_sum(a4[q]);
                                    if (q < nq) {
                                        const int prq = pairs[q0 + q];
                                        const int t = prq < T * K ? prq / K : prq - T * K;
                                        if (lane == t) bacc[k] = __fadd_rn(bacc[k], __fmul_rn(s.pg[prq], tot));
                                    }
                                }
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.empty[slot]);
                ++si;
            }
            if (!signalled) signal_phase_a();
            if (!s.abort && lane < T) {
#pragma unroll
                for (int k = 0; k < MAXBK; ++k) {
                    const int o = b_lo + warp + NCW * k;
                    if (o < b_hi) {
                        float v = bacc[k];
                        if (p.residual) v = __fadd_rn(p.residual[(size_t)lane * H + o], v);
                        p.out[(size_t)lane * H + o] = v;
                    }
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
    if ((H + num_sms - 1) / num_sms > NCW * MAXBK) return 0;
    const int max_rows = (E + (SI ? 1 : 0) + num_sms - 1) / num_sms;  // router rows staged per CTA
    // staged router rows + the rms weight vector (stack mode) must fit the ring
    if ((size_t)(max_rows + 1) * H * 4 > (size_t)RING_BYTES || 2 * H > STAGE_BYTES) return 0;
    if (I > STAGE_BYTES || SI > STAGE_BYTES) return 0;
    const int HS = I > SI ? I : SI;
    const int tx = XH_BYTES / (H * (x_bf16 ? 2 : 4));
    const int th = XH_BYTES / ((K + (SI ? 1 : 0)) * HS * 4);
    int t = tx < th ? tx : th;
    if (t > MAXT) t = MAXT;
    return t > 0 ? t : 0;
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
