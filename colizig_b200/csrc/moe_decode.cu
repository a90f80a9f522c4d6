// Decode-regime MoE layer (1..32 tokens) as ONE persistent cooperative kernel.
//
// Reference path (src/qwen38/moe.zig): route (435-463) -> per expert gate/up
// (fp8.zig:165-257, S small) -> silu(g)*u (activation.zig:8-20) -> down ->
// out += gate * eo, plus the always-on shared expert (467-479).
//
// Phases inside the launch (grid = one CTA per SM, 8 consumer warps + 1
// producer warp per CTA):
//   R  router logits.  CTA c owns router rows [c*E/G, (c+1)*E/G); the rows and
//      the token block are staged into shared memory with bulk (TMA) copies and
//      every logit is formed in the reference's exact f32 order (dotF32,
//      matmul.zig:60-82: 32 FMA chains = one per lane, lane-ordered combine).
//      The shared expert's gate x.sh_gate is one more row.  A grid-wide arrive
//      counter closes the phase.
//   K  top-k.  Every CTA redundantly computes softmax/top-k for all tokens
//      (identical, deterministic), groups the (token, slot) pairs by expert
//      (ascending id; the shared expert last) and derives the work split.
//   A  gate/up.  The flattened list of (group, row) pairs is split evenly over
//      CTAs.  The producer warp streams gate+up weight rows through a ring of
//      shared-memory stages with bulk copies; consumer warps decode E4M3
//      in registers, multiply by the per-128-block scale once per 16-column
//      chunk, reduce with warp shuffles and write h = silu(g)*u (f32) to HBM.
//   B  down + combine.  CTA c owns output rows [c*H/G, (c+1)*H/G) for every
//      group.  The producer starts streaming these down-weight rows while phase
//      A is still running (weights do not depend on h); consumers wait only for
//      the per-group h-ready counters.  Each (token, row) accumulates
//      gate * dot(h, w) in ascending expert order in registers — no atomics, a
//      fixed order, deterministic — and is written once.
//
// Every wait is bounded; a CTA that gives up sets a bit in the device error
// word, stops early (draining its in-flight copies) and the host returns -7.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cz_common.cuh"
#include "cz_internal.h"

namespace cz {

constexpr int NCW = 8;                      // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;    // + 1 producer warp
constexpr int STAGE_BYTES = 32 * 1024;
constexpr int NSTAGES = 6;
constexpr int RING_BYTES = STAGE_BYTES * NSTAGES;
constexpr int MAXT = kDecodeMaxTokens;      // 32: one lane per token in phase B
constexpr int MAXK = kMaxTopk;              // 16
constexpr int MAXE = kMaxExperts;           // 512
constexpr int MAXG = MAXE + 1;              // routed experts + shared
constexpr int MAXP = MAXT * (MAXK + 1);     // pairs incl. shared-expert pairs
constexpr int MAXBK = 8;                    // phase-B rows per warp (rows per CTA <= 64)
constexpr int MAXM = MAXE / 32;             // router values per lane

struct __align__(128) DecodeSmem {
    uint8_t ring[RING_BYTES];
    uint64_t full[NSTAGES];
    uint64_t empty[NSTAGES];
    uint64_t rbar;
    int abort;
    int U;
    int P;
    int seq;
    float rsc[MAXT];
    int pe[MAXP];
    float pg[MAXP];
    int cnt[MAXG + 1];
    int goff[MAXG + 1];
    int g_expert[MAXG];
    int g_pair0[MAXG];
    int g_npairs[MAXG];
    int g_rowA[MAXG + 1];
    int gidx[MAXG + 1];
    int sorted_pairs[MAXP];
};

static_assert(sizeof(DecodeSmem) <= 227 * 1024, "decode smem too large");

// ---- sync-word layout ------------------------------------------------------
// sync[0] = launch sequence number, sync[1] = error word, then two regions of
// kSyncRegionWords words: [0] router arrive count, [1] done count, [2..] per-group
// h-ready row counters.  A launch uses region seq&1 and zeroes the other one.
__device__ __forceinline__ uint32_t* region(uint32_t* sync, int par) {
    return sync + 2 + par * kSyncRegionWords;
}

struct Stage {
    int phase;  // 0 = A (gate/up), 1 = B (down)
    int u;      // group
    int r0;     // A: first row within the group; B: first absolute output row
    int n;      // rows
};

// Deterministic stage schedule shared by the producer and the consumers.
struct StageIter {
    int phase, u, a, a_hi, b_lo, b_hi, brow, U, RA;
    const int* rowA;
    const int* g_expert;
    int E, I, SI;

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
                int n = RA;
                n = min(n, rowA[u + 1] - a);
                n = min(n, a_hi - a);
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
        const int inter = inter_of(u);
        const int rb = max(1, STAGE_BYTES / inter);
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

__device__ __forceinline__ void group_ptrs(const DecodeParams& p, int e, const uint8_t*& gw, const uint8_t*& uw,
                                           const uint8_t*& dw, const float*& gs, const float*& us,
                                           const float*& ds, int& inter) {
    if (e == p.E) {
        inter = p.SI;
        gw = p.sh_gate_w;
        uw = p.sh_up_w;
        dw = p.sh_down_w;
        gs = p.sh_gate_s;
        us = p.sh_up_s;
        ds = p.sh_down_s;
    } else {
        inter = p.I;
        const size_t wsz = (size_t)p.I * p.H;
        gw = p.gate_w + (size_t)e * wsz;
        uw = p.up_w + (size_t)e * wsz;
        dw = p.down_w + (size_t)e * wsz;
        const size_t ssz = (size_t)cz_nblk(p.I) * cz_nblk(p.H);
        gs = p.gate_s + (size_t)e * ssz;
        us = p.up_s + (size_t)e * ssz;
        ds = p.down_s + (size_t)e * ssz;
    }
}

// Token value the MoE sees: the caller's x, or rms(h) in stack mode
// (rmsnorm.zig:32-40: out = v * r * w, two f32 multiplies).
__device__ __forceinline__ float xval_global(const DecodeParams& p, const float* rsc, int t, int i) {
    if (p.x_bf16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p.x)[(size_t)t * p.H + i]);
    const float v = reinterpret_cast<const float*>(p.x)[(size_t)t * p.H + i];
    if (p.rms_w) return __fmul_rn(__fmul_rn(v, rsc[t]), p.rms_w[i]);
    return v;
}

__device__ __forceinline__ float xval_smem(const DecodeParams& p, const uint8_t* xs, const float* rsc, int t,
                                           int i) {
    if (p.x_bf16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(xs)[(size_t)t * p.H + i]);
    const float v = reinterpret_cast<const float*>(xs)[(size_t)t * p.H + i];
    if (p.rms_w) return __fmul_rn(__fmul_rn(v, rsc[t]), p.rms_w[i]);
    return v;
}

__device__ void set_error(const DecodeParams& p, DecodeSmem& s, uint32_t bit) {
    atomicOr(p.sync + 1, bit);
    s.abort = 1;
}

// Exclusive scan of n (<= MAXG+1) ints by one warp; writes out[], returns total.
// With `flags`, scans (in[i] > 0 ? 1 : 0) instead of in[i].
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

// Top-k of one token (moe.zig:435-463) by one warp.  Lane l holds experts
// l, l+32, ...  Selection keys are the f32 bit patterns of exp(v - max) + 1
// (non-negative floats order like their bits; 0 marks "not a candidate":
// already chosen, NaN, or beyond E).  Each round takes the largest key and,
// among equal keys, the smallest expert id — the reference's strict-greater
// scan from e = 0 with bv = -1.  A round with no candidate yields id 0, as in
// the reference.
__device__ void route_token(const DecodeParams& p, DecodeSmem& s, int t, int lane) {
    const int E = p.E, K = p.K;
    const float* lg = p.logits + (size_t)t * (E + 1);
    float v[MAXM];
    float mx = __int_as_float(0xffc00000);  // NaN: fmaxf ignores it
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        const int e = lane + 32 * m;
        v[m] = (e < E) ? __ldcg(lg + e) : __int_as_float(0xffc00000);
        mx = fmaxf(mx, v[m]);
    }
    mx = warp_max(mx);
    uint32_t key[MAXM];
    double all = 0.0;
    float ex0 = 0.0f;
#pragma unroll
    for (int m = 0; m < MAXM; ++m) {
        const int e = lane + 32 * m;
        float ex = 0.0f;
        key[m] = 0u;
        if (e < E) {
            ex = cz_expf(__fsub_rn(v[m], mx));
            all += (double)ex;
            if (ex > -1.0f) key[m] = __float_as_uint(ex) + 1u;
        }
        if (m == 0) ex0 = ex;
    }
    all = warp_sum_d(all);
    const float ex_e0 = __shfl_sync(0xffffffffu, ex0, 0);
    double top = 0.0;
    float val[MAXK];
    int idx[MAXK];
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
        idx[z] = best;
        val[z] = bv;
        top = __dadd_rn(top, (double)bv);
    }
    const double den = p.norm_topk ? top : all;
    if (lane == 0) {
        for (int z = 0; z < K; ++z) {
            const float g = __double2float_rn(__ddiv_rn((double)val[z], den));
            s.pe[t * K + z] = idx[z];
            s.pg[t * K + z] = g;
            if (blockIdx.x == 0) {
                if (p.topk_idx) p.topk_idx[(size_t)t * K + z] = (uint32_t)idx[z];
                if (p.topk_gates) p.topk_gates[(size_t)t * K + z] = g;
            }
        }
        if (p.SI) {
            s.pe[p.T * K + t] = E;
            s.pg[p.T * K + t] = cz_sigmoid(__ldcg(lg + E));
        }
    }
}

__global__ void __launch_bounds__(NTHREADS, 1) moe_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    DecodeSmem& s = *reinterpret_cast<DecodeSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int T = p.T, H = p.H, E = p.E, K = p.K;
    const int Er = E + (p.SI ? 1 : 0);

    const uint32_t seq = ld_relaxed_gpu(p.sync);
    uint32_t* reg = region(p.sync, seq & 1);
    if (c == 0) {
        uint32_t* other = region(p.sync, (seq & 1) ^ 1);
        for (int i = tid; i < kSyncRegionWords; i += NTHREADS) other[i] = 0u;
    }
    if (tid == 0) {
        for (int i = 0; i < NSTAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], NCW);
        }
        mbar_init(&s.rbar, 1);
        s.abort = 0;
        fence_mbarrier_init();
    }
    __syncthreads();

    // ---------------- phase R: router logits ----------------
    const int row_lo = (int)((long long)c * Er / G), row_hi = (int)((long long)(c + 1) * Er / G);
    const int nrows = row_hi - row_lo;
    const size_t xelt = p.x_bf16 ? 2 : 4;
    const size_t xbytes = (size_t)T * H * xelt;
    const size_t rbytes = (size_t)nrows * H * 4;
    const bool xfits = xbytes + rbytes <= (size_t)RING_BYTES;
    uint8_t* xs = s.ring;
    float* rows = reinterpret_cast<float*>(s.ring + (xfits ? xbytes : 0));
    const bool need_x_smem = (nrows > 0 || p.rms_w != nullptr);
    if (tid == 0) {
        uint32_t bytes = (uint32_t)rbytes + ((need_x_smem && xfits) ? (uint32_t)xbytes : 0u);
        mbar_arrive_expect_tx(&s.rbar, bytes);
        if (need_x_smem && xfits) bulk_g2s(xs, p.x, (uint32_t)xbytes, &s.rbar);
        for (int r = 0; r < nrows; ++r) {
            const int e = row_lo + r;
            const float* src = (e < E) ? p.router + (size_t)e * H : p.sh_gate;
            bulk_g2s(rows + (size_t)r * H, src, (uint32_t)H * 4u, &s.rbar);
        }
    }
    if (!mbar_wait_bounded(&s.rbar, 0, &s.abort)) {
        if (lane == 0) set_error(p, s, CZ_DERR_FULL_WAIT);
    }
    __syncthreads();
    const bool xs_ok = need_x_smem && xfits;

    if (p.rms_w) {
        // rms scale per token (every CTA, redundantly): f64 sum of squares, mean
        // rounded to f32, r = 1/sqrt(mean + eps) in f32.
        for (int t = warp; t < T; t += NCW + 1) {
            double ss = 0.0;
            for (int i = lane; i < H; i += 32) {
                const float v = xs_ok ? reinterpret_cast<const float*>(xs)[(size_t)t * H + i]
                                      : reinterpret_cast<const float*>(p.x)[(size_t)t * H + i];
                ss = __fma_rn((double)v, (double)v, ss);
            }
            ss = warp_sum_d(ss);
            if (lane == 0) {
                const float mean = __double2float_rn(__ddiv_rn(ss, (double)H));
                s.rsc[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            }
        }
        __syncthreads();
    }

    // Normalised f32 copy of the tokens for phase A (CTA c writes its slice).
    if (p.xf) {
        const size_t TH = (size_t)T * H;
        const size_t lo = (size_t)c * TH / G, hi = (size_t)(c + 1) * TH / G;
        for (size_t k = lo + tid; k < hi; k += NTHREADS) {
            const int t = (int)(k / H), i = (int)(k % H);
            p.xf[k] = xval_global(p, s.rsc, t, i);
        }
    }

    {
        const int ntg = (T + 3) / 4;
        const int nitems = nrows * ntg;
        for (int it = warp; it < nitems; it += NCW + 1) {
            const int r = it / ntg, t0 = (it % ntg) * 4;
            const int nt = min(4, T - t0);
            const float* wrow = rows + (size_t)r * H;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            int i = 0;
            for (; i + 32 <= H; i += 32) {
                const float wv = wrow[i + lane];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (q < nt) {
                        const float xv = xs_ok ? xval_smem(p, xs, s.rsc, t0 + q, i + lane)
                                               : xval_global(p, s.rsc, t0 + q, i + lane);
                        acc[q] = __fmaf_rn(xv, wv, acc[q]);
                    }
                }
            }
            for (; i + 8 <= H; i += 8) {
                if (lane < 8) {
                    const float wv = wrow[i + lane];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (q < nt) {
                            const float xv = xs_ok ? xval_smem(p, xs, s.rsc, t0 + q, i + lane)
                                                   : xval_global(p, s.rsc, t0 + q, i + lane);
                            acc[q] = __fmaf_rn(xv, wv, acc[q]);
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                // total[l] = (((0 + acc0[l]) + acc1[l]) + acc2[l]) + acc3[l], chain k = lanes 8k..8k+7
                const float a = acc[q];
                const float a8 = __shfl_down_sync(0xffffffffu, a, 8);
                const float a16 = __shfl_down_sync(0xffffffffu, a, 16);
                const float a24 = __shfl_down_sync(0xffffffffu, a, 24);
                const float tl = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, a), a8), a16), a24);
                float sum = __shfl_sync(0xffffffffu, tl, 0);
#pragma unroll
                for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, tl, l));
                for (int ii = i; ii < H && q < nt; ++ii) {
                    const float xv = xs_ok ? xval_smem(p, xs, s.rsc, t0 + q, ii) : xval_global(p, s.rsc, t0 + q, ii);
                    sum = __fmaf_rn(xv, wrow[ii], sum);
                }
                if (lane == 0 && q < nt) p.logits[(size_t)(t0 + q) * (E + 1) + row_lo + r] = sum;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        red_release_add_gpu(&reg[0], 1u);
        if (!wait_geq_bounded(&reg[0], (uint32_t)G, p.sync + 1)) set_error(p, s, CZ_DERR_ROUTER_BARRIER);
    }
    __syncthreads();

    // ---------------- phase K: top-k + grouping (every CTA) ----------------
    if (s.abort) goto finish;  // uniform: s.abort was settled before the barrier above
    for (int t = warp; t < T; t += NCW + 1) route_token(p, s, t, lane);
    {
        const int P = T * K + (p.SI ? T : 0);
        for (int i = tid; i <= Er; i += NTHREADS) s.cnt[i] = 0;
        __syncthreads();
        for (int i = tid; i < P; i += NTHREADS) atomicAdd(&s.cnt[s.pe[i]], 1);
        __syncthreads();
        if (warp == 0) {
            warp_exclusive_scan(s.cnt, s.goff, Er, lane, false);
        } else if (warp == 1) {
            // group index of every expert with a non-zero count (ascending id)
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
        // routed groups have p.I rows each; the shared expert (id E) is last
        for (int u = tid; u <= U; u += NTHREADS) s.g_rowA[u] = u * p.I;
        __syncthreads();
        if (tid == 0 && U > 0 && s.g_expert[U - 1] == E) s.g_rowA[U] = (U - 1) * p.I + p.SI;
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
    const int HS = max(p.I, p.SI);
    const float* xf = p.xf ? p.xf : reinterpret_cast<const float*>(p.x);
    uint32_t* ready = reg + 2;

    if (warp == NCW) {
        // ---- producer ----
        if (lane == 0 && !s.abort) {
            fence_proxy_async_smem();
            StageIter itr;
            itr.init(s, a_lo, a_hi, b_lo, b_hi, RA, E, p.I, p.SI);
            Stage st;
            int si = 0;
            while (itr.next(st)) {
                const int slot = si % NSTAGES, round = si / NSTAGES;
                if (round > 0 && !mbar_wait_bounded(&s.empty[slot], (round - 1) & 1, &s.abort)) {
                    if (!s.abort) set_error(p, s, CZ_DERR_EMPTY_WAIT);
                    break;
                }
                const uint8_t *gw, *uw, *dw;
                const float *gs, *us, *ds;
                int inter;
                group_ptrs(p, s.g_expert[st.u], gw, uw, dw, gs, us, ds, inter);
                uint8_t* dst = s.ring + (size_t)slot * STAGE_BYTES;
                if (st.phase == 0) {
                    const uint32_t bytes = (uint32_t)st.n * H;
                    mbar_arrive_expect_tx(&s.full[slot], 2 * bytes);
                    bulk_g2s(dst, gw + (size_t)st.r0 * H, bytes, &s.full[slot]);
                    bulk_g2s(dst + bytes, uw + (size_t)st.r0 * H, bytes, &s.full[slot]);
                } else {
                    const uint32_t bytes = (uint32_t)st.n * inter;
                    mbar_arrive_expect_tx(&s.full[slot], bytes);
                    bulk_g2s(dst, dw + (size_t)st.r0 * inter, bytes, &s.full[slot]);
                }
                ++si;
            }
            // drain: no copy may land after this CTA exits
            for (int k = max(0, si - NSTAGES); k < si; ++k) {
                const int slot = k % NSTAGES;
                bool ok = false;
                for (uint32_t it2 = 0; it2 < CZ_SPIN_LIMIT && !ok; ++it2) {
                    ok = mbar_try_wait(&s.full[slot], (k / NSTAGES) & 1);
                    if (!ok) __nanosleep(64);
                }
                if (!ok) atomicOr(p.sync + 1, CZ_DERR_DRAIN_WAIT);
            }
        }
        __syncwarp();
    } else {
        // ---- consumers ----
        float bacc[MAXBK];
#pragma unroll
        for (int k = 0; k < MAXBK; ++k) bacc[k] = 0.0f;
        StageIter itr;
        itr.init(s, a_lo, a_hi, b_lo, b_hi, RA, E, p.I, p.SI);
        Stage st;
        int si = 0;
        bool signalled = false;
        const int nbH = cz_nblk(H);
        auto signal_phase_a = [&]() {
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
            if (tid == 0) {
                __threadfence();
                for (int u = 0; u < U; ++u) {
                    const int lo = max(a_lo, s.g_rowA[u]), hi = min(a_hi, s.g_rowA[u + 1]);
                    if (hi > lo) red_release_add_gpu(&ready[u], (uint32_t)(hi - lo));
                }
            }
            signalled = true;
        };
        while (!s.abort && itr.next(st)) {
            if (st.phase == 1 && !signalled) signal_phase_a();
            const uint8_t *gw, *uw, *dw;
            const float *gs, *us, *ds;
            int inter;
            const int e = s.g_expert[st.u];
            group_ptrs(p, e, gw, uw, dw, gs, us, ds, inter);
            if (st.phase == 1) {
                bool ok = true;
                if (lane == 0) ok = wait_geq_bounded(&ready[st.u], (uint32_t)inter, p.sync + 1);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                __syncwarp();
                if (!ok) {
                    if (lane == 0) set_error(p, s, CZ_DERR_READY_WAIT);
                    break;
                }
            }
            const int slot = si % NSTAGES;
            const bool full_ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s.full[slot], (si / NSTAGES) & 1, &s.abort));
            if (!full_ok) {
                if (lane == 0 && !s.abort) set_error(p, s, CZ_DERR_FULL_WAIT);
                break;
            }
            const uint8_t* stage = s.ring + (size_t)slot * STAGE_BYTES;
            const int np = s.g_npairs[st.u];
            const int* pairs = s.sorted_pairs + s.g_pair0[st.u];
            if (st.phase == 0) {
                // gate/up rows st.r0 .. st.r0+n of group u
                const int nch = H >> 4;
                for (int r = warp; r < st.n; r += NCW) {
                    const int j = st.r0 + r;
                    const uint8_t* wg = stage + (size_t)r * H;
                    const uint8_t* wu = stage + (size_t)st.n * H + (size_t)r * H;
                    const float* sgr = gs + (size_t)(j >> 7) * nbH;
                    const float* sur = us + (size_t)(j >> 7) * nbH;
                    for (int q0 = 0; q0 < np; q0 += 4) {
                        const int nq = min(4, np - q0);
                        int tok[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int pr = pairs[q0 + min(q, nq - 1)];
                            tok[q] = pr < T * K ? pr / K : pr - T * K;
                        }
                        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
                        for (int ch = lane; ch < nch; ch += 32) {
                            float fg[16], fu[16];
                            decode16(*reinterpret_cast<const uint4*>(wg + ch * 16), fg);
                            decode16(*reinterpret_cast<const uint4*>(wu + ch * 16), fu);
                            const float scg = __ldg(sgr + (ch >> 3)), scu = __ldg(sur + (ch >> 3));
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                if (q < nq) {
                                    const float4* xp =
                                        reinterpret_cast<const float4*>(xf + (size_t)tok[q] * H + ch * 16);
                                    float pg0 = 0.f, pg1 = 0.f, pu0 = 0.f, pu1 = 0.f;
#pragma unroll
                                    for (int v4 = 0; v4 < 4; ++v4) {
                                        const float4 xv = __ldcg(xp + v4);
                                        pg0 = __fmaf_rn(xv.x, fg[4 * v4 + 0], pg0);
                                        pg1 = __fmaf_rn(xv.y, fg[4 * v4 + 1], pg1);
                                        pg0 = __fmaf_rn(xv.z, fg[4 * v4 + 2], pg0);
                                        pg1 = __fmaf_rn(xv.w, fg[4 * v4 + 3], pg1);
                                        pu0 = __fmaf_rn(xv.x, fu[4 * v4 + 0], pu0);
                                        pu1 = __fmaf_rn(xv.y, fu[4 * v4 + 1], pu1);
                                        pu0 = __fmaf_rn(xv.z, fu[4 * v4 + 2], pu0);
                                        pu1 = __fmaf_rn(xv.w, fu[4 * v4 + 3], pu1);
                                    }
                                    ag[q] = __fmaf_rn(scg, pg0 + pg1, ag[q]);
                                    au[q] = __fmaf_rn(scu, pu0 + pu1, au[q]);
                                }
                            }
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float g = warp_sum(ag[q]);
                            const float uu = warp_sum(au[q]);
                            if (lane == q && q < nq) {
                                const int pr = pairs[q0 + q];
                                p.hbuf[(size_t)pr * HS + j] = cz_silu(g) * uu;
                            }
                        }
                    }
                }
            } else {
                // down rows st.r0 .. st.r0+n (absolute) of group u
                const int nbI = cz_nblk(inter);
                const int nch = inter >> 4;
#pragma unroll
                for (int k = 0; k < MAXBK; ++k) {
                    const int o = b_lo + warp + NCW * k;
                    if (o >= b_hi) break;
                    if (o < st.r0 || o >= st.r0 + st.n) continue;
                    const uint8_t* wr = stage + (size_t)(o - st.r0) * inter;
                    const float* sr = ds + (size_t)(o >> 7) * nbI;
                    for (int q0 = 0; q0 < np; q0 += 4) {
                        const int nq = min(4, np - q0);
                        int pr[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) pr[q] = pairs[q0 + min(q, nq - 1)];
                        float a4[4] = {0.f, 0.f, 0.f, 0.f};
                        for (int ch = lane; ch < nch; ch += 32) {
                            float f[16];
                            decode16(*reinterpret_cast<const uint4*>(wr + ch * 16), f);
                            const float sc = __ldg(sr + (ch >> 3));
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                if (q < nq) {
                                    const float4* hp =
                                        reinterpret_cast<const float4*>(p.hbuf + (size_t)pr[q] * HS + ch * 16);
                                    float d0 = 0.f, d1 = 0.f;
#pragma unroll
                                    for (int v4 = 0; v4 < 4; ++v4) {
                                        const float4 hv = __ldcg(hp + v4);
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

int decode_launch(const DecodeParams& prm, int num_sms, cudaStream_t stream) {
    if (prm.T < 1 || prm.T > MAXT || prm.K < 1 || prm.K > MAXK || prm.E < prm.K || prm.E > MAXE) return CZ_ESHAPE;
    if (prm.H % 16 || prm.I % 16 || prm.SI % 16) return CZ_ESHAPE;
    if ((prm.H + num_sms - 1) / num_sms > NCW * MAXBK) return CZ_ESHAPE;
    const int max_rows = (prm.E + 1 + num_sms - 1) / num_sms;  // router rows staged per CTA
    if ((size_t)max_rows * prm.H * 4 > (size_t)RING_BYTES || 2 * prm.H > STAGE_BYTES) return CZ_ESHAPE;
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
