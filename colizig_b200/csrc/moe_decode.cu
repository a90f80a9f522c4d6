// Decode-regime MoE layer (up to 4 tokens per launch) as ONE persistent
// cooperative kernel.
//
// Reference path (src/qwen38/moe.zig): route (435-463) -> per expert gate/up
// (fp8.zig:165-257) -> silu(g)*u (activation.zig:8-20) -> down -> out += gate*eo,
// plus the always-on shared expert (467-479).
//
// Grid = one CTA per SM: 8 consumer warps, 1 producer warp, 1 h warp.  The
// weights go HBM -> shared memory through a ring of bulk-copy (TMA) stages
// filled by one producer thread; no weight is read from global memory inside a
// compute loop.
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
//      holds experts [e_lo, e_hi) only; the other groups get no work here and
//      the GPUs' outputs are summed by one all-reduce after the launch.
//   C  gate/up.  Each group's intermediate rows are cut into chunks of 16; the
//      flattened chunk list is split evenly over the CTAs.  Per chunk the
//      producer streams gate rows [r0, r0+16) x 2048-column slabs of H and the
//      same for up; the consumer warps split the K blocks and reduce, and the
//      h warp writes hw = gate * silu(g) * u of every routed token to the
//      pair's h row in global scratch.  A grid-wide arrive counter closes the
//      phase (the producer keeps streaming meanwhile, see D).
//   D  down.  CTA c owns output rows [c*H/G, (c+1)*H/G).  While C still runs,
//      the producer streams those rows of every group's down matrix (with their
//      128 x 128 scales), packed several groups to a ring stage.  After the
//      counter, consumer warp j takes pairs j, j+8, ...: the pair's h row
//      (from L2) becomes f16 hi/lo terms, and f16 MMAs against the down rows
//      give one partial per (pair, row).  Out = residual + each token's pair
//      partials in ascending expert order: no second reduction over CTAs.
//      The weight copies carry an L2 evict-first hint: streamed once, they
//      should not push the kernel's code, the router rows or the scratch out
//      of L2.
//
// Arithmetic.  Gate/up: mma.sync m16n8k32 E4M3 x E4M3 -> f32, which forms and
// sums the exact products (checked on B200 to round like f32).  The weights
// enter as their stored bytes.  The token is split exactly into E4M3 terms: x
// (scaled by 2^s so that max|x| lies in [128, 256)) = t1 + t2 (+ t3), every
// term a column of the MMA; a bf16 token is exact in 2 terms, an f32 token is
// kept to 12 bits in 3.  Down: mma.sync m16n8k16 f16 x f16 -> f32 with the
// E4M3 weights converted exactly to f16 and h (scaled by a power of two per
// pair into the f16 range) as hi + lo f16 terms (22 bits).  Each 128-column
// block's sum is multiplied by its 128 x 128 scale in f32.  Every sum has a
// fixed order: deterministic, no float atomics.
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
constexpr int GU_BYTES = CR * KS;         // a gate/up stage: [K block][16 rows][128 B], 128-byte swizzled
constexpr int SC_BYTES = 1024;            // block scales carried with every stage (hidden <= 32768)
constexpr int SLOT_BYTES = 33 * 1024;     // >= GU_BYTES + SC_BYTES; also one pack of down rows
constexpr int NSLOT = 4;                  // ring slots at least (more when shared memory allows)
constexpr int MAXSLOT = 6;
constexpr int RING_BYTES = NSLOT * SLOT_BYTES;  // the smallest ring (also stages phase R)
constexpr int MAXT = kDecodeMaxTokens;    // 8
constexpr int DHW = 1024;                 // phase D: words of a warp's f16 h terms (intermediate <= 1024)
constexpr int DMR = 32;                   // phase D: output rows per CTA at most
constexpr int MAXK = kMaxTopk;            // 16
constexpr int MAXE = kMaxExperts;         // 512
// (token, slot) pairs of one launch incl. shared-expert pairs: at most 68 (four
// tokens at the largest top-k; eight at top-8), decode_max_tokens keeps T * (K + 1)
// below; the grouping warp sorts up to 96 (3 positions a lane)
constexpr int MAXSORT = 4 * (MAXK + 1);
constexpr int MAXP = MAXSORT;
static_assert(MAXP <= 96, "the grouping warp's 3 positions a lane");
constexpr int MAXG = MAXP;                // groups <= pairs
constexpr int SMEM_LIMIT = 227 * 1024;

static_assert(GU_BYTES + SC_BYTES <= SLOT_BYTES, "slot");
// routing scratch in the ring: logits + exps [T][LS] f32, two candidate buffers
// [T][ceil(E/32)][K] and the winners [T][MAXK] (8-byte entries)
static_assert(2 * ((kDecodeMaxTokens * ((kMaxExperts + 4) & ~3) * 4 + 15) & ~15) +
                      2 * kDecodeMaxTokens * ((kMaxExperts + 31) / 32) * kMaxTopk * 8 + kDecodeMaxTokens * kMaxTopk * 8 <=
                  NSLOT * SLOT_BYTES,
              "routing scratch");
static_assert(SLOT_BYTES % 1024 == 0, "TMA destinations stay 1024-aligned");

// Small shared state (after the large regions).
struct __align__(16) DecodeMisc {
    uint64_t full[MAXSLOT];
    uint64_t empty[MAXSLOT];
    uint64_t rbar;
    int abort;
    int U, P, NC;
    uint32_t xmax[MAXT];  // max |x_t| (f32 bits)
    int xexp[MAXT];       // s per token (terms hold x_t * 2^s)
    float xscale[MAXT];   // 2^-s per token
    int fastgroup;        // the groups were formed by the top-k warp (one token, distinct experts)
    int dots_done;        // one token: warps of this CTA that have published their router logits
    int exact[MAXT];      // token t was routed by the exact exp-keyed selection (its gates are set)
    float pd[MAXP];       // logit - max of the winner of pair p (the gates are formed from it later)
    float shlog[MAXT];    // the shared expert's gate logit per token
    int geo_drows, geo_nrb, geo_rbytes, geo_per;  // phase D geometry of this CTA (output rows, packs)
    int pe[MAXP];         // expert of pair p = t*K + z (shared: p = T*K + t -> E)
    float pg[MAXP];       // gate of pair p
    int order[MAXP];      // pairs sorted by (expert, pair)
    int g_expert[MAXG];
    int g_pair0[MAXG];
    int g_npairs[MAXG];
    int g_chunk0[MAXG + 1];
    int g_pack[MAXG];     // phase D: the pack (ring stage) holding the group's down rows (-1: not held here)
    int g_poff[MAXG];     // byte offset of the group's rows in its pack
    int npk;              // packs of this CTA
    int rtok[MAXP];       // token of sorted pair r when its group is held here, else -1
};

// Shared-memory map of one launch: [ring][x terms][red][dsum][misc].
// red holds the consumer warps' partial gate/up sums of two chunks in flight,
// [chunk parity][warp][gate/up][16 rows][rc columns]; phase D then keeps each
// warp's f16 h terms (DHW words a warp) in red, or, with hslot, in the ring slot
// after the last pack (free: its last stage was a consumed gate/up slab), which
// lets red shrink to 8 columns and one more ring slot fit.  The host picks hslot
// when every group fits 8 MMA columns and every CTA's packs leave a slot free.
struct Carve {
    int JX, CS;  // E4M3 terms per token; byte stride of one term column
    int ns;      // ring slots
    int rc;      // columns of a warp's partial sums in red (16, or 8 with hslot)
    uint32_t xterm, red, dsum, misc, total;
};

__host__ __device__ inline Carve carve(int T, int H, int x_bf16, int hslot) {
    Carve c;
    c.JX = x_bf16 ? 2 : 3;
    c.CS = ((H + 127) & ~127) + 64;  // column stride = 64 mod 128: lanes of 2 columns hit disjoint banks
    c.rc = hslot ? 8 : 16;
    const uint32_t red_bytes = 2u * NCW * 2 * 16 * (uint32_t)c.rc * 4;  // 16 KB, or 32 KB = NCW * DHW words
    const uint32_t dsum_bytes = (uint32_t)T * (MAXK + 1) * DMR * 4;     // [sorted pair][output row]
    // the rest of the map decides how many slots fit
    const uint32_t rest = (((uint32_t)(T * c.JX * c.CS) + 127u) & ~127u) + red_bytes + dsum_bytes +
                          (((uint32_t)sizeof(DecodeMisc) + 127u) & ~127u);
    const int fit = ((int)SMEM_LIMIT - 1024 - (int)rest) / SLOT_BYTES;
    c.ns = fit < NSLOT ? NSLOT : (fit > MAXSLOT ? MAXSLOT : fit);
    uint32_t off = (uint32_t)c.ns * SLOT_BYTES;
    c.xterm = off;
    off += ((uint32_t)(T * c.JX * c.CS) + 127u) & ~127u;
    c.red = off;
    off += red_bytes;
    c.dsum = off;
    off += dsum_bytes;
    c.misc = off;
    off += ((uint32_t)sizeof(DecodeMisc) + 127u) & ~127u;
    c.total = off;
    return c;
}

// ---- sync words ------------------------------------------------------------
// sync[0] = launch sequence number, sync[1] = error word, then two regions of
// kSyncRegionWords: [0] router arrivals, [1] CTAs done, [2] h rows
// written.  A launch uses region seq&1 and zeroes the other one, so a launch
// that stopped early leaves nothing behind.
__device__ __forceinline__ uint32_t* region(uint32_t* sync, int par) { return sync + 2 + par * kSyncRegionWords; }

struct GroupW {
    const uint8_t *gw, *uw;
    const float *gs, *us, *ds;
    int inter;
    int gu_row0;                  // first row of this expert in its gate/up tensor maps
    const CUtensorMap *gmap, *umap;
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
        g.gu_row0 = 0;
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
        g.gu_row0 = e * p.I;
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

// Two E4M3 bytes (low byte = element 0) -> f16x2, exactly.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v) {
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
    return h;
}

__device__ __forceinline__ void mma_f16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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
// tail).  wrow / xs are shared memory.  Returns the logit in every lane.
template <bool BF16>
__device__ __forceinline__ float router_dot(const float* __restrict__ wrow, const uint8_t* __restrict__ xs, int H,
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
    float tv[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) tv[l] = __shfl_sync(0xffffffffu, tl, l);  // independent: issued together
    float sum = tv[0];
#pragma unroll
    for (int l = 1; l < 8; ++l) sum = __fadd_rn(sum, tv[l]);
#pragma unroll 1
    for (; i < H; ++i) sum = __fmaf_rn(xv(i), wrow[i], sum);
    return sum;
}

// Start of part c of n items split over G parts: floor(c * n / G).  32-bit: c <= G <= 160 and
// n <= 5120 for every caller (hidden, router rows, chunks; decode_max_tokens bounds them).
__device__ __forceinline__ int split_at(int c, int n, int G) {
    return (int)(((uint32_t)c * (uint32_t)n) / (uint32_t)G);
}

__device__ __forceinline__ int pair_token(int pr, int T, int K) { return pr < T * K ? pr / K : pr - T * K; }

// Bounded wait of all lanes on an mbarrier phase; warp-uniform result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, DecodeMisc& s) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, &s.abort));
}

// ---- routing (moe.zig:435-463) ----------------------------------------------
// The reference picks, K times, the unchosen expert with the largest
// exp(logit - max) by a strict-greater scan from expert 0 (ties to the lowest
// id).  That order is a total order on (key, id): a larger key first, among
// equal keys the smaller id, where key = f32 bits of exp(logit - max) + 1
// (non-negative floats order like their bits; 0 = not a candidate: NaN, or past
// the last expert).  The top K of a set under a total order are the union of
// the top K of its parts, so each warp ranks a part of 32 entries by counting
// the entries that beat each one, keeps its top K, and the survivors are ranked
// again until one part is left.  A selection round without a candidate (every
// remaining key 0) yields id 0 with expert 0's value, as the reference's scan
// does.

// Empty entries (key 0, ids from 0x80000000 up) rank after every expert.  Every
// entry of a part must differ from the others, so that the counted ranks are
// 0, 1, 2, ... and the top K slots are all written: past-the-end experts carry
// 0x80000000 + their index, merge padding 0xc0000000 + its position.
__device__ __forceinline__ unsigned long long empty_entry(uint32_t unique) {
    return (unsigned long long)unique;
}

__device__ __forceinline__ unsigned long long route_entry(uint32_t key, uint32_t id) {
    return ((unsigned long long)key << 32) | id;
}

// How many of the warp's 32 entries beat this lane's entry.
__device__ __forceinline__ int rank_in_warp(unsigned long long v) {
    const uint32_t key = (uint32_t)(v >> 32), id = (uint32_t)v;
    int r = 0;
#pragma unroll 8
    for (int m = 0; m < 32; ++m) {
        const unsigned long long w = __shfl_sync(0xffffffffu, v, m);
        const uint32_t km = (uint32_t)(w >> 32), im = (uint32_t)w;
        r += (km > key) || (km == key && im < id);
    }
    return r;
}

// Shared-memory scratch of the routing step (carved from the ring, which is
// free between the token term split and the first weight copy).
struct RouteScratch {
    float* lg;                // [T][LS] logits (+ the shared gate logit at column E)
    float* ex;                // [T][LS] exp(logit - max), kept for the all-expert sum
    unsigned long long* ca;   // [T][nch * K] candidates (two buffers for the merge rounds)
    unsigned long long* cb;
    unsigned long long* fin;  // [T][MAXK] the winners in selection order
};

// Largest non-NaN value of the warp (NaN when every lane holds NaN): the
// reference's @max fold over the logits (moe.zig:441), one instruction.
__device__ __forceinline__ float warp_max_f32(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// Order-preserving key of an f32 logit: a larger logit gives a larger key, -0
// and +0 the same key, NaN 0 (never ahead of a number).
__device__ __forceinline__ uint32_t logit_key(float v) {
    const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));  // -0 -> +0
    if (v != v) return 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_logit(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Exact selection for one token (moe.zig:435-463, the reference's own rules), by
// one warp: every exp(logit - max) is formed; K rounds take the largest value,
// among equal values the smallest id (a strict-greater scan from expert 0 with
// bv = -1); a round without a candidate (every remaining value NaN) yields id 0
// with expert 0's value.  Writes the token's ids and gates.  The fast path below
// falls back to it when the logit order might not be the exp order.
__device__ __noinline__ void route_exact(const float* __restrict__ lg, float* __restrict__ ex, int E, int K,
                                         int norm_topk, int t, DecodeMisc& s, uint32_t* topk_idx,
                                         float* topk_gates, bool write_out) {
    const int lane = threadIdx.x & 31;
    float mx = __int_as_float(0xffc00000);
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
    mx = warp_max_f32(mx);
    for (int e = lane; e < E; e += 32) ex[e] = cz_expf(__fsub_rn(lg[e], mx));
    __syncwarp();
    double top = 0.0;
    int my_e = 0;
    float my_v = 0.0f;
    unsigned long long chosen[(MAXE + 63) / 64] = {};
    for (int z = 0; z < K; ++z) {
        // largest value (then smallest id) among the unchosen, NaN never taken
        uint32_t bk = 0u;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            const float v = ex[e];
            const uint32_t k = (!(chosen[e >> 6] >> (e & 63) & 1ull) && v > -1.0f) ? __float_as_uint(v) + 1u : 0u;
            if (k > bk) {
                bk = k;
                bi = e;
            }
        }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        const int best = kmax == 0u ? 0 : (int)__reduce_min_sync(0xffffffffu, bk == kmax ? (uint32_t)bi : 0x7fffffffu);
        const float bv = kmax == 0u ? ex[0] : __uint_as_float(kmax - 1u);
        if (kmax) chosen[best >> 6] |= 1ull << (best & 63);
        if (lane == z) {
            my_e = best;
            my_v = bv;
        }
        top = __dadd_rn(top, (double)bv);
    }
    double den = top;
    if (!norm_topk) {
        double all = 0.0;
        if (lane == 0)
            for (int e = 0; e < E; ++e) all = __dadd_rn(all, (double)ex[e]);
        den = __shfl_sync(0xffffffffu, all, 0);
    }
    if (lane < K) {
        const float g = __double2float_rn(__ddiv_rn((double)my_v, den));
        s.pe[t * K + lane] = my_e;
        s.pg[t * K + lane] = g;
        if (write_out) {
            if (topk_idx) topk_idx[(size_t)t * K + lane] = (uint32_t)my_e;
            if (topk_gates) topk_gates[(size_t)t * K + lane] = g;
        }
    }
    if (lane == 0) s.exact[t] = 1;
    __syncwarp();
}

// Top-k ids of every token by the whole CTA (all threads call it).  The experts
// are ranked by their f32 logits, which is the reference's exp order (exp is
// monotone) except where two different logits give the same f32 exp; ties of
// equal logits go to the smaller id as in the reference.  Each warp ranks a part
// of 32 experts by counting the entries that beat each one and keeps its top K;
// the survivors are ranked again until one part is left (the top K of a set
// under a total order are the union of its parts' top K).  The winners are then
// checked: finite, their exps clear of underflow, and every two consecutive
// winners with different logits, and the last winner and the largest logit
// below it, at least 2^-22 apart after the subtraction of the max, so that
// their f32 exps differ.  A token that fails the check (or with norm_topk off)
// is routed again by route_exact.  Writes s.pe, s.pd (logit - max of each
// winner, for route_gates) and, from CTA 0, the top-k ids.  Token t's results
// are written by warp t % NWARPS; the caller synchronises before other warps
// read them.
__device__ __forceinline__ void route_all(const RouteScratch& rs, int T, int E, int K, int LS, int norm_topk,
                                          int has_shared, DecodeMisc& s, uint32_t* topk_idx, float* topk_gates,
                                          bool write_out) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nch = (E + 31) >> 5;
    const int stride = nch * K;  // entries per token in the candidate buffers
    // stage 1: (token, 32 experts) per warp, ids following the lanes
    for (int it = warp; it < T * nch; it += NWARPS) {
        const int t = it / nch, j = it - t * nch;
        const int e = 32 * j + lane;
        const uint32_t key = e < E ? logit_key(rs.lg[(size_t)t * LS + e]) : 0u;
        int r = 0;
#pragma unroll 4
        for (int m = 0; m < 32; ++m) {
            const uint32_t km = __shfl_sync(0xffffffffu, key, m);
            r += (km > key) | ((km == key) & (m < lane));
        }
        if (r < K) rs.ca[((size_t)t * nch + j) * K + r] = route_entry(key, e < E ? (uint32_t)e : 0x80000000u + (uint32_t)e);
    }
    __syncthreads();
    // merge rounds: parts of 32 survivors -> their top K, until one part is left
    unsigned long long* cur = rs.ca;
    unsigned long long* nxt = rs.cb;
    int n = stride;
    while (n > 32) {
        const int ng = (n + 31) >> 5;
        for (int it = warp; it < T * ng; it += NWARPS) {
            const int t = it / ng, gi = it - t * ng, k = 32 * gi + lane;
            const unsigned long long v = k < n ? cur[(size_t)t * stride + k] : empty_entry(0xc0000000u + (uint32_t)k);
            const int r = rank_in_warp(v);
            if (r < K) nxt[(size_t)t * stride + gi * K + r] = v;
        }
        __syncthreads();
        unsigned long long* tmp = cur;
        cur = nxt;
        nxt = tmp;
        n = ng * K;
    }
    // final part: warp t ranks token t's last <= 32 entries, checks the winners
    for (int t = warp; t < T; t += NWARPS) {
        const float* lt = rs.lg + (size_t)t * LS;
        const unsigned long long v = lane < n ? cur[(size_t)t * stride + lane] : empty_entry(0xc0000000u + lane);
        const int r = rank_in_warp(v);
        unsigned long long* fin = rs.fin + (size_t)t * MAXK;
        if (r < K) fin[r] = v;
        __syncwarp();
        const unsigned long long w = lane < K ? fin[lane] : 0ull;
        const uint32_t key = (uint32_t)(w >> 32);
        const int id = (int)(uint32_t)w;
        const float val = lane < K ? key_logit(key) : 0.0f;
        const float mx = __shfl_sync(0xffffffffu, val, 0);
        const float d = __fsub_rn(val, mx);
        const float vn = __shfl_down_sync(0xffffffffu, val, 1), dn = __shfl_down_sync(0xffffffffu, d, 1);
        const uint32_t klast = __shfl_sync(0xffffffffu, key, K - 1);
        // the largest key strictly below the last winner's (0: none, or NaN only)
        uint32_t wk = 0u;
        for (int e = lane; e < E; e += 32) {
            const uint32_t ke = logit_key(lt[e]);
            if (ke < klast && ke > wk) wk = ke;
        }
        wk = __reduce_max_sync(0xffffffffu, wk);
        bool ok = true;
        if (lane < K) {
            ok = key != 0u && fabsf(val) <= 3.0e38f;
            if (lane + 1 < K) ok = ok && (vn == val || __fsub_rn(d, dn) >= 0x1p-22f);
            if (lane + 1 == K) {
                ok = ok && d >= -80.0f;
                if (wk) ok = ok && __fsub_rn(d, __fsub_rn(key_logit(wk), mx)) >= 0x1p-22f;
            }
        }
        const bool fast = __all_sync(0xffffffffu, ok) && norm_topk;
        if (fast) {
            if (lane < K) {
                s.pe[t * K + lane] = id;
                s.pd[t * K + lane] = d;
                if (write_out && topk_idx) topk_idx[(size_t)t * K + lane] = (uint32_t)id;
            }
            if (lane == 0) s.exact[t] = 0;
        } else {
            route_exact(lt, rs.ex + (size_t)t * LS, E, K, norm_topk, t, s, topk_idx, topk_gates, write_out);
        }
        if (lane == 0 && has_shared) {
            s.pe[T * K + t] = E;
            s.shlog[t] = lt[E];
        }
    }
}

// The gates of the tokens routed by the fast path (route_all), by one warp:
// g_z = f32(f64(exp(d_z)) / top) with top the f64 sum of the winners' exps in
// selection order (moe.zig:447-462; the same exp as the reference's @exp,
// cz_expf), and the shared expert's sigmoid gate.  Off the critical path: only
// the h warp reads the gates, and it runs this itself before its first chunk.
__device__ __noinline__ void route_gates(int T, int K, int has_shared, DecodeMisc& s, float* topk_gates,
                                         bool write_out) {
    const int lane = threadIdx.x & 31;
    for (int t = 0; t < T; ++t) {
        if (!s.exact[t]) {
            const float ex = lane < K ? cz_expf(s.pd[t * K + lane]) : 0.0f;
            double top = 0.0;
#pragma unroll 1
            for (int z = 0; z < MAXK; ++z) {
                const float vz = __shfl_sync(0xffffffffu, ex, z);
                if (z < K) top = __dadd_rn(top, (double)vz);
            }
            if (lane < K) {
                const float g = __double2float_rn(__ddiv_rn((double)ex, top));
                s.pg[t * K + lane] = g;
                if (write_out && topk_gates) topk_gates[(size_t)t * K + lane] = g;
            }
        }
        if (lane == 0 && has_shared) s.pg[T * K + t] = cz_sigmoid(s.shlog[t]);
    }
    __syncwarp();
}

// One gate/up stage into ring slot `slot` (one thread): slab st/2 of chunk rows
// [r0, r0+16) of group weights gw, gate (st even) or up (st odd), column blocks
// [kb0, kb0 + nkbs) as [block][row][128 B] (128-byte swizzle), plus the row block's
// scales after the slab.
__device__ __forceinline__ void issue_gu_stage(const DecodeParams& p, DecodeMisc& s, uint8_t* ring, const GroupW& gw,
                                               int r0, int st, int slot, int nkbH, int nbpH, uint64_t pol) {
    uint8_t* dst = ring + (size_t)slot * SLOT_BYTES;
    float* sdst = reinterpret_cast<float*>(dst + GU_BYTES);
    const bool up = st & 1;
    const int kb0 = (st >> 1) * (KS / 128), nkbs = min(KS / 128, nkbH - kb0);
    const CUtensorMap* map = up ? gw.umap : gw.gmap;
    const float* ssrc = (up ? gw.us : gw.gs) + (size_t)(r0 >> 7) * nbpH;
    const uint32_t wb = (uint32_t)(CR * 128) * (uint32_t)(p.gu3d ? p.gu_kb : nkbs);
    mbar_arrive_expect_tx(&s.full[slot], wb + (uint32_t)(nbpH * 4));
    if (p.gu3d) {
        tma_box3_g2s(dst, map, 0, gw.gu_row0 + r0, kb0, &s.full[slot], pol);
    } else {
        for (int kb = 0; kb < nkbs; ++kb)
            tma_box_g2s(dst + (size_t)kb * CR * 128, map, (kb0 + kb) * 128, gw.gu_row0 + r0, &s.full[slot], pol);
    }
    bulk_g2s(sdst, ssrc, (uint32_t)nbpH * 4u, &s.full[slot]);
}

// Producer: wait until ring slot `slot` is free for its use number `round`
// (bounded); false = stop.
__device__ __forceinline__ bool slot_acquire(DecodeMisc& s, uint32_t* err, int slot, int round) {
    if (round == 0) return true;
    bool ok = false;
    for (uint32_t it = 0; it < CZ_SPIN_LIMIT && !ok && !s.abort; ++it) {
        ok = mbar_try_wait(&s.empty[slot], (round - 1) & 1);
        if (!ok && it > 64) __nanosleep(64);
    }
    if (!ok && !s.abort) set_error(err, s, CZ_DERR_EMPTY_WAIT);
    return ok;
}

// Producer, once the ring is full (stage NS is next): everything this CTA streams
// later is prefetched into L2, so that the HBM reads of the whole layer call are
// in flight from the start and a stage issued when its slot frees up finds its
// bytes in L2.  nst = this CTA's gate/up stages; the packs of down rows follow.
__device__ __forceinline__ void prefetch_rest(const DecodeParams& p, const DecodeMisc& s, int ch_lo, int ch_hi, int nks,
                                              int NS, int nst, int drows, int o_lo, int o_hi, bool packs) {
    const int H = p.H, E = p.E, SI = p.SI, Ir = p.I;
    int u = 0;
    for (int ch = ch_lo; ch < ch_hi; ++ch) {
        while (s.g_chunk0[u + 1] <= ch) ++u;
        if (2 * nks * (ch - ch_lo + 1) <= NS) continue;  // inside the first ring fill
        const GroupW gw = group_w(p, s.g_expert[u]);
        const size_t r0 = (size_t)(ch - s.g_chunk0[u]) * CR;
        prefetch_l2(gw.gw + r0 * H, (uint32_t)(CR * H));  // 16 whole rows, contiguous
        prefetch_l2(gw.uw + r0 * H, (uint32_t)(CR * H));
    }
    if (packs && drows > 0) {
        const int rb0 = o_lo >> 7, nrb = ((o_hi - 1) >> 7) - rb0 + 1;
        const int nkbH = cz_nblk(H);
        for (int v = 0; v < s.U; ++v) {
            if (s.g_pack[v] < 0 || nst + s.g_pack[v] < NS) continue;
            const int ev = s.g_expert[v];
            const bool sh = ev == E;
            const int iu = sh ? SI : Ir;
            prefetch_l2(sh ? p.sh_down_w + (size_t)o_lo * SI : p.down_w + ((size_t)(ev - p.e_lo) * H + o_lo) * Ir,
                        (uint32_t)drows * (uint32_t)iu);
            prefetch_l2(sh ? p.sh_down_s + (size_t)rb0 * cz_nbp(SI)
                           : p.down_s + ((size_t)(ev - p.e_lo) * nkbH + rb0) * cz_nbp(Ir),
                        (uint32_t)(nrb * cz_nbp(iu) * 4));
        }
    }
}

// One token (T = 1), by one warp and with no CTA barrier: route_all's selection,
// check and the one-token grouping in a compact form.  The warp polls the tagged
// router logits straight into registers (expert 32j + lane in key[j]), then takes
// K + 1 selection rounds: the largest key left, among equal keys the smallest id
// (the reference's strict-greater scan from expert 0); the round after the K-th
// only reads the largest key left, which the check compares with the last winner.
// The winners are distinct, so each is a group of its own; its place in ascending
// expert order comes from ballots of the taken flags.  Returns false when the
// check fails (the caller then routes through route_all / route_exact), when
// norm_topk is off, or when a logit never arrives (error word set).  Writes what
// route_all and the one-token grouping write: pe, pd, exact, shlog, the groups,
// U, P, NC, npk, fastgroup, and from CTA 0 the top-k ids.
template <int NJ>
__device__ __forceinline__ bool route_one(const DecodeParams& p, DecodeMisc& s, int ns, int E, int K, int SI,
                                          int Ir, uint32_t tag, uint32_t limit, uint32_t* err, bool write_out) {
    const int lane = threadIdx.x & 31;
    uint32_t key[NJ];  // logit bits while polling, then the order-preserving keys
    uint32_t pend = 0u;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        key[j] = 0u;
        if (32 * j + lane < E) pend |= 1u << j;
    }
    // the shared expert's gate logit (word E), by lane 0 (kept out of key[], which
    // is only ever indexed by constants and so stays in registers)
    bool psh = SI && lane == 0;
    uint32_t shb = 0u;
    for (uint32_t it = 0; it < limit; ++it) {
        // every pending word's load first, then the tag checks: the loads overlap
        unsigned long long w[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) w[j] = (pend & (1u << j)) ? ld_relaxed_u64(p.logits + 32 * j + lane) : 0ull;
        const unsigned long long ws = psh ? ld_relaxed_u64(p.logits + E) : 0ull;
#pragma unroll
        for (int j = 0; j < NJ; ++j)
            if ((pend & (1u << j)) && (uint32_t)(w[j] >> 32) == tag) {
                key[j] = (uint32_t)w[j];
                pend &= ~(1u << j);
            }
        if (psh && (uint32_t)(ws >> 32) == tag) {
            shb = (uint32_t)ws;
            psh = false;
        }
        if (!__any_sync(0xffffffffu, pend != 0u || psh)) break;
        if (*(volatile int*)&s.abort) break;
        __nanosleep(it < 256 ? 50 : 200);
    }
    if (__any_sync(0xffffffffu, pend != 0u || psh)) {
        if (lane == 0) set_error(err, s, CZ_DERR_ROUTER_BARRIER);
        return false;
    }
    const float shl = __uint_as_float(shb);  // lane 0's
#pragma unroll
    for (int j = 0; j < NJ; ++j) key[j] = 32 * j + lane < E ? logit_key(__uint_as_float(key[j])) : 0u;
    if (!p.norm_topk) return false;

    uint32_t taken = 0u, mykey = 0u, wk = 0u;
    int myid = 0;
#pragma unroll 1
    for (int z = 0; z <= K; ++z) {
        uint32_t bk = 0u;
        int bj = 0;
#pragma unroll
        for (int j = 0; j < NJ; ++j)
            if (key[j] > bk) {
                bk = key[j];
                bj = j;
            }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        if (z == K) {
            wk = kmax;
            break;
        }
        const uint32_t win = __reduce_min_sync(0xffffffffu, bk == kmax ? (uint32_t)(32 * bj + lane) : 0xffffffffu);
        // the winner's key is cleared by arithmetic on every j (a store to key[win >> 5]
        // would put key[] in local memory)
        const uint32_t hit = lane == (int)(win & 31u) ? 1u << (win >> 5) : 0u;
#pragma unroll
        for (int j = 0; j < NJ; ++j) key[j] &= ((hit >> j) & 1u) - 1u;
        taken |= hit;
        if (lane == z) {
            myid = (int)win;
            mykey = kmax;
        }
    }
    // the check of route_all: finite winners, exps clear of underflow, f32 exps that
    // differ between consecutive winners of different logits and between the last
    // winner and the largest logit left
    const float val = lane < K ? key_logit(mykey) : 0.0f;
    const float mx = __shfl_sync(0xffffffffu, val, 0);
    const float d = __fsub_rn(val, mx);
    const float vn = __shfl_down_sync(0xffffffffu, val, 1), dn = __shfl_down_sync(0xffffffffu, d, 1);
    bool ok = true;
    if (lane < K) {
        ok = mykey != 0u && fabsf(val) <= 3.0e38f;
        if (lane + 1 < K) ok = ok && (vn == val || __fsub_rn(d, dn) >= 0x1p-22f);
        if (lane + 1 == K) {
            ok = ok && d >= -80.0f;
            if (wk) ok = ok && __fsub_rn(d, __fsub_rn(key_logit(wk), mx)) >= 0x1p-22f;
        }
    }
    if (!__all_sync(0xffffffffu, ok)) return false;

    const bool act = lane < K;
    if (act) {
        s.pe[lane] = myid;
        s.pd[lane] = d;
        if (write_out && p.topk_idx) p.topk_idx[lane] = (uint32_t)myid;
    }
    // rank of this lane's winner among the winners, by expert id
    int rho = 0;
    {
        const int jj = myid >> 5, ll = myid & 31;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const uint32_t m = __ballot_sync(0xffffffffu, (taken >> j) & 1u);
            if (j < jj) rho += __popc(m);
            if (j == jj) rho += __popc(m & ((1u << ll) - 1u));
        }
    }
    const int drows = s.geo_drows, per = s.geo_per, rbytes = s.geo_rbytes;
    const bool held = act && myid >= p.e_lo && myid < p.e_hi;
    const uint32_t hm = __reduce_or_sync(0xffffffffu, held ? (1u << rho) : 0u);
    const int k = __popc(hm & ((1u << rho) - 1u));  // index among held routed groups
    const int nr = __popc(hm);
    if (act) {
        s.g_expert[rho] = myid;
        s.g_pair0[rho] = rho;
        s.g_npairs[rho] = 1;
        s.order[rho] = lane;
        s.rtok[rho] = held ? 0 : -1;
        s.g_chunk0[rho] = k * (Ir / CR);
        s.g_pack[rho] = held && drows > 0 ? k / per : -1;
        s.g_poff[rho] = held && drows > 0 ? (k % per) * rbytes : 0;
    }
    if (lane == 0) {
        s.exact[0] = 0;
        int U = K, nc = nr * (Ir / CR);
        int npk = nr > 0 && drows > 0 ? (nr - 1) / per + 1 : 0;
        if (SI) {  // the shared expert: pair K, the last group
            s.pe[K] = E;
            s.shlog[0] = shl;
            s.g_expert[K] = E;
            s.g_pair0[K] = K;
            s.g_npairs[K] = 1;
            s.order[K] = K;
            s.rtok[K] = p.shared_here ? 0 : -1;
            s.g_chunk0[K] = nc;
            s.g_pack[K] = -1;
            s.g_poff[K] = 0;
            if (p.shared_here) {
                nc += SI / CR;
                if (drows > 0) {
                    const int sbytes = drows * SI + s.geo_nrb * cz_nbp(SI) * 4;
                    const int fill = nr > 0 ? (nr - (npk - 1) * per) * rbytes : SLOT_BYTES;
                    if (npk > 0 && fill + sbytes <= SLOT_BYTES) {
                        s.g_pack[K] = npk - 1;
                        s.g_poff[K] = fill;
                    } else {
                        s.g_pack[K] = npk;
                        ++npk;
                    }
                }
            }
            U = K + 1;
        }
        if (p.hslot && npk > ns - 1) set_error(err, s, CZ_DERR_SHAPE);
        s.g_chunk0[U] = nc;
        s.U = U;
        s.P = K + (SI ? 1 : 0);
        s.NC = nc;
        s.npk = npk;
    }
    return true;
}

// Phase D, one consumer warp: wait for and release packs [pk_done, j_end) (stages
// si0 + j of the ring); ok turns false when a wait gives up.
__device__ __forceinline__ void release_packs(DecodeMisc& s, int si0, int NS, int j_end, int& pk_done, bool& ok) {
    for (; pk_done < j_end; ++pk_done) {
        const int sidx = si0 + pk_done;
        if (ok) ok = warp_wait(&s.full[sidx % NS], (sidx / NS) & 1, s);
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.empty[sidx % NS]);
    }
}

// Named barriers between the consumer warps and the h warp (288 threads each):
// RED_FULL(b): the consumers' partial gate/up sums of a chunk of parity b are in
// red[b]; RED_FREE(b): the h warp has read them; H_DONE: the h warp has read
// every chunk of this CTA (red is free for phase D).  The producer warp takes
// part in none of them: it may still be waiting for ring slots that only phase D
// frees.
constexpr int BAR_RED_FULL = 2, BAR_RED_FREE = 4, BAR_H_DONE = 6;
// One-token prologue (every warp but the producer, or all threads): XMAX: max |x|
// is complete (288 threads); SPLIT: the token's terms are written and the ring's
// copy of the token is dead; ROUTED: the producer warp has routed and grouped.
constexpr int BAR_XMAX = 7, BAR_ROUTED = 8, BAR_SPLIT = 9;
__device__ __forceinline__ void bar_sync_n(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"((NCW + 1) * 32) : "memory"); }
__device__ __forceinline__ void bar_sync_all(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(NTHREADS) : "memory"); }
__device__ __forceinline__ void bar_arrive_all(int id) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "n"(NTHREADS) : "memory"); }
__device__ __forceinline__ void bar_arrive_n(int id) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "n"((NCW + 1) * 32) : "memory"); }

// Bounded poll of tagged exchange words into f32 values.  Every thread polls its
// words p[k] (k = tid, tid + NTHREADS, ... < n) until each carries `tag`, issuing
// all of its loads before checking any.  Returns false if it gave up (spin limit,
// or another warp of the CTA already gave up).
template <int NPW>
__device__ __forceinline__ bool poll_words(const unsigned long long* __restrict__ src, int n, int row_words,
                                        int src_stride, float* __restrict__ dst, int dst_stride, uint32_t tag,
                                        uint32_t limit, DecodeMisc& s) {
    const int tid = threadIdx.x;
    uint32_t pend = 0;
    const unsigned long long* a[NPW];
    float* d[NPW];
#pragma unroll
    for (int i = 0; i < NPW; ++i) {
        const int k = tid + i * NTHREADS;
        a[i] = src;
        d[i] = dst;
        if (k < n) {
            const int r = k / row_words, cix = k - r * row_words;
            a[i] = src + (size_t)r * src_stride + cix;
            d[i] = dst + (size_t)r * dst_stride + cix;
            pend |= 1u << i;
        }
    }
    for (uint32_t it = 0; pend && it < limit; ++it) {
        unsigned long long w[NPW];
#pragma unroll
        for (int i = 0; i < NPW; ++i)
            if (pend & (1u << i)) w[i] = ld_relaxed_u64(a[i]);
#pragma unroll
        for (int i = 0; i < NPW; ++i)
            if ((pend & (1u << i)) && (uint32_t)(w[i] >> 32) == tag) {
                *d[i] = __uint_as_float((uint32_t)w[i]);
                pend &= ~(1u << i);
            }
        if (pend) {
            if (*(volatile int*)&s.abort) break;
            __nanosleep(it < 64 ? 20 : 200);
        }
    }
    return pend == 0;
}

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
    const Carve cv = carve(T, H, p.x_bf16, p.hslot);
    DecodeMisc& s = *reinterpret_cast<DecodeMisc*>(sb + cv.misc);
    uint8_t* const ring = sb;
    uint8_t* const xterm = sb + cv.xterm;
    float* const red = reinterpret_cast<float*>(sb + cv.red);
    uint32_t* const err = p.sync + 1;
    const uint32_t limit = p.spin_limit ? p.spin_limit : CZ_SPIN_LIMIT;

    // ---------------- phase R: router logits ----------------
    const int row_lo = split_at(c, Er, G), row_hi = split_at(c + 1, Er, G);
    const int nrows = row_hi - row_lo;
    const uint32_t xbytes = (uint32_t)T * H * (xbf ? 2u : 4u);
    const uint32_t rbytes = (uint32_t)nrows * H * 4u;
    // ring during phase R: [router rows][tokens][rms weight]
    float* rows = reinterpret_cast<float*>(ring);
    uint8_t* xs = ring + rbytes;
    float* wnorm = reinterpret_cast<float*>(ring + rbytes + xbytes);
    // The next launch in the stream may start its CTAs as this launch's CTAs end.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        // the barriers, then the router rows at once: weights, which no kernel writes,
        // so the copy goes out before the wait for the previous kernel
        for (int i = 0; i < cv.ns; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], NCW);
        }
        mbar_init(&s.rbar, 1);
        s.abort = 0;
        s.dots_done = 0;
        fence_mbarrier_init();
        const uint32_t wbytes = p.rms_w ? (uint32_t)H * 4u : 0u;
        mbar_arrive_expect_tx(&s.rbar, xbytes + rbytes + wbytes);
        for (int r = 0; r < nrows; ++r) {
            const int e = row_lo + r;
            bulk_g2s(rows + (size_t)r * H, (e < E) ? p.router + (size_t)e * H : p.sh_gate, (uint32_t)H * 4u, &s.rbar);
        }
        // the tokens (and the sequence word) may come from the previous kernel
        asm volatile("griddepcontrol.wait;" ::: "memory");
        bulk_g2s(xs, p.x, xbytes, &s.rbar);
        if (wbytes) bulk_g2s(wnorm, p.rms_w, wbytes, &s.rbar);
    } else if (tid == 64) {
        // phase D geometry of this CTA: output rows [o_lo, o_hi), their row blocks, the
        // bytes one routed group's rows take in a pack, and the groups a pack holds
        const int o_lo = split_at(c, H, G), o_hi = split_at(c + 1, H, G);
        const int drows = o_hi - o_lo;
        const int nrb = drows > 0 ? ((o_hi - 1) >> 7) - (o_lo >> 7) + 1 : 0;
        const int rbytes = drows * Ir + nrb * cz_nbp(Ir) * 4;
        s.geo_drows = drows;
        s.geo_nrb = nrb;
        s.geo_rbytes = rbytes;
        s.geo_per = drows > 0 ? SLOT_BYTES / rbytes : 1;
    } else if (tid == 32) {
        // the weight stream's tensor maps: fetched now, not at the first weight copy
        prefetch_tensormap(&p.gate_map);
        prefetch_tensormap(&p.up_map);
        if (SI) {
            prefetch_tensormap(&p.sh_gate_map);
            prefetch_tensormap(&p.sh_up_map);
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the previous kernel's writes are visible
    const uint32_t seq = ld_relaxed_gpu(p.sync);
    const uint32_t tag = seq + 1u;  // this launch's exchange tag (zeroed scratch never matches)
    // expert parallelism: this launch's counter, the same on every rank
    const uint32_t eseq = p.ep_world > 1 ? ld_relaxed_gpu(p.ep_seq) : 0u;
    uint32_t* reg = region(p.sync, seq & 1);
    if (c == 0 && tid < kSyncRegionWords) region(p.sync, (seq & 1) ^ 1)[tid] = 0u;
    if (tid < MAXT) s.xmax[tid] = 0u;
    __syncthreads();
    // this CTA has read the sequence words: every thread's loads are ordered before
    // the count-in by the barrier above
    if (tid == 0) red_relaxed_add_gpu(&reg[0], 1u);
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
    const int nitems = nrows * T;
    int si_early = 0;  // gate/up stages the producer issued right after routing (one token)
    if constexpr (T == 1) {
        // One token: the producer warp routes and groups it alone (route_one) while
        // the other warps form this CTA's router logits, max |x| and the token's
        // E4M3 terms (x * 2^s = term 0 + term 1 (+ term 2), term j at xterm + j*CS);
        // the producer then waits only for the terms (SPLIT: the ring's copy of the
        // token is dead) before it streams.
        if (warp == PW) {
            // Polls from every CTA while the logits are still being formed slow their
            // publication down (the words share a few L2 lines): the first poll waits
            // until this CTA has published its own logits, the grid's others being
            // due about then, or about a microsecond in a CTA without router rows.
            {
                const int nd = nitems < NCW ? nitems : NCW;
                if (nd == 0) __nanosleep(1000);
                for (uint32_t it = 0; it < limit && *(volatile int*)&s.dots_done < nd && !*(volatile int*)&s.abort; ++it)
                    __nanosleep(32);
            }
            bool ok = false;
            if (!s.abort)
                ok = E <= 128 ? route_one<4>(p, s, cv.ns, E, K, SI, Ir, tag, limit, err, c == 0)
                              : route_one<16>(p, s, cv.ns, E, K, SI, Ir, tag, limit, err, c == 0);
            if (lane == 0) s.fastgroup = ok ? 1 : 0;
            __syncwarp();
            bar_arrive_all(BAR_ROUTED);
            bar_sync_all(BAR_SPLIT);
            // The first ring fill goes out here, in the code right after routing (the
            // phase C loop below, cold in the instruction cache when it is first
            // reached, skips these stages).
            if (ok && lane == 0 && !s.abort) {
                fence_proxy_async_smem();  // the ring's generic accesses precede the copies
                const uint64_t pol = l2_evict_first_policy();
                const int NC = s.NC, ch_lo = split_at(c, NC, G), ch_hi = split_at(c + 1, NC, G);
                const int nks = (H + KS - 1) / KS, nkbH = cz_nblk(H), nbpH = cz_nbp(H);
                int u = 0;
                for (int ch = ch_lo; ch < ch_hi && si_early < cv.ns; ++ch) {
                    while (s.g_chunk0[u + 1] <= ch) ++u;
                    const GroupW gw = group_w(p, s.g_expert[u]);
                    const int r0 = (ch - s.g_chunk0[u]) * CR;
                    for (int st = 0; st < 2 * nks && si_early < cv.ns; ++st, ++si_early)
                        issue_gu_stage(p, s, ring, gw, r0, st, si_early, nkbH, nbpH, pol);
                }
            }
        } else {
            const int nd = nitems < NCW ? nitems : NCW;     // warps on the router dot
            const int wt = tid < PW * 32 ? tid : tid - 32;  // thread index among the 288
            if (!s.abort && warp < nd) {
                for (int r = warp; r < nrows; r += nd) {
                    const float* wr = rows + (size_t)r * H;
                    const float v = xbf ? router_dot<true>(wr, xs, H, lane) : router_dot<false>(wr, xs, H, lane);
                    if (lane == 0 && !(p.dbg_hold && row_lo + r == 0))
                        st_relaxed_u64(p.logits + row_lo + r, tag_word(tag, v));
                }
                if (lane == 0) atomicAdd(&s.dots_done, 1);
            }
            if (!s.abort) {
                float m = 0.0f;
                for (int i = wt; i < H; i += NTHREADS - 32) {
                    const float a = fabsf(xval(i));
                    if (a < 3.0e38f) m = fmaxf(m, a);
                }
                m = warp_max_f32(m);
                if (lane == 0 && m > 0.0f) atomicMax(&s.xmax[0], __float_as_uint(m));
            }
            bar_sync_n(BAR_XMAX);
            if (!s.abort && warp >= nd) {
                const int nsw = NWARPS - 1 - nd;  // warps on the split
                const int st0 = (warp - nd - (warp > PW ? 1 : 0)) * 32 + lane;
                const int sx = prescale_exp(__uint_as_float(s.xmax[0]));
                for (int i = 2 * st0; i < H; i += 2 * 32 * nsw) {
                    float a = scale2(xval(i), sx), b = scale2(xval(i + 1), sx);
                    for (int j = 0; j < cv.JX; ++j) {
                        const uint16_t d = e4m3_term2(a, b);
                        *reinterpret_cast<uint16_t*>(xterm + (size_t)j * cv.CS + i) = d;
                    }
                }
            }
            if (tid == 0) {
                const int e = prescale_exp(__uint_as_float(s.xmax[0]));
                s.xexp[0] = e;
                s.xscale[0] = scale2(1.0f, -e);
            }
            fence_proxy_async_smem();  // the token's generic reads precede the producer's copies
            bar_arrive_all(BAR_SPLIT);
            bar_sync_all(BAR_ROUTED);
        }
    } else {
        // max |x_t| for the per-token power-of-two prescale (one atomic per warp)
        if (!s.abort) {
            for (int t = 0; t < T; ++t) {
                float m = 0.0f;
                for (int i = tid; i < H; i += NTHREADS) {
                    const float a = fabsf(xval(t * H + i));
                    if (a < 3.0e38f) m = fmaxf(m, a);
                }
                m = warp_max_f32(m);
                if (lane == 0 && m > 0.0f) atomicMax(&s.xmax[t], __float_as_uint(m));
            }
        }
        __syncthreads();
        // The first nd warps form the router logits (one (row, token) item each, in
        // turn); each logit goes out as one tagged word the moment it is formed.  Then
        // every warp (the others at once) splits the tokens into E4M3 terms:
        //   x_t * 2^s_t = term 0 + term 1 (+ term 2), column (t, j) holding term j of
        //   token t, H bytes at xterm + (t*JX + j)*CS.
        // The CTA polls the grid's logits only after the split, so the split is shared
        // by all warps rather than left to the few without a router item.
        const int nd = nitems < NWARPS ? nitems : NWARPS;
        if (!s.abort) {
            if (warp < nd) {
                for (int it = warp; it < nitems; it += NWARPS) {
                    const int r = it / T, t = it - r * T;
                    const float* wr = rows + (size_t)r * H;
                    const float v = xbf ? router_dot<true>(wr, xs + (size_t)t * H * 2, H, lane)
                                        : router_dot<false>(wr, xs + (size_t)t * H * 4, H, lane);
                    if (lane == 0 && !(p.dbg_hold && row_lo + r == 0))
                        st_relaxed_u64(p.logits + (size_t)t * LS + row_lo + r, tag_word(tag, v));
                }
            }
            {
                const int nsw = NWARPS;  // warps on the split
                const int st0 = warp * 32 + lane;
                for (int t = 0; t < T; ++t) {
                    const int sx = prescale_exp(__uint_as_float(s.xmax[t]));
                    uint8_t* col = xterm + (size_t)(t * cv.JX) * cv.CS;
                    for (int i = 2 * st0; i < H; i += 2 * 32 * nsw) {
                        float a = scale2(xval(t * H + i), sx), b = scale2(xval(t * H + i + 1), sx);
                        for (int j = 0; j < cv.JX; ++j) {
                            const uint16_t d = e4m3_term2(a, b);
                            *reinterpret_cast<uint16_t*>(col + (size_t)j * cv.CS + i) = d;
                        }
                    }
                }
            }
        }
        if (tid < T) {
            const int e = prescale_exp(__uint_as_float(s.xmax[tid]));
            s.xexp[tid] = e;
            s.xscale[tid] = scale2(1.0f, -e);
        }
    }
    // ---------------- phase K: every logit of the grid, top-k, grouping (every CTA) ----------------
    // (one token: only when route_one gave up)
    const int P = T * K + (SI ? T : 0);
    bool general = true;
    if constexpr (T == 1) general = s.fastgroup == 0;
    if (general) {
        __syncthreads();  // the ring's tokens are dead from here on: it holds the routing scratch

        RouteScratch rs;
        {
            const int nch = (E + 31) >> 5;
            const uint32_t lgb = ((uint32_t)T * LS * 4u + 15u) & ~15u;
            const uint32_t cab = (uint32_t)T * nch * K * 8u;
            rs.lg = reinterpret_cast<float*>(ring);
            rs.ex = reinterpret_cast<float*>(ring + lgb);
            rs.ca = reinterpret_cast<unsigned long long*>(ring + 2 * lgb);
            rs.cb = reinterpret_cast<unsigned long long*>(ring + 2 * lgb + cab);
            rs.fin = reinterpret_cast<unsigned long long*>(ring + 2 * lgb + 2 * cab);
        }
        if (!s.abort) {
            constexpr int NPW = (T * (MAXE + 1) + NTHREADS - 1) / NTHREADS;
            if (!poll_words<NPW>(p.logits, T * Er, Er, LS, rs.lg, LS, tag, limit, s))
                set_error(err, s, CZ_DERR_ROUTER_BARRIER);
        }
        __syncthreads();
        if (tid == 0) s.fastgroup = 0;
        if (!s.abort) {
            route_all(rs, T, E, K, LS, p.norm_topk, SI != 0, s, p.topk_idx, p.topk_gates, c == 0);
            if (T == 1 && warp == 0) {
                // One token: its K experts are distinct unless a selection round found no
                // candidate (NaN logits), so each pair is a group of its own, in ascending
                // expert order.  The warp that ranked the token forms the groups in a few
                // shuffles; duplicates fall through to the general path below.
                __syncwarp();
                const bool act = lane < K;
                const int myid = act ? s.pe[lane] : 0x7fffffff;
                int rho = 0;
                bool dup = false;
    #pragma unroll 4
                for (int m = 0; m < MAXK; ++m) {
                    const int im = __shfl_sync(0xffffffffu, myid, m);
                    rho += (m < K) & (im < myid);
                    dup |= act & (m < K) & (m != lane) & (im == myid);
                }
                if (!__any_sync(0xffffffffu, dup)) {
                    const int drows = s.geo_drows, per = s.geo_per, rbytes = s.geo_rbytes;
                    const bool held = act && myid >= p.e_lo && myid < p.e_hi;
                    const uint32_t hm = __reduce_or_sync(0xffffffffu, held ? (1u << rho) : 0u);
                    const int k = __popc(hm & ((1u << rho) - 1u));  // index among held routed groups
                    const int nr = __popc(hm);
                    if (act) {
                        s.g_expert[rho] = myid;
                        s.g_pair0[rho] = rho;
                        s.g_npairs[rho] = 1;
                        s.order[rho] = lane;
                        s.rtok[rho] = held ? 0 : -1;
                        s.g_chunk0[rho] = k * (Ir / CR);
                        s.g_pack[rho] = held && drows > 0 ? k / per : -1;
                        s.g_poff[rho] = held && drows > 0 ? (k % per) * rbytes : 0;
                    }
                    if (lane == 0) {
                        int U = K, nc = nr * (Ir / CR);
                        int npk = nr > 0 && drows > 0 ? (nr - 1) / per + 1 : 0;
                        if (SI) {  // the shared expert: pair T*K = K, the last group
                            s.g_expert[K] = E;
                            s.g_pair0[K] = K;
                            s.g_npairs[K] = 1;
                            s.order[K] = K;
                            s.rtok[K] = p.shared_here ? 0 : -1;
                            s.g_chunk0[K] = nc;
                            s.g_pack[K] = -1;
                            s.g_poff[K] = 0;
                            if (p.shared_here) {
                                nc += SI / CR;
                                if (drows > 0) {
                                    const int sbytes = drows * SI + s.geo_nrb * cz_nbp(SI) * 4;
                                    const int fill = nr > 0 ? (nr - (npk - 1) * per) * rbytes : SLOT_BYTES;
                                    if (npk > 0 && fill + sbytes <= SLOT_BYTES) {
                                        s.g_pack[K] = npk - 1;
                                        s.g_poff[K] = fill;
                                    } else {
                                        s.g_pack[K] = npk;
                                        ++npk;
                                    }
                                }
                            }
                            U = K + 1;
                        }
                        if (p.hslot && npk > cv.ns - 1) set_error(err, s, CZ_DERR_SHAPE);
                        s.g_chunk0[U] = nc;
                        s.U = U;
                        s.P = P;
                        s.NC = nc;
                        s.npk = npk;
                        s.fastgroup = 1;
                    }
                }
            }
        }
        // the ring held generic-proxy data (the routing scratch) and is next written by
        // bulk copies: order every thread's accesses before them
        fence_proxy_async_smem();
        __syncthreads();
        if (!s.abort && !s.fastgroup) {
            // pairs sorted by (expert, pair) with ranks: P <= 68
            for (int i = tid; i < P; i += NTHREADS) {
                const int e = s.pe[i];
                int r = 0;
                for (int j = 0; j < P; ++j) {
                    const int ej = s.pe[j];
                    r += (ej < e) | ((ej == e) & (j < i));
                }
                s.order[r] = i;
            }
        }
        __syncthreads();
        if (warp == 0 && !s.fastgroup) {
            if (!s.abort) {
                // Groups: runs of one expert in sorted order.  A token picks an expert at
                // most once, except in selection rounds without a candidate (every
                // remaining logit NaN), which all pick expert 0; a run longer than the
                // gate/up MMA columns hold (maxq pairs) is split into groups of maxq pairs
                // (each reads the expert's weights again).  Up to 3 sorted positions per
                // lane: r = 32 w + lane.
                const int maxq = cv.rc / cv.JX;
                int pe_r[3];
                uint32_t chg[3];
    #pragma unroll
                for (int w = 0; w < 3; ++w) {
                    const int r = 32 * w + lane;
                    pe_r[w] = r < P ? s.pe[s.order[r]] : -1;
                    const int prev = __shfl_up_sync(0xffffffffu, pe_r[w], 1);
                    const int prev_w = w > 0 ? __shfl_sync(0xffffffffu, pe_r[w > 0 ? w - 1 : 0], 31) : -1;
                    const int pv = lane == 0 ? prev_w : prev;
                    chg[w] = __ballot_sync(0xffffffffu, r < P && (r == 0 || pe_r[w] != pv));
                }
                // a position starts a group when its distance to its run's first position
                // is a multiple of maxq
                uint32_t stw[3];
                int u_base[3];
                int base = 0;
    #pragma unroll
                for (int w = 0; w < 3; ++w) {
                    const int r = 32 * w + lane;
                    int rs0 = -1;  // the run's first position: the last change at or before r
                    const uint32_t below = lane == 31 ? 0xffffffffu : ((2u << lane) - 1u);
    #pragma unroll
                    for (int v = w; v >= 0; --v) {
                        const uint32_t m = v == w ? (chg[v] & below) : chg[v];
                        if (rs0 < 0 && m) rs0 = 32 * v + 31 - __clz(m);
                    }
                    const bool start = r < P && (r - rs0) % maxq == 0;
                    stw[w] = __ballot_sync(0xffffffffu, start);
                    u_base[w] = base;
                    if (start) {
                        const int u = base + __popc(stw[w] & ((1u << lane) - 1u));
                        s.g_expert[u] = pe_r[w];
                        s.g_pair0[u] = r;
                    }
                    base += __popc(stw[w]);
                }
                __syncwarp();
                // per group (up to 3 per lane, u = 32 v + lane): size, held here, first
                // chunk, phase D pack.  Routed groups all have Ir/CR chunks and rb bytes
                // of down rows per pack; the shared expert (expert E) is the last group.
                const int drows = s.geo_drows, nrb = s.geo_nrb, rbytes = s.geo_rbytes, per = s.geo_per;
                int nr = 0;  // held routed groups before this batch
    #pragma unroll
                for (int v = 0; v < 3; ++v) {
                    const int u = 32 * v + lane;
                    const bool in = u < base;
                    const int eu = in ? s.g_expert[u] : -1;
                    const int p0 = in ? s.g_pair0[u] : 0;
                    const int p1 = u + 1 < base ? s.g_pair0[u + 1] : P;
                    const bool here = in && (eu == E ? p.shared_here != 0 : (eu >= p.e_lo && eu < p.e_hi));
                    const bool routed = here && eu != E;
                    const uint32_t rm = __ballot_sync(0xffffffffu, routed);
                    const int k = nr + __popc(rm & ((1u << lane) - 1u));  // index among held routed groups
                    if (in) {
                        s.g_npairs[u] = p1 - p0;
                        s.g_chunk0[u] = k * (Ir / CR);
                        s.g_pack[u] = routed && drows > 0 ? k / per : -1;
                        s.g_poff[u] = routed && drows > 0 ? (k % per) * rbytes : 0;
                        for (int q = p0; q < p1; ++q) s.rtok[q] = here ? pair_token(s.order[q], T, K) : -1;
                    }
                    nr += __popc(rm);
                }
                __syncwarp();
                if (lane == 0) {
                    int nc = nr * (Ir / CR);
                    int npk = nr > 0 && drows > 0 ? (nr - 1) / per + 1 : 0;
                    if (base > 0 && s.g_expert[base - 1] == E && p.shared_here) {
                        nc += SI / CR;
                        if (drows > 0) {
                            const int sbytes = drows * SI + nrb * cz_nbp(SI) * 4;
                            const int fill = nr > 0 ? (nr - (npk - 1) * per) * rbytes : SLOT_BYTES;
                            if (npk > 0 && fill + sbytes <= SLOT_BYTES) {
                                s.g_pack[base - 1] = npk - 1;
                                s.g_poff[base - 1] = fill;
                            } else {
                                s.g_pack[base - 1] = npk;
                                s.g_poff[base - 1] = 0;
                                ++npk;
                            }
                        }
                    }
                    // hslot: the slot after the last pack must be free (the host checked the worst case)
                    if (p.hslot && npk > cv.ns - 1) set_error(err, s, CZ_DERR_SHAPE);
                    s.g_chunk0[base] = nc;
                    s.U = base;
                    s.P = P;
                    s.NC = nc;
                    s.npk = npk;
                }
            } else if (lane == 0) {
                s.U = 0;
                s.NC = 0;
                s.npk = 0;
            }
        }
        __syncthreads();
    }

    // ---------------- phase C: this CTA's chunks; phase D: this CTA's output rows ----------------
    const int o_lo = split_at(c, H, G), o_hi = split_at(c + 1, H, G);
    const int drows = o_hi - o_lo;
    const int ldh = Ir > SI ? Ir : SI;  // row stride of the h rows in global scratch
    float* const dsum = reinterpret_cast<float*>(sb + cv.dsum);  // phase D: [sorted pair][row] sums
    {
        const int NC = s.NC;
        const int NS = cv.ns;
        const int ch_lo = split_at(c, NC, G), ch_hi = split_at(c + 1, NC, G);
        const int nks = (H + KS - 1) / KS;     // gate (and up) stages per chunk
        const int nbpH = cz_nbp(H);
        const int nkbH = cz_nblk(H);           // 128-column blocks of H

        if (warp == PW) {
            // ---------------- producer (one thread) ----------------
            if (lane == 0) {
                fence_proxy_async_smem();  // generic reads of the ring (logits) precede the async writes
                const uint64_t pol = l2_evict_first_policy();
                int si = 0;
                const int nst = 2 * nks * (ch_hi - ch_lo);  // gate/up stages; the packs follow
                // phase C: gate/up slabs of every chunk
                {
                    int u = 0;
                    for (int ch = ch_lo; ch < ch_hi && !s.abort; ++ch) {
                        while (s.g_chunk0[u + 1] <= ch) ++u;
                        const GroupW gw = group_w(p, s.g_expert[u]);
                        const int r0 = (ch - s.g_chunk0[u]) * CR;
                        for (int st = 0; st < 2 * nks && !s.abort; ++st, ++si) {
                            if (si < si_early) continue;  // issued right after routing
                            const int slot = si % NS;
                            if (si == NS) prefetch_rest(p, s, ch_lo, ch_hi, nks, NS, nst, drows, o_lo, o_hi, T != 1);
                            if (!slot_acquire(s, err, slot, si / NS)) break;
                            issue_gu_stage(p, s, ring, gw, r0, st, slot, nkbH, nbpH, pol);
                        }
                    }
                }
                // phase D: the packs of down rows [o_lo, o_hi) (+ their 128 x 128 scales) of
                // every group held here; they stream in while phase C still runs
                if (drows > 0) {
                    const int rb0 = o_lo >> 7, nrb = ((o_hi - 1) >> 7) - rb0 + 1;
                    int u = 0;
                    for (int j = 0; j < s.npk && !s.abort; ++j, ++si) {
                        while (u < s.U && s.g_pack[u] != j) ++u;
                        int u1 = u;
                        uint32_t bytes = 0;  // what the copies below deliver (rows x iu is a multiple of 16)
                        for (; u1 < s.U && (s.g_pack[u1] == j || s.g_pack[u1] < 0); ++u1) {
                            if (s.g_pack[u1] < 0) continue;
                            const int iu = s.g_expert[u1] == E ? SI : Ir;
                            bytes += (uint32_t)(drows * iu + nrb * cz_nbp(iu) * 4);
                        }
                        const int slot = si % NS;
                        if (si == NS) prefetch_rest(p, s, ch_lo, ch_hi, nks, NS, nst, drows, o_lo, o_hi, T != 1);
                        if (!slot_acquire(s, err, slot, si / NS)) break;
                        uint8_t* dst = ring + (size_t)slot * SLOT_BYTES;
                        mbar_arrive_expect_tx(&s.full[slot], bytes);
                        for (int v = u; v < u1; ++v) {
                            if (s.g_pack[v] < 0) continue;
                            const int ev = s.g_expert[v];
                            const bool sh = ev == E;
                            const int iu = sh ? SI : Ir;
                            const uint8_t* wsrc = sh ? p.sh_down_w + (size_t)o_lo * SI
                                                     : p.down_w + ((size_t)(ev - p.e_lo) * H + o_lo) * Ir;
                            const float* ssrc = sh ? p.sh_down_s + (size_t)rb0 * cz_nbp(SI)
                                                   : p.down_s + ((size_t)(ev - p.e_lo) * nkbH + rb0) * cz_nbp(Ir);
                            uint8_t* d = dst + s.g_poff[v];
                            const uint32_t wbytes = (uint32_t)drows * (uint32_t)iu;  // a multiple of 16
                            bulk_g2s_hint(d, wsrc, wbytes, &s.full[slot], pol);
                            bulk_g2s(d + wbytes, ssrc, (uint32_t)(nrb * cz_nbp(iu) * 4), &s.full[slot]);
                        }
                        u = u1;
                    }
                }
                // CTA 0 advances the launch sequence (the next launch's tag) once every
                // CTA has counted itself in (reg[0], right after it read the sequence):
                // no CTA of this launch reads it later, and the next launch starts only
                // after this one has ended.  A count that never completes leaves the
                // sequence as it is and sets an error bit.
                if (c == 0) {
                    bool in = false;
                    for (uint32_t it = 0; it < limit && !in; ++it) {
                        in = ld_relaxed_gpu(&reg[0]) >= (uint32_t)G;
                        if (!in) __nanosleep(100);
                    }
                    if (in) {
                        st_relaxed_u32(p.sync, seq + 1u);
                        if (p.ep_world > 1) st_relaxed_u32(p.ep_seq, eseq + 1u);
                    } else {
                        atomicOr(err, CZ_DERR_SEQ_WAIT);
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
            // First the gates of the tokens the fast path routed (while the first
            // stages land), then per chunk, once the consumers' partial gate/up sums
            // are in red[b]: hw = gate * silu(g) * u per (row r, routed token) into the
            // pair's h row in global scratch.  Runs beside the next chunk's MMAs.
            if (!s.abort) route_gates(T, K, SI != 0, s, p.topk_gates, c == 0);
            const int nch = ch_hi - ch_lo;
            int u = 0;
            for (int ch = ch_lo; ch < ch_hi; ++ch) {
                while (s.g_chunk0[u + 1] <= ch) ++u;
                const int ci = ch - ch_lo, b = ci & 1;
                const int np = s.g_npairs[u];
                const int* pairs = s.order + s.g_pair0[u];
                const int r0 = (ch - s.g_chunk0[u]) * CR;
                bar_sync_n(BAR_RED_FULL + b);
                const int wst = 2 * 16 * cv.rc;  // floats of one warp's gate + up partial sums
                const float* rb = red + b * (NCW * wst);
#pragma unroll 1
                for (int q0 = 0; q0 < np; q0 += 2) {  // lanes: two pairs x 16 rows
                    const int q = q0 + (lane >> 4), r = lane & 15;
                    const int tk = q < np ? pair_token(pairs[q], T, K) : 0;
                    if (q < np && !s.abort) {
                        float gs = 0.0f, us = 0.0f;
                        const float* rg = rb + r * cv.rc + q * cv.JX;
                        float gv[NCW][3], uv[NCW][3];
#pragma unroll
                        for (int w = 0; w < NCW; ++w)
#pragma unroll
                            for (int j = 0; j < 3; ++j) {
                                gv[w][j] = j < cv.JX ? rg[w * wst + j] : 0.0f;
                                uv[w][j] = j < cv.JX ? rg[w * wst + 16 * cv.rc + j] : 0.0f;
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
                        st_relaxed_u64(p.hrows + (size_t)pairs[q] * ldh + r0 + r,
                                       tag_word(tag, s.pg[pairs[q]] * (silu_fast(gs * xsc) * (us * xsc))));
                    }
                }
                __threadfence_block();
                if (ci + 2 < nch) bar_arrive_n(BAR_RED_FREE + b);
            }
        } else {
            // ---------------- consumers ----------------
            const int g = lane >> 2, t = lane & 3;  // MMA fragment coordinates
            // MMA rows g, g + 8 hold chunk rows rho, rho + 8: the two rows a quarter-warp
            // reads then sit 4 apart in the swizzle pattern, so their chunks use disjoint banks
            const int rho = (g >> 1) + 4 * (g & 1);
            int si = 0;
            int u = 0;
            // ==== phase C: gate/up of every chunk (h is formed by the h warp) ====
            for (int ch = ch_lo; ch < ch_hi; ++ch) {
                while (s.g_chunk0[u + 1] <= ch) ++u;
                const int ci = ch - ch_lo, b = ci & 1;
                // red[b] is reused: the h warp must be done with chunk ci-2
                if (ci >= 2) bar_sync_n(BAR_RED_FREE + b);
                const int np = s.g_npairs[u];
                const int* pairs = s.order + s.g_pair0[u];
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
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&s.empty[slg]);
                        mbar_arrive(&s.empty[slu]);
                    }
                }

                // ---- this warp's partial gate/up sums of the chunk -> red[b] (h warp) ----
                {
                    const int rc = cv.rc;
                    float* rg = red + (b * NCW * 2 + warp * 2 + 0) * (16 * rc);
                    float* ru = rg + 16 * rc;
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        if (8 * m >= rc) break;  // rc = 8: every group's columns fit MMA tile 0
                        const int col = 8 * m + 2 * t;
                        rg[rho * rc + col] = accg[m][0];
                        rg[rho * rc + col + 1] = accg[m][1];
                        rg[(rho + 8) * rc + col] = accg[m][2];
                        rg[(rho + 8) * rc + col + 1] = accg[m][3];
                        ru[rho * rc + col] = accu[m][0];
                        ru[rho * rc + col + 1] = accu[m][1];
                        ru[(rho + 8) * rc + col] = accu[m][2];
                        ru[(rho + 8) * rc + col + 1] = accu[m][3];
                    }
                }
                __threadfence_block();
                bar_arrive_n(BAR_RED_FULL + b);
            }
        }
    }

    // No grid-wide barrier: phase D reads every h row as tagged words and polls
    // until each carries this launch's tag.  Only the h warp must be done reading
    // red, which phase D reuses for the h terms.  The producer keeps issuing the
    // phase D packs meanwhile (it joins the block again at the end).
    if (warp < NCW || warp == HW) bar_sync_n(BAR_H_DONE);

    // ---------------- phase D: output rows [o_lo, o_hi) over every pair held here ----------------
    // Pair j (in group order) goes to consumer warp j % NCW.  For one pair and one row:
    // sum over 128-column blocks of scale(row block, column block) x (down row . h row),
    // lanes on 8-column pieces.  Every warp waits for and releases every pack in order.
    if (warp < NCW && drows > 0) {
        const int NS = cv.ns;
        const int nch = s.NC;
        const int si0 = 2 * ((H + KS - 1) / KS) * (split_at(c + 1, nch, G) - split_at(c, nch, G));
        const int rb0 = o_lo >> 7;
        // this warp's DHW words of f16 h terms: in red, or (hslot) in the ring slot after
        // the last pack, whose last stage was a gate/up slab consumed in phase C
        uint32_t* const hb = (p.hslot ? reinterpret_cast<uint32_t*>(ring + (size_t)((si0 + s.npk) % NS) * SLOT_BYTES)
                                      : reinterpret_cast<uint32_t*>(red)) +
                             warp * DHW;
        int pk_done = 0;   // packs waited for and released by this warp
        bool ok = !s.abort;
        int jp = 0;  // running index of held pairs
        for (int u = 0; u < s.U; ++u) {
            const int pk = s.g_pack[u];
            if (pk < 0) continue;
            const int np = s.g_npairs[u];
            const bool sh = s.g_expert[u] == E;
            const int iu = sh ? SI : Ir, nbpI = cz_nbp(iu);
            for (int q = 0; q < np; ++q, ++jp) {
                if (jp % NCW != warp) continue;
                // the pair's h row (loads in flight while the pack is waited for); below it becomes,
                // x 2^e (max |h| x 2^e in [2^14, 2^15), inside the f16 range), f16 pairs of hi and lo
                // terms (22 bits) in this warp's share of the idle reduction buffer: words [0, iu/2)
                // hi, [iu/2, iu) lo
                const int pr = s.order[s.g_pair0[u] + q];
                // The row is tagged words written by other CTAs' h warps: poll until every
                // word carries this launch's tag (the first loads go out before the pack wait).
                const unsigned long long* hrow = p.hrows + (size_t)pr * ldh;
                const int nw2 = iu >> 1;
                float2 hv[DHW / 64];
                unsigned long long wa[DHW / 64], wb[DHW / 64];
                uint32_t pend = 0;
#pragma unroll
                for (int j = 0; j < DHW / 64; ++j) {
                    hv[j] = make_float2(0.f, 0.f);
                    if (lane + 32 * j < nw2) {
                        pend |= 1u << j;
                        ld_relaxed_u64x2(hrow + 2 * (lane + 32 * j), wa[j], wb[j]);
                    }
                }
                release_packs(s, si0, NS, pk, pk_done, ok);  // every earlier pack is done for this warp
                const int sidx = si0 + pk;
                if (ok) ok = warp_wait(&s.full[sidx % NS], (sidx / NS) & 1, s);
                for (uint32_t it = 0; ok; ++it) {
#pragma unroll
                    for (int j = 0; j < DHW / 64; ++j)
                        if ((pend & (1u << j)) && (uint32_t)(wa[j] >> 32) == tag && (uint32_t)(wb[j] >> 32) == tag) {
                            hv[j] = make_float2(__uint_as_float((uint32_t)wa[j]), __uint_as_float((uint32_t)wb[j]));
                            pend &= ~(1u << j);
                        }
                    if (__all_sync(0xffffffffu, pend == 0)) break;
                    if (it >= limit || *(volatile int*)&s.abort) {
                        ok = false;
                        break;
                    }
                    __nanosleep(it < 64 ? 20 : 200);
#pragma unroll
                    for (int j = 0; j < DHW / 64; ++j)
                        if (pend & (1u << j)) ld_relaxed_u64x2(hrow + 2 * (lane + 32 * j), wa[j], wb[j]);
                }
                if (!ok) {
                    if (lane == 0 && !s.abort) set_error(err, s, CZ_DERR_READY_WAIT);
                    continue;
                }
                const uint8_t* wr = ring + (size_t)(sidx % NS) * SLOT_BYTES + s.g_poff[u];
                const float* sc = reinterpret_cast<const float*>(wr + (size_t)drows * iu);
                float hm = 0.0f;
#pragma unroll
                for (int j = 0; j < DHW / 64; ++j) hm = fmaxf(hm, fmaxf(fabsf(hv[j].x), fabsf(hv[j].y)));
                hm = warp_max(hm);
                const int he = !(hm < 3.0e38f) ? 0 : prescale_exp(hm) + 7;  // [128, 256) x 2^7
                const float hs = scale2(1.0f, he), hsi = scale2(1.0f, -he);
#pragma unroll
                for (int j = 0; j < DHW / 64; ++j)
                    if (lane + 32 * j < nw2) {
                        const float ax = hv[j].x * hs, ay = hv[j].y * hs;
                        const __half2 hi = __floats2half2_rn(ax, ay);
                        const float2 back = __half22float2(hi);
                        const __half2 lo = __floats2half2_rn(ax - back.x, ay - back.y);
                        hb[lane + 32 * j] = *reinterpret_cast<const uint32_t*>(&hi);
                        hb[nw2 + lane + 32 * j] = *reinterpret_cast<const uint32_t*>(&lo);
                    }
                __syncwarp();
                // f16 MMAs m16n8k16: A = 16 of the pack's down rows (E4M3 -> f16, exact), B columns
                // 0 / 1 = the hi / lo terms of h.  The K order inside a 64-column group is permuted
                // (A and B alike): step j's columns {2t, 2t+1, 2t+8, 2t+9} of lane t are the bytes
                // 16t + 4j .. 16t + 4j + 3, so one 16-byte load of a row feeds four steps.  Each
                // 128-column block's sum is scaled once.
                const int g = lane >> 2, t = lane & 3;
                for (int rt = 0; rt * 16 < drows; ++rt) {
                    const int ra = rt * 16 + g, rb = ra + 8;
                    const bool va = ra < drows, vb = rb < drows;
                    const uint8_t* wa = wr + (size_t)(va ? ra : 0) * iu + 16 * t;
                    const uint8_t* wb = wr + (size_t)(vb ? rb : 0) * iu + 16 * t;
                    const float* sca = sc + (size_t)(((o_lo + (va ? ra : 0)) >> 7) - rb0) * nbpI;
                    const float* scb = sc + (size_t)(((o_lo + (vb ? rb : 0)) >> 7) - rb0) * nbpI;
                    const uint32_t* hbc = hb + (g == 1 ? nw2 : 0) + 8 * t;
                    float acca = 0.0f, accb = 0.0f;
                    for (int kb = 0; kb < (iu >> 7); ++kb) {
                        float cc[4][4] = {};
#pragma unroll
                        for (int k64 = 0; k64 < 2; ++k64) {
                            const int kbase = kb * 128 + k64 * 64;
                            const uint4 xa = va ? *reinterpret_cast<const uint4*>(wa + kbase) : make_uint4(0u, 0u, 0u, 0u);
                            const uint4 xb = vb ? *reinterpret_cast<const uint4*>(wb + kbase) : make_uint4(0u, 0u, 0u, 0u);
                            const uint4 b01 = g < 2 ? *reinterpret_cast<const uint4*>(hbc + (kbase >> 1)) : make_uint4(0u, 0u, 0u, 0u);
                            const uint4 b23 = g < 2 ? *reinterpret_cast<const uint4*>(hbc + (kbase >> 1) + 4) : make_uint4(0u, 0u, 0u, 0u);
                            const uint32_t av[4] = {xa.x, xa.y, xa.z, xa.w}, bw[4] = {xb.x, xb.y, xb.z, xb.w};
                            const uint32_t h0[4] = {b01.x, b01.z, b23.x, b23.z}, h1[4] = {b01.y, b01.w, b23.y, b23.w};
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                mma_f16(cc[j], e4m3x2_to_f16x2(av[j] & 0xffffu), e4m3x2_to_f16x2(bw[j] & 0xffffu),
                                        e4m3x2_to_f16x2(av[j] >> 16), e4m3x2_to_f16x2(bw[j] >> 16), h0[j], h1[j]);
                        }
                        const float ra0 = (cc[0][0] + cc[1][0]) + (cc[2][0] + cc[3][0]);
                        const float ra1 = (cc[0][1] + cc[1][1]) + (cc[2][1] + cc[3][1]);
                        const float rb0 = (cc[0][2] + cc[1][2]) + (cc[2][2] + cc[3][2]);
                        const float rb1 = (cc[0][3] + cc[1][3]) + (cc[2][3] + cc[3][3]);
                        acca = __fmaf_rn(sca[kb], ra0 + ra1, acca);
                        accb = __fmaf_rn(scb[kb], rb0 + rb1, accb);
                    }
                    if (t == 0) {
                        if (va) dsum[(s.g_pair0[u] + q) * drows + ra] = acca * hsi;
                        if (vb) dsum[(s.g_pair0[u] + q) * drows + rb] = accb * hsi;
                    }
                }
                __syncwarp();
            }
        }
        release_packs(s, si0, NS, s.npk, pk_done, ok);
        if (!ok && lane == 0 && !s.abort) set_error(err, s, CZ_DERR_FULL_WAIT);
    }
    __syncthreads();
    if (!s.abort && drows > 0) {
        // out[t][o] = (residual) + the token's pairs in group (ascending expert) order
        for (int k = tid; k < T * drows; k += NTHREADS) {
            const int tk = k / drows, r = k - tk * drows;
            float sum = 0.0f;
            bool any = false;
            for (int rp = 0; rp < s.P; ++rp) {  // sorted pairs: groups in ascending expert order
                if (s.rtok[rp] != tk) continue;
                const float v = dsum[rp * drows + r];
                sum = any ? sum + v : v;
                any = true;
            }
            const size_t o = (size_t)tk * H + o_lo + r;
            const float v = p.residual ? __fadd_rn(p.residual[o], sum) : sum;
            if (p.ep_world > 1) {
                // this rank's partial sum goes to slot [par][ep_rank] of every rank
                const size_t w = ((size_t)((eseq & 1u) * kEpMaxRanks + p.ep_rank) * kDecodeMaxTokens + tk) *
                                     kEpMaxHidden + o_lo + r;
                const unsigned long long tw = tag_word(eseq + 1u, v);
                for (int q = 0; q < p.ep_world; ++q) st_relaxed_sys_u64(p.ep_recv[q] + w, tw);
            } else {
                p.out[o] = v;
            }
        }
        if (p.ep_world > 1) {
            // out = the ranks' partial sums added in ascending rank order (ascending
            // expert ranges), polled from this rank's own receive slots
            const uint32_t etag = eseq + 1u;
            const int W = p.ep_world;
            // a deadline, not a poll count: peers may reach this launch seconds apart
            const uint64_t t_end = global_ns() + p.ep_wait_ns;
            for (int k = tid; k < T * drows; k += NTHREADS) {
                const int tk = k / drows, r = k - tk * drows;
                const unsigned long long* src = p.ep_recv[p.ep_rank] +
                                                ((size_t)(eseq & 1u) * kEpMaxRanks * kDecodeMaxTokens + tk) *
                                                    kEpMaxHidden + o_lo + r;
                constexpr size_t RS = (size_t)kDecodeMaxTokens * kEpMaxHidden;  // between senders
                unsigned long long wv[kEpMaxRanks] = {};
                uint32_t pend = (1u << W) - 1u;
                for (uint32_t it = 0; pend; ++it) {
#pragma unroll
                    for (int q = 0; q < kEpMaxRanks; ++q)
                        if (pend & (1u << q)) wv[q] = ld_relaxed_sys_u64(src + q * RS);
#pragma unroll
                    for (int q = 0; q < kEpMaxRanks; ++q)
                        if ((pend & (1u << q)) && (uint32_t)(wv[q] >> 32) == etag) pend &= ~(1u << q);
                    if (!pend) break;
                    if ((it & 63u) == 63u && global_ns() > t_end) break;
                    __nanosleep(it < 64 ? 32 : 1024);
                }
                if (pend) {
                    atomicOr(err, CZ_DERR_EP_WAIT);
                    continue;
                }
                float sum = __uint_as_float((uint32_t)wv[0]);
#pragma unroll
                for (int q = 1; q < kEpMaxRanks; ++q)
                    if (q < W) sum = __fadd_rn(sum, __uint_as_float((uint32_t)wv[q]));
                p.out[(size_t)tk * H + o_lo + r] = sum;
            }
        }
    }

    // ---------------- completion: advance the launch sequence ----------------
    // With a status slot the last CTA to finish copies the error word there (every
    // CTA's bits are in it by then).  The sequence was advanced by CTA 0's producer.
    if (p.status_out) {
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            const uint32_t old = atomicAdd(&reg[1], 1u);
            if (old == (uint32_t)G - 1u) {
                __threadfence();
                *p.status_out = ld_relaxed_gpu(err);
            }
        }
    }
}

// ---- host side --------------------------------------------------------------

static bool g_attr_set = false;

size_t decode_smem_bytes(int T, int H, int x_bf16, int hslot) { return carve(T, H, x_bf16, hslot).total + 1024; }

// Whether a launch can keep phase D's h terms in a ring slot (carve): every group's
// term columns (at most T tokens x JX) fit one 8-column MMA tile, and on every CTA
// the packs of down rows (routed groups <= T*K, at least `per` a pack with the most
// output rows and two row blocks of scales, + one for the shared expert) leave one
// of the ring's slots unused.
int decode_hslot(int T, int H, int K, int I, int SI, int x_bf16, int num_sms) {
    if (T * (x_bf16 ? 2 : 3) > 8) return 0;
    const int ns = carve(T, H, x_bf16, 1).ns;
    const int drows = (H + num_sms - 1) / num_sms;
    const int rbytes = drows * I + 2 * cz_nbp(I) * 4;
    const int per = SLOT_BYTES / rbytes;
    if (per < 1) return 0;
    const int npk = (T * K + per - 1) / per + (SI ? 1 : 0);
    return npk <= ns - 1 ? 1 : 0;
}

int decode_max_tokens(int H, int E, int K, int I, int SI, int x_bf16, int num_sms) {
    if (K < 1 || K > MAXK || E < K || E > MAXE || H % 16 || I % 16 || SI % 16 || H < 16 || I < 16) return 0;
    if (num_sms > kMaxGrid) return 0;
    const int IM = I > SI ? I : SI;
    // scales carried with a gate/up stage: its row block of the scale table
    if ((size_t)cz_nbp(H) * 4 > (size_t)SC_BYTES) return 0;
    // phase D: a CTA's output rows of one group (+ their <= 2 row blocks of scales) fit one ring stage
    const int orows = (H + num_sms - 1) / num_sms;
    if (orows > DMR || (size_t)orows * IM + (size_t)2 * cz_nbp(IM) * 4 > (size_t)SLOT_BYTES) return 0;
    if (IM > DHW || IM % 128) return 0;  // phase D: a warp's h terms; whole 128-column blocks
    const int max_rows = (E + (SI ? 1 : 0) + num_sms - 1) / num_sms;  // router rows staged per CTA
    int t = MAXT;
    while (t > 0) {
        // gate/up MMA columns: a group holds at most t pairs, each as JX E4M3 term columns (<= 16);
        // a launch holds at most MAXSORT (token, slot) pairs
        if (t * (x_bf16 ? 2 : 3) > 16 || t * (K + (SI ? 1 : 0)) > MAXSORT) {
            --t;
            continue;
        }
        const size_t stage_r = (size_t)max_rows * H * 4 + (size_t)t * H * (x_bf16 ? 2 : 4) + (size_t)H * 4;
        const size_t lg = (size_t)t * logit_stride(E) * 4;
        if (stage_r <= (size_t)RING_BYTES && lg <= (size_t)RING_BYTES && decode_smem_bytes(t, H, x_bf16, 0) <= SMEM_LIMIT)
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
    static_assert(MAXT == 8, "one kernel instance per token count");
    static void (*const kern[MAXT])(DecodeParams) = {moe_decode_kernel<1>, moe_decode_kernel<2>, moe_decode_kernel<3>,
                                                      moe_decode_kernel<4>, moe_decode_kernel<5>, moe_decode_kernel<6>,
                                                      moe_decode_kernel<7>, moe_decode_kernel<8>};
    if (!g_attr_set) {
        for (int i = 0; i < MAXT; ++i)
            if (cudaFuncSetAttribute(kern[i], cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT) != cudaSuccess)
                return CZ_ELAUNCH;
        g_attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(NTHREADS);
    DecodeParams p = prm;
    p.hslot = decode_hslot(p.T, p.H, p.K, p.I, p.SI, p.x_bf16, num_sms);
    cfg.dynamicSmemBytes = decode_smem_bytes(p.T, p.H, p.x_bf16, p.hslot);
    cfg.stream = stream;
    // Cooperative (every CTA resident: they exchange words), and programmatic
    // dependent launch: the launch may begin while the previous kernel of the stream
    // ends (its CTAs take the SMs that kernel's CTAs leave); it reads nothing that
    // kernel writes before its griddepcontrol.wait.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern[p.T - 1], p) != cudaSuccess) return CZ_ELAUNCH;
    return CZ_OK;
}

}  // namespace cz
