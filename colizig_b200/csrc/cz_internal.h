// Host/device shared definitions of the colizig B200 library (not part of the
// public C ABI; see include/colizig_cuda.h for that).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cz {

constexpr int kDecodeMaxTokens = 8;   // per decode launch (one kernel instance per count; tokens sharing an expert read its rows once)
constexpr int kMaxTopk = 16;
constexpr int kMaxExperts = 512;
constexpr int kMaxGrid = 160;         // decode CTAs (one per SM) the no-allocation scratch is sized for
constexpr int kSyncRegionWords = 8;   // [1] = CTAs done (the other words are unused padding)
constexpr int kSyncWords = 2 + 2 * kSyncRegionWords;  // seq, err, two regions
// Expert-parallel decode with the ranks' partial outputs summed inside the decode
// kernel (peer stores over NVLink): at most this many ranks and this hidden size.
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxHidden = 8192;
// Receive buffer of that combine, per rank: a 256-byte header (word 0 = the EP
// launch counter) and [2 parities][kEpMaxRanks senders][kDecodeMaxTokens][kEpMaxHidden]
// tagged words.
constexpr size_t kEpRecvHeader = 256;
constexpr size_t kEpRecvWords = (size_t)2 * kEpMaxRanks * kDecodeMaxTokens * kEpMaxHidden;
constexpr size_t kEpRecvBytes = kEpRecvHeader + kEpRecvWords * 8;

__host__ __device__ inline int cz_nblk(int x) { return (x + 127) / 128; }
// Row stride (floats) of the router-logit scratch: E experts + the shared
// expert's gate, rounded up to 4 floats (rows start on 16-byte boundaries).
__host__ __device__ inline int logit_stride(int E) { return (E + 1 + 3) & ~3; }
// Row length (floats) of a resident block-scale table: nblk rounded up to 4, so
// every row starts on a 16-byte boundary.
__host__ __device__ inline int cz_nbp(int x) { return (cz_nblk(x) + 3) & ~3; }

// Everything the decode kernel reads or writes; passed by value (a
// __grid_constant__ kernel parameter, so the tensor maps can be used in place).
struct alignas(64) DecodeParams {
    CUtensorMap gate_map;     // gate_w u8 [E*I rows][H]: boxes of 16 rows x 128 columns (x gu_kb blocks), 128-byte swizzle
    CUtensorMap up_map;
    CUtensorMap sh_gate_map;  // shared expert [SI rows][H] (SI > 0)
    CUtensorMap sh_up_map;
    int gu3d, gu_kb;          // gate/up boxes span gu_kb 128-column blocks (3D map) or one (2D map)
    int hslot;                // phase D's h terms in a free ring slot (set by decode_launch)
    const void* x;           // [T, H] f32 or bf16 (stack mode: h, f32)
    int x_bf16;
    int T;
    const float* rms_w;      // stack mode: rmsnorm weight [H] (else null)
    float eps;
    const float* residual;   // stack mode: h (out = residual + moe) (else null)
    float* out;              // [T, H] f32
    uint32_t* topk_idx;      // [T, K] or null
    float* topk_gates;       // [T, K] or null
    const float* router;     // [E, H]
    const uint8_t* gate_w;   // [E, I, H]
    const uint8_t* up_w;     // [E, I, H]
    const uint8_t* down_w;   // [E, H, I]
    const float* gate_s;     // [E, nb(I), nbp(H)]  (rows padded to 4 floats)
    const float* up_s;
    const float* down_s;     // [E, nb(H), nbp(I)]
    const uint8_t* sh_gate_w;  // shared expert (SI > 0)
    const uint8_t* sh_up_w;
    const uint8_t* sh_down_w;
    const float* sh_gate_s;
    const float* sh_up_s;
    const float* sh_down_s;
    const float* sh_gate;    // [H]
    int H, E, K, I, SI, norm_topk;
    int e_lo, e_hi;          // routed experts held (and computed) here: [e_lo, e_hi); stacked from e_lo
    int shared_here;         // the shared expert is computed here
    // Tagged exchange words: (tag << 32) | f32 bits, tag = launch sequence + 1.  A
    // reader polls a word until it carries the current tag, so the data itself is
    // the flag (no grid counter, no fence); both buffers are zeroed at allocation.
    unsigned long long* logits;  // scratch [kDecodeMaxTokens, logit_stride(E)]: router logits
    unsigned long long* hrows;   // scratch [T*(K+1)][max(I, SI)]: the h row of every (token, expert) pair
    uint32_t* sync;          // kSyncWords words, zeroed once at allocation
    uint32_t* status_out;    // nullable: the last CTA copies the device error word here
    uint32_t spin_limit;     // polls before a wait gives up (0 = CZ_SPIN_LIMIT)
    int dbg_hold;            // failure-path tests: router row 0's logits are never published
    // Expert parallelism with replicated tokens, ranks summed in the kernel
    // (ep_world > 1; else 0 and out is this rank's own sum).  Each CTA stores its
    // output rows' partial sums as tagged words (tag = EP launch counter + 1) into
    // slot [par][ep_rank] of every rank's receive buffer (peer-mapped), then polls
    // slots [par][0..ep_world) of its own and adds them in ascending rank order;
    // par = counter & 1.  The counter advances once per such launch on every rank.
    unsigned long long* ep_recv[kEpMaxRanks];  // word 0 of each rank's slot area (header skipped)
    uint32_t* ep_seq;        // this rank's EP launch counter (receive buffer header)
    int ep_world, ep_rank;
    uint64_t ep_wait_ns;     // how long a CTA waits for the peers' rows before it gives up
};

// Bytes of the decode kernel's tagged scratch for these dims (logits, h rows).
inline size_t decode_logit_words(int E) { return (size_t)kDecodeMaxTokens * logit_stride(E); }
inline size_t decode_hrow_words(int K, int I, int SI) {
    return (size_t)kDecodeMaxTokens * (K + 1) * (size_t)(I > SI ? I : SI);
}

// Decode-kernel tensor map of gate/up weights: u8 [rows][H] in 128-byte-swizzled
// boxes of 16 rows x 128 columns, up to 16 column blocks deep when H % 128 == 0
// (*kb = depth, else 0 = 2D).
bool make_gu_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t H, int* kb);

size_t decode_smem_bytes(int T, int H, int x_bf16, int hslot);
int decode_hslot(int T, int H, int K, int I, int SI, int x_bf16, int num_sms);
// Largest token count one decode launch takes for these dims (tokens and the
// gate/up outputs must fit the kernel's shared staging area); 0 = unsupported.
int decode_max_tokens(int H, int E, int K, int I, int SI, int x_bf16, int num_sms);
int decode_launch(const DecodeParams& p, int num_sms, cudaStream_t stream);

// ---- prefill: token batches on tcgen05 grouped GEMMs (moe_prefill.cu) ----

// One layer's weights as the prefill kernels see them (experts [e_lo, e_hi)
// held here, stacked from e_lo; the shared expert when shared_here).
struct PrefillLayer {
    CUtensorMap gate_map, up_map;  // u8 [(e_hi-e_lo)*I][H], box 128 x 128, 128-byte swizzle
    CUtensorMap down_map;          // u8 [(e_hi-e_lo)*H][I], box 128 x 128, 128-byte swizzle
    CUtensorMap sh_gate_map, sh_up_map, sh_down_map;  // shared expert (SI x H, H x SI)
    const float *router, *sh_gate;
    const float *gate_s, *up_s, *down_s;  // [EL][nb(I)][nbp(H)], [EL][nb(H)][nbp(I)]
    const float *sh_gate_s, *sh_up_s, *sh_down_s;
    int H, E, K, I, SI, norm_topk, e_lo, e_hi, shared_here;
};

// Whether the prefill path takes these dims (multiples of 128, sizes it was built for).
bool prefill_supported(int H, int E, int K, int I, int SI);
// Scratch bytes one prefill call of T tokens needs.
size_t prefill_scratch_bytes(int T, int H, int E, int K, int I, int SI, int num_sms);
// A u8 [rows][cols] tensor map, box 128 cols x box_rows rows, 128-byte swizzle.
bool make_sw128_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// out[T, H] (+ residual) = MoE(x) for a batch of T tokens; x f32 or bf16
// (rms_w: x = rms(x, rms_w), eps).  topk_idx / topk_gates nullable.  err = the
// device error word.  Stream-ordered; the scratch stays in use until the
// stream reaches the end of the call.
// Records a timer event on `st`: an external event-record node when the stream
// is being captured into a CUDA graph (so every replay re-records it), a plain
// record otherwise.
inline bool record_timer_event(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) return false;
    return (cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal)
                                                : cudaEventRecord(ev, st)) == cudaSuccess;
}

int prefill_run(const PrefillLayer& L, const void* x, int x_bf16, int T, const float* rms_w, float eps,
                const float* residual, float* out, uint32_t* topk_idx, float* topk_gates, void* scratch,
                size_t scratch_bytes, uint32_t* err, int num_sms, cudaStream_t st,
                cudaEvent_t* gemm_ev = nullptr, const uint32_t* pre_idx = nullptr, const float* pre_gates = nullptr);
// The routing part alone: idx/gates [T][K] of T tokens (stack mode: xn = rms(x, rms_w), f32 [T][H]).
int prefill_route(const PrefillLayer& L, const void* x, int x_bf16, int T, const float* rms_w, float eps,
                  uint32_t* idx, float* gates, float* xn, void* scratch, size_t scratch_bytes, cudaStream_t st);

// Expert parallelism with sharded tokens (moe_ep.cu).  Rank r holds experts
// [r*E/W, (r+1)*E/W).  ep_plan: per token the W destination slots (-1 = not sent)
// in a send buffer ordered by destination then token, and the W row counts.
int ep_plan(const uint32_t* idx, int T, int K, int E, int W, int* slot, int* counts, void* tmp, size_t tmp_bytes,
            cudaStream_t st);
// Rows of the send buffer: [H x elt bytes of the token row][K u32 ids][K f32 gates], stride rs bytes.
int ep_pack(const void* x, size_t xrow_bytes, const uint32_t* idx, const float* gates, int T, int K, int W,
            const int* slot, uint8_t* send, size_t rs, cudaStream_t st);
// Received rows -> contiguous x [R][H], idx [R][K], gates [R][K].
int ep_unpack(const uint8_t* recv, size_t rs, int R, size_t xrow_bytes, int K, void* x, uint32_t* idx, float* gates,
              cudaStream_t st);
// out[t] = residual[t] + sum over destinations d (ascending) of back[slot[t][d]] (f32 [.][H]).
int ep_combine(const float* back, const int* slot, int T, int W, int H, const float* residual, float* out,
               cudaStream_t st);

// BF16 shared expert (moe_shared_bf16.cu), for layers whose shared expert is the
// reference's BF16 NativeMatrix (moe.zig:297-338).  gate_up: hsh[T][SI] =
// silu(x.Wg)*(x.Wu) and sg[T] = sigmoid(x.sh_gate), x rms-normalised when rms_w;
// else out[T][H] += sg * (hsh . Wd).  Stream-ordered.
struct ShbParams {
    const void* x;            // [T][H] f32 or bf16
    int x_bf16, T, H, SI;
    const float* rms_w;       // stack mode: rmsnorm weight [H] (else null)
    float eps;
    const uint16_t *wg, *wu;  // bf16 [SI][H]
    const uint16_t* wd;       // bf16 [H][SI]
    const float* sh_gate;     // [H]
    float* hsh;               // scratch [T][SI]
    float* sg;                // scratch [T]
    float* out;               // [T][H]
};
bool shb_supported(int H, int SI);
size_t shb_scratch_bytes(int T, int SI);  // hsh, then sg at a 256-byte boundary
int shb_launch(const ShbParams& p, bool gate_up, cudaStream_t st);

// Legacy per-matrix block-FP8 matmul (device pointers, stream-ordered).
int fp8_matmul_launch(float* y, const float* x, const uint8_t* w, const float* scales, int S, int I, int O,
                      cudaStream_t stream);

int debug_expf_launch(const float* x, float* y, size_t n, cudaStream_t stream);

}  // namespace cz
