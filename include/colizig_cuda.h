/* colizig_cuda.h — C ABI of libcolizig_cuda.so, the B200 (sm_100a) backend for
 * colizig's block-FP8 MoE expert path.
 *
 * Part 1 is the reference's runtime-loaded backend surface, the six symbols
 * that src/backend/gpu.zig:84-89 resolves by name.  Each declaration names the
 * reference function it replaces (src/backend/cuda/colizig_cuda.cu).  Names,
 * argument meaning and return codes are kept; the CUDA runtime's habit of
 * changing the host MXCSR is undone on every entry, as in the reference.
 *
 * Part 2 adds MoE-level entry points.  The reference only offers a per-matrix
 * matmul, so its MoE layer (src/qwen38/moe.zig:409-426 forward) crosses the host
 * boundary ~3*topk times per token.  These calls run the whole layer — router
 * softmax/top-k, token-to-expert gather, gate/up with SiLU*mul, down, weighted
 * combine — on resident weights in one call.
 *
 * Return codes (reference convention, colizig_cuda.cu:228-284, extended):
 *    0 ok
 *   -1 bad arguments / not initialised       -2 device allocation failed
 *   -3 host->device copy failed              -4 kernel launch failed
 *   -5 device->host copy failed              -6 layer not registered
 *   -7 a device-side wait timed out (the kernel stopped early; the context is
 *      still usable and the next call starts clean)
 *   -8 shape not supported by this build     -9 NCCL / expert-parallel error
 *  -10 checkpoint file missing, unreadable or malformed, or a tensor missing
 *
 * Threading: one process-wide context, internally serialised by a mutex.
 * Ownership: callers own every buffer they pass; no pointer is retained after
 * a call returns, except that registered weights are copied into the
 * library's resident device storage.
 */
#ifndef COLIZIG_CUDA_H
#define COLIZIG_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Part 1: the reference backend surface --------------------------- */

/* colizig_cuda.cu:171-187 colizig_cuda_init.  Idempotent.  0 ok, -1 no device,
 * -2 cudaSetDevice failed, -3 properties failed, -4 device setup failed. */
int colizig_cuda_init(void);

/* colizig_cuda_init on an explicit device ordinal (one process per GPU for
 * expert parallelism).  No reference counterpart: the reference always uses
 * device 0 (colizig_cuda.cu:176). */
int colizig_cuda_init_device(int device);

/* colizig_cuda.cu:189-191.  "<name> (sm_XY, N MiB)" or "" before init. */
const char* colizig_cuda_device_name(void);

/* colizig_cuda.cu:195-202.  Capacity, in bytes, of the keyed resident weight
 * store used by colizig_cuda_matmul_fp8 (0 = keyed calls upload every time).
 * Clamped to 7/8 of the free device memory. */
void colizig_cuda_set_vram_budget(uint64_t bytes);

/* colizig_cuda.cu:204-209.  Null-safe.  hits/misses of keyed lookups, MiB of
 * weights uploaded host->device, and resident keyed matrices. */
void colizig_cuda_stats(uint64_t* hits, uint64_t* misses, uint64_t* uploaded_mib, uint64_t* resident);

/* colizig_cuda.cu:211-224.  Frees every device buffer (keyed store, MoE layers,
 * scratch, expert-parallel state) and returns to the uninitialised state. */
void colizig_cuda_shutdown(void);

/* colizig_cuda.cu:228-284 colizig_cuda_matmul_fp8.  Synchronous, host pointers.
 *   y[S,O] = x[S,I] @ (e4m3(w[O,I]) * scales[o/128, i/128])^T
 * w row-major E4M3 bytes, scales row-major [ceil(O/128), ceil(I/128)] f32
 * multipliers.  key 0 = upload w every call; otherwise the weights stay
 * resident under `key` (the moe.zig:97-99 key scheme) within the budget. */
int colizig_cuda_matmul_fp8(float* y, const float* x, const unsigned char* w, const float* scales, int S,
                            int I, int O, uint64_t key);

/* No reference counterpart: colizig_cuda_matmul_fp8 on device pointers, queued
 * on `stream` (NULL = the default stream) and returning at once; weights and
 * scales are the caller's device arrays (no keyed store).  For hosts that keep
 * activations on the GPU, e.g. the attention projections of a decoder loop
 * captured into a CUDA graph.  0, -1 (arguments), -4 (launch). */
int colizig_cuda_matmul_fp8_device(float* y, const float* x, const unsigned char* w, const float* scales, int S,
                                   int I, int O, void* stream);

/* ---- Part 2: MoE layer entry points (no reference counterpart) ---------- */

/* Mirrors moe.zig:23-30 Dims.  shared_inter == 0 -> no shared expert. */
typedef struct colizig_moe_dims {
    uint32_t hidden;
    uint32_t experts;
    uint32_t topk;
    uint32_t inter;
    uint32_t shared_inter;
    uint32_t norm_topk;
} colizig_moe_dims;

/* One expert's three projections in the reference layout (moe.zig:50-117):
 * gate/up u8 [inter, hidden] + f32 [nblk(inter), nblk(hidden)] scales, down
 * u8 [hidden, inter] + f32 [nblk(hidden), nblk(inter)]. */
typedef struct colizig_moe_expert {
    const uint8_t* gate_w;
    const float* gate_s;
    const uint8_t* up_w;
    const float* up_s;
    const uint8_t* down_w;
    const float* down_s;
} colizig_moe_expert;

/* flags */
#define COLIZIG_PTR_DEVICE 1u /* every data pointer is a device pointer; the call is
                                 asynchronous on `stream` (else: host pointers,
                                 synchronous, like colizig_cuda_matmul_fp8) */

#define COLIZIG_EP 2u /* register_layer: hold only this rank's experts (expert parallelism,
                         after colizig_cuda_ep_init); every forward of the layer then sums
                         the ranks' outputs on `stream`: inside the decode kernel for
                         decode batches (see colizig_cuda_ep_combine_mode), else with one
                         NCCL all-reduce */

#define COLIZIG_EP_SHARDED 4u /* moe_forward / moe_stack_forward on COLIZIG_EP layers: x (h)
    holds this rank's own tokens (T may differ between ranks, 0 included) and
    out/topk are for them; the ranks exchange token rows and partial sums with
    NCCL send/recv (expert-parallel prefill).  Every rank of the group makes the
    call.  Layers with a shared expert are not supported here (-8). */

#define COLIZIG_SHARED_BF16 8u /* register_layer: the shared expert is the reference's BF16
    NativeMatrix (src/qwen38/moe.zig:297-338, tensors.zig:65-120), as real Qwen4-Exp
    checkpoints hold it: shared->gate_w / up_w point at bf16 [shared_inter, hidden]
    and shared->down_w at bf16 [hidden, shared_inter] (raw bf16 bits, cast the
    pointers), the scale pointers are ignored.  Computed from the layer input
    (after rms in stack mode) beside the routed experts and added to out with its
    sigmoid gate; under COLIZIG_EP it is held and computed on every rank.  Not
    with COLIZIG_EP_SHARDED nor colizig_cuda_moe_forward_noalloc (-8). */

/* x dtypes */
#define COLIZIG_X_F32 0
#define COLIZIG_X_BF16 1

/* Register (or replace) MoE layer `layer`: copies the f32 router [experts,
 * hidden] and every expert's E4M3 weights and scales into resident device
 * memory (replaces moe.zig's ExpertCache / the VRAM LRU, colizig_cuda.cu:80-169).
 * shared / shared_gate describe an always-on block-FP8 shared expert whose
 * output is scaled by sigmoid(x . shared_gate) (moe.zig:467-479); both NULL
 * when dims->shared_inter == 0.  hidden, inter and shared_inter must be
 * multiples of 16; topk <= 16. */
int colizig_cuda_moe_register_layer(uint32_t layer, const colizig_moe_dims* dims, const float* router,
                                    const colizig_moe_expert* experts, const colizig_moe_expert* shared,
                                    const float* shared_gate, uint32_t flags);

int colizig_cuda_moe_unregister_layer(uint32_t layer);

/* Registers MoE layer `layer` straight from a safetensors checkpoint: the
 * reference's host indexes the shards (src/model/manifest.zig,
 * src/model/weights.zig:198-235) and loads each routed expert from the mmap on
 * demand (src/qwen38/moe.zig:251-292 loadExpert, 306-329 Layer.load); here the
 * shards are parsed and mapped once and checkpoint layer `layer_index`'s router,
 * experts and shared expert go into resident device memory in this one call.
 * Tensor names are tried as "<prefix>.<suffix>", then as the bare suffix, with
 * suffixes layers.L.mlp.gate.weight (router [E, H], F32 or BF16),
 * layers.L.mlp.experts.e.{gate,up,down}_proj.weight (F8_E4M3) and
 * .weight_scale_inv (F32, BF16 or F16 [nblk, nblk]), and for dims->shared_inter
 * > 0 layers.L.mlp.shared_expert.{gate,up,down}_proj.weight(_scale_inv)
 * (F8_E4M3; or BF16 [SI, H] / [H, SI] without scales, registered as
 * COLIZIG_SHARED_BF16) and layers.L.mlp.shared_expert_gate.weight ([H] or [1, H]).  BF16 /
 * F16 values are widened exactly to f32 (a BF16 router then gives the logits of
 * the reference's dotBf16, matmul.zig:84-110).  prefix may be NULL; flags: 0 or
 * COLIZIG_EP.  Returns 0, -10 when a shard cannot be read or parsed or a
 * tensor is missing (checked before anything else, so also without a device),
 * -8 on a dtype or shape that does not match dims, or register_layer's codes. */
int colizig_cuda_moe_load_safetensors(uint32_t layer, const char* const* shard_paths, int n_shards,
                                      const char* prefix, uint32_t layer_index, const colizig_moe_dims* dims,
                                      uint32_t flags);

/* moe.zig:409-426 forward for T tokens: out[T, hidden] f32 =
 * sum_k gate_k * down_k(silu(gate_k(x)) * up_k(x)) (+ shared expert).
 * x is [T, hidden] f32 or bf16.  topk_idx / topk_gates (nullable) receive each
 * token's router pick [T, topk] (u32 ids / f32 gates). */
int colizig_cuda_moe_forward(uint32_t layer, const void* x, int x_dtype, int T, float* out, uint32_t* topk_idx,
                             float* topk_gates, uint32_t flags, void* stream);

/* The per-layer caller of the MoE (src/qwen3moe/model.zig:227-232) over layers
 * first..first+n-1, with the attention sublayer as identity:
 *   n = rms(h, norm_w[l]) ; h += moe_l(n)        (rmsnorm.zig:32-40, eps)
 * h [T, hidden] f32 is updated in place; norm_w [n_layers, hidden] f32 or NULL
 * (all ones). */
int colizig_cuda_moe_stack_forward(uint32_t first_layer, uint32_t n_layers, const float* norm_w, float eps,
                                   float* h, int T, uint32_t flags, void* stream);

/* Expert parallelism over W GPUs of one node (one process per GPU), the
 * partition of src/qwen38/moe.zig's experts that forwardGrouped (moe.zig:637-664)
 * makes possible.  Rank r holds experts [r*E/W, (r+1)*E/W) (rank 0 also the
 * shared expert); router and top-k run replicated.  colizig_cuda_ep_unique_id
 * fills 128 bytes on one rank, the caller hands them to every rank, and every
 * rank calls colizig_cuda_ep_init once (after colizig_cuda_init_device).
 * Returns -9 when NCCL (libnccl.so.2) is unavailable or fails. */
int colizig_cuda_ep_unique_id(void* id_out);
int colizig_cuda_ep_init(int rank, int world, const void* id);
int colizig_cuda_ep_shutdown(void);

/* No reference counterpart.  Deadline (ms) of the library's host waits while an
 * EP communicator is active (default 60000; <= 0 waits without one).  A wait
 * that runs out, or an asynchronous NCCL error, aborts the communicator
 * (ncclCommAbort: its kernels return) and the call returns -9; every EP call
 * then returns -9 until colizig_cuda_ep_shutdown and colizig_cuda_ep_init. */
int colizig_cuda_ep_set_timeout(int ms);

/* No reference counterpart.  Abort the EP communicator now, as the deadline
 * does (for a host watchdog that learned between steps that a peer has left).
 * No device work; returns 0. */
int colizig_cuda_ep_abort(void);

/* No reference counterpart (the reference runs on one process).  How
 * expert-parallel decode calls (replicated tokens, fewer than 32 per call) sum
 * the ranks' outputs.  colizig_cuda_ep_init maps every rank's receive buffer
 * into every other rank (CUDA IPC, up to 8 ranks); when all ranks succeed, the
 * decode kernel itself stores its partial output rows into every rank's buffer
 * and adds the ranks' rows in ascending rank order, with no NCCL call.
 * Otherwise, and for prefill-sized batches, one NCCL all-reduce sums them.
 * colizig_cuda_ep_combine_mode returns 1 (in the kernel) or 0 (NCCL);
 * colizig_cuda_ep_set_combine(0 or 1) chooses; every rank must choose the same
 * before its next EP call.  The kernel waits for a peer's rows as long as the
 * host waits for a collective (colizig_cuda_ep_set_timeout, 60 s by default);
 * rows that never arrive make the call (or colizig_cuda_moe_check) return -7. */
int colizig_cuda_ep_combine_mode(void);

/* No reference counterpart.  How many tokens one decode launch of registered
 * layer `layer` takes for x_dtype (COLIZIG_X_F32 / COLIZIG_X_BF16): a call of T
 * tokens below the prefill size (32) runs ceil(T / n) decode launches.  0 when
 * the layer is unknown.  For hosts that budget launches (and the benchmark). */
int colizig_cuda_moe_decode_batch(uint32_t layer, int x_dtype);
int colizig_cuda_ep_set_combine(int in_kernel);

/* Device-side error word of the last asynchronous call(s) on the library's
 * MoE scratch (0 = none); reading it synchronises `stream` (NULL = the default
 * stream, as in the device-pointer forward) and clears it.  Returns 0, or -7
 * when a bounded wait in a kernel gave up since the last read. */
int colizig_cuda_moe_check(void* stream);

/* No counterpart in the reference.  The same computation as
 * colizig_cuda_moe_forward with COLIZIG_PTR_DEVICE (device pointers, async on
 * `stream`), for callers that must not allocate device memory during a call:
 * an engine that has already handed all of HBM to its own pool or to
 * colizig_cuda_set_vram_budget, or a decode loop where a cudaMalloc/cudaFree
 * (which synchronises the device) would stall every stream.  The scratch lives
 * in one static device array of 574,336 bytes inside the library, so no
 * call allocates.  Limits: hidden <= 4096, experts <= 512, topk <= 16,
 * moe_intermediate and shared_intermediate <= 1024, a device of at most 160 SMs (launches of up to 4 tokens; larger T runs as
 * several launches); a layer beyond
 * them returns -8 before anything is launched.  The FIRST call on a device does set-up (it looks up the
 * scratch address and configures the kernel), so make it before any stream
 * capture.  The scratch is shared: calls whose executions overlap (two
 * streams, two threads) race on it and give wrong results; serialise them.
 * Only the scratch's sync words must start at zero; static storage is zero
 * when the library loads and every call leaves them ready for the next.
 * status (nullable, device u32): after the launches the call's device error
 * word is copied there (0 = ok; non-zero = a bounded wait in the kernel gave
 * up and the outputs are invalid), then cleared.  With a NULL status the word
 * is kept, so a wait that gave up is reported by the next call that passes a
 * status.  T == 0 launches nothing.  colizig_cuda_shutdown forgets the
 * scratch address, so the first call after a new init (for instance after the
 * host application reset the device) is a set-up call again. */
int colizig_cuda_moe_forward_noalloc(uint32_t layer, const void* x, int x_dtype, int T, float* out,
                                     uint32_t* topk_idx, float* topk_gates, uint32_t* status, void* stream);

/* No counterpart in the reference: a kernel timer for benchmarks.
 * colizig_cuda_kernel_timer(capacity > 0) arms it with room for `capacity`
 * launch pairs (and clears it); capacity 0 turns it off.  While armed, every
 * MoE forward records a CUDA event pair around each decode kernel launch and
 * around each of the two grouped GEMM launches of a prefill forward; the
 * records are external event nodes when the forward is captured into a CUDA
 * graph, so graph replays are timed too; so does every colizig_cuda_matmul_fp8
 * call around its kernel.  colizig_cuda_kernel_timer_read waits for the events
 * and writes, per recorded pair, its kind (1 decode kernel, 2 prefill gate/up
 * GEMM, 3 prefill down GEMM, 4 per-matrix block-FP8 matmul) and device time in
 * ms; it
 * returns the number of pairs written, or -2 when pairs were dropped because
 * the timer was full. */
int colizig_cuda_kernel_timer(int capacity);
int colizig_cuda_kernel_timer_read(int* kinds, float* ms, int max_n);

/* Diagnostics used by the parity tests: the router's exp (the reference's
 * @exp(f32) restated in double precision) over n device floats. */
int colizig_cuda_debug_expf(const float* x_dev, float* y_dev, size_t n);

/* Failure-path test hook, no reference counterpart.  Arms a one-shot hold for
 * the next decode launch: router row 0's logits are never published, so every
 * CTA's bounded wait for them gives up after spin_limit polls (about 0.2 us
 * each) and the call reports -7 (or the no-allocation call's status is
 * non-zero).  Nothing faults or hangs; the next call starts clean.  0 ok, -1
 * not initialised or spin_limit == 0. */
int colizig_cuda_debug_hold_router(uint32_t spin_limit);

/* Diagnostics (no reference counterpart): the device error word's bits as they
 * stand once all device work so far has finished, not cleared (1 router wait,
 * 2/4 ring waits, 8 h-row wait, 16 drain, 32 shape, 64 sequence, 128 a peer
 * rank's partial sums).  0 before any MoE call. */
int colizig_cuda_debug_error_bits(uint32_t* bits);

/* Test hook for the watched host wait (colizig_cuda_ep_set_timeout), over
 * caller-provided fakes: query(ctx) 0 done, 1 pending, < 0 failed;
 * async_error(ctx) non-zero = the communicator reports an error; abort_comm(ctx)
 * is called once when the wait gives up.  Returns 0, -5 (query failed) or -9
 * (aborted: deadline or error); -1 for a null callback. */
int colizig_cuda_debug_watch_wait(int (*query)(void*), int (*async_error)(void*), void (*abort_comm)(void*),
                                  void* ctx, int timeout_ms);

#ifdef __cplusplus
}
#endif
#endif
