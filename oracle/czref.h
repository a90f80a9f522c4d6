/* czref — CPU restatement of colizig's block-FP8 MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity oracle and the timed
 * CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it; the product library
 * (libcolizig_cuda.so) never links or calls it.
 *
 * Every function restates a reference function (paths relative to the
 * colizig source tree):
 *   czref_e4m3_lut        src/ops/fp8.zig:29-64    (decodeE4M3, e4m3_lut)
 *   czref_dequant_row     src/ops/fp8.zig:80-130   (decodeLane, dequantRow)
 *   czref_dot_fp8_row     src/ops/fp8.zig:137-160  (dotFp8Row, 2 chains x 8 lanes)
 *   czref_matmul_fp8      src/ops/fp8.zig:215-257  (matmulFp8Cpu)
 *   czref_dot_f32         src/ops/matmul.zig:60-82 (dotF32, 4 chains x 8 lanes)
 *   czref_matmul_f32      src/ops/matmul.zig:21-33 (matmul)
 *   czref_sigmoid/silu    src/ops/activation.zig:8-20
 *   czref_set_threads     src/runtime/parallel.zig:50-76 (enable/disable/chunks)
 *   czref_rms             src/ops/rmsnorm.zig:32-40
 *   czref_route           src/qwen38/moe.zig:435-463
 *   czref_moe_forward     src/qwen38/moe.zig:409-426, 481-539 (dense), 597-665 (grouped),
 *                         467-479 (shared expert)
 *
 * The vector width is the reference box's AVX2 width, L = 8 f32 lanes
 * (std.simd.suggestVectorLength on an AVX2 target).  Zig's default float mode is
 * strict: `a + b*c` is a multiply and an add (two roundings) and only @mulAdd is
 * fused; @reduce(.Add) on floats sums lanes 0..L-1 in order.  This file is built
 * with -ffp-contract=off and uses fmaf()/FMA intrinsics exactly where the
 * reference uses @mulAdd.
 *
 * Zig's @exp(f32) is restated by czref_expf: a double-precision Cody-Waite
 * reduction plus a degree-13 Taylor polynomial, rounded once to f32 (error far
 * below half an f32 ulp, i.e. correctly rounded except in vanishingly rare
 * midpoint cases).  The CUDA router evaluates the identical sequence of IEEE
 * double operations, so top-k parity against this oracle is bit-exact.
 */
#ifndef CZREF_H
#define CZREF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    size_t hidden;
    size_t experts;
    size_t topk;
    size_t inter;
    size_t shared_inter; /* 0 = no shared expert (Qwen3-MoE) */
    int norm_topk;
} czref_dims;

/* One MoE layer's weights, reference layout (moe.zig:50-117, 297-338).
 * Per expert e: gate_w[e] u8 [inter, hidden] E4M3, gate_s[e] f32
 * [nblk(inter), nblk(hidden)]; up likewise; down_w[e] u8 [hidden, inter],
 * down_s[e] f32 [nblk(hidden), nblk(inter)].
 * The shared expert (optional) is an always-on block-FP8 expert with the
 * reference's sigmoid gate vector sh_gate [hidden]; when sh_gate_bf16 is set it
 * is instead the reference's BF16 NativeMatrix shared expert (moe.zig:297-338,
 * tensors.zig:65-120): sh_{gate,up}_bf16 [shared_inter, hidden] and
 * sh_down_bf16 [hidden, shared_inter] raw bf16 bits, run through dotBf16. */
typedef struct {
    const float* router; /* [experts, hidden] f32 */
    const uint8_t* const* gate_w;
    const float* const* gate_s;
    const uint8_t* const* up_w;
    const float* const* up_s;
    const uint8_t* const* down_w;
    const float* const* down_s;
    const uint8_t* sh_gate_w;
    const float* sh_gate_s;
    const uint8_t* sh_up_w;
    const float* sh_up_s;
    const uint8_t* sh_down_w;
    const float* sh_down_s;
    const float* sh_gate; /* [hidden] */
    const uint16_t* sh_gate_bf16;
    const uint16_t* sh_up_bf16;
    const uint16_t* sh_down_bf16;
} czref_layer;

size_t czref_nblk(size_t x);
void czref_e4m3_lut(float out[256]);
float czref_expf(float x);
void czref_expf_n(const float* x, float* y, size_t n);
float czref_sigmoid(float x);
float czref_silu(float x);
void czref_dequant_row(float* out, const uint8_t* w, const float* scale_row, size_t n);
float czref_dot_fp8_row(const float* x, const uint8_t* w, const float* scale_row, size_t n);
float czref_dot_f32(const float* a, const float* b, size_t n);
void czref_matmul_f32(float* y, const float* x, const float* w, size_t S, size_t I, size_t O);
float czref_dot_bf16(const float* a, const uint16_t* b, size_t n);
void czref_matmul_bf16(float* y, const float* x, const uint16_t* w, size_t S, size_t I, size_t O);
void czref_matmul_fp8(float* y, const float* x, const uint8_t* w, const float* scales,
                      size_t S, size_t I, size_t O);

void czref_rms(float* out, const float* x, const float* w, size_t n, float eps);

/* parallel.enable(io, n) for n > 1, parallel.disable() for n <= 1.
 * Results are bit-identical for every thread count. */
void czref_set_threads(int n);
int czref_get_threads(void);

/* route() for one token: idx[K] expert ids, gates[K]. */
void czref_route(const czref_layer* L, const czref_dims* d, const float* xs,
                 uint32_t* idx, float* gates);

/* forward(): S == 1 -> forwardDense, S > 1 -> forwardGrouped.
 * x [S, hidden] f32 -> out [S, hidden] f32.  idx_out/gates_out (nullable)
 * receive every token's top-k pick [S, topk].  Returns 0, or -1 on bad args. */
int czref_moe_forward(const czref_layer* L, const czref_dims* d, const float* x, size_t S,
                      float* out, uint32_t* idx_out, float* gates_out);

#ifdef __cplusplus
}
#endif
#endif
