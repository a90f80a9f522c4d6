/* Native caller loop for benchmarks: times host-pointer MoE forwards through the
 * library's C ABI the way a compiled host (the reference's Zig program,
 * src/backend/gpu.zig) calls it, without an interpreter between the calls.
 * The caller passes the entry point (colizig_cuda_moe_forward) as a function
 * pointer, so this file links against nothing but libc. */
#include <stdint.h>
#include <time.h>

typedef int (*cz_forward_fn)(uint32_t layer, const void* x, int x_dtype, int T, float* out, uint32_t* topk_idx,
                             float* topk_gates, uint32_t flags, void* stream);

/* n synchronous forwards, layer i % nl on tokens xs[i % nx]; returns the elapsed
 * seconds (CLOCK_MONOTONIC), or a negative value after a failed call, whose
 * code is written to *rc. */
__attribute__((visibility("default"))) double cz_hostbench_forwards(void* fn, int n, const uint32_t* layers, int nl,
                                                                    const void* const* xs, int nx, int dtype, int T,
                                                                    float* out, uint32_t* idx, float* gates, int* rc) {
    cz_forward_fn f = (cz_forward_fn)fn;
    struct timespec a, b;
    *rc = 0;
    clock_gettime(CLOCK_MONOTONIC, &a);
    for (int i = 0; i < n; ++i) {
        const int r = f(layers[i % nl], xs[i % nx], dtype, T, out, idx, gates, 0u, (void*)0);
        if (r) {
            *rc = r;
            return -1.0;
        }
    }
    clock_gettime(CLOCK_MONOTONIC, &b);
    return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}
