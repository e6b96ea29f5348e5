// Host-side interfaces between the C ABI (block.cu) and the kernels
// (router.cu, expert.cu).
#pragma once

#include "common.cuh"

namespace vqmoe {

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T,
                           int H, int E, int k, float *logits, int32_t *inds, float *scores,
                           float *sgate, uint16_t *x16, cudaStream_t stream);
vqmoe_status launch_route(const int32_t *inds, int P, int E, int32_t *cnt, int32_t *off,
                          int32_t *list, int32_t *active, int32_t *rank_scratch, uint32_t *zero,
                          int zero_words, cudaStream_t stream);
vqmoe_status launch_router_route(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T,
                                 int H, int E, int k, float *logits, int32_t *inds, float *scores,
                                 float *sgate, uint16_t *x16, int32_t *cnt, int32_t *off,
                                 int32_t *list, int32_t *active, int32_t *rank_scratch,
                                 uint32_t *zero, int zero_words, cudaStream_t stream);
vqmoe_status launch_to_f16(const uint16_t *x, uint16_t *x16, size_t n, cudaStream_t stream);

// The routed experts of one stage: pairs grouped by expert (route_kernel).
struct RoutedIO {
    const int32_t *cnt, *off, *list, *active;
    int E, k, P;
    const void *x;          // fp16 rows for VQ weights, bf16 for dense
    int x_per_pair;         // 1: x row = pair, 0: x row = pair / k
    void *out;              // [P][OUT]
    int out_f16;            // fp16 (saturated) output instead of bf16
    const float *pair_scale;
    float *part;            // [ks][P][NMAT][OUT] when ks > 1
    uint32_t *sem;          // [E][row blocks]
    int ks;
};

// The shared expert of one stage: dense bf16, every token.
struct SharedIO {
    const void *x;          // [T][IN] bf16
    const void *w0, *w1;    // [OUT][IN] bf16
    int T, IN, OUT;
    void *out;              // [T][OUT] bf16
    float *part;            // [ks][T][NMAT][OUT] when ks > 1
    uint32_t *sem;          // [row blocks]
    int ks;
};

vqmoe_status launch_expert_stage(const vqmoe_linear *w0, const vqmoe_linear *w1, const RoutedIO *r,
                                 const SharedIO *s, uint32_t *work, cudaStream_t stream);
// K slices and 32-row blocks of a routed stage; K slices and 16-row blocks
// of a shared stage.
void plan_routed(int E, int P, int IN, int OUT, int *ks, int *rb);
void plan_shared(int IN, int OUT, int *ks, int *rb);
// The shared expert's dense matmul (+ SwiGLU when w1 is set): K slicing,
// its partial buffer [ks][T][nmat][OUT] float and [ceil(OUT/32)] semaphores.
void plan_shared_dense(int IN, int OUT, int nmat, int *ks, int *kslice, size_t *smem);
vqmoe_status launch_shared_dense(const void *x, const void *w0, const void *w1, int T, int IN, int OUT,
                                 void *out, float *part, uint32_t *sem, cudaStream_t stream);

}  // namespace vqmoe
