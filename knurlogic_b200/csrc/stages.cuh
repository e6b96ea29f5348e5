// Host-side interfaces between the C ABI (block.cu) and the kernels
// (router.cu, expert.cu).
#pragma once

#include "common.cuh"

namespace vqmoe {

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T,
                           int H, int E, int k, float *logits, int32_t *inds, float *scores,
                           float *sgate, uint16_t *x16, int mode, const float *escale,
                           cudaStream_t stream);
vqmoe_status launch_route(const int32_t *inds, int P, int E, int32_t *cnt, int32_t *off,
                          int32_t *list, int32_t *active, int32_t *rank_scratch, uint32_t *zero,
                          int zero_words, cudaStream_t stream);
vqmoe_status launch_router_route(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T,
                                 int H, int E, int k, float *logits, int32_t *inds, float *scores,
                                 float *sgate, uint16_t *x16, int32_t *cnt, int32_t *off,
                                 int32_t *list, int32_t *active, int32_t *rank_scratch,
                                 uint32_t *zero, int zero_words, int mode, cudaStream_t stream);
vqmoe_status launch_to_f16(const uint16_t *x, uint16_t *x16, size_t n, cudaStream_t stream);
// The router's pieces, for the tensor split's router: exact logits of T
// tokens ([T][E1] float; zero2[0 .. nzero2) cleared on the way), and the
// top-k + routing sort of up to kSelectMaxTok tokens from given logits
// (cnt[0 .. E] zero on entry).
constexpr int kSelectMaxTok = 512;
vqmoe_status launch_logits(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T, int H, int E, int E1,
                           float *logits, uint16_t *x16, cudaStream_t stream, uint32_t *zero2 = nullptr,
                           int nzero2 = 0);
vqmoe_status launch_select(const float *logits, int T, int E, int E1, int k, bool has_shared, int32_t *inds,
                           float *scores, float *sgate, int32_t *cnt, int32_t *off, int32_t *list, int32_t *active,
                           int32_t *rank_scratch, uint32_t *zero, int zero_words, int mode, cudaStream_t stream);
vqmoe_status launch_rms_norm(const uint16_t *x, const uint16_t *w, int T, int H, float eps, uint16_t *out,
                             cudaStream_t stream);

// The routed experts of one stage: pairs grouped by expert (route_kernel).
struct RoutedIO {
    const int32_t *cnt, *off, *list, *active;
    int E, k, P;
    const void *x;          // fp16 rows for VQ weights, bf16 for dense
    int x_per_pair;         // 1: x row = pair, 0: x row = pair / k
    void *out;              // [P][OUT]
    int out_f16;            // fp16 (saturated) output instead of bf16
    const float *pair_scale;
    int act;                // a gate/up stage's VQMOE_ACT_*
    void *xs;               // [P][IN] fp16 scratch (the prefill path's sorted inputs), or null
};

// The prefill path (tcgen05 grouped GEMM) serves a call with VQ experts and
// at least 32 pairs per expert on average; it needs the xs scratch.
inline bool prefill_regime(bool vq, int E, int P) { return vq && E <= 512 && (long long)P >= 32LL * E; }

// Words of the expert kernel's control block: tile counter, an unused word,
// and one finished-tile count per expert. Zeroed by the routing kernel.
inline int expert_ctl_words(int E) { return 2 + E; }

// The routed experts of a layer in one launch: phase 1 = gate/up + SwiGLU
// (r1, may be null), then phase 2 = w2 (down, or the only linear) on r2.
// err: the call's status word; wait_polls: the phase 2 dependency wait's
// poll limit (0: the default, about four seconds); after_permute (optional):
// an event recorded once the prefill path's inputs are in expert order
// (right away on the decode path).
vqmoe_status launch_experts(const vqmoe_linear *gate, const vqmoe_linear *up, const RoutedIO *r1,
                            const vqmoe_linear *w2, const RoutedIO &r2, uint32_t *ctl, uint32_t *err,
                            uint32_t wait_polls, cudaStream_t stream, cudaEvent_t after_permute = nullptr);
// The tensor split's combine + float32 reduction over peer memory
// (tp_reduce.cu). base[q]: rank q's symmetric buffer as this rank addresses
// it: kTpFlagBytes of flags, then its partial [T][H] bf16, then its result
// region [T][H] bf16.
constexpr int kTpMaxRanks = 8;
constexpr size_t kTpFlagBytes = 256;
struct TpArgs {
    int rank, n;
    uint8_t *base[kTpMaxRanks];
    uint32_t *err;             // the call's status word
    uint32_t wait_polls;       // polls of each barrier wait (0: about four seconds)
    int ep_local;              // expert split: experts per rank (0: the tensor split)
};
vqmoe_status launch_tp_reduce(const uint16_t *ybuf, int T, int k, int H, const uint16_t *sh, const float *sg,
                              const TpArgs &a, uint16_t *out, cudaStream_t stream);
// The expert split (TpArgs with ep_local = E / n experts per rank): each
// rank's buffer holds kTpFlagBytes of flags, its expert outputs [T*k][H] bf16
// (the pairs of the experts it owns), then its result region [T][H] bf16.
size_t ep_buffer_bytes(int T, int k, int H);
vqmoe_status launch_ep_reduce(const int32_t *inds, int T, int k, int H, int ep_local, const uint16_t *sh,
                              const float *sg, const TpArgs &a, uint16_t *out, cudaStream_t stream);
// The split router's routing region in each rank's buffer, after the
// partial and the result: kTpRouteWords 32-bit words per token (the router's
// logits, E + 1 <= 1025 of them, or its expert ids, weights and gate), and
// the exchange that fills every rank's arrays (up to three, `widths` words
// per token each) from the ranks' row slices [r0, r1); with x16 it also
// writes the fp16 copy of x [T][H] the VQ experts read.
constexpr int kTpRouteWords = 1025;
size_t tp_route_offset(int T, int H);
size_t tp_route_bytes(int T);
vqmoe_status launch_tp_gather(void *const *arrays, const int *widths, int T, int H, int r0, int r1, uint32_t *zero,
                              int nzero, const uint16_t *x, uint16_t *x16, const TpArgs &a, cudaStream_t stream);

// The routed experts with reference-layout VQ weights (VQMOE_FMT_VQ_REF):
// phase 1 (r1, may be null) then phase 2, two launches.
vqmoe_status launch_experts_ref(const vqmoe_linear *gate, const vqmoe_linear *up, const RoutedIO *r1,
                                const vqmoe_linear *w2, const RoutedIO &r2, cudaStream_t stream);
// The shared expert's dense matmul (+ SwiGLU when w1 is set): K slicing,
// its partial buffer [ks][T][nmat][OUT] float and [ceil(OUT/32)] semaphores.
void plan_shared_dense(int IN, int OUT, int nmat, int *ks, int *kslice, size_t *smem);
// The same on tcgen05 for many tokens (IN a multiple of 64); `err` is a
// word for the kernel's bounded waits.
vqmoe_status launch_dense_prefill(const void *x, const void *w0, const void *w1, int T, int IN, int OUT,
                                  void *out, uint32_t *err, cudaStream_t stream);
vqmoe_status launch_shared_dense(const void *x, const void *w0, const void *w1, int T, int IN, int OUT,
                                 void *out, float *part, uint32_t *sem, cudaStream_t stream);

}  // namespace vqmoe
