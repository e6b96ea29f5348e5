/*
 * vqmoe.h -- C ABI of the B200 VQ-MoE expert layer (libvqmoe.so).
 *
 * Drop-in for the expert path of Knurlogic's Qwen3.5-MoE sparse block with
 * VQ-quantised experts. Every entry point takes plain device pointers,
 * sizes and a cudaStream_t (passed as void*), allocates no device memory
 * (callers pass a workspace sized by the *_workspace_size queries), never
 * throws, and returns a vqmoe_status. Every call only enqueues work on
 * `stream` (no host synchronisation).
 *
 * Reference interfaces each entry point replaces (paths inside the
 * Knurlogic project):
 *   vqmoe_sparse_moe_block  SparseMoeBlock.__call__
 *       src/knurlogic/engine/families/qwen/architecture/qwen3_5.py:170-192
 *   vqmoe_switch_glu        SwitchGLU.__call__
 *       .../glm5_next/_mlx_vlm/models/switch_layers.py:172-193
 *   vqmoe_switch_linear     VQSwitchLinear.__call__ (artifact model.py; the
 *       contract is engine/families/deepseek/heads/deepseek_v4.py:77-130)
 *       and SwitchLinear.__call__ (switch_layers.py:116-125) for bf16 experts
 *   vqmoe_router            the router lines qwen3_5.py:174-179 (+ the
 *       shared_expert_gate Linear of qwen3_5.py:186)
 *   vqmoe_dequant           the VQ runtime's dense fp16 expert decode
 *       (src/knurlogic/tuning/measured.py:21-33, VQ_DECODE_CHUNK)
 *   vqmoe_prepare_vq        loading VQSwitchLinear.codes / .vq_scales
 *       (deepseek_v4.py:111-130 layout) into the device layout the kernels
 *       read
 *   vqmoe_sparse_moe_block_tp  the tensor-split block with its Reduce
 *       (src/knurlogic/engine/split/tensor.py:159-187) fused over NVLink
 *       peer memory; vqmoe_sparse_moe_block_ep the same block with whole
 *       experts split by id (no counterpart in the reference)
 *   vqmoe_add_rms_norm      the decoder's residual add + RMSNorm
 *       (qwen3_5.py:120-130, 578-587)
 *
 * Numerics (matching the reference's rounding order, qwen3_5.py:35-40,
 * 108-112, 170-192): bf16 matmul outputs; fp32 softmax / top-k /
 * renormalisation with weights rounded to bf16; silu / sigmoid in fp32
 * rounded once; the top-k sum in fp32 rounded once. VQ weights dequantise
 * to W = fp16(f32(codebook[code][j]) * f32(vq_scale)) (vqmoe_dequant, bit
 * for bit, on every expert path: decode, prefill and the reference-layout
 * kernel) and the VQ matmul takes the bf16 activations as fp16 (saturated
 * at +-65504), with fp16 x fp16 products accumulated in fp32.
 */
#ifndef VQMOE_H_
#define VQMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 2: vqmoe_linear.activation (was reserved), vqmoe_block.router_mode and
 * its trailing reserved word, vqmoe_router_ex, vqmoe_moe_experts.
 * 3: vqmoe_block.wait_polls (was reserved), vqmoe_workspace_status; every
 * workspace starts with VQMOE_STATUS_BYTES of status words.
 * 4: vqmoe_linear.biases / .bits / .reserved (affine-quantized experts,
 * VQMOE_FMT_AFFINE). */
#define VQMOE_ABI_VERSION 4

#if defined(__GNUC__)
#define VQMOE_API __attribute__((visibility("default")))
#else
#define VQMOE_API
#endif

typedef enum {
    VQMOE_OK = 0,
    VQMOE_BAD_SHAPE = 1,         /* a size is out of range or does not divide */
    VQMOE_BAD_FORMAT = 2,        /* unknown weight format / unsupported dim, K */
    VQMOE_BAD_POINTER = 3,       /* null or misaligned pointer */
    VQMOE_WORKSPACE_TOO_SMALL = 4,
    VQMOE_BAD_CODE = 5,          /* a VQ code >= codebook size */
    VQMOE_LAUNCH_FAILED = 6,     /* a CUDA launch or call returned an error */
    VQMOE_TIMEOUT = 7,           /* a bounded device wait ran out (vqmoe_workspace_status) */
    VQMOE_NOT_SUPPORTED = 8
} vqmoe_status;

/* Weight formats of one switch (expert) linear. */
enum {
    VQMOE_FMT_DENSE_BF16 = 0,    /* weight [E, OUT, IN] bf16 (SwitchLinear) */
    VQMOE_FMT_VQ_U8 = 1,         /* codes and scales in the device layout
                                    (vqmoe_prepare_vq); codebook [K, dim] fp16
                                    (the reference's, shared by all experts) */
    VQMOE_FMT_VQ_REF = 2,        /* codes and scales in the reference layout
                                    (deepseek_v4.py:111-130): codes [E, OUT,
                                    IN/dim], one code per entry, uint8 when
                                    K <= 256, uint16 above; vq_scales [E, OUT,
                                    IN/group]; codebook [K, dim] fp16 with dim
                                    2, 4 or 8, K <= 65536 (the wider formats
                                    the tiled fast path does not take) */
    VQMOE_FMT_AFFINE = 3         /* affine-quantized experts, mlx-lm's
                                    QuantizedSwitchLinear (switch_layers.py:
                                    24-86, mx.gather_qmm mode "affine"):
                                    weight [E, OUT, IN*bits/32] uint32, each row
                                    a little-endian bit stream of `bits`-bit
                                    values q (element j at bits [j*bits,
                                    (j+1)*bits)); scales and biases [E, OUT,
                                    IN/group] bf16; W = bf16(fmaf(scale, q,
                                    bias)); activations stay bf16 */
};

/* One switch linear: y[r] = x[r] @ W[expert(r)]^T, W [E, OUT, IN].
 * Mirrors VQSwitchLinear(codes, codebook, vq_scales, group_size=,
 * pack_bits=0) (deepseek_v4.py:126-130). VQ_U8: dim 4, K <= 256,
 * group_size 64, IN % 64 == 0, OUT % 16 == 0. VQ_REF: dim 2, 4 or 8,
 * K <= 65536, group_size a multiple of dim dividing IN, IN % 64 == 0,
 * OUT % 16 == 0. AFFINE (QuantizedSwitchLinear): bits 2, 3, 4, 5, 6 or 8,
 * group_size 32, 64 or 128, IN % 64 == 0, OUT % 16 == 0. A SwitchGLU's
 * three linears share one of VQ_REF and AFFINE, or use neither.
 * Dense: IN % 16 == 0, OUT % 16 == 0. Pointers 16-byte aligned. */
typedef struct {
    int32_t format;
    int32_t num_experts;
    int32_t out_features;
    int32_t in_features;
    const void *weight;          /* DENSE_BF16 */
    const void *codes;           /* VQ_U8 (device layout) */
    const void *codebook;        /* VQ_U8 */
    const void *scales;          /* VQ_U8 */
    int32_t codebook_size;       /* K */
    int32_t dim;                 /* code vector length */
    int32_t group_size;          /* inputs per vq_scales entry */
    int32_t activation;          /* on the gate linear of a SwitchGLU: VQMOE_ACT_*;
                                    0 elsewhere */
    const void *biases;          /* AFFINE: [E, OUT, IN/group] bf16 */
    int32_t bits;                /* AFFINE: 2, 3, 4, 5, 6 or 8 */
    int32_t reserved;            /* 0 */
} vqmoe_linear;

/* Activation between the gate and up projections of a SwitchGLU, set on its
 * gate linear. Both round the activation of the bf16 gate output to bf16
 * once and the product with the bf16 up output to bf16 once. */
enum {
    VQMOE_ACT_SWIGLU = 0,        /* _SwiGLU, qwen3_5.py:108-112: silu in fp32 */
    VQMOE_ACT_GEGLU = 1          /* geglu, gemma4_text.py:131-135 (GeGLU
                                    186-189): gelu's tanh form in fp32 */
};

/* Router variants: how the k weights come from the logits (the top-k
 * itself is always by descending logit, ties to the lower expert). */
enum {
    VQMOE_ROUTER_SOFTMAX_TOPK_RENORM = 0, /* Qwen3.5, qwen3_5.py:174-179: fp32
                                             softmax over all experts, the top
                                             k renormalised in fp32 */
    VQMOE_ROUTER_TOPK_SOFTMAX = 1,        /* Qwen4-exp with norm_topk_prob,
                                             qwen4_exp.py:806-810: fp32 softmax
                                             over the k selected logits */
    VQMOE_ROUTER_SOFTMAX_TOPK = 2         /* Qwen4-exp without norm_topk_prob,
                                             qwen4_exp.py:811-814: the top-k of
                                             the fp32 softmax over all experts,
                                             not renormalised */
};

/* One Qwen3.5-MoE sparse block (qwen3_5.py:170-192). The shared expert is
 * optional (shared_inter == 0 disables it and its gate). */
typedef struct {
    int32_t hidden;              /* H */
    int32_t num_experts;         /* E (<= 512) */
    int32_t top_k;               /* k (<= 32, <= E) */
    int32_t shared_inter;        /* I_s, 0 = no shared expert */
    const void *router_w;        /* mlp.gate.weight [E, H] bf16 */
    vqmoe_linear gate;           /* mlp.switch_mlp.gate_proj [E, I, H] */
    vqmoe_linear up;             /* mlp.switch_mlp.up_proj   [E, I, H] */
    vqmoe_linear down;           /* mlp.switch_mlp.down_proj [E, H, I] */
    const void *shared_gate_w;   /* mlp.shared_expert.gate_proj [I_s, H] bf16 */
    const void *shared_up_w;     /* mlp.shared_expert.up_proj   [I_s, H] bf16 */
    const void *shared_down_w;   /* mlp.shared_expert.down_proj [H, I_s] bf16 */
    const void *shared_expert_gate_w; /* mlp.shared_expert_gate [1, H] bf16 */
    int32_t router_mode;         /* VQMOE_ROUTER_* (0: Qwen3.5) */
    int32_t wait_polls;          /* polls before a phase 2 tile gives up waiting
                                    for its expert's phase 1 tiles; 0: the
                                    default (about four seconds) */
} vqmoe_block;

/* Output dtype of vqmoe_sparse_moe_block. F32 holds the bf16 block output
 * widened to float32: the tensor split sums rank partials in float32
 * (src/knurlogic/engine/split/tensor.py:159-187). */
enum { VQMOE_OUT_BF16 = 0, VQMOE_OUT_F32 = 1 };

/* Workspace bytes for vqmoe_sparse_moe_block / vqmoe_switch_glu /
 * vqmoe_switch_linear / vqmoe_router at T tokens (host-only queries). */
VQMOE_API size_t vqmoe_block_workspace_size(const vqmoe_block *blk, int32_t tokens);
VQMOE_API size_t vqmoe_switch_glu_workspace_size(const vqmoe_linear *gate,
                                                 const vqmoe_linear *down,
                                                 int32_t tokens, int32_t top_k);
VQMOE_API size_t vqmoe_switch_linear_workspace_size(const vqmoe_linear *w,
                                                    int32_t tokens,
                                                    int32_t top_k,
                                                    int32_t x_per_pair);
VQMOE_API size_t vqmoe_router_workspace_size(int32_t tokens, int32_t num_experts);

/* SparseMoeBlock.__call__: out[T, H] = routed combine + gated shared expert.
 * x [T, H] bf16; out bf16 or f32 (out_dtype). With a shared expert, its two
 * kernels run on a side stream forked from `stream` (an event recorded on
 * `stream`) and joined back before the combine, so the call is still
 * ordered on `stream` as a whole. The side stream and its two events are
 * created by the first such call of each host thread on each device: make
 * that call before capturing `stream` into a CUDA graph. */
VQMOE_API vqmoe_status vqmoe_sparse_moe_block(const vqmoe_block *blk, const void *x,
                                    int32_t tokens, void *out,
                                    int32_t out_dtype, void *workspace,
                                    size_t workspace_bytes, void *stream);

/* vqmoe_sparse_moe_block that also records five caller-created CUDA events
 * (cudaEvent_t, passed as void*) on `stream`: before the router, then after
 * the router and routing sort, the routed experts (gate/up + SwiGLU and
 * down, one launch), the join of the shared expert's side stream, and the
 * combine. A sixth event, when n_events >= 6, is recorded between the
 * prefill path's input permute and its grouped GEMM (right after the
 * routing on the decode path). For profiling; tokens <= 2048. */
VQMOE_API vqmoe_status vqmoe_sparse_moe_block_timed(
    const vqmoe_block *blk, const void *x, int32_t tokens, void *out,
    int32_t out_dtype, void *workspace, size_t workspace_bytes, void *stream,
    void *const *events, int32_t n_events);

/* A tensor-split rank's view of its split's symmetric buffers, for
 * vqmoe_sparse_moe_block_tp: this rank, the number of ranks (<= 8), and
 * every rank's buffer (buffer_bytes >= vqmoe_tp_buffer_bytes) as this rank
 * addresses it -- peer memory over NVLink (CUDA IPC or symmetric memory).
 * The caller zeroes each buffer once, before the split's first call, and
 * has every rank see that done (a barrier) before any rank calls. */
typedef struct {
    int32_t rank;
    int32_t world;
    void *buffers[8];
    int64_t buffer_bytes;
    int32_t wait_polls;          /* polls of each cross-rank wait; 0: about four seconds */
    int32_t reserved;            /* 0 */
} vqmoe_tp;

/* Bytes of one rank's buffer for blocks of `hidden` at up to `tokens`
 * tokens per call. */
VQMOE_API size_t vqmoe_tp_buffer_bytes(int32_t hidden, int32_t tokens);

/* The tensor-split SparseMoeBlock: this rank's cut of the block (router,
 * experts, shared expert on its cut), then ONE kernel that combines the
 * rank's bf16 partial and reduces it with the other ranks' over peer memory
 * -- the float32 sum in rank order, rounded once to bf16 (Reduce,
 * src/knurlogic/engine/split/tensor.py:159-187) -- into out [T, H] bf16 on
 * every rank. Every rank of the split makes the same calls in the same
 * order (the ranks meet inside the kernel at bounded barriers; a wait that
 * runs out is reported by vqmoe_workspace_status). hidden % (8 * world)
 * == 0. */
VQMOE_API vqmoe_status vqmoe_sparse_moe_block_tp(const vqmoe_block *blk, const vqmoe_tp *tp,
                                                 const void *x, int32_t tokens, void *out,
                                                 void *workspace, size_t workspace_bytes,
                                                 void *stream);

/* vqmoe_sparse_moe_block_tp that also records five caller-created CUDA
 * events on `stream` (as vqmoe_sparse_moe_block_timed): before the router,
 * after the split router and the routing exchange and sort, after the routed
 * experts, after the join of the shared expert's side stream, and after the
 * fused combine + reduction. For profiling; tokens <= 2048. */
VQMOE_API vqmoe_status vqmoe_sparse_moe_block_tp_timed(const vqmoe_block *blk, const vqmoe_tp *tp,
                                                       const void *x, int32_t tokens, void *out,
                                                       void *workspace, size_t workspace_bytes, void *stream,
                                                       void *const *events, int32_t n_events);

/* Bytes of one rank's buffer for the expert split (its expert outputs
 * [T*k][H] bf16 and its result region [T][H] bf16 behind the flags), for
 * up to `tokens` tokens per call. */
VQMOE_API size_t vqmoe_ep_buffer_bytes(int32_t hidden, int32_t tokens, int32_t top_k);

/* The SparseMoeBlock with its experts split by id across the ranks (expert
 * parallelism, an alternative to the tensor split at large E; the reference
 * has no EP): rank r of n holds experts [r*E/n, (r+1)*E/n) whole -- the
 * three linears carry E/n experts, uint8 dim-4 VQ in the device layout --
 * and the full router and shared expert. Every rank routes every token, runs
 * the pairs of its own experts, writing their outputs into its buffer, and
 * ONE kernel then sums each token's k slots in slot order over peer memory,
 * reading each slot from its expert's owner, and adds the gated shared
 * expert: the unsplit block's combine bit for bit, into out [T, H] bf16 on
 * every rank. Same call rules as vqmoe_sparse_moe_block_tp (the vqmoe_tp
 * descriptor, buffer_bytes >= vqmoe_ep_buffer_bytes, zeroed once). The
 * decode path only: fewer than 32 pairs per expert per 2048-token chunk. */
VQMOE_API vqmoe_status vqmoe_sparse_moe_block_ep(const vqmoe_block *blk, const vqmoe_tp *ep, const void *x,
                                                 int32_t tokens, void *out, void *workspace,
                                                 size_t workspace_bytes, void *stream);

/* SwitchGLU.__call__: y[T, k, H] bf16 = down(bf16(act(gate(x))) * up(x))
 * for each (token, slot) of indices [T, k] int32; act = gate->activation
 * (SwiGLU or GeGLU). */
VQMOE_API vqmoe_status vqmoe_switch_glu(const vqmoe_linear *gate,
                              const vqmoe_linear *up,
                              const vqmoe_linear *down, const void *x,
                              const int32_t *indices, int32_t tokens,
                              int32_t top_k, void *y, void *workspace,
                              size_t workspace_bytes, void *stream);

/* Size of the fixed per-device scratch of vqmoe_switch_glu_noalloc. */
#define VQMOE_NOALLOC_SCRATCH_BYTES (4 << 20)

/* vqmoe_switch_glu without a caller workspace: the workspace is a fixed
 * VQMOE_NOALLOC_SCRATCH_BYTES array of this library on each device, so the
 * call allocates nothing. No counterpart in the reference (MLX allocates
 * its temporaries itself); it serves callers that cannot allocate device
 * memory at call time, such as an FFI host with no device allocator or an
 * allocator's out-of-memory handler. Returns VQMOE_WORKSPACE_TOO_SMALL
 * when vqmoe_switch_glu_workspace_size(gate, down, tokens, top_k) exceeds
 * the scratch. The first call on a device takes the scratch's address
 * (cudaGetSymbolAddress) and keeps it for that device index: make it before
 * any stream capture, in the device's primary context (a driver-API context
 * of the caller's own, or a call after cudaDeviceReset, is not supported).
 * Nothing in the scratch needs to start at zero. One scratch per device:
 * calls that overlap on the same device race; the caller must order them. */
VQMOE_API vqmoe_status vqmoe_switch_glu_noalloc(const vqmoe_linear *gate,
                              const vqmoe_linear *up,
                              const vqmoe_linear *down, const void *x,
                              const int32_t *indices, int32_t tokens,
                              int32_t top_k, void *y, void *stream);

/* VQSwitchLinear.__call__ / SwitchLinear.__call__: y[T, k, OUT] bf16 with
 * y[t, s] = x_row @ W[indices[t, s]]^T. x_per_pair = 0: x is [T, IN] (one
 * row per token, shared by its k slots); 1: x is [T*k, IN] (one row per
 * (token, slot), e.g. the down projection's input). */
VQMOE_API vqmoe_status vqmoe_switch_linear(const vqmoe_linear *w, const void *x,
                                 int32_t x_per_pair, const int32_t *indices,
                                 int32_t tokens, int32_t top_k, void *y,
                                 void *workspace, size_t workspace_bytes,
                                 void *stream);

/* Router: inds [T, k] int32 (descending logit, ties to the lower expert),
 * scores [T, k] float32 holding bf16 values, and, when shared_expert_gate_w
 * is not NULL, sgate [T] float32 = bf16(sigmoid(bf16(x @ w_sg^T))). */
VQMOE_API vqmoe_status vqmoe_router(const void *x, const void *router_w,
                          const void *shared_expert_gate_w, int32_t tokens,
                          int32_t hidden, int32_t num_experts, int32_t top_k,
                          int32_t *inds, float *scores, float *sgate,
                          void *workspace, size_t workspace_bytes,
                          void *stream);

/* vqmoe_router with the weights of a router variant (VQMOE_ROUTER_*):
 * Qwen4-exp's SparseMoeBlock router, qwen4_exp.py:800-815. expert_scale
 * (optional, [num_experts] float): each selected weight becomes
 * bf16(weight * expert_scale[expert]) -- Gemma-4's Router.per_expert_scale
 * (gemma4_text.py:156-182, with VQMOE_ROUTER_TOPK_SOFTMAX; its RMS norm
 * of the input is the caller's). */
VQMOE_API vqmoe_status vqmoe_router_ex(const void *x, const void *router_w,
                          const void *shared_expert_gate_w, int32_t tokens,
                          int32_t hidden, int32_t num_experts, int32_t top_k,
                          int32_t router_mode, const float *expert_scale,
                          int32_t *inds, float *scores, float *sgate,
                          void *workspace, size_t workspace_bytes, void *stream);

/* Gemma-4's router input, mx.fast.rms_norm(x, weight, eps) of Router.__call__
 * (gemma4_text.py:171): out[T, H] bf16 = bf16(bf16(x * r) * weight), r =
 * 1 / sqrt(mean(x^2) + eps) in float32, the mean of the squares summed
 * exactly and rounded once to float32. x, weight [H] (Router.scale *
 * hidden^-0.5, rounded to bf16) and out are bf16. */
VQMOE_API vqmoe_status vqmoe_rms_norm(const void *x, const void *weight, int32_t tokens,
                                      int32_t hidden, float eps, void *out, void *stream);

/* The decoder stack's residual add and RMSNorm, one pass per row
 * (DecoderLayer.__call__ and RMSNorm.__call__, qwen3_5.py:120-130, 578-587):
 * sum = bf16(x + residual) when residual is given (written to sum_out when
 * that is given), then norm_out = bf16(f32(f32(sum) * rs) * weight) with
 * rs = 1 / sqrt(mean(sum^2) + eps) in float32 (the mean of the squares
 * summed exactly, rounded once to float32) and weight [hidden] float32 --
 * the (1 + weight) gain the reference keeps in float32. Also the per-head
 * q/k norms of the attention (rows = tokens x heads, hidden = head_dim).
 * x, residual, sum_out, norm_out: [rows, hidden] bf16. */
VQMOE_API vqmoe_status vqmoe_add_rms_norm(const void *x, const void *residual, const float *weight,
                                          int32_t rows, int32_t hidden, float eps, void *sum_out,
                                          void *norm_out, void *stream);

/* Gemma-4's Experts.__call__ (gemma4_text.py:196-214): out[T, H] bf16 =
 * sum over the k slots of bf16(y[t, s] * scores[t, s]), in fp32 and rounded
 * once, with y = vqmoe_switch_glu(gate, up, down, x, indices) (GeGLU via
 * gate->activation). */
VQMOE_API size_t vqmoe_moe_experts_workspace_size(const vqmoe_linear *gate,
                                                  const vqmoe_linear *down,
                                                  int32_t tokens, int32_t top_k);
VQMOE_API vqmoe_status vqmoe_moe_experts(const vqmoe_linear *gate,
                          const vqmoe_linear *up, const vqmoe_linear *down,
                          const void *x, const int32_t *indices,
                          const float *scores, int32_t tokens, int32_t top_k,
                          void *out, void *workspace, size_t workspace_bytes,
                          void *stream);

/* Dense weights of experts [first, first + count): out [count, OUT, IN],
 * fp16 W = fp16(codebook[code][j] * scale) for the VQ formats, bf16 W =
 * bf16(fmaf(scale, q, bias)) for AFFINE. */
VQMOE_API vqmoe_status vqmoe_dequant(const vqmoe_linear *w, int32_t first,
                                     int32_t count, void *out, void *stream);

/* Device layout of one VQ switch linear (what vqmoe_linear.codes / .scales
 * point to): bytes of its codes and of its scales. Rows are padded to a
 * multiple of 32 and inputs to a multiple of 256, then cut into tiles of
 * 32 rows x 256 inputs ordered for the kernels' loads (padded weights are
 * exactly zero). */
VQMOE_API vqmoe_status vqmoe_vq_layout_bytes(int32_t num_experts,
                                             int32_t out_features,
                                             int32_t in_features,
                                             int64_t *code_bytes,
                                             int64_t *scale_bytes);

/* Reference-layout codes [E, OUT, IN/4] uint8 and vq_scales [E, OUT, IN/64]
 * fp16 (device buffers) -> the device layout, into caller buffers sized by
 * vqmoe_vq_layout_bytes. Requires IN % 64 == 0 and OUT % 16 == 0. */
VQMOE_API vqmoe_status vqmoe_prepare_vq(const uint8_t *codes,
                                        const void *scales,
                                        int32_t num_experts,
                                        int32_t out_features,
                                        int32_t in_features,
                                        uint8_t *codes_dev, void *scales_dev,
                                        void *stream);

/* Device-layout codes -> reference-layout codes [E, OUT, IN/4]. */
VQMOE_API vqmoe_status vqmoe_unprepare_codes(const uint8_t *codes_dev,
                                             int32_t num_experts,
                                             int32_t out_features,
                                             int32_t in_features,
                                             uint8_t *codes, void *stream);

/* *bad_count (device uint32, zeroed by the caller) += the number of codes
 * >= codebook_size among codes[0, count). A loader calls it once; the
 * kernels trust the codes. */
VQMOE_API vqmoe_status vqmoe_count_bad_codes_u16(const uint16_t *codes,
                                                 int64_t count,
                                                 int32_t codebook_size,
                                                 uint32_t *bad_count,
                                                 void *stream);
/* The same over uint8 codes. */
VQMOE_API vqmoe_status vqmoe_count_bad_codes(const uint8_t *codes,
                                             int64_t count,
                                             int32_t codebook_size,
                                             uint32_t *bad_count,
                                             void *stream);

/* Every workspace (of vqmoe_sparse_moe_block, vqmoe_switch_glu,
 * vqmoe_switch_linear, vqmoe_moe_experts) starts with this many bytes of
 * status words, cleared at the start of each call on its stream. */
#define VQMOE_STATUS_BYTES 256

/* The device-side status of the last call that used `workspace`: waits for
 * `stream` (host synchronisation), then returns VQMOE_TIMEOUT when one of
 * the call's bounded device waits ran out (its outputs are then wrong; the
 * message names the stage and the wait), else VQMOE_OK. Every device wait is
 * bounded, so a kernel never hangs on one: the Knurlogic runtime treats a
 * stalled peer as an event (src/knurlogic/engine/split/liveness.py), and this
 * is the event's device-side form. Read it between calls; the next call
 * clears it. */
VQMOE_API vqmoe_status vqmoe_workspace_status(const void *workspace, void *stream);

/* Message of the last non-OK status returned on this host thread. */
VQMOE_API const char *vqmoe_last_error(void);

VQMOE_API int32_t vqmoe_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VQMOE_H_ */
