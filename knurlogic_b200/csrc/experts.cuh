// Structures shared by the routed-expert kernels (expert.cu: mma.sync, the
// decode regime; expert_prefill.cu: tcgen05, the prefill regime).
#pragma once

#include "common.cuh"

namespace vqmoe {

struct LinearDev {
    const uint8_t *codes;      // VQ device layout (layout.cuh)
    const uint16_t *codebook;  // [K][4] fp16 bits
    const uint16_t *scales;    // VQ device layout (layout.cuh), fp16 bits
    const uint16_t *weight;    // dense [E][OUT][IN] bf16 bits
    int K;
};

struct RoutedSet {
    const int32_t *cnt, *off, *list, *active;  // routing; active[E] = #active
    int E, k, x_per_pair, P;
    const uint16_t *x;           // input rows: fp16 (VQ) or bf16 (dense)
    LinearDev w0, w1;            // w1: up_proj of the fused gate/up stage
    int IN, OUT;
    uint16_t *out;               // [P][OUT]
    int out_f16;                 // 1: fp16 (saturated) output, 0: bf16
    const float *pair_scale;     // optional [P]: y = bf16(bf16(acc) * s)
    int act;                     // gate/up stage: VQMOE_ACT_SWIGLU or VQMOE_ACT_GEGLU
    int out_sorted;              // prefill path: output row = the pair's sorted position
};

struct PipeArgs {
    RoutedSet s1;                // phase 1: fused gate/up (when has1)
    RoutedSet s2;                // phase 2: down, or the one switch linear
    int has1;
    // [0] tile counter, [1] unused, [2 + i] finished phase 1 tiles of
    // active expert i; zeroed by the routing kernel
    uint32_t *ctl;
    uint32_t *err;               // the call's status word (kWait* when a wait ran out)
    uint32_t wait_polls;         // polls of a phase 2 tile's dependency wait (0: the default)
};

template <bool DUAL>
__device__ __forceinline__ uint16_t epilogue_value(float g, float u, const float *pair_scale,
                                                   int pair, int out_f16, int act = VQMOE_ACT_SWIGLU) {
    float v;
    if (DUAL) {
        // _SwiGLU (qwen3_5.py:108-112) / geglu (gemma4_text.py:131-135):
        // bf16(bf16(act(g)) * u), g and u the bf16 outputs of the gate and
        // up matmuls, act in fp32
        const float gb = bf16r(g);
        v = bf16r(bf16r(act == VQMOE_ACT_GEGLU ? gelu_tanh_f32(gb) : silu_f32(gb)) * bf16r(u));
    } else {
        v = bf16r(g);
        if (pair_scale) v = bf16r(v * pair_scale[pair]);
    }
    if (out_f16) return bf16_to_f16_sat(f32_to_bf16(v));
    return f32_to_bf16(v);
}

// epilogue_value with the routing weight already in hand (scaled: multiply
// by s), for callers that stage the weights of a tile in shared memory
template <bool DUAL>
__device__ __forceinline__ uint16_t epilogue_value_s(float g, float u, bool scaled, float s, int out_f16) {
    float v;
    if (DUAL) {
        v = bf16r(bf16r(silu_f32(bf16r(g))) * bf16r(u));
    } else {
        v = bf16r(g);
        if (scaled) v = bf16r(v * s);
    }
    if (out_f16) return bf16_to_f16_sat(f32_to_bf16(v));
    return f32_to_bf16(v);
}

struct TileInfo {
    int phase;      // 1: gate/up, 2: down / single linear
    int ai;         // index among the active experts
    int e, n, base; // expert, its pair count, list offset
    int row0;       // first output row of the tile
};

// The prefill path (tcgen05): both stages of the routed VQ experts in one
// launch, for layers whose experts see many tokens each.
// xs: [P][IN of the first stage] fp16 scratch for the expert-ordered inputs.
vqmoe_status launch_experts_prefill(const PipeArgs &a, void *xs, cudaStream_t stream,
                                    cudaEvent_t after_permute = nullptr);

}  // namespace vqmoe
