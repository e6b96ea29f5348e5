// The whole Qwen3.5-MoE sparse block and the C-ABI entry points.
//
// SparseMoeBlock.__call__ (qwen3_5.py:170-192) as a fixed launch sequence on
// one stream (graph-capturable: no host sync, no allocation):
//   router logits (+ shared_expert_gate row)  -> router top-k
//   fused gate/up + SwiGLU over routed pairs   -> act  [T*k, I]
//   shared expert gate/up + SwiGLU (dense)     -> acts [T, I_s]
//   down over routed pairs, x routing weight   -> ybuf [T*k, H]
//   shared expert down (dense)                 -> sh   [T, H]
//   combine: bf16(sum_k ybuf) + bf16(sg * sh)  -> out  [T, H]
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "layout.cuh"
#include "stages.cuh"

namespace vqmoe {

static thread_local char g_err[512] = "";

vqmoe_status set_error(vqmoe_status s, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return s;
}

vqmoe_status check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(VQMOE_LAUNCH_FAILED, "%s: %s", what, cudaGetErrorString(e));
    return VQMOE_OK;
}

int sm_count() {
    static std::atomic<int> cached[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
        const int c = cached[dev].load(std::memory_order_relaxed);
        if (c) return c;
    }
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

vqmoe_status ensure_dynamic_smem(const void *fn, size_t bytes, const char *what) {
    if (bytes <= 48 * 1024) return VQMOE_OK;
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, size_t> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(what);
    std::lock_guard<std::mutex> lock(mu);
    size_t &have = done[{fn, dev}];
    if (have >= bytes) return VQMOE_OK;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(VQMOE_LAUNCH_FAILED, "%s: %zu bytes of shared memory", what, bytes);
    }
    have = bytes;
    return VQMOE_OK;
}

// ------------------------------------------------------------- combine

// out[t, h] = bf16( bf16(sum_s ybuf[t*k+s, h]) + bf16(sg[t] * sh[t, h]) )
// (qwen3_5.py:181-187: the k-sum in fp32 rounded once; the gated shared
// expert rounded once; their sum rounded once).
__global__ void __launch_bounds__(256)
combine_kernel(const uint16_t *__restrict__ ybuf, int T, int k, int H,
               const uint16_t *__restrict__ sh, const float *__restrict__ sg,
               void *__restrict__ out, int out_f32) {
    const int vpr = H / 8;
    const size_t nvec = (size_t)T * vpr;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nvec;
         v += (size_t)gridDim.x * blockDim.x) {
        const int tkn = (int)(v / vpr), c8 = (int)(v - (size_t)tkn * vpr);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll 8
        for (int s = 0; s < k; ++s) {
            uint4 y = __ldg(reinterpret_cast<const uint4 *>(ybuf + ((size_t)tkn * k + s) * H + c8 * 8));
            const uint32_t u[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] += bf16_to_f32(u[j] & 0xFFFFu);
                acc[2 * j + 1] += bf16_to_f32(u[j] >> 16);
            }
        }
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = bf16r(acc[i]);
        if (sh) {
            const float gate = sg[tkn];
            uint4 sv = *reinterpret_cast<const uint4 *>(sh + (size_t)tkn * H + c8 * 8);
            const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[2 * j] = bf16r(r[2 * j] + bf16r(gate * bf16_to_f32(u[j] & 0xFFFFu)));
                r[2 * j + 1] = bf16r(r[2 * j + 1] + bf16r(gate * bf16_to_f32(u[j] >> 16)));
            }
        }
        if (out_f32) {
            float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)tkn * H + c8 * 8);
            o[0] = make_float4(r[0], r[1], r[2], r[3]);
            o[1] = make_float4(r[4], r[5], r[6], r[7]);
        } else {
            uint32_t p[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                p[j] = (uint32_t)f32_to_bf16(r[2 * j]) | ((uint32_t)f32_to_bf16(r[2 * j + 1]) << 16);
            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + (size_t)tkn * H + c8 * 8) =
                make_uint4(p[0], p[1], p[2], p[3]);
        }
    }
}

// ---------------------------------------------------------- validation

static bool aligned_ptr(const void *p) { return p && aligned16(p); }

static vqmoe_status check_linear(const vqmoe_linear *w, const char *name) {
    if (!w) return set_error(VQMOE_BAD_POINTER, "%s: null descriptor", name);
    if (w->num_experts <= 0 || w->out_features <= 0 || w->in_features <= 0)
        return set_error(VQMOE_BAD_SHAPE, "%s: non-positive shape", name);
    if (w->out_features % 16)
        return set_error(VQMOE_BAD_SHAPE, "%s: out_features %d is not a multiple of 16", name,
                         w->out_features);
    if (w->format == VQMOE_FMT_DENSE_BF16) {
        if (w->in_features % 16)
            return set_error(VQMOE_BAD_SHAPE, "%s: in_features %d is not a multiple of 16", name,
                             w->in_features);
        if (!w->weight || !aligned16(w->weight))
            return set_error(VQMOE_BAD_POINTER, "%s: weight null or not 16-byte aligned", name);
        return VQMOE_OK;
    }
    if (w->format == VQMOE_FMT_AFFINE) {
        const int b = w->bits;
        if (b != 2 && b != 3 && b != 4 && b != 5 && b != 6 && b != 8)
            return set_error(VQMOE_BAD_FORMAT, "%s: affine bits %d (2, 3, 4, 5, 6 or 8)", name, b);
        if (w->group_size != 32 && w->group_size != 64 && w->group_size != 128)
            return set_error(VQMOE_BAD_FORMAT, "%s: affine group_size %d (32, 64 or 128)", name, w->group_size);
        if (w->in_features % 64 || w->in_features % w->group_size)
            return set_error(VQMOE_BAD_SHAPE, "%s: in_features %d (a multiple of 64 and of the group)", name,
                             w->in_features);
        if (!aligned_ptr(w->weight) || !aligned_ptr(w->scales) || !aligned_ptr(w->biases))
            return set_error(VQMOE_BAD_POINTER, "%s: weight/scales/biases null or not 16-byte aligned", name);
        return VQMOE_OK;
    }
    if (w->format == VQMOE_FMT_VQ_REF) {
        if ((w->dim != 2 && w->dim != 4 && w->dim != 8) || w->codebook_size <= 0 || w->codebook_size > 65536)
            return set_error(VQMOE_BAD_FORMAT, "%s: VQ dim %d / K %d unsupported (dim 2, 4 or 8; K <= 65536)",
                             name, w->dim, w->codebook_size);
        if (w->group_size <= 0 || w->group_size % w->dim || w->in_features % w->group_size)
            return set_error(VQMOE_BAD_FORMAT, "%s: VQ group_size %d (a multiple of dim %d dividing in %d)",
                             name, w->group_size, w->dim, w->in_features);
        if (w->in_features % 64)
            return set_error(VQMOE_BAD_SHAPE, "%s: in_features %d is not a multiple of 64", name,
                             w->in_features);
        if (!w->codes || !w->codebook || !w->scales || !aligned16(w->codes) || !aligned16(w->codebook) ||
            !aligned16(w->scales))
            return set_error(VQMOE_BAD_POINTER, "%s: codes/codebook/scales null or not 16-byte aligned", name);
        return VQMOE_OK;
    }
    if (w->format != VQMOE_FMT_VQ_U8)
        return set_error(VQMOE_BAD_FORMAT, "%s: unknown format %d", name, w->format);
    if (w->dim != 4 || w->codebook_size <= 0 || w->codebook_size > 256)
        return set_error(VQMOE_BAD_FORMAT, "%s: VQ dim %d / K %d unsupported (dim 4, K <= 256)",
                         name, w->dim, w->codebook_size);
    if (w->group_size != 64)
        return set_error(VQMOE_BAD_FORMAT, "%s: VQ group_size %d unsupported (64)", name,
                         w->group_size);
    if (w->in_features % 64)
        return set_error(VQMOE_BAD_SHAPE, "%s: in_features %d is not a multiple of 64", name,
                         w->in_features);
    if (!w->codes || !w->codebook || !w->scales || !aligned16(w->codes) ||
        !aligned16(w->codebook) || !aligned16(w->scales))
        return set_error(VQMOE_BAD_POINTER, "%s: codes/codebook/scales null or not 16-byte aligned",
                         name);
    return VQMOE_OK;
}

// a SwitchGLU's linears share one general-kernel format (reference-layout
// VQ or affine) or use none
static vqmoe_status check_glu_formats(const vqmoe_linear *g, const vqmoe_linear *u, const vqmoe_linear *d) {
    if ((is_general(g->format) || is_general(u->format) || is_general(d->format)) &&
        (g->format != u->format || g->format != d->format))
        return set_error(VQMOE_BAD_FORMAT,
                         "gate/up/down: reference-layout VQ or affine on some linears but not all");
    return VQMOE_OK;
}

// workspace carving: each region 256-byte aligned
struct Carve {
    char *base;
    size_t off = 0;
    template <typename T>
    T *take(size_t count) {
        off = align_up(off, 256);
        T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
};

// Routing tables + the zeroed words (work counters, split-K semaphores)
// of a routed gate/up stage followed by a routed down stage.
struct RouteWs {
    int32_t *cnt, *off, *list, *active, *rank;
    uint32_t *zero;      // the expert kernel's control block (expert_ctl_words)
    int zero_words;
    uint32_t *szero;     // the shared expert's semaphores (zeroed on its own stream)
    int szero_words;
    uint32_t *ssem_gu, *ssem_dn;
    float *spart_gu, *spart_dn;
    int sks_gu, sks_dn;
};

static void carve_route(Carve &c, RouteWs &w, int E, int P, int H, int T, int Is) {
    w.cnt = c.take<int32_t>(E + 1);            // cnt[E]: the routing kernel's finished-CTA count
    w.off = c.take<int32_t>(E + 1);
    w.list = c.take<int32_t>(P);
    w.active = c.take<int32_t>(E + 1);
    w.rank = c.take<int32_t>(P);
    w.zero_words = expert_ctl_words(E);
    w.zero = c.take<uint32_t>(w.zero_words);
    int srb_gu = 0, srb_dn = 0;
    w.sks_gu = w.sks_dn = 1;
    if (Is > 0) {
        int kl = 0;
        size_t sm = 0;
        plan_shared_dense(H, Is, 2, &w.sks_gu, &kl, &sm);
        plan_shared_dense(Is, H, 1, &w.sks_dn, &kl, &sm);
        srb_gu = (Is + 31) / 32;
        srb_dn = (H + 31) / 32;
    }
    w.szero_words = srb_gu + srb_dn;
    w.szero = w.szero_words ? c.take<uint32_t>(w.szero_words) : nullptr;
    w.ssem_gu = w.szero;
    w.ssem_dn = w.szero ? w.szero + srb_gu : nullptr;
    // shared expert partials: T is at most one launch of tokens
    w.spart_gu = Is > 0 && w.sks_gu > 1 ? c.take<float>((size_t)w.sks_gu * T * 2 * Is) : nullptr;
    w.spart_dn = Is > 0 && w.sks_dn > 1 ? c.take<float>((size_t)w.sks_dn * T * H) : nullptr;
}

struct BlockWs {
    uint32_t *status;    // kStatusBytes at offset 0: [0] routed experts, [1] shared expert
    float *logits;
    int32_t *inds;
    float *scores;
    float *sgate;
    uint16_t *x16;
    RouteWs rt;
    uint16_t *act;
    uint16_t *act_s;
    uint16_t *ybuf;
    uint16_t *sh;
    uint16_t *xs;        // the prefill path's expert-ordered inputs, or null
    size_t bytes;
};

static BlockWs carve_block(void *ws, const vqmoe_block *b, int T) {
    Carve c{static_cast<char *>(ws)};
    BlockWs w{};
    const int E = b->num_experts, k = b->top_k, H = b->hidden;
    const int I = b->gate.out_features, Is = std::max(b->shared_inter, 0);
    const int P = T * k;
    w.status = c.take<uint32_t>(kStatusBytes / sizeof(uint32_t));
    w.logits = c.take<float>((size_t)T * (E + 1));
    w.inds = c.take<int32_t>(P);
    w.scores = c.take<float>(P);
    w.sgate = c.take<float>(T);
    w.x16 = is_vq(b->gate.format) ? c.take<uint16_t>((size_t)T * H) : nullptr;
    carve_route(c, w.rt, E, P, H, T, Is);
    w.act = c.take<uint16_t>((size_t)P * I);
    w.act_s = c.take<uint16_t>((size_t)T * Is);
    w.ybuf = c.take<uint16_t>((size_t)P * H);
    w.sh = c.take<uint16_t>((size_t)T * H);
    const bool vq = b->gate.format == VQMOE_FMT_VQ_U8 && b->down.format == VQMOE_FMT_VQ_U8;
    w.xs = prefill_regime(vq, E, P) ? c.take<uint16_t>((size_t)P * H) : nullptr;
    w.bytes = align_up(c.off, 256);
    return w;
}

// The status words of a call start at zero (before the shared expert's side
// stream forks, so both streams see it); they stay set across the token
// chunks of the call.
static vqmoe_status clear_status(uint32_t *status, cudaStream_t st) {
    if (cudaMemsetAsync(status, 0, 2 * sizeof(uint32_t), st) != cudaSuccess) return check_launch("status words");
    return VQMOE_OK;
}

// Tokens per launch sequence; a larger T runs as independent token chunks
// (bounds the workspace).
constexpr int kMaxTokensPerLaunch = 2048;

// the gate linear of a SwitchGLU names its activation
static vqmoe_status check_glu_activation(const vqmoe_linear *gate) {
    if (gate->activation != VQMOE_ACT_SWIGLU && gate->activation != VQMOE_ACT_GEGLU)
        return set_error(VQMOE_BAD_FORMAT, "gate_proj activation %d (0 SwiGLU, 1 GeGLU)", gate->activation);
    return VQMOE_OK;
}

static vqmoe_status check_block(const vqmoe_block *b, int T) {
    if (!b) return set_error(VQMOE_BAD_POINTER, "null block");
    if (T <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d", T);
    const int H = b->hidden, E = b->num_experts, k = b->top_k;
    if (H <= 0 || H % 16) return set_error(VQMOE_BAD_SHAPE, "hidden %d is not a multiple of 16", H);
    if (E <= 0 || E > 512) return set_error(VQMOE_BAD_SHAPE, "num_experts %d (1..512)", E);
    if (k <= 0 || k > 32 || k > E) return set_error(VQMOE_BAD_SHAPE, "top_k %d (1..min(32, E))", k);
    if (b->wait_polls < 0) return set_error(VQMOE_BAD_SHAPE, "wait_polls %d (>= 0)", b->wait_polls);
    vqmoe_status s;
    if ((s = check_linear(&b->gate, "gate_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(&b->up, "up_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(&b->down, "down_proj")) != VQMOE_OK) return s;
    const int I = b->gate.out_features;
    const vqmoe_linear *L[3] = {&b->gate, &b->up, &b->down};
    const int outs[3] = {I, I, H}, ins[3] = {H, H, I};
    for (int i = 0; i < 3; ++i)
        if (L[i]->num_experts != E || L[i]->out_features != outs[i] || L[i]->in_features != ins[i])
            return set_error(VQMOE_BAD_SHAPE,
                             "switch_mlp shapes: gate/up must be [E=%d, I, H=%d], down [E, H, I]", E, H);
    if (b->gate.format != b->up.format)
        return set_error(VQMOE_BAD_FORMAT, "gate_proj and up_proj formats differ");
    if ((s = check_glu_formats(&b->gate, &b->up, &b->down)) != VQMOE_OK) return s;
    if ((s = check_glu_activation(&b->gate)) != VQMOE_OK) return s;
    if (b->router_mode < VQMOE_ROUTER_SOFTMAX_TOPK_RENORM || b->router_mode > VQMOE_ROUTER_SOFTMAX_TOPK)
        return set_error(VQMOE_BAD_FORMAT, "router_mode %d (0..2)", b->router_mode);
    if (!aligned_ptr(b->router_w)) return set_error(VQMOE_BAD_POINTER, "router_w");
    if (b->shared_inter < 0 || b->shared_inter % 16)
        return set_error(VQMOE_BAD_SHAPE, "shared_inter %d is not a multiple of 16", b->shared_inter);
    if (b->shared_inter > 0 &&
        (!aligned_ptr(b->shared_gate_w) || !aligned_ptr(b->shared_up_w) ||
         !aligned_ptr(b->shared_down_w) || !aligned_ptr(b->shared_expert_gate_w)))
        return set_error(VQMOE_BAD_POINTER, "shared expert weights null or not 16-byte aligned");
    return VQMOE_OK;
}

// events (optional, n_ev >= 5): recorded before the router, after the
// routing, after the routed experts, after the join of the shared expert's
// side stream, and after the combine; a sixth, when given, after the
// prefill path's input permute (with the routing's when there is none).
static vqmoe_status mark(cudaEvent_t *ev, int n_ev, int i, cudaStream_t st) {
    if (ev && i < n_ev && cudaEventRecord(ev[i], st) != cudaSuccess)
        return set_error(VQMOE_LAUNCH_FAILED, "event %d", i);
    return VQMOE_OK;
}

static RoutedIO routed_io(const RouteWs &rt, int E, int k, int P, const void *x, int x_per_pair,
                          void *out, int out_f16, const float *scale) {
    RoutedIO r{};
    r.cnt = rt.cnt;
    r.off = rt.off;
    r.list = rt.list;
    r.active = rt.active;
    r.E = E;
    r.k = k;
    r.P = P;
    r.x = x;
    r.x_per_pair = x_per_pair;
    r.out = out;
    r.out_f16 = out_f16;
    r.pair_scale = scale;
    return r;
}

// The shared expert runs on a side stream forked from the caller's stream
// (an event after the caller's prior work) and joined before the combine, so
// it overlaps the routing and the routed experts. One side stream and event
// pair per host thread and device, created on the first call on that device
// (make that call before capturing the stream into a CUDA graph).
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
constexpr int kMaxDevices = 64;

static vqmoe_status side_stream(SideStream **out) {
    static thread_local SideStream per_dev[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(VQMOE_LAUNCH_FAILED, "side stream: cudaGetDevice");
    SideStream &ss = per_dev[dev];
    if (!ss.s) {
        int lo = 0, hi = 0;
        cudaDeviceGetStreamPriorityRange(&lo, &hi);
        if (cudaStreamCreateWithPriority(&ss.s, cudaStreamNonBlocking, hi) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return set_error(VQMOE_LAUNCH_FAILED, "side stream: create");
        }
    }
    *out = &ss;
    return VQMOE_OK;
}

// The shared expert on stream st: gate/up + SwiGLU into act_s, then down
// into sh. Where both matmuls take 64-input windows, the tcgen05 kernel at
// every token count: on its side stream it holds few SMs (one CTA per 128
// weight rows) for longer, which costs the routed-expert kernel running
// beside it less than a kernel spread over every SM (measured at c2: 118 us
// per block against 121 us for the K-sliced kernels and 123 us for a
// cluster K-split on all SMs); else the K-sliced mma.sync kernels.
static vqmoe_status run_shared(const vqmoe_block *b, const uint16_t *x, int T, const BlockWs &w,
                               cudaStream_t st) {
    const RouteWs &rt = w.rt;
    if (b->hidden % 64 == 0 && b->shared_inter % 64 == 0) {
        vqmoe_status s = launch_dense_prefill(x, b->shared_gate_w, b->shared_up_w, T, b->hidden,
                                              b->shared_inter, w.act_s, w.status + 1, st);
        if (s != VQMOE_OK) return s;
        return launch_dense_prefill(w.act_s, b->shared_down_w, nullptr, T, b->shared_inter, b->hidden,
                                    w.sh, w.status + 1, st);
    }
    if (rt.szero_words &&
        cudaMemsetAsync(rt.szero, 0, (size_t)rt.szero_words * sizeof(uint32_t), st) != cudaSuccess)
        return check_launch("shared expert semaphores");
    vqmoe_status s = launch_shared_dense(x, b->shared_gate_w, b->shared_up_w, T, b->hidden,
                                         b->shared_inter, w.act_s, rt.spart_gu, rt.ssem_gu, st);
    if (s != VQMOE_OK) return s;
    return launch_shared_dense(w.act_s, b->shared_down_w, nullptr, T, b->shared_inter, b->hidden,
                               w.sh, rt.spart_dn, rt.ssem_dn, st);
}

// The expert split: keep only this rank's experts [own0, own1) in the list
// of active experts the expert kernel takes its tiles from (in order).
__global__ void __launch_bounds__(1024) filter_active_kernel(int32_t *__restrict__ active, int E, int own0, int own1) {
    __shared__ int s_keep[1024];
    __shared__ int s_n;
    const int tid = threadIdx.x;
    const int n = active[E];
    const int e = tid < n ? active[tid] : -1;
    const int keep = e >= own0 && e < own1;
    s_keep[tid] = keep;
    __syncthreads();
    if (tid == 0) {
        int c = 0;
        for (int i = 0; i < n; ++i) {
            const int kk = s_keep[i];
            s_keep[i] = c;
            c += kk;
        }
        s_n = c;
    }
    __syncthreads();
    if (keep) active[s_keep[tid]] = e;
    __syncthreads();
    if (tid == 0) active[E] = s_n;
}

static vqmoe_status run_block(const vqmoe_block *b, const uint16_t *x, int T,
                              void *out, int out_f32, const BlockWs &w,
                              cudaStream_t st, cudaEvent_t *ev = nullptr, int n_ev = 0,
                              const TpArgs *tp = nullptr) {
    const int H = b->hidden, E = b->num_experts, k = b->top_k, P = T * k;
    const bool shared = b->shared_inter > 0;
    const bool vq_in = is_vq(b->gate.format);
    const bool vq_dn = is_vq(b->down.format);
    vqmoe_status s;
    if ((s = mark(ev, n_ev, 0, st)) != VQMOE_OK) return s;
    SideStream *side = nullptr;
    if (shared) {
        if ((s = side_stream(&side)) != VQMOE_OK) return s;
        if (cudaEventRecord(side->fork, st) != cudaSuccess ||
            cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess)
            return check_launch("side stream fork");
        if ((s = run_shared(b, x, T, w, side->s)) != VQMOE_OK) return s;
        if (cudaEventRecord(side->join, side->s) != cudaSuccess)
            return check_launch("side stream join");
    }
    const RouteWs &rt = w.rt;
    const uint16_t *rw = static_cast<const uint16_t *>(b->router_w);
    const uint16_t *sgw = shared ? static_cast<const uint16_t *>(b->shared_expert_gate_w) : nullptr;
    if (tp && tp->ep_local) {
        // the expert split: every rank routes every token, then keeps the
        // experts it owns
        s = launch_router_route(x, rw, sgw, T, H, E, k, w.logits, w.inds, w.scores, w.sgate, w.x16, rt.cnt, rt.off,
                                rt.list, rt.active, rt.rank, rt.zero, rt.zero_words, b->router_mode, st);
        if (s != VQMOE_OK) return s;
        const int own0 = tp->rank * tp->ep_local;
        filter_active_kernel<<<1, 1024, 0, st>>>(rt.active, E, own0, own0 + tp->ep_local);
        if ((s = check_launch("filter_active_kernel")) != VQMOE_OK) return s;
    } else if (tp) {
        // under a split each rank computes the exact logits of T / n of the
        // tokens (the router's cost, the same on every rank otherwise); the
        // ranks exchange them over peer memory and every rank selects and
        // sorts the whole routing (with one rank, the same path over its own
        // buffer). Above the select kernel's size the ranks route their own
        // tokens and exchange the routing instead.
        const int r0 = (int)((long long)T * tp->rank / tp->n), r1 = (int)((long long)T * (tp->rank + 1) / tp->n);
        const int E1 = E + (sgw ? 1 : 0);
        TpArgs g = *tp;
        g.err = w.status;
        uint16_t *x16 = vq_in ? w.x16 : nullptr;
        if (T <= kSelectMaxTok && E <= 1024) {
            if (r1 > r0 && (s = launch_logits(x + (size_t)r0 * H, rw, sgw, r1 - r0, H, E, E1,
                                              w.logits + (size_t)r0 * E1, nullptr, st)) != VQMOE_OK)
                return s;
            void *arrays[3] = {w.logits, nullptr, nullptr};
            const int widths[3] = {E1, 0, 0};
            if ((s = launch_tp_gather(arrays, widths, T, H, r0, r1, reinterpret_cast<uint32_t *>(rt.cnt), E + 1, x,
                                      x16, g, st)) != VQMOE_OK ||
                (s = launch_select(w.logits, T, E, E1, k, sgw != nullptr, w.inds, w.scores, w.sgate, rt.cnt, rt.off,
                                   rt.list, rt.active, rt.rank, rt.zero, rt.zero_words, b->router_mode, st)) != VQMOE_OK)
                return s;
        } else {
            if (r1 > r0 && (s = launch_router(x + (size_t)r0 * H, rw, sgw, r1 - r0, H, E, k,
                                              w.logits + (size_t)r0 * E1, w.inds + (size_t)r0 * k,
                                              w.scores + (size_t)r0 * k, w.sgate + r0, nullptr, b->router_mode,
                                              nullptr, st)) != VQMOE_OK)
                return s;
            void *arrays[3] = {w.inds, w.scores, sgw ? w.sgate : nullptr};
            const int widths[3] = {k, k, sgw ? 1 : 0};
            if ((s = launch_tp_gather(arrays, widths, T, H, r0, r1, nullptr, 0, x, x16, g, st)) != VQMOE_OK ||
                (s = launch_route(w.inds, P, E, rt.cnt, rt.off, rt.list, rt.active, rt.rank, rt.zero, rt.zero_words,
                                  st)) != VQMOE_OK)
                return s;
        }
    } else {
        s = launch_router_route(x, rw, sgw, T, H, E, k, w.logits, w.inds, w.scores, w.sgate, w.x16, rt.cnt, rt.off,
                                rt.list, rt.active, rt.rank, rt.zero, rt.zero_words, b->router_mode, st);
        if (s != VQMOE_OK) return s;
    }
    if ((s = mark(ev, n_ev, 1, st)) != VQMOE_OK) return s;
    // the routed experts: gate/up + SwiGLU, then down (x routing weight)
    RoutedIO r1 = routed_io(rt, E, k, P, vq_in ? (const void *)w.x16 : (const void *)x, 0, w.act,
                            vq_dn, nullptr);
    r1.xs = w.xs;
    r1.act = b->gate.activation;
    // the expert split: the owned pairs' outputs go straight into this
    // rank's buffer, where the other ranks read them
    uint16_t *ybuf = tp && tp->ep_local ? reinterpret_cast<uint16_t *>(tp->base[tp->rank] + kTpFlagBytes) : w.ybuf;
    RoutedIO r2 = routed_io(rt, E, k, P, w.act, 1, ybuf, 0, w.scores);
    s = launch_experts(&b->gate, &b->up, &r1, &b->down, r2, rt.zero, w.status, (uint32_t)b->wait_polls, st,
                       ev && n_ev > 5 ? ev[5] : nullptr);
    if (s != VQMOE_OK || (s = mark(ev, n_ev, 2, st)) != VQMOE_OK) return s;
    if (shared && cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess)
        return check_launch("side stream join");
    if ((s = mark(ev, n_ev, 3, st)) != VQMOE_OK) return s;
    if (tp && tp->ep_local) {
        TpArgs a = *tp;
        a.err = w.status;
        if ((s = launch_ep_reduce(w.inds, T, k, H, tp->ep_local, shared ? w.sh : nullptr, w.sgate, a,
                                  static_cast<uint16_t *>(out), st)) != VQMOE_OK)
            return s;
        return mark(ev, n_ev, 4, st);
    }
    if (tp) {
        // the combine and the split's reduction, one kernel over peer memory
        TpArgs a = *tp;
        a.err = w.status;
        if ((s = launch_tp_reduce(w.ybuf, T, k, H, shared ? w.sh : nullptr, w.sgate, a,
                                  static_cast<uint16_t *>(out), st)) != VQMOE_OK)
            return s;
        return mark(ev, n_ev, 4, st);
    }
    const size_t nvec = (size_t)T * (H / 8);
    const int grid = (int)std::min<size_t>((nvec + 255) / 256, (size_t)sm_count() * 8);
    combine_kernel<<<grid, 256, 0, st>>>(w.ybuf, T, k, H, shared ? w.sh : nullptr, w.sgate, out, out_f32);
    if ((s = check_launch("combine_kernel")) != VQMOE_OK) return s;
    return mark(ev, n_ev, 4, st);
}

// Workspace of vqmoe_switch_glu / vqmoe_switch_linear at T tokens.
struct GluWs {
    uint32_t *status;    // kStatusBytes at offset 0: [0] routed experts
    uint16_t *x16;
    RouteWs rt;
    uint16_t *act;
    uint16_t *xs;        // the prefill path's expert-ordered inputs, or null
    size_t bytes;
};

static GluWs carve_glu(void *ws, const vqmoe_linear *first, const vqmoe_linear *down, int T, int k,
                       int rows_x) {
    Carve c{static_cast<char *>(ws)};
    GluWs w{};
    const int E = first->num_experts, P = T * k;
    const bool dual = down != nullptr;
    w.status = c.take<uint32_t>(kStatusBytes / sizeof(uint32_t));
    w.x16 = is_vq(first->format) ? c.take<uint16_t>((size_t)rows_x * first->in_features)
                                             : nullptr;
    const int H = first->in_features, I = first->out_features;
    carve_route(c, w.rt, E, P, H, T, 0);
    w.act = dual ? c.take<uint16_t>((size_t)P * I) : nullptr;
    const bool vq = first->format == VQMOE_FMT_VQ_U8 && (!dual || down->format == VQMOE_FMT_VQ_U8);
    w.xs = prefill_regime(vq, E, P) ? c.take<uint16_t>((size_t)P * H) : nullptr;
    w.bytes = align_up(c.off, 256);
    return w;
}

// x (bf16) -> fp16 (saturated), 8 elements per thread
__global__ void to_f16_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ y, size_t n8) {
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < n8;
         v += (size_t)gridDim.x * blockDim.x) {
        uint4 val = reinterpret_cast<const uint4 *>(x)[v];
        uint32_t u[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            u[j] = (uint32_t)bf16_to_f16_sat(u[j] & 0xFFFFu) | ((uint32_t)bf16_to_f16_sat(u[j] >> 16) << 16);
        reinterpret_cast<uint4 *>(y)[v] = make_uint4(u[0], u[1], u[2], u[3]);
    }
}

vqmoe_status launch_to_f16(const uint16_t *x, uint16_t *x16, size_t n, cudaStream_t stream) {
    const size_t n8 = n / 8;
    const int grid = (int)std::min<size_t>((n8 + 255) / 256, (size_t)sm_count() * 8);
    to_f16_kernel<<<std::max(grid, 1), 256, 0, stream>>>(x, x16, n8);
    return check_launch("to_f16_kernel");
}

}  // namespace vqmoe

using namespace vqmoe;

// ------------------------------------------------------------ C ABI

extern "C" {

int32_t vqmoe_abi_version(void) { return VQMOE_ABI_VERSION; }

vqmoe_status vqmoe_workspace_status(const void *workspace, void *stream) {
    if (!aligned_ptr(workspace)) return set_error(VQMOE_BAD_POINTER, "workspace_status: workspace");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t w[2] = {0, 0};
    if (cudaMemcpyAsync(w, workspace, sizeof(w), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_launch("workspace_status");
    if (!w[0] && !w[1]) return VQMOE_OK;
    auto kind = [](uint32_t v) {
        return v == kWaitDependency ? "a phase 2 tile's wait for its expert's phase 1 tiles"
               : v == kWaitPipeline ? "a tcgen05 pipeline barrier"
                                    : "none";
    };
    return set_error(VQMOE_TIMEOUT, "a bounded device wait ran out: routed experts: %s; shared expert: %s",
                     kind(w[0]), kind(w[1]));
}

const char *vqmoe_last_error(void) { return g_err; }

size_t vqmoe_router_workspace_size(int32_t tokens, int32_t num_experts) {
    return align_up((size_t)tokens * (num_experts + 1) * sizeof(float), 256);
}

size_t vqmoe_switch_glu_workspace_size(const vqmoe_linear *gate, const vqmoe_linear *down,
                                       int32_t tokens, int32_t top_k) {
    if (!gate || !down || tokens <= 0 || top_k <= 0) return 0;
    const int T = std::min<int>(tokens, kMaxTokensPerLaunch);
    return carve_glu(nullptr, gate, down, T, top_k, T).bytes;
}

size_t vqmoe_switch_linear_workspace_size(const vqmoe_linear *w, int32_t tokens, int32_t top_k,
                                          int32_t x_per_pair) {
    if (!w || tokens <= 0 || top_k <= 0) return 0;
    const int T = std::min<int>(tokens, kMaxTokensPerLaunch);
    return carve_glu(nullptr, w, nullptr, T, top_k, x_per_pair ? T * top_k : T).bytes;
}

size_t vqmoe_block_workspace_size(const vqmoe_block *blk, int32_t tokens) {
    if (!blk || tokens <= 0) return 0;
    return carve_block(nullptr, blk, tokens).bytes;
}

static vqmoe_status block_impl(const vqmoe_block *blk, const void *x, int32_t tokens, void *out,
                               int32_t out_dtype, void *workspace, size_t workspace_bytes,
                               void *stream, cudaEvent_t *ev, int n_ev, const TpArgs *tp = nullptr) {
    vqmoe_status s = check_block(blk, tokens);
    if (s != VQMOE_OK) return s;
    if (!aligned_ptr(x) || !aligned_ptr(out) || !aligned_ptr(workspace))
        return set_error(VQMOE_BAD_POINTER, "x / out / workspace null or not 16-byte aligned");
    if (out_dtype != VQMOE_OUT_BF16 && out_dtype != VQMOE_OUT_F32)
        return set_error(VQMOE_BAD_FORMAT, "out_dtype %d", out_dtype);
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    BlockWs w = carve_block(workspace, blk, chunk);
    if (workspace_bytes < w.bytes)
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "workspace %zu < %zu bytes", workspace_bytes, w.bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((s = clear_status(w.status, st)) != VQMOE_OK) return s;
    const size_t osz = out_dtype == VQMOE_OUT_F32 ? 4 : 2;
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0);
        s = run_block(blk, static_cast<const uint16_t *>(x) + (size_t)t0 * blk->hidden, T,
                      static_cast<char *>(out) + (size_t)t0 * blk->hidden * osz,
                      out_dtype == VQMOE_OUT_F32, w, st, t0 == 0 ? ev : nullptr, n_ev, tp);
        if (s != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

vqmoe_status vqmoe_sparse_moe_block(const vqmoe_block *blk, const void *x, int32_t tokens,
                                    void *out, int32_t out_dtype, void *workspace,
                                    size_t workspace_bytes, void *stream) {
    return block_impl(blk, x, tokens, out, out_dtype, workspace, workspace_bytes, stream,
                      nullptr, 0);
}

size_t vqmoe_tp_buffer_bytes(int32_t hidden, int32_t tokens) {
    if (hidden <= 0 || tokens <= 0) return 0;
    const size_t T = (size_t)std::min<int>(tokens, kMaxTokensPerLaunch);
    return tp_route_offset((int)T, hidden) + tp_route_bytes((int)T);
}

static vqmoe_status block_tp_impl(const vqmoe_block *blk, const vqmoe_tp *tp, const void *x, int32_t tokens,
                                  void *out, void *workspace, size_t workspace_bytes, void *stream,
                                  cudaEvent_t *ev, int n_ev) {
    if (!tp) return set_error(VQMOE_BAD_POINTER, "block_tp: null split descriptor");
    if (tp->world < 1 || tp->world > kTpMaxRanks || tp->rank < 0 || tp->rank >= tp->world)
        return set_error(VQMOE_BAD_SHAPE, "block_tp: rank %d of %d (at most %d ranks)", tp->rank, tp->world,
                         kTpMaxRanks);
    if (tp->wait_polls < 0) return set_error(VQMOE_BAD_SHAPE, "block_tp: wait_polls %d", tp->wait_polls);
    if (!blk || blk->hidden % (8 * tp->world))
        return set_error(VQMOE_BAD_SHAPE, "block_tp: hidden %d is not a multiple of 8 x %d ranks",
                         blk ? blk->hidden : 0, tp->world);
    if (tokens <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d", tokens);
    if ((size_t)tp->buffer_bytes < vqmoe_tp_buffer_bytes(blk->hidden, tokens))
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "block_tp: buffers of %lld < %zu bytes",
                         (long long)tp->buffer_bytes, vqmoe_tp_buffer_bytes(blk->hidden, tokens));
    TpArgs a{};
    a.rank = tp->rank;
    a.n = tp->world;
    a.wait_polls = (uint32_t)tp->wait_polls;
    for (int q = 0; q < tp->world; ++q) {
        if (!aligned_ptr(tp->buffers[q])) return set_error(VQMOE_BAD_POINTER, "block_tp: buffer of rank %d", q);
        a.base[q] = static_cast<uint8_t *>(tp->buffers[q]);
    }
    return block_impl(blk, x, tokens, out, VQMOE_OUT_BF16, workspace, workspace_bytes, stream, ev, n_ev, &a);
}

vqmoe_status vqmoe_sparse_moe_block_tp(const vqmoe_block *blk, const vqmoe_tp *tp, const void *x, int32_t tokens,
                                       void *out, void *workspace, size_t workspace_bytes, void *stream) {
    return block_tp_impl(blk, tp, x, tokens, out, workspace, workspace_bytes, stream, nullptr, 0);
}

size_t vqmoe_ep_buffer_bytes(int32_t hidden, int32_t tokens, int32_t top_k) {
    if (hidden <= 0 || tokens <= 0 || top_k <= 0) return 0;
    return ep_buffer_bytes(std::min<int>(tokens, kMaxTokensPerLaunch), top_k, hidden);
}

vqmoe_status vqmoe_sparse_moe_block_ep(const vqmoe_block *blk, const vqmoe_tp *ep, const void *x, int32_t tokens,
                                       void *out, void *workspace, size_t workspace_bytes, void *stream) {
    if (!blk || !ep) return set_error(VQMOE_BAD_POINTER, "block_ep: null descriptor");
    const int n = ep->world, E = blk->num_experts, H = blk->hidden, k = blk->top_k;
    if (n < 1 || n > kTpMaxRanks || ep->rank < 0 || ep->rank >= n)
        return set_error(VQMOE_BAD_SHAPE, "block_ep: rank %d of %d (at most %d ranks)", ep->rank, n, kTpMaxRanks);
    if (ep->wait_polls < 0) return set_error(VQMOE_BAD_SHAPE, "block_ep: wait_polls %d", ep->wait_polls);
    if (E <= 0 || E % n) return set_error(VQMOE_BAD_SHAPE, "block_ep: %d experts over %d ranks", E, n);
    if (H <= 0 || H % (8 * n)) return set_error(VQMOE_BAD_SHAPE, "block_ep: hidden %d, %d ranks", H, n);
    if (tokens <= 0 || k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, k);
    const int El = E / n, own0 = ep->rank * El;
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    if (prefill_regime(true, E, chunk * k))
        return set_error(VQMOE_BAD_SHAPE, "block_ep: %d pairs over %d experts (the decode path: fewer than 32 a "
                         "expert)", chunk * k, E);
    if ((size_t)ep->buffer_bytes < vqmoe_ep_buffer_bytes(H, tokens, k))
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "block_ep: buffers of %lld < %zu bytes",
                         (long long)ep->buffer_bytes, vqmoe_ep_buffer_bytes(H, tokens, k));
    // the rank's E / n experts are addressed by their global ids: each VQ
    // layout pointer is moved back by own0 experts' worth of tiles
    vqmoe_block b2 = *blk;
    vqmoe_linear *L[3] = {&b2.gate, &b2.up, &b2.down};
    for (vqmoe_linear *l : L) {
        if (l->format != VQMOE_FMT_VQ_U8)
            return set_error(VQMOE_BAD_FORMAT, "block_ep: experts in the uint8 dim-4 VQ layout only");
        if (l->num_experts != El)
            return set_error(VQMOE_BAD_SHAPE, "block_ep: a rank holds %d experts, got %d", El, l->num_experts);
        const VqGeom G{1, l->out_features, l->in_features};
        const size_t cstride = (size_t)G.code_bytes(), sstride = (size_t)G.scale_elems() * 2;
        const uintptr_t c = reinterpret_cast<uintptr_t>(l->codes), sc = reinterpret_cast<uintptr_t>(l->scales);
        if (!c || !sc || c < own0 * cstride || sc < own0 * sstride)
            return set_error(VQMOE_BAD_POINTER, "block_ep: expert weights");
        l->codes = reinterpret_cast<const void *>(c - own0 * cstride);
        l->scales = reinterpret_cast<const void *>(sc - own0 * sstride);
        l->num_experts = E;
    }
    TpArgs a{};
    a.rank = ep->rank;
    a.n = n;
    a.wait_polls = (uint32_t)ep->wait_polls;
    a.ep_local = El;
    for (int q = 0; q < n; ++q) {
        if (!aligned_ptr(ep->buffers[q])) return set_error(VQMOE_BAD_POINTER, "block_ep: buffer of rank %d", q);
        a.base[q] = static_cast<uint8_t *>(ep->buffers[q]);
    }
    return block_impl(&b2, x, tokens, out, VQMOE_OUT_BF16, workspace, workspace_bytes, stream, nullptr, 0, &a);
}

vqmoe_status vqmoe_sparse_moe_block_tp_timed(const vqmoe_block *blk, const vqmoe_tp *tp, const void *x,
                                             int32_t tokens, void *out, void *workspace, size_t workspace_bytes,
                                             void *stream, void *const *events, int32_t n_events) {
    if (!events || n_events < 5) return set_error(VQMOE_BAD_POINTER, "block_tp_timed: five events needed");
    if (tokens > kMaxTokensPerLaunch)
        return set_error(VQMOE_BAD_SHAPE, "timed block: at most %d tokens", kMaxTokensPerLaunch);
    return block_tp_impl(blk, tp, x, tokens, out, workspace, workspace_bytes, stream,
                         reinterpret_cast<cudaEvent_t *>(const_cast<void **>(events)), n_events);
}

vqmoe_status vqmoe_sparse_moe_block_timed(const vqmoe_block *blk, const void *x, int32_t tokens,
                                          void *out, int32_t out_dtype, void *workspace,
                                          size_t workspace_bytes, void *stream,
                                          void *const *events, int32_t n_events) {
    if (!events || n_events < 5)
        return set_error(VQMOE_BAD_POINTER, "timed block: needs 5 events");
    if (tokens > kMaxTokensPerLaunch)
        return set_error(VQMOE_BAD_SHAPE, "timed block: at most %d tokens", kMaxTokensPerLaunch);
    return block_impl(blk, x, tokens, out, out_dtype, workspace, workspace_bytes, stream,
                      reinterpret_cast<cudaEvent_t *>(const_cast<void **>(events)), n_events);
}

vqmoe_status vqmoe_switch_glu(const vqmoe_linear *gate, const vqmoe_linear *up,
                              const vqmoe_linear *down, const void *x,
                              const int32_t *indices, int32_t tokens, int32_t top_k,
                              void *y, void *workspace, size_t workspace_bytes,
                              void *stream) {
    vqmoe_status s;
    if ((s = check_linear(gate, "gate_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(up, "up_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(down, "down_proj")) != VQMOE_OK) return s;
    if ((s = check_glu_activation(gate)) != VQMOE_OK) return s;
    if (tokens <= 0 || top_k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, top_k);
    const int I = gate->out_features, H = gate->in_features, E = gate->num_experts;
    if (up->out_features != I || up->in_features != H || down->out_features != H ||
        down->in_features != I || up->num_experts != E || down->num_experts != E ||
        gate->format != up->format)
        return set_error(VQMOE_BAD_SHAPE, "switch_glu: inconsistent gate/up/down shapes");
    if ((s = check_glu_formats(gate, up, down)) != VQMOE_OK) return s;
    if (E > 1024) return set_error(VQMOE_BAD_SHAPE, "switch_glu: %d experts (<= 1024)", E);
    if (!aligned_ptr(x) || !aligned_ptr(y) || !indices || !aligned_ptr(workspace))
        return set_error(VQMOE_BAD_POINTER, "x / indices / y / workspace");
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    GluWs w = carve_glu(workspace, gate, down, chunk, top_k, chunk);
    if (workspace_bytes < w.bytes)
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "workspace %zu < %zu bytes", workspace_bytes, w.bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((s = clear_status(w.status, st)) != VQMOE_OK) return s;
    const bool vq_in = is_vq(gate->format), vq_dn = is_vq(down->format);
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0), P = T * top_k;
        const int32_t *ind = indices + (size_t)t0 * top_k;
        const uint16_t *xt = static_cast<const uint16_t *>(x) + (size_t)t0 * H;
        const RouteWs &rt = w.rt;
        if (vq_in && (s = launch_to_f16(xt, w.x16, (size_t)T * H, st)) != VQMOE_OK) return s;
        if ((s = launch_route(ind, P, E, rt.cnt, rt.off, rt.list, rt.active, rt.rank, rt.zero,
                              rt.zero_words, st)) != VQMOE_OK)
            return s;
        RoutedIO r1 = routed_io(rt, E, top_k, P, vq_in ? (const void *)w.x16 : (const void *)xt, 0,
                                w.act, vq_dn, nullptr);
        r1.xs = w.xs;
        r1.act = gate->activation;
        RoutedIO r2 = routed_io(rt, E, top_k, P, w.act, 1,
                                static_cast<uint16_t *>(y) + (size_t)t0 * top_k * H, 0, nullptr);
        if ((s = launch_experts(gate, up, &r1, down, r2, rt.zero, w.status, 0, st)) != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

// Experts.__call__ of gemma4_text.py:196-214: y = SwitchGLU(x, indices),
// out[t] = sum_s w[t, s] * y[t, s] -- per pair bf16(y * w), summed over the
// k slots in fp32 and rounded once (the block's combine without a shared
// expert). Workspace: the SwitchGLU workspace, then the [T, k, H] bf16
// expert outputs.
static size_t moe_experts_ybuf_offset(const GluWs &w) { return align_up(w.bytes, 256); }

size_t vqmoe_moe_experts_workspace_size(const vqmoe_linear *gate, const vqmoe_linear *down, int32_t tokens,
                                        int32_t top_k) {
    if (!gate || !down || tokens <= 0 || top_k <= 0) return 0;
    const int T = std::min<int>(tokens, kMaxTokensPerLaunch);
    const GluWs w = carve_glu(nullptr, gate, down, T, top_k, T);
    return align_up(moe_experts_ybuf_offset(w) + (size_t)T * top_k * gate->in_features * sizeof(uint16_t), 256);
}

vqmoe_status vqmoe_moe_experts(const vqmoe_linear *gate, const vqmoe_linear *up, const vqmoe_linear *down,
                               const void *x, const int32_t *indices, const float *scores, int32_t tokens,
                               int32_t top_k, void *out, void *workspace, size_t workspace_bytes, void *stream) {
    vqmoe_status s;
    if ((s = check_linear(gate, "gate_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(up, "up_proj")) != VQMOE_OK) return s;
    if ((s = check_linear(down, "down_proj")) != VQMOE_OK) return s;
    if ((s = check_glu_activation(gate)) != VQMOE_OK) return s;
    if (tokens <= 0 || top_k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, top_k);
    const int I = gate->out_features, H = gate->in_features, E = gate->num_experts;
    if (up->out_features != I || up->in_features != H || down->out_features != H ||
        down->in_features != I || up->num_experts != E || down->num_experts != E ||
        gate->format != up->format)
        return set_error(VQMOE_BAD_SHAPE, "moe_experts: inconsistent gate/up/down shapes");
    if ((s = check_glu_formats(gate, up, down)) != VQMOE_OK) return s;
    if (E > 1024) return set_error(VQMOE_BAD_SHAPE, "moe_experts: %d experts (<= 1024)", E);
    if (!aligned_ptr(x) || !aligned_ptr(out) || !indices || !scores || !aligned_ptr(workspace))
        return set_error(VQMOE_BAD_POINTER, "x / indices / scores / out / workspace");
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    GluWs w = carve_glu(workspace, gate, down, chunk, top_k, chunk);
    const size_t need = vqmoe_moe_experts_workspace_size(gate, down, tokens, top_k);
    if (workspace_bytes < need)
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "workspace %zu < %zu bytes", workspace_bytes, need);
    uint16_t *ybuf = reinterpret_cast<uint16_t *>(static_cast<char *>(workspace) + moe_experts_ybuf_offset(w));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((s = clear_status(w.status, st)) != VQMOE_OK) return s;
    const bool vq_in = is_vq(gate->format), vq_dn = is_vq(down->format);
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0), P = T * top_k;
        const int32_t *ind = indices + (size_t)t0 * top_k;
        const uint16_t *xt = static_cast<const uint16_t *>(x) + (size_t)t0 * H;
        const RouteWs &rt = w.rt;
        if (vq_in && (s = launch_to_f16(xt, w.x16, (size_t)T * H, st)) != VQMOE_OK) return s;
        if ((s = launch_route(ind, P, E, rt.cnt, rt.off, rt.list, rt.active, rt.rank, rt.zero,
                              rt.zero_words, st)) != VQMOE_OK)
            return s;
        RoutedIO r1 = routed_io(rt, E, top_k, P, vq_in ? (const void *)w.x16 : (const void *)xt, 0,
                                w.act, vq_dn, nullptr);
        r1.xs = w.xs;
        r1.act = gate->activation;
        RoutedIO r2 = routed_io(rt, E, top_k, P, w.act, 1, ybuf, 0, scores + (size_t)t0 * top_k);
        if ((s = launch_experts(gate, up, &r1, down, r2, rt.zero, w.status, 0, st)) != VQMOE_OK) return s;
        const size_t nvec = (size_t)T * (H / 8);
        const int grid = (int)std::min<size_t>((nvec + 255) / 256, (size_t)sm_count() * 8);
        combine_kernel<<<grid, 256, 0, st>>>(ybuf, T, top_k, H, nullptr, nullptr,
                                             static_cast<uint16_t *>(out) + (size_t)t0 * H, 0);
        if ((s = check_launch("combine_kernel")) != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

vqmoe_status vqmoe_switch_linear(const vqmoe_linear *w, const void *x, int32_t x_per_pair,
                                 const int32_t *indices, int32_t tokens, int32_t top_k,
                                 void *y, void *workspace, size_t workspace_bytes, void *stream) {
    vqmoe_status s;
    if ((s = check_linear(w, "switch_linear")) != VQMOE_OK) return s;
    if (tokens <= 0 || top_k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, top_k);
    if (w->num_experts > 1024) return set_error(VQMOE_BAD_SHAPE, "switch_linear: %d experts (<= 1024)", w->num_experts);
    if (!aligned_ptr(x) || !aligned_ptr(y) || !indices || !aligned_ptr(workspace))
        return set_error(VQMOE_BAD_POINTER, "x / indices / y / workspace");
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    const int rows_x = x_per_pair ? chunk * top_k : chunk;
    GluWs ws = carve_glu(workspace, w, nullptr, chunk, top_k, rows_x);
    if (workspace_bytes < ws.bytes)
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "workspace %zu < %zu bytes", workspace_bytes, ws.bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((s = clear_status(ws.status, st)) != VQMOE_OK) return s;
    const bool vq = is_vq(w->format);
    const int IN = w->in_features, E = w->num_experts;
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0), P = T * top_k;
        const size_t xrow0 = x_per_pair ? (size_t)t0 * top_k : (size_t)t0;
        const size_t nrows = x_per_pair ? (size_t)P : (size_t)T;
        const uint16_t *xt = static_cast<const uint16_t *>(x) + xrow0 * IN;
        const RouteWs &rt = ws.rt;
        if (vq && (s = launch_to_f16(xt, ws.x16, nrows * IN, st)) != VQMOE_OK) return s;
        if ((s = launch_route(indices + (size_t)t0 * top_k, P, E, rt.cnt, rt.off, rt.list, rt.active,
                              rt.rank, rt.zero, rt.zero_words, st)) != VQMOE_OK)
            return s;
        RoutedIO r = routed_io(rt, E, top_k, P, vq ? (const void *)ws.x16 : (const void *)xt,
                               x_per_pair, static_cast<uint16_t *>(y) + (size_t)t0 * top_k * w->out_features,
                               0, nullptr);
        r.xs = ws.xs;
        if ((s = launch_experts(nullptr, nullptr, nullptr, w, r, rt.zero, ws.status, 0, st)) != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

vqmoe_status vqmoe_router_ex(const void *x, const void *router_w, const void *sgw,
                             int32_t tokens, int32_t hidden, int32_t num_experts,
                             int32_t top_k, int32_t router_mode, const float *expert_scale, int32_t *inds,
                             float *scores, float *sgate, void *workspace, size_t workspace_bytes, void *stream) {
    if (tokens <= 0 || hidden <= 0 || hidden % 8 || num_experts <= 0 || num_experts > 512 ||
        top_k <= 0 || top_k > 32 || top_k > num_experts)
        return set_error(VQMOE_BAD_SHAPE, "router: T %d H %d E %d k %d", tokens, hidden,
                         num_experts, top_k);
    if (!aligned_ptr(x) || !aligned_ptr(router_w) || (sgw && !aligned16(sgw)) || !inds ||
        !scores || (sgw && !sgate) || !workspace)
        return set_error(VQMOE_BAD_POINTER, "router pointers");
    if (router_mode < VQMOE_ROUTER_SOFTMAX_TOPK_RENORM || router_mode > VQMOE_ROUTER_SOFTMAX_TOPK)
        return set_error(VQMOE_BAD_FORMAT, "router_mode %d (0..2)", router_mode);
    if (workspace_bytes < vqmoe_router_workspace_size(tokens, num_experts))
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "router workspace");
    return launch_router(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(router_w),
                         static_cast<const uint16_t *>(sgw), tokens, hidden, num_experts, top_k,
                         static_cast<float *>(workspace), inds, scores, sgate, nullptr, router_mode,
                         expert_scale, static_cast<cudaStream_t>(stream));
}

vqmoe_status vqmoe_rms_norm(const void *x, const void *weight, int32_t tokens, int32_t hidden, float eps,
                            void *out, void *stream) {
    if (tokens <= 0 || hidden <= 0) return set_error(VQMOE_BAD_SHAPE, "rms_norm: T %d H %d", tokens, hidden);
    if (!(eps >= 0.0f)) return set_error(VQMOE_BAD_SHAPE, "rms_norm: eps %g", (double)eps);
    if (!x || !weight || !out) return set_error(VQMOE_BAD_POINTER, "rms_norm: x / weight / out");
    return launch_rms_norm(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(weight), tokens, hidden,
                           eps, static_cast<uint16_t *>(out), static_cast<cudaStream_t>(stream));
}

vqmoe_status vqmoe_router(const void *x, const void *router_w, const void *sgw, int32_t tokens, int32_t hidden,
                          int32_t num_experts, int32_t top_k, int32_t *inds, float *scores, float *sgate,
                          void *workspace, size_t workspace_bytes, void *stream) {
    return vqmoe_router_ex(x, router_w, sgw, tokens, hidden, num_experts, top_k, VQMOE_ROUTER_SOFTMAX_TOPK_RENORM,
                           nullptr, inds, scores, sgate, workspace, workspace_bytes, stream);
}

}  // extern "C"
