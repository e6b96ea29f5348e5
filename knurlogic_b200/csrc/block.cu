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
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace vqmoe {

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w,
                           const uint16_t *wsg, int T, int H, int E, int k,
                           float *logits, int32_t *inds, float *scores,
                           float *sgate, cudaStream_t stream);
vqmoe_status launch_expert(const vqmoe_linear *w0, const vqmoe_linear *w1,
                           const int32_t *inds, int P, int k, const void *x,
                           int x_per_pair, void *out, const float *pair_scale,
                           int list_cap, cudaStream_t stream);

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
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
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
        for (int s = 0; s < k; ++s) {
            uint4 y = *reinterpret_cast<const uint4 *>(ybuf + ((size_t)tkn * k + s) * H + c8 * 8);
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

static bool aligned_ptr(const void *p) { return p && aligned16(p); }

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

struct BlockWs {
    float *logits;
    int32_t *inds;
    float *scores;
    float *sgate;
    uint16_t *act;
    uint16_t *act_s;
    uint16_t *ybuf;
    uint16_t *sh;
    size_t bytes;
};

static BlockWs carve_block(void *ws, const vqmoe_block *b, int T) {
    Carve c{static_cast<char *>(ws)};
    BlockWs w{};
    const int E1 = b->num_experts + 1;
    const int I = b->gate.out_features;
    (void)E1;
    w.logits = c.take<float>((size_t)T * E1);
    w.inds = c.take<int32_t>((size_t)T * b->top_k);
    w.scores = c.take<float>((size_t)T * b->top_k);
    w.sgate = c.take<float>((size_t)T);
    w.act = c.take<uint16_t>((size_t)T * b->top_k * I);
    w.act_s = c.take<uint16_t>((size_t)T * std::max(b->shared_inter, 0));
    w.ybuf = c.take<uint16_t>((size_t)T * b->top_k * b->hidden);
    w.sh = c.take<uint16_t>((size_t)T * b->hidden);
    w.bytes = align_up(c.off, 256);
    return w;
}

// Tokens per launch of the expert kernels: the per-CTA pair list lives in
// shared memory; a larger T is processed in independent token chunks.
constexpr int kMaxTokensPerLaunch = 2048;

static vqmoe_status check_block(const vqmoe_block *b, int T) {
    if (!b) return set_error(VQMOE_BAD_POINTER, "null block");
    if (T <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d", T);
    const int H = b->hidden, E = b->num_experts, k = b->top_k;
    if (H <= 0 || H % 16) return set_error(VQMOE_BAD_SHAPE, "hidden %d is not a multiple of 16", H);
    if (E <= 0 || E > 512) return set_error(VQMOE_BAD_SHAPE, "num_experts %d (1..512)", E);
    if (k <= 0 || k > 32 || k > E) return set_error(VQMOE_BAD_SHAPE, "top_k %d (1..min(32, E))", k);
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
    if (!aligned_ptr(b->router_w)) return set_error(VQMOE_BAD_POINTER, "router_w");
    if (b->shared_inter < 0 || b->shared_inter % 16)
        return set_error(VQMOE_BAD_SHAPE, "shared_inter %d is not a multiple of 16", b->shared_inter);
    if (b->shared_inter > 0 &&
        (!aligned_ptr(b->shared_gate_w) || !aligned_ptr(b->shared_up_w) ||
         !aligned_ptr(b->shared_down_w) || !aligned_ptr(b->shared_expert_gate_w)))
        return set_error(VQMOE_BAD_POINTER, "shared expert weights null or not 16-byte aligned");
    return VQMOE_OK;
}

static vqmoe_linear dense_linear(const void *w, int out, int in) {
    vqmoe_linear d{};
    d.format = VQMOE_FMT_DENSE_BF16;
    d.num_experts = 1;
    d.out_features = out;
    d.in_features = in;
    d.weight = w;
    return d;
}

// events (optional, n_ev >= 6): recorded before the router and after the
// router, the routed gate/up, the routed down, the shared expert, combine.
static vqmoe_status mark(cudaEvent_t *ev, int n_ev, int i, cudaStream_t st) {
    if (ev && i < n_ev && cudaEventRecord(ev[i], st) != cudaSuccess)
        return set_error(VQMOE_LAUNCH_FAILED, "event %d", i);
    return VQMOE_OK;
}

static vqmoe_status run_block(const vqmoe_block *b, const uint16_t *x, int T,
                              void *out, int out_f32, const BlockWs &w,
                              cudaStream_t st, cudaEvent_t *ev = nullptr, int n_ev = 0) {
    const int H = b->hidden, E = b->num_experts, k = b->top_k;
    const int Is = b->shared_inter;
    const bool shared = Is > 0;
    vqmoe_status s;
    if ((s = mark(ev, n_ev, 0, st)) != VQMOE_OK) return s;
    s = launch_router(x, static_cast<const uint16_t *>(b->router_w),
                                   shared ? static_cast<const uint16_t *>(b->shared_expert_gate_w) : nullptr,
                                   T, H, E, k, w.logits, w.inds, w.scores, w.sgate, st);
    if (s != VQMOE_OK || (s = mark(ev, n_ev, 1, st)) != VQMOE_OK) return s;
    s = launch_expert(&b->gate, &b->up, w.inds, T * k, k, x, 0, w.act, nullptr, T, st);
    if (s != VQMOE_OK || (s = mark(ev, n_ev, 2, st)) != VQMOE_OK) return s;
    s = launch_expert(&b->down, nullptr, w.inds, T * k, k, w.act, 1, w.ybuf, w.scores, T, st);
    if (s != VQMOE_OK || (s = mark(ev, n_ev, 3, st)) != VQMOE_OK) return s;
    if (shared) {
        vqmoe_linear sg = dense_linear(b->shared_gate_w, Is, H);
        vqmoe_linear su = dense_linear(b->shared_up_w, Is, H);
        vqmoe_linear sd = dense_linear(b->shared_down_w, H, Is);
        s = launch_expert(&sg, &su, nullptr, T, 1, x, 1, w.act_s, nullptr, 0, st);
        if (s != VQMOE_OK) return s;
        s = launch_expert(&sd, nullptr, nullptr, T, 1, w.act_s, 1, w.sh, nullptr, 0, st);
        if (s != VQMOE_OK) return s;
    }
    if ((s = mark(ev, n_ev, 4, st)) != VQMOE_OK) return s;
    const size_t nvec = (size_t)T * (H / 8);
    const int grid = (int)std::min<size_t>((nvec + 255) / 256, (size_t)sm_count() * 8);
    combine_kernel<<<grid, 256, 0, st>>>(w.ybuf, T, k, H, shared ? w.sh : nullptr, w.sgate, out, out_f32);
    if ((s = check_launch("combine_kernel")) != VQMOE_OK) return s;
    return mark(ev, n_ev, 5, st);
}

// ------------------------------------------------------ prepare / dequant

// code 4q+t of a chunk of 4*nq codes <-> device position t*nq+q
__global__ void permute_codes_kernel(const uint8_t *__restrict__ src,
                                     uint8_t *__restrict__ dst, long long rows,
                                     int ncodes, int to_device) {
    const long long total = rows * ncodes;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / ncodes;
        const int c = (int)(i - r * ncodes);
        const int c0 = c & ~63, n = min(64, ncodes - c0), nq = n >> 2;
        const int u = c - c0;                     // reference position in chunk
        const int d = c0 + (u & 3) * nq + (u >> 2);  // device position
        if (to_device)
            dst[r * ncodes + d] = src[r * ncodes + c];
        else
            dst[r * ncodes + c] = src[r * ncodes + d];
    }
}

// *bad_count += number of codes >= K (the caller zeroes it first)
__global__ void count_bad_codes_kernel(const uint8_t *__restrict__ codes, long long n, int K,
                                       uint32_t *__restrict__ bad_count) {
    uint32_t bad = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        bad += codes[i] >= K;
    for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(bad_count, bad);
}

__global__ void dequant_kernel(const uint8_t *__restrict__ codes,
                               const uint16_t *__restrict__ cb,
                               const uint16_t *__restrict__ scales, int OUT,
                               int IN, long long first_row, long long rows,
                               uint16_t *__restrict__ out) {
    const int ncodes = IN / 4;
    const long long total = rows * ncodes;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / ncodes;
        const int c = (int)(i - r * ncodes);
        const int c0 = c & ~63, n = min(64, ncodes - c0), nq = n >> 2;
        const int u = c - c0;
        const int d = c0 + (u & 3) * nq + (u >> 2);
        const long long rr = first_row + r;
        const uint32_t code = codes[rr * ncodes + d];
        const uint16_t s = scales[rr * (IN / 64) + (c * 4) / 64];
        const uint32_t s2 = (uint32_t)s | ((uint32_t)s << 16);
        const uint2 e = *reinterpret_cast<const uint2 *>(cb + code * 4);
        const uint2 w = make_uint2(hmul2_u32(e.x, s2), hmul2_u32(e.y, s2));
        *reinterpret_cast<uint2 *>(out + r * IN + c * 4) = w;
    }
}

}  // namespace vqmoe

using namespace vqmoe;

// ------------------------------------------------------------ C ABI

extern "C" {

int32_t vqmoe_abi_version(void) { return VQMOE_ABI_VERSION; }

const char *vqmoe_last_error(void) { return g_err; }

size_t vqmoe_router_workspace_size(int32_t tokens, int32_t num_experts) {
    return align_up((size_t)tokens * (num_experts + 1) * sizeof(float), 256);
}

size_t vqmoe_switch_glu_workspace_size(int32_t tokens, int32_t top_k, int32_t inter) {
    return align_up((size_t)tokens * top_k * inter * 2, 256);
}

size_t vqmoe_block_workspace_size(const vqmoe_block *blk, int32_t tokens) {
    if (!blk || tokens <= 0) return 0;
    return carve_block(nullptr, blk, tokens).bytes;
}

static vqmoe_status block_impl(const vqmoe_block *blk, const void *x, int32_t tokens, void *out,
                               int32_t out_dtype, void *workspace, size_t workspace_bytes,
                               void *stream, cudaEvent_t *ev, int n_ev) {
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
    const size_t osz = out_dtype == VQMOE_OUT_F32 ? 4 : 2;
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0);
        s = run_block(blk, static_cast<const uint16_t *>(x) + (size_t)t0 * blk->hidden, T,
                      static_cast<char *>(out) + (size_t)t0 * blk->hidden * osz,
                      out_dtype == VQMOE_OUT_F32, w, st, t0 == 0 ? ev : nullptr, n_ev);
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

vqmoe_status vqmoe_sparse_moe_block_timed(const vqmoe_block *blk, const void *x, int32_t tokens,
                                          void *out, int32_t out_dtype, void *workspace,
                                          size_t workspace_bytes, void *stream,
                                          void *const *events, int32_t n_events) {
    if (!events || n_events < 6)
        return set_error(VQMOE_BAD_POINTER, "timed block: needs 6 events");
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
    if (tokens <= 0 || top_k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, top_k);
    const int I = gate->out_features, H = gate->in_features;
    if (up->out_features != I || up->in_features != H || down->out_features != H ||
        down->in_features != I || up->num_experts != gate->num_experts ||
        down->num_experts != gate->num_experts || gate->format != up->format)
        return set_error(VQMOE_BAD_SHAPE, "switch_glu: inconsistent gate/up/down shapes");
    if (!aligned_ptr(x) || !aligned_ptr(y) || !indices || !aligned_ptr(workspace))
        return set_error(VQMOE_BAD_POINTER, "x / indices / y / workspace");
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    const size_t need = vqmoe_switch_glu_workspace_size(chunk, top_k, I);
    if (workspace_bytes < need)
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint16_t *act = static_cast<uint16_t *>(workspace);
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0);
        const int32_t *ind = indices + (size_t)t0 * top_k;
        s = launch_expert(gate, up, ind, T * top_k, top_k,
                          static_cast<const uint16_t *>(x) + (size_t)t0 * H, 0, act, nullptr, T, st);
        if (s != VQMOE_OK) return s;
        s = launch_expert(down, nullptr, ind, T * top_k, top_k, act, 1,
                          static_cast<uint16_t *>(y) + (size_t)t0 * top_k * H, nullptr, T, st);
        if (s != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

vqmoe_status vqmoe_switch_linear(const vqmoe_linear *w, const void *x, int32_t x_per_pair,
                                 const int32_t *indices, int32_t tokens, int32_t top_k,
                                 void *y, void *stream) {
    vqmoe_status s;
    if ((s = check_linear(w, "switch_linear")) != VQMOE_OK) return s;
    if (tokens <= 0 || top_k <= 0) return set_error(VQMOE_BAD_SHAPE, "tokens %d top_k %d", tokens, top_k);
    if (!aligned_ptr(x) || !aligned_ptr(y) || !indices)
        return set_error(VQMOE_BAD_POINTER, "x / indices / y");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int chunk = std::min<int>(tokens, kMaxTokensPerLaunch);
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int T = std::min(chunk, tokens - t0);
        const size_t xrow0 = x_per_pair ? (size_t)t0 * top_k : (size_t)t0;
        s = launch_expert(w, nullptr, indices + (size_t)t0 * top_k, T * top_k, top_k,
                          static_cast<const uint16_t *>(x) + xrow0 * w->in_features, x_per_pair,
                          static_cast<uint16_t *>(y) + (size_t)t0 * top_k * w->out_features,
                          nullptr, T, st);
        if (s != VQMOE_OK) return s;
    }
    return VQMOE_OK;
}

vqmoe_status vqmoe_router(const void *x, const void *router_w, const void *sgw,
                          int32_t tokens, int32_t hidden, int32_t num_experts,
                          int32_t top_k, int32_t *inds, float *scores, float *sgate,
                          void *workspace, size_t workspace_bytes, void *stream) {
    if (tokens <= 0 || hidden <= 0 || hidden % 8 || num_experts <= 0 || num_experts > 512 ||
        top_k <= 0 || top_k > 32 || top_k > num_experts)
        return set_error(VQMOE_BAD_SHAPE, "router: T %d H %d E %d k %d", tokens, hidden,
                         num_experts, top_k);
    if (!aligned_ptr(x) || !aligned_ptr(router_w) || (sgw && !aligned16(sgw)) || !inds ||
        !scores || (sgw && !sgate) || !workspace)
        return set_error(VQMOE_BAD_POINTER, "router pointers");
    if (workspace_bytes < vqmoe_router_workspace_size(tokens, num_experts))
        return set_error(VQMOE_WORKSPACE_TOO_SMALL, "router workspace");
    return launch_router(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(router_w),
                         static_cast<const uint16_t *>(sgw), tokens, hidden, num_experts, top_k,
                         static_cast<float *>(workspace), inds, scores, sgate,
                         static_cast<cudaStream_t>(stream));
}

vqmoe_status vqmoe_dequant(const vqmoe_linear *w, int32_t first, int32_t count, void *out,
                           void *stream) {
    vqmoe_status s;
    if ((s = check_linear(w, "dequant")) != VQMOE_OK) return s;
    if (w->format != VQMOE_FMT_VQ_U8) return set_error(VQMOE_BAD_FORMAT, "dequant: not a VQ linear");
    if (first < 0 || count <= 0 || first + count > w->num_experts)
        return set_error(VQMOE_BAD_SHAPE, "dequant: experts [%d, %d) of %d", first, first + count,
                         w->num_experts);
    if (!aligned_ptr(out)) return set_error(VQMOE_BAD_POINTER, "dequant: out");
    const long long rows = (long long)count * w->out_features;
    const long long total = rows * (w->in_features / 4);
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)sm_count() * 16);
    dequant_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(w->codes), static_cast<const uint16_t *>(w->codebook),
        static_cast<const uint16_t *>(w->scales), w->out_features, w->in_features,
        (long long)first * w->out_features, rows, static_cast<uint16_t *>(out));
    return check_launch("dequant_kernel");
}

static vqmoe_status permute(const uint8_t *src, uint8_t *dst, int64_t rows, int32_t ncodes,
                            int to_device, void *stream) {
    if (!src || !dst || rows <= 0 || ncodes <= 0 || ncodes % 16)
        return set_error(VQMOE_BAD_SHAPE, "codes: rows %lld codes_per_row %d (a multiple of 16)",
                         (long long)rows, ncodes);
    if (src == dst) return set_error(VQMOE_BAD_POINTER, "codes: src and dst must not overlap");
    const long long total = (long long)rows * ncodes;
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)sm_count() * 16);
    permute_codes_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(src, dst, rows, ncodes,
                                                                            to_device);
    return check_launch("permute_codes_kernel");
}

vqmoe_status vqmoe_prepare_codes(const uint8_t *src, uint8_t *dst, int64_t rows,
                                 int32_t codes_per_row, void *stream) {
    return permute(src, dst, rows, codes_per_row, 1, stream);
}

vqmoe_status vqmoe_unprepare_codes(const uint8_t *src, uint8_t *dst, int64_t rows,
                                   int32_t codes_per_row, void *stream) {
    return permute(src, dst, rows, codes_per_row, 0, stream);
}

vqmoe_status vqmoe_count_bad_codes(const uint8_t *codes, int64_t count, int32_t codebook_size,
                                   uint32_t *bad_count, void *stream) {
    if (!codes || !bad_count || count <= 0)
        return set_error(VQMOE_BAD_POINTER, "count_bad_codes: pointers / count");
    if (codebook_size <= 0 || codebook_size > 256)
        return set_error(VQMOE_BAD_FORMAT, "codebook_size %d (1..256)", codebook_size);
    const int grid = (int)std::min<long long>((count + 255) / 256, (long long)sm_count() * 16);
    count_bad_codes_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, count,
                                                                              codebook_size, bad_count);
    return check_launch("count_bad_codes_kernel");
}

}  // extern "C"
