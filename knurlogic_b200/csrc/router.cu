// Router of the Qwen3.5-MoE sparse block on B200.
//
// Reference: src/knurlogic/engine/families/qwen/architecture/qwen3_5.py:174-179
//   logits = self.gate(x)                                (bf16 Linear)
//   probs  = softmax(logits.astype(float32))
//   inds   = argpartition(probs, -k)[..., -k:]
//   scores = (p[inds] / p[inds].sum()).astype(bf16)
// and the shared-expert gate of qwen3_5.py:186, bf16(sigmoid(bf16(x @ w_sg))).
//
// Kernel 1 (router_logits_kernel) computes the [T, E(+1)] logits. Each
// product of two bf16 values is exact in float64 and the dot product
// accumulates in float64, then rounds ONCE to bf16: the logits are the
// correctly rounded values (up to a ~2^-45 relative error), so the expert
// choice downstream is the same as any exact implementation's.
// Kernel 2 (router_topk_kernel) runs one warp per token: float32 softmax,
// k rounds of a warp arg-max on (logit, -index), float32 renormalisation.
#include "common.cuh"

namespace vqmoe {

constexpr int kRouterTok = 8;       // tokens per CTA (staged in SMEM)
constexpr int kRouterRows = 8;      // router rows per CTA (one per warp)

__global__ void __launch_bounds__(256)
router_logits_kernel(const uint16_t *__restrict__ x,
                     const uint16_t *__restrict__ w,
                     const uint16_t *__restrict__ wsg, int T, int H, int E,
                     int E1, float *__restrict__ logits) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.y * kRouterTok;
    // stage kRouterTok token rows (zero past T), 16 bytes per access
    const int vec_per_row = H / 8;
    for (int v = tid; v < kRouterTok * vec_per_row; v += blockDim.x) {
        int r = v / vec_per_row, c = v - r * vec_per_row;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (t0 + r < T)
            val = *reinterpret_cast<const uint4 *>(x + (size_t)(t0 + r) * H + c * 8);
        *reinterpret_cast<uint4 *>(xs + (size_t)r * H + c * 8) = val;
    }
    __syncthreads();
    const int row = blockIdx.x * kRouterRows + warp;
    if (row >= E1) return;
    const uint16_t *wr = row < E ? w + (size_t)row * H : wsg;
    double acc[kRouterTok];
#pragma unroll
    for (int i = 0; i < kRouterTok; ++i) acc[i] = 0.0;
    for (int h = lane * 8; h < H; h += 256) {
        uint4 wv = *reinterpret_cast<const uint4 *>(wr + h);
        const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
        double wd[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wd[2 * j] = (double)bf16_to_f32(wu[j] & 0xFFFFu);
            wd[2 * j + 1] = (double)bf16_to_f32(wu[j] >> 16);
        }
#pragma unroll
        for (int i = 0; i < kRouterTok; ++i) {
            uint4 xv = *reinterpret_cast<const uint4 *>(xs + (size_t)i * H + h);
            const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[i] = fma((double)bf16_to_f32(xu[j] & 0xFFFFu), wd[2 * j], acc[i]);
                acc[i] = fma((double)bf16_to_f32(xu[j] >> 16), wd[2 * j + 1], acc[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kRouterTok; ++i) {
        double v = acc[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[i] = v;
    }
    if (lane < kRouterTok && t0 + lane < T) {
        double v = acc[0];
#pragma unroll
        for (int i = 1; i < kRouterTok; ++i)
            if (lane == i) v = acc[i];
        logits[(size_t)(t0 + lane) * E1 + row] = bf16_to_f32(f64_to_bf16(v));
    }
}

constexpr int kMaxExpertsPerLane = 16;   // E <= 512

__global__ void __launch_bounds__(256)
router_topk_kernel(const float *__restrict__ logits, int T, int E, int E1,
                   int k, int has_shared, int32_t *__restrict__ inds,
                   float *__restrict__ scores, float *__restrict__ sgate) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= T) return;
    const float *lr = logits + (size_t)t * E1;
    float l[kMaxExpertsPerLane];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
        int j = lane + 32 * i;
        l[i] = j < E ? lr[j] : -INFINITY;
        m = fmaxf(m, l[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float ex[kMaxExpertsPerLane];
    float z = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
        int j = lane + 32 * i;
        ex[i] = j < E ? expf(l[i] - m) : 0.0f;
        z += ex[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    uint32_t taken = 0;
    float psel[32];
    int isel[32];
    for (int s = 0; s < k; ++s) {
        float bl = -INFINITY;
        int bj = 0x7fffffff;
        float be = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxExpertsPerLane; ++i) {
            int j = lane + 32 * i;
            bool ok = j < E && !((taken >> i) & 1u);
            // ascending j inside the lane: strict > keeps the lower index
            if (ok && (l[i] > bl || bj == 0x7fffffff)) {
                bl = l[i];
                bj = j;
                be = ex[i];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ol = __shfl_xor_sync(0xffffffffu, bl, o);
            int oj = __shfl_xor_sync(0xffffffffu, bj, o);
            float oe = __shfl_xor_sync(0xffffffffu, be, o);
            bool better = (oj != 0x7fffffff) &&
                          (bj == 0x7fffffff || ol > bl || (ol == bl && oj < bj));
            if (better) {
                bl = ol;
                bj = oj;
                be = oe;
            }
        }
        if ((bj & 31) == lane) taken |= 1u << (bj >> 5);
        isel[s] = bj;
        psel[s] = be / z;
    }
    if (lane == 0) {
        float den = 0.0f;
        for (int s = 0; s < k; ++s) den += psel[s];
        for (int s = 0; s < k; ++s) {
            inds[(size_t)t * k + s] = isel[s];
            scores[(size_t)t * k + s] = bf16r(psel[s] / den);
        }
        if (has_shared) sgate[t] = bf16r(sigmoid_f32(lr[E]));
    }
}

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w,
                           const uint16_t *wsg, int T, int H, int E, int k,
                           float *logits, int32_t *inds, float *scores,
                           float *sgate, cudaStream_t stream) {
    const int E1 = E + (wsg ? 1 : 0);
    size_t smem = (size_t)kRouterTok * H * sizeof(uint16_t);
    static int configured_smem[64] = {0};   // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && (dev < 0 || dev >= 64 || (int)smem > configured_smem[dev])) {
        if (cudaFuncSetAttribute(router_logits_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return set_error(VQMOE_LAUNCH_FAILED, "router: smem %zu", smem);
        if (dev >= 0 && dev < 64) configured_smem[dev] = (int)smem;
    }
    dim3 g1((E1 + kRouterRows - 1) / kRouterRows, (T + kRouterTok - 1) / kRouterTok);
    router_logits_kernel<<<g1, 256, smem, stream>>>(x, w, wsg, T, H, E, E1, logits);
    vqmoe_status s = check_launch("router_logits_kernel");
    if (s != VQMOE_OK) return s;
    router_topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(logits, T, E, E1, k,
                                                        wsg != nullptr, inds,
                                                        scores, sgate);
    return check_launch("router_topk_kernel");
}

}  // namespace vqmoe
