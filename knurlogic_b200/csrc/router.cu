// Router of the Qwen3.5-MoE sparse block on B200, and the routing tables
// the expert kernels read.
//
// Reference: src/knurlogic/engine/families/qwen/architecture/qwen3_5.py:174-179
//   logits = self.gate(x)                                (bf16 Linear)
//   probs  = softmax(logits.astype(float32))
//   inds   = argpartition(probs, -k)[..., -k:]
//   scores = (p[inds] / p[inds].sum()).astype(bf16)
// and the shared-expert gate of qwen3_5.py:186, bf16(sigmoid(bf16(x @ w_sg))).
//
// router_logits_kernel (any H % 16 == 0) / router_logits_dmma_kernel
//   (H % 128 == 0, fp64 tensor cores): the [T, E(+1)] logits. Each product of two bf16
//   values is exact in float64 and the dot product accumulates in float64,
//   then rounds ONCE to bf16: the logits are correctly rounded (up to a
//   ~2^-45 relative error), so the expert choice is the one any exact
//   implementation makes. Each lane holds its slice of a router row in
//   registers; the CTA's tokens are staged in shared memory. The CTAs of the
//   first row block also write x as fp16 (saturated) for the VQ experts.
// router_topk_kernel: one warp per token: float32 softmax, k rounds of a
//   warp arg-max on (logit, -index), float32 renormalisation.
// route_kernel: one CTA: counting sort of the T*k (token, slot) pairs by
//   expert -> per-expert count / offset / pair list, the list of experts
//   that received pairs, and zeroed work counters for the expert kernels.
#include "common.cuh"

namespace vqmoe {

constexpr int kRouterTok = 16;      // tokens per CTA (staged in SMEM)
constexpr int kRouterRows = 8;      // router rows per CTA (one per warp)
constexpr int kRouterMaxSeg = 8;    // 8 * 256 inputs of a row in registers per pass

__global__ void __launch_bounds__(256)
router_logits_kernel(const uint16_t *__restrict__ x,
                     const uint16_t *__restrict__ w,
                     const uint16_t *__restrict__ wsg, int T, int H, int E,
                     int E1, float *__restrict__ logits,
                     uint16_t *__restrict__ x16) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.y * kRouterTok;
    const int vec_per_row = H / 8;
    for (int v = tid; v < kRouterTok * vec_per_row; v += blockDim.x) {
        int r = v / vec_per_row, c = v - r * vec_per_row;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (t0 + r < T) {
            val = *reinterpret_cast<const uint4 *>(x + (size_t)(t0 + r) * H + c * 8);
            if (x16 && blockIdx.x == 0) {
                uint32_t u[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    u[j] = (uint32_t)bf16_to_f16_sat(u[j] & 0xFFFFu) |
                           ((uint32_t)bf16_to_f16_sat(u[j] >> 16) << 16);
                *reinterpret_cast<uint4 *>(x16 + (size_t)(t0 + r) * H + c * 8) =
                    make_uint4(u[0], u[1], u[2], u[3]);
            }
        }
        *reinterpret_cast<uint4 *>(xs + (size_t)r * H + c * 8) = val;
    }
    __syncthreads();
    const int row = blockIdx.x * kRouterRows + warp;
    if (row >= E1) return;
    const uint16_t *wr = row < E ? w + (size_t)row * H : wsg;
    const int ntok = min(kRouterTok, T - t0);
    double acc[kRouterTok];
#pragma unroll
    for (int i = 0; i < kRouterTok; ++i) acc[i] = 0.0;
    for (int h0 = 0; h0 < H; h0 += kRouterMaxSeg * 256) {
        // this lane's slice of the row, all loads in flight at once
        uint4 wv[kRouterMaxSeg];
#pragma unroll
        for (int s = 0; s < kRouterMaxSeg; ++s) {
            const int h = h0 + s * 256 + lane * 8;
            wv[s] = h < H ? *reinterpret_cast<const uint4 *>(wr + h) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int s = 0; s < kRouterMaxSeg; ++s) {
            const int h = h0 + s * 256 + lane * 8;
            if (h >= H) break;
            const uint32_t wu[4] = {wv[s].x, wv[s].y, wv[s].z, wv[s].w};
            double wd[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                wd[2 * j] = (double)bf16_to_f32(wu[j] & 0xFFFFu);
                wd[2 * j + 1] = (double)bf16_to_f32(wu[j] >> 16);
            }
#pragma unroll
            for (int i = 0; i < kRouterTok; ++i) {
                if (i < ntok) {
                    uint4 xv = *reinterpret_cast<const uint4 *>(xs + (size_t)i * H + h);
                    const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[i] = fma((double)bf16_to_f32(xu[j] & 0xFFFFu), wd[2 * j], acc[i]);
                        acc[i] = fma((double)bf16_to_f32(xu[j] >> 16), wd[2 * j + 1], acc[i]);
                    }
                }
            }
        }
    }
    double mine = 0.0;
#pragma unroll
    for (int i = 0; i < kRouterTok; ++i) {
        double v = acc[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == i) mine = v;
    }
    if (lane < ntok)
        logits[(size_t)(t0 + lane) * E1 + row] = bf16_to_f32(f64_to_bf16(mine));
}

// Tensor-core variant (H % 128 == 0): fp64 MMA m8n8k4 (A = 8 tokens x 4
// inputs, B = 4 inputs x 8 router rows, fp64 accumulate). bf16 values
// convert exactly to fp64 and each product is exact, as in the CUDA-core
// kernel. A CTA owns an 8 x 8 tile of logits; its 4 warps split H; lane
// (g, t) feeds inputs [q*H/4 + t*H/16, +H/16) of warp q in order -- one
// permutation of the k axis applied to A and B alike -- so every lane
// reads contiguous 16-byte vectors. The 4 warp partials (each summed over
// two interleaved accumulators) are added in a fixed order.
__device__ __forceinline__ void dmma_f64(double (&d)[2], double a, double b) {
    asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
        : "+d"(d[0]), "+d"(d[1])
        : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(128)
router_logits_dmma_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                          const uint16_t *__restrict__ wsg, int T, int H, int E, int E1,
                          float *__restrict__ logits, uint16_t *__restrict__ x16) {
    __shared__ double part[4][8][8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int t0 = blockIdx.y * 8, e0 = blockIdx.x * 8;
    if (x16 && blockIdx.x == 0) {   // fp16 copy of this CTA's tokens for the VQ experts
        const int vpr = H / 8;
        for (int v = tid; v < 8 * vpr; v += blockDim.x) {
            const int r = v / vpr, c = v - r * vpr;
            if (t0 + r >= T) continue;
            const uint4 val = *reinterpret_cast<const uint4 *>(x + (size_t)(t0 + r) * H + c * 8);
            uint32_t u[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                u[j] = (uint32_t)bf16_to_f16_sat(u[j] & 0xFFFFu) | ((uint32_t)bf16_to_f16_sat(u[j] >> 16) << 16);
            *reinterpret_cast<uint4 *>(x16 + (size_t)(t0 + r) * H + c * 8) = make_uint4(u[0], u[1], u[2], u[3]);
        }
    }
    const int seg = H >> 4;                      // inputs per lane
    const int k0 = warp * (H >> 2) + t * seg;
    const int tok = t0 + g, row = e0 + g;
    const bool tok_ok = tok < T, row_ok = row < E1;
    const uint16_t *xp = x + (size_t)(tok_ok ? tok : 0) * H + k0;
    const uint16_t *wp = (row < E ? w + (size_t)row * H : wsg) + k0;
    double d0[2] = {0.0, 0.0}, d1[2] = {0.0, 0.0};
    for (int j = 0; j < seg; j += 8) {
        const uint4 xv = tok_ok ? *reinterpret_cast<const uint4 *>(xp + j) : make_uint4(0, 0, 0, 0);
        const uint4 wv = row_ok ? *reinterpret_cast<const uint4 *>(wp + j) : make_uint4(0, 0, 0, 0);
        const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dmma_f64(d0, (double)bf16_to_f32(xu[i] & 0xFFFFu), (double)bf16_to_f32(wu[i] & 0xFFFFu));
            dmma_f64(d1, (double)bf16_to_f32(xu[i] >> 16), (double)bf16_to_f32(wu[i] >> 16));
        }
    }
    // D fragment: (token g, rows 2t, 2t+1)
    part[warp][g][2 * t] = d0[0] + d1[0];
    part[warp][g][2 * t + 1] = d0[1] + d1[1];
    __syncthreads();
    if (tid < 64) {
        const int tg = tid >> 3, rr = tid & 7;
        const double v = ((part[0][tg][rr] + part[1][tg][rr]) + part[2][tg][rr]) + part[3][tg][rr];
        if (t0 + tg < T && e0 + rr < E1)
            logits[(size_t)(t0 + tg) * E1 + e0 + rr] = bf16_to_f32(f64_to_bf16(v));
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
    float den = 0.0f, my_p = 0.0f;
    int my_j = 0;
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
        const float p = be / z;
        den += p;                 // sequential float32 sum, selection order
        if (lane == s) {          // lane s keeps slot s (k <= 32)
            my_p = p;
            my_j = bj;
        }
    }
    if (lane < k) {
        inds[(size_t)t * k + lane] = my_j;
        scores[(size_t)t * k + lane] = bf16r(my_p / den);
    }
    if (lane == 0 && has_shared) sgate[t] = bf16r(sigmoid_f32(lr[E]));
}

// Counting sort of pairs by expert (one CTA). Out-of-range expert ids are
// dropped (their pairs get no output). Also zeroes `zero_words` words at
// `zero` (the expert kernels' work counters and split-K semaphores).
__global__ void __launch_bounds__(1024)
route_kernel(const int32_t *__restrict__ inds, int P, int E,
             int32_t *__restrict__ cnt, int32_t *__restrict__ off,
             int32_t *__restrict__ list, int32_t *__restrict__ active,
             int32_t *__restrict__ rank_scratch, uint32_t *__restrict__ zero,
             int zero_words) {
    extern __shared__ int32_t s_route[];
    int32_t *s_cnt = s_route;          // [E]
    int32_t *s_off = s_route + E;      // [E]
    __shared__ int32_t s_wsum[32], s_asum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < zero_words; i += blockDim.x) zero[i] = 0u;
    for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = inds[p];
        rank_scratch[p] = (e >= 0 && e < E) ? atomicAdd(&s_cnt[e], 1) : -1;
    }
    __syncthreads();
    // exclusive scan of counts and of (count > 0), E <= 1024
    const int e = tid;
    const int c = e < E ? s_cnt[e] : 0;
    const int a = c > 0;
    int ic = c, ia = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, ic, o);
        int v = __shfl_up_sync(0xffffffffu, ia, o);
        if (lane >= o) {
            ic += u;
            ia += v;
        }
    }
    if (lane == 31) {
        s_wsum[warp] = ic;
        s_asum[warp] = ia;
    }
    __syncthreads();
    if (warp == 0) {
        int wc = s_wsum[lane], wa = s_asum[lane];
        int xc = wc, xa = wa;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int u = __shfl_up_sync(0xffffffffu, xc, o);
            int v = __shfl_up_sync(0xffffffffu, xa, o);
            if (lane >= o) {
                xc += u;
                xa += v;
            }
        }
        s_wsum[lane] = xc - wc;   // exclusive warp prefix
        s_asum[lane] = xa - wa;
    }
    __syncthreads();
    if (e < E) {
        const int oc = s_wsum[warp] + ic - c;
        const int oa = s_asum[warp] + ia - a;
        s_off[e] = oc;
        cnt[e] = c;
        off[e] = oc;
        if (a) active[oa] = e;
        if (e == E - 1) {
            off[E] = oc + c;
            active[E] = oa + a;   // number of active experts
        }
    }
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int r = rank_scratch[p];
        if (r >= 0) list[s_off[inds[p]] + r] = p;
    }
}

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w,
                           const uint16_t *wsg, int T, int H, int E, int k,
                           float *logits, int32_t *inds, float *scores,
                           float *sgate, uint16_t *x16, cudaStream_t stream) {
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
    vqmoe_status s;
    if (H % 128 == 0) {
        dim3 gt((E1 + 7) / 8, (T + 7) / 8);
        router_logits_dmma_kernel<<<gt, 128, 0, stream>>>(x, w, wsg, T, H, E, E1, logits, x16);
        s = check_launch("router_logits_dmma_kernel");
    } else {
        dim3 g1((E1 + kRouterRows - 1) / kRouterRows, (T + kRouterTok - 1) / kRouterTok);
        router_logits_kernel<<<g1, 256, smem, stream>>>(x, w, wsg, T, H, E, E1, logits, x16);
        s = check_launch("router_logits_kernel");
    }
    if (s != VQMOE_OK) return s;
    router_topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(logits, T, E, E1, k,
                                                        wsg != nullptr, inds,
                                                        scores, sgate);
    return check_launch("router_topk_kernel");
}

vqmoe_status launch_route(const int32_t *inds, int P, int E, int32_t *cnt,
                          int32_t *off, int32_t *list, int32_t *active,
                          int32_t *rank_scratch, uint32_t *zero, int zero_words,
                          cudaStream_t stream) {
    if (E > 1024) return set_error(VQMOE_BAD_SHAPE, "route: %d experts (<= 1024)", E);
    route_kernel<<<1, 1024, 2 * E * sizeof(int32_t), stream>>>(
        inds, P, E, cnt, off, list, active, rank_scratch, zero, zero_words);
    return check_launch("route_kernel");
}

}  // namespace vqmoe
