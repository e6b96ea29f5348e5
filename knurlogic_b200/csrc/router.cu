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
//   (H % 256 == 0, fp64 tensor cores): the [T, E(+1)] logits. Each product of two bf16
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
#include "stages.cuh"

namespace vqmoe {

constexpr int kRouterTok = 16;      // tokens per CTA (staged in SMEM)
constexpr int kRouterRows = 8;      // router rows per CTA (one per warp)
constexpr int kRouterMaxSeg = 8;    // 8 * 256 inputs of a row in registers per pass

__global__ void __launch_bounds__(256)
router_logits_kernel(const uint16_t *__restrict__ x,
                     const uint16_t *__restrict__ w,
                     const uint16_t *__restrict__ wsg, int T, int H, int E,
                     int E1, float *__restrict__ logits,
                     uint16_t *__restrict__ x16, uint32_t *__restrict__ zero2, int nzero2) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (zero2 && blockIdx.x == 0 && blockIdx.y == 0)   // the routing kernel's counters
        for (int i = tid; i < nzero2; i += blockDim.x) zero2[i] = 0u;
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

// Tensor-core variant (H % 256 == 0): fp64 MMA m8n8k4 (A = 8 tokens x 4
// inputs, B = 4 inputs x 8 router rows, fp64 accumulate). bf16 values
// convert exactly to fp64 and each product is exact, as in the CUDA-core
// kernel. A CTA owns an 8 x 8 tile of logits; its 8 warps split H; lane
// (g, t) feeds inputs [q*H/8 + t*H/32, +H/32) of warp q in order -- one
// permutation of the k axis applied to A and B alike -- so every lane
// reads contiguous 16-byte vectors, all issued before the first MMA. The
// warp partials (each summed over two interleaved accumulators) are added
// in a fixed order.
__device__ __forceinline__ void dmma_f64(double (&d)[2], double a, double b) {
    asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
        : "+d"(d[0]), "+d"(d[1])
        : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256)
router_logits_dmma_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                          const uint16_t *__restrict__ wsg, int T, int H, int E, int E1,
                          float *__restrict__ logits, uint16_t *__restrict__ x16, uint32_t *__restrict__ zero2,
                          int nzero2) {
    constexpr int NW = 8;                        // warps splitting H
    __shared__ double part[NW][8][8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (zero2 && blockIdx.x == 0 && blockIdx.y == 0)   // the routing kernel's counters
        for (int i = tid; i < nzero2; i += blockDim.x) zero2[i] = 0u;
    const int g = lane >> 2, t = lane & 3;
    const int t0 = blockIdx.y * 8, e0 = blockIdx.x * 8;
    pdl_trigger();                   // the routing kernel may launch and wait for these logits
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
    const int seg = H / (4 * NW);                // inputs per lane (multiple of 8)
    const int k0 = warp * (H / NW) + t * seg;
    const int tok = t0 + g, row = e0 + g;
    const bool tok_ok = tok < T, row_ok = row < E1;
    const uint16_t *xp = x + (size_t)(tok_ok ? tok : 0) * H + k0;
    const uint16_t *wp = (row < E ? w + (size_t)row * H : (wsg ? wsg : w)) + k0;
    double d0[2] = {0.0, 0.0}, d1[2] = {0.0, 0.0}, d2[2] = {0.0, 0.0}, d3[2] = {0.0, 0.0};
    for (int j0 = 0; j0 < seg; j0 += 64) {       // up to 8 vectors of each in flight
        uint4 xv[8], wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool in = j0 + 8 * i < seg;
            xv[i] = (tok_ok && in) ? __ldg(reinterpret_cast<const uint4 *>(xp + j0 + 8 * i)) : make_uint4(0, 0, 0, 0);
            wv[i] = (row_ok && in) ? __ldg(reinterpret_cast<const uint4 *>(wp + j0 + 8 * i)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t xu[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
            const uint32_t wu[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
            for (int q = 0; q < 4; q += 2) {
                dmma_f64(d0, (double)bf16_to_f32(xu[q] & 0xFFFFu), (double)bf16_to_f32(wu[q] & 0xFFFFu));
                dmma_f64(d1, (double)bf16_to_f32(xu[q] >> 16), (double)bf16_to_f32(wu[q] >> 16));
                dmma_f64(d2, (double)bf16_to_f32(xu[q + 1] & 0xFFFFu), (double)bf16_to_f32(wu[q + 1] & 0xFFFFu));
                dmma_f64(d3, (double)bf16_to_f32(xu[q + 1] >> 16), (double)bf16_to_f32(wu[q + 1] >> 16));
            }
        }
    }
    // D fragment: (token g, rows 2t, 2t+1)
    part[warp][g][2 * t] = (d0[0] + d1[0]) + (d2[0] + d3[0]);
    part[warp][g][2 * t + 1] = (d0[1] + d1[1]) + (d2[1] + d3[1]);
    __syncthreads();
    if (tid < 64) {
        const int tg = tid >> 3, rr = tid & 7;
        double v = part[0][tg][rr];
#pragma unroll
        for (int q = 1; q < NW; ++q) v += part[q][tg][rr];
        if (t0 + tg < T && e0 + rr < E1)
            logits[(size_t)(t0 + tg) * E1 + e0 + rr] = bf16_to_f32(f64_to_bf16(v));
    }
}

// Register-blocked variant for many tokens (T >= kBlkMinTok, E1 <= 144,
// H % 256 == 0): a CTA owns 8 MT tokens x every logit column. Its 8 warps
// are NG column groups x 8 / NG slices of H; a warp keeps the fp64
// accumulators of its MT x (up to NPG) tiles of 8 x 8, reusing each token
// fragment for all its column tiles and each (converted) weight fragment
// for all MT token tiles. Lane (g, t) of slice q feeds inputs
// q*H/KS + t*H/(4 KS) + j of MMA j (one permutation of the k axis for A and
// B alike), read as 16-byte vectors one batch of 8 MMAs ahead. The slice
// partials are added in a fixed order (slice 0 first), then rounded once to
// bf16.
constexpr int kBlkMinTok = 1024;
constexpr int kBlkMaxNt = 18;                    // E1 <= 144

__device__ __forceinline__ double bf16_f64(uint32_t h) { return (double)__uint_as_float(h << 16); }

template <int MT, int NG>
__global__ void __launch_bounds__(256)
router_logits_dmma_blk_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                              const uint16_t *__restrict__ wsg, int T, int H, int E, int E1,
                              float *__restrict__ logits, uint16_t *__restrict__ x16) {
    constexpr int KS = 8 / NG;
    constexpr int NPG = (kBlkMaxNt + NG - 1) / NG;
    __shared__ double part[KS][8 * MT][kBlkMaxNt * 8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kq = warp % KS, ng = warp / KS;
    const int NT = (E1 + 7) >> 3, per = (NT + NG - 1) / NG;
    const int nt0 = min(ng * per, NT), nnt = min(per, NT - nt0);   // this warp's column tiles
    const int t0 = blockIdx.x * 8 * MT;
    pdl_trigger();                   // the routing kernel may launch and wait for these logits
    const int S = H / (4 * KS);      // inputs per lane per slice (multiple of 8)
    const int k0 = kq * (H / KS) + t * S;
    const uint16_t *xp[MT];
    bool tok_ok[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int tok = t0 + 8 * mt + g;
        tok_ok[mt] = tok < T;
        xp[mt] = x + (size_t)(tok_ok[mt] ? tok : 0) * H + k0;
    }
    const uint16_t *wp[NPG];
    bool row_ok[NPG];
#pragma unroll
    for (int n = 0; n < NPG; ++n) {
        const int row = (nt0 + n) * 8 + g;
        row_ok[n] = n < nnt && row < E1;
        wp[n] = (row < E ? w + (size_t)row * H : (wsg ? wsg : w)) + k0;
    }
    double acc[MT][NPG][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int n = 0; n < NPG; ++n) acc[mt][n][0] = acc[mt][n][1] = 0.0;
    uint4 xv[MT], wv[NPG];
    auto load = [&](int j0) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
            xv[mt] = tok_ok[mt] ? __ldg(reinterpret_cast<const uint4 *>(xp[mt] + j0)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int n = 0; n < NPG; ++n)
            wv[n] = row_ok[n] ? __ldg(reinterpret_cast<const uint4 *>(wp[n] + j0)) : make_uint4(0, 0, 0, 0);
    };
    load(0);
    for (int j0 = 0; j0 < S; j0 += 8) {
        uint4 xc[MT], wc[NPG];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) xc[mt] = xv[mt];
#pragma unroll
        for (int n = 0; n < NPG; ++n) wc[n] = wv[n];
        if (j0 + 8 < S) load(j0 + 8);
        if (x16 && ng == 0) {                // fp16 copy of the tokens for the VQ experts
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                if (!tok_ok[mt]) continue;
                const uint32_t u[4] = {xc[mt].x, xc[mt].y, xc[mt].z, xc[mt].w};
                uint32_t h[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    h[q] = (uint32_t)bf16_to_f16_sat(u[q] & 0xFFFFu) | ((uint32_t)bf16_to_f16_sat(u[q] >> 16) << 16);
                *reinterpret_cast<uint4 *>(x16 + (size_t)(t0 + 8 * mt + g) * H + k0 + j0) =
                    make_uint4(h[0], h[1], h[2], h[3]);
            }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            double a[MT];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint32_t xq = (q >> 1) == 0 ? xc[mt].x : (q >> 1) == 1 ? xc[mt].y : (q >> 1) == 2 ? xc[mt].z : xc[mt].w;
                a[mt] = bf16_f64((xq >> (16 * (q & 1))) & 0xFFFFu);
            }
#pragma unroll
            for (int n = 0; n < NPG; ++n) {
                if (n < nnt) {
                    const uint32_t wq = (q >> 1) == 0 ? wc[n].x : (q >> 1) == 1 ? wc[n].y : (q >> 1) == 2 ? wc[n].z : wc[n].w;
                    const double b = bf16_f64((wq >> (16 * (q & 1))) & 0xFFFFu);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) dmma_f64(acc[mt][n], a[mt], b);
                }
            }
        }
    }
    // D fragment of tile (mt, n): (token 8mt + g, columns 8 (nt0 + n) + 2t, + 1)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int n = 0; n < NPG; ++n)
            if (n < nnt) {
                part[kq][8 * mt + g][(nt0 + n) * 8 + 2 * t] = acc[mt][n][0];
                part[kq][8 * mt + g][(nt0 + n) * 8 + 2 * t + 1] = acc[mt][n][1];
            }
    __syncthreads();
    const int cols = NT * 8;
    for (int o = tid; o < 8 * MT * cols; o += 256) {
        const int tg = o / cols, c = o - tg * cols;
        double v = part[0][tg][c];
#pragma unroll
        for (int q = 1; q < KS; ++q) v += part[q][tg][c];
        if (t0 + tg < T && c < E1) logits[(size_t)(t0 + tg) * E1 + c] = bf16_to_f32(f64_to_bf16(v));
    }
}

// The same with the m16n8k8 fp64 MMA and 16 tokens per CTA: per MMA lane
// (g, t) feeds k-slots t and t + 4 with two consecutive inputs of its
// segment (a0 / a1: tokens g / g + 8 at slot t, a2 / a3 at slot t + 4;
// b0 / b1: column g at slots t / t + 4), so a 16-byte vector covers 4 MMAs.
__device__ __forceinline__ void dmma_f64_k8(double (&d)[4], double a0, double a1, double a2, double a3, double b0,
                                            double b1) {
    asm("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(a2), "d"(a3), "d"(b0), "d"(b1));
}

template <int NG>
__global__ void __launch_bounds__(256)
router_logits_dmma16_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                            const uint16_t *__restrict__ wsg, int T, int H, int E, int E1,
                            float *__restrict__ logits, uint16_t *__restrict__ x16) {
    constexpr int KS = 8 / NG;
    constexpr int NPG = (kBlkMaxNt + NG - 1) / NG;
    __shared__ double part[KS][16][kBlkMaxNt * 8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kq = warp % KS, ng = warp / KS;
    const int NT = (E1 + 7) >> 3, per = (NT + NG - 1) / NG;
    const int nt0 = min(ng * per, NT), nnt = min(per, NT - nt0);
    const int t0 = blockIdx.x * 16;
    pdl_trigger();
    const int S = H / (4 * KS);
    const int k0 = kq * (H / KS) + t * S;
    const uint16_t *xp[2];
    bool tok_ok[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int tok = t0 + 8 * h + g;
        tok_ok[h] = tok < T;
        xp[h] = x + (size_t)(tok_ok[h] ? tok : 0) * H + k0;
    }
    const uint16_t *wp[NPG];
    bool row_ok[NPG];
#pragma unroll
    for (int n = 0; n < NPG; ++n) {
        const int row = (nt0 + n) * 8 + g;
        row_ok[n] = n < nnt && row < E1;
        wp[n] = (row < E ? w + (size_t)row * H : (wsg ? wsg : w)) + k0;
    }
    double acc[NPG][4];
#pragma unroll
    for (int n = 0; n < NPG; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0;
    uint4 xv[2], wv[NPG];
    auto load = [&](int j0) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
            xv[h] = tok_ok[h] ? __ldg(reinterpret_cast<const uint4 *>(xp[h] + j0)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int n = 0; n < NPG; ++n)
            wv[n] = row_ok[n] ? __ldg(reinterpret_cast<const uint4 *>(wp[n] + j0)) : make_uint4(0, 0, 0, 0);
    };
    load(0);
    for (int j0 = 0; j0 < S; j0 += 8) {
        uint4 xc[2], wc[NPG];
        xc[0] = xv[0];
        xc[1] = xv[1];
#pragma unroll
        for (int n = 0; n < NPG; ++n) wc[n] = wv[n];
        if (j0 + 8 < S) load(j0 + 8);
        if (x16 && ng == 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (!tok_ok[h]) continue;
                const uint32_t u[4] = {xc[h].x, xc[h].y, xc[h].z, xc[h].w};
                uint32_t f[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    f[q] = (uint32_t)bf16_to_f16_sat(u[q] & 0xFFFFu) | ((uint32_t)bf16_to_f16_sat(u[q] >> 16) << 16);
                *reinterpret_cast<uint4 *>(x16 + (size_t)(t0 + 8 * h + g) * H + k0 + j0) = make_uint4(f[0], f[1], f[2], f[3]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {        // word q: inputs j0 + 2q (slot t), j0 + 2q + 1 (slot t + 4)
            const uint32_t x0 = q == 0 ? xc[0].x : q == 1 ? xc[0].y : q == 2 ? xc[0].z : xc[0].w;
            const uint32_t x1 = q == 0 ? xc[1].x : q == 1 ? xc[1].y : q == 2 ? xc[1].z : xc[1].w;
            const double a0 = bf16_f64(x0 & 0xFFFFu), a2 = bf16_f64(x0 >> 16);
            const double a1 = bf16_f64(x1 & 0xFFFFu), a3 = bf16_f64(x1 >> 16);
#pragma unroll
            for (int n = 0; n < NPG; ++n) {
                if (n < nnt) {
                    const uint32_t wq = q == 0 ? wc[n].x : q == 1 ? wc[n].y : q == 2 ? wc[n].z : wc[n].w;
                    dmma_f64_k8(acc[n], a0, a1, a2, a3, bf16_f64(wq & 0xFFFFu), bf16_f64(wq >> 16));
                }
            }
        }
    }
    // D fragment: c0 / c1 (token g, columns 2t / 2t + 1), c2 / c3 (token g + 8)
#pragma unroll
    for (int n = 0; n < NPG; ++n)
        if (n < nnt) {
            const int c = (nt0 + n) * 8 + 2 * t;
            part[kq][g][c] = acc[n][0];
            part[kq][g][c + 1] = acc[n][1];
            part[kq][g + 8][c] = acc[n][2];
            part[kq][g + 8][c + 1] = acc[n][3];
        }
    __syncthreads();
    const int cols = NT * 8;
    for (int o = tid; o < 16 * cols; o += 256) {
        const int tg = o / cols, c = o - tg * cols;
        double v = part[0][tg][c];
#pragma unroll
        for (int q = 1; q < KS; ++q) v += part[q][tg][c];
        if (t0 + tg < T && c < E1) logits[(size_t)(t0 + tg) * E1 + c] = bf16_to_f32(f64_to_bf16(v));
    }
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

// Top-k of one token by one warp (E <= 32 * EPL): float32 softmax over the
// bf16 logits, then the k largest by (logit, lower expert first) and
// float32 renormalisation in selection order; lane s (< k) returns slot s.
// Each logit becomes a unique 32-bit key (order-preserving bf16 bits above
// 0xFFFF - expert), each lane sorts its EPL keys, and k rounds take the
// warp maximum of the lanes' heads (one shuffle per level) and pop it.
__device__ __forceinline__ uint32_t logit_key(float l, int j) {
    uint32_t b = __float_as_uint(l) >> 16;       // a bf16 value
    if (b == 0x8000u) b = 0;                     // -0 ties with +0
    const uint32_t ob = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
    return (ob << 16) | (0xFFFFu - (uint32_t)j);
}

template <int EPL>
__device__ __forceinline__ void topk_warp(const float *__restrict__ lr, int E, int k, int lane, int mode,
                                          int &my_j, float &my_score) {
    float l[EPL], ex[EPL];
    uint32_t key[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int j = lane + 32 * i;
        l[i] = j < E ? lr[j] : -INFINITY;
        m = fmaxf(m, l[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float z = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int j = lane + 32 * i;
        ex[i] = j < E ? expf(l[i] - m) : 0.0f;
        z += ex[i];
        key[i] = j < E ? logit_key(l[i], j) : 0u;   // 0: below every real key
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    // sort this lane's keys (with their exponentials) descending
#pragma unroll
    for (int a = 0; a < EPL; ++a)
#pragma unroll
        for (int b = EPL - 1; b > a; --b)
            if (key[b] > key[b - 1]) {
                const uint32_t tk = key[b]; key[b] = key[b - 1]; key[b - 1] = tk;
                const float te = ex[b]; ex[b] = ex[b - 1]; ex[b - 1] = te;
            }
    float den = 0.0f, my_p = 0.0f, my_e = 0.0f;
    my_j = 0;
    for (int s = 0; s < k; ++s) {
        uint32_t best = key[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        const int j = 0xFFFF - (int)(best & 0xFFFFu);
        const int owner = j & 31;
        const float e = __shfl_sync(0xffffffffu, ex[0], owner);
        if (lane == owner) {           // pop the head
#pragma unroll
            for (int i = 0; i + 1 < EPL; ++i) {
                key[i] = key[i + 1];
                ex[i] = ex[i + 1];
            }
            key[EPL - 1] = 0u;
        }
        const float p = e / z;
        // sequential float32 sum, selection order: of the probabilities, or
        // (softmax over the top k: its max is the top-1 logit, the global
        // max) of the exponentials
        den += mode == VQMOE_ROUTER_TOPK_SOFTMAX ? e : p;
        if (lane == s) {
            my_p = p;
            my_e = e;
            my_j = j;
        }
    }
    my_score = mode == VQMOE_ROUTER_SOFTMAX_TOPK   ? bf16r(my_p)
               : mode == VQMOE_ROUTER_TOPK_SOFTMAX ? bf16r(my_e / den)
                                                   : bf16r(my_p / den);
}

// Routing for one launch of up to kSelectMaxTok tokens: top-k of every
// token (a warp per token, 8 tokens per CTA), each (token, slot) pair's rank
// within its expert from a global atomic on cnt[expert], then the CTA that
// finishes last (an atomic on cnt[E]) scans the counts and scatters the
// pairs into per-expert lists. cnt[0..E] start at zero: the logits kernel
// zeroes them, and this kernel reads nothing before it has waited for that
// kernel. The order of pairs inside an expert's list is the atomics'
// (each pair's output does not depend on it). Zeroes `zero`.
constexpr int kSelectWarps = 8;
template <int EPL>
__global__ void __launch_bounds__(kSelectWarps * 32)
router_select_kernel(const float *__restrict__ logits, int T, int E, int E1, int k, int has_shared,
                     int32_t *__restrict__ inds, float *__restrict__ scores, float *__restrict__ sgate,
                     int32_t *__restrict__ cnt, int32_t *__restrict__ off, int32_t *__restrict__ list,
                     int32_t *__restrict__ active, int32_t *__restrict__ rank, uint32_t *__restrict__ zero,
                     int zero_words, int mode, const float *__restrict__ escale) {
    __shared__ int32_t s_off[1024];
    __shared__ int32_t s_wc[kSelectWarps], s_wa[kSelectWarps];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // (the previous block call's expert kernel, the reader of `zero`, finished
    // before this call's logits kernel began)
    if (blockIdx.x == 0)
        for (int i = tid; i < zero_words; i += blockDim.x) zero[i] = 0u;
    pdl_trigger();                   // the expert kernel may launch and stage its codebooks
    pdl_wait();                      // the logits kernel's results (and its zeroed cnt)
    const int t = blockIdx.x * kSelectWarps + warp;
    if (t < T) {
        const float *lr = logits + (size_t)t * E1;
        int j;
        float sc;
        topk_warp<EPL>(lr, E, k, lane, mode, j, sc);
        if (lane < k) {
            if (escale) sc = bf16r(sc * escale[j]);
            inds[(size_t)t * k + lane] = j;
            scores[(size_t)t * k + lane] = sc;
            rank[(size_t)t * k + lane] = atomicAdd(&cnt[j], 1);
        }
        if (lane == 0 && has_shared) sgate[t] = bf16r(sigmoid_f32(lr[E]));
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(reinterpret_cast<uint32_t *>(cnt + E), 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // exclusive scans of counts and of (count > 0): 4 experts per thread
    const int P = T * k;
    int c[4], a[4], sc_ = 0, sa = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int e = 4 * tid + q;
        c[q] = e < E ? __ldcg(cnt + e) : 0;
        a[q] = c[q] > 0;
        sc_ += c[q];
        sa += a[q];
    }
    int ic = sc_, ia = sa;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, ic, o);
        const int v = __shfl_up_sync(0xffffffffu, ia, o);
        if (lane >= o) {
            ic += u;
            ia += v;
        }
    }
    if (lane == 31) {
        s_wc[warp] = ic;
        s_wa[warp] = ia;
    }
    __syncthreads();
    int bc = 0, ba = 0;
    for (int w2 = 0; w2 < warp; ++w2) {
        bc += s_wc[w2];
        ba += s_wa[w2];
    }
    int oc = bc + ic - sc_, oa = ba + ia - sa;   // exclusive prefix of this thread's first expert
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int e = 4 * tid + q;
        if (e < E) {
            s_off[e] = oc;
            off[e] = oc;
            if (a[q]) active[oa] = e;
            if (e == E - 1) {
                off[E] = oc + c[q];
                active[E] = oa + a[q];   // number of active experts
            }
        }
        oc += c[q];
        oa += a[q];
    }
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) list[s_off[__ldcg(inds + p)] + __ldcg(rank + p)] = p;
}

template <int EPL>
__global__ void __launch_bounds__(256)
router_topk_kernel_t(const float *__restrict__ logits, int T, int E, int E1, int k, int has_shared,
                     int32_t *__restrict__ inds, float *__restrict__ scores, float *__restrict__ sgate, int mode,
                     const float *__restrict__ escale) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= T) return;
    const float *lr = logits + (size_t)t * E1;
    int j;
    float sc;
    topk_warp<EPL>(lr, E, k, lane, mode, j, sc);
    if (lane < k) {
        if (escale) sc = bf16r(sc * escale[j]);
        inds[(size_t)t * k + lane] = j;
        scores[(size_t)t * k + lane] = sc;
    }
    if (lane == 0 && has_shared) sgate[t] = bf16r(sigmoid_f32(lr[E]));
}

template <int EPL>
static void launch_topk_t(const float *logits, int T, int E, int E1, int k, int has_shared, int32_t *inds,
                          float *scores, float *sgate, int mode, const float *escale, cudaStream_t st) {
    router_topk_kernel_t<EPL><<<(T + 7) / 8, 256, 0, st>>>(logits, T, E, E1, k, has_shared, inds, scores, sgate,
                                                           mode, escale);
}

static vqmoe_status launch_topk(const float *logits, int T, int E, int E1, int k, int has_shared,
                                int32_t *inds, float *scores, float *sgate, int mode, const float *escale,
                                cudaStream_t st) {
    const int epl = (E + 31) / 32;
    if (epl <= 1) launch_topk_t<1>(logits, T, E, E1, k, has_shared, inds, scores, sgate, mode, escale, st);
    else if (epl <= 2) launch_topk_t<2>(logits, T, E, E1, k, has_shared, inds, scores, sgate, mode, escale, st);
    else if (epl <= 4) launch_topk_t<4>(logits, T, E, E1, k, has_shared, inds, scores, sgate, mode, escale, st);
    else if (epl <= 8) launch_topk_t<8>(logits, T, E, E1, k, has_shared, inds, scores, sgate, mode, escale, st);
    else launch_topk_t<16>(logits, T, E, E1, k, has_shared, inds, scores, sgate, mode, escale, st);
    return check_launch("router_topk_kernel");
}

// zero2 (optional, nzero2 words): zeroed by the small-launch kernels (the
// routing kernel's counters; only launches of up to kSelectMaxTok tokens pass it)
vqmoe_status launch_logits(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T, int H,
                           int E, int E1, float *logits, uint16_t *x16, cudaStream_t stream,
                           uint32_t *zero2, int nzero2) {
    size_t smem = (size_t)kRouterTok * H * sizeof(uint16_t);
    vqmoe_status s = ensure_dynamic_smem(reinterpret_cast<const void *>(router_logits_kernel), smem, "router");
    if (s != VQMOE_OK) return s;
    if (H % 256 == 0 && T >= kBlkMinTok && E1 <= kBlkMaxNt * 8 && !zero2) {
        if (T >= 2 * kBlkMinTok)
            router_logits_dmma16_kernel<4><<<(T + 15) / 16, 256, 0, stream>>>(x, w, wsg, T, H, E, E1, logits, x16);
        else
            router_logits_dmma_blk_kernel<1, 2><<<(T + 7) / 8, 256, 0, stream>>>(x, w, wsg, T, H, E, E1, logits,
                                                                                   x16);
        s = check_launch("router_logits_dmma_blk_kernel");
    } else if (H % 256 == 0) {
        dim3 gt((E1 + 7) / 8, (T + 7) / 8);
        router_logits_dmma_kernel<<<gt, 256, 0, stream>>>(x, w, wsg, T, H, E, E1, logits, x16, zero2, nzero2);
        s = check_launch("router_logits_dmma_kernel");
    } else {
        dim3 g1((E1 + kRouterRows - 1) / kRouterRows, (T + kRouterTok - 1) / kRouterTok);
        router_logits_kernel<<<g1, 256, smem, stream>>>(x, w, wsg, T, H, E, E1, logits, x16, zero2, nzero2);
        s = check_launch("router_logits_kernel");
    }
    return s;
}

vqmoe_status launch_router(const uint16_t *x, const uint16_t *w,
                           const uint16_t *wsg, int T, int H, int E, int k,
                           float *logits, int32_t *inds, float *scores,
                           float *sgate, uint16_t *x16, int mode, const float *escale, cudaStream_t stream) {
    const int E1 = E + (wsg ? 1 : 0);
    vqmoe_status s = launch_logits(x, w, wsg, T, H, E, E1, logits, x16, stream);
    if (s != VQMOE_OK) return s;
    return launch_topk(logits, T, E, E1, k, wsg != nullptr, inds, scores, sgate, mode, escale, stream);
}

// Logits, then top-k + counting sort in one CTA when the launch is small
// enough, else top-k and the route kernel separately.
vqmoe_status launch_router_route(const uint16_t *x, const uint16_t *w, const uint16_t *wsg, int T,
                                 int H, int E, int k, float *logits, int32_t *inds, float *scores,
                                 float *sgate, uint16_t *x16, int32_t *cnt, int32_t *off,
                                 int32_t *list, int32_t *active, int32_t *rank_scratch,
                                 uint32_t *zero, int zero_words, int mode, cudaStream_t stream) {
    const int E1 = E + (wsg ? 1 : 0);
    if (T > kSelectMaxTok || E > 1024) {
        vqmoe_status s = launch_router(x, w, wsg, T, H, E, k, logits, inds, scores, sgate, x16, mode, nullptr,
                                       stream);
        if (s != VQMOE_OK) return s;
        return launch_route(inds, T * k, E, cnt, off, list, active, rank_scratch, zero, zero_words, stream);
    }
    // cnt[0..E]: the select kernel's counters (cnt[E] counts finished CTAs)
    vqmoe_status s = launch_logits(x, w, wsg, T, H, E, E1, logits, x16, stream,
                                   reinterpret_cast<uint32_t *>(cnt), E + 1);
    if (s != VQMOE_OK) return s;
    return launch_select(logits, T, E, E1, k, wsg != nullptr, inds, scores, sgate, cnt, off, list, active,
                         rank_scratch, zero, zero_words, mode, stream);
}

vqmoe_status launch_select(const float *logits, int T, int E, int E1, int k, bool has_shared, int32_t *inds,
                           float *scores, float *sgate, int32_t *cnt, int32_t *off, int32_t *list, int32_t *active,
                           int32_t *rank_scratch, uint32_t *zero, int zero_words, int mode, cudaStream_t stream) {
    if (T > kSelectMaxTok || E > 1024) return set_error(VQMOE_BAD_SHAPE, "select: T %d E %d", T, E);
    const int epl = (E + 31) / 32;
    auto fn = epl <= 1 ? router_select_kernel<1>
              : epl <= 2 ? router_select_kernel<2>
              : epl <= 4 ? router_select_kernel<4>
              : epl <= 8 ? router_select_kernel<8>
                         : router_select_kernel<16>;
    if (launch_pdl(fn, dim3((T + kSelectWarps - 1) / kSelectWarps), dim3(kSelectWarps * 32), 0, stream, logits, T,
                   E, E1, k, (int)has_shared, inds, scores, sgate, cnt, off, list, active, rank_scratch, zero,
                   zero_words, mode, static_cast<const float *>(nullptr)) != cudaSuccess)
        return check_launch("router_select_kernel");
    return check_launch("router_select_kernel");
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

// ------------------------------------------------------------ RMS norm
// Gemma-4's router input, mx.fast.rms_norm(x, w, eps) (gemma4_text.py:
// 171): out = bf16(bf16(x * r) * w), r = 1 / sqrt(ms + eps) in float32
// (IEEE square root and division), ms the mean of the squares: each square
// of a bf16 value is exact in fp64, their sum is accumulated in fp64 and the
// mean rounded once to float32. One CTA per row.
__global__ void __launch_bounds__(256)
rms_norm_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w, int H, float eps,
                uint16_t *__restrict__ out) {
    __shared__ double s_part[8];
    const int row = blockIdx.x, tid = threadIdx.x;
    const uint16_t *xr = x + (size_t)row * H;
    double acc = 0.0;
    for (int i = tid; i < H; i += blockDim.x) {
        const double v = (double)bf16_to_f32(xr[i]);
        acc += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((tid & 31) == 0) s_part[tid >> 5] = acc;
    __syncthreads();
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += s_part[i];
    const float ms = (float)(sum / (double)H);
    const float r = 1.0f / sqrtf(ms + eps);
    for (int i = tid; i < H; i += blockDim.x)
        out[(size_t)row * H + i] = f32_to_bf16(bf16r(bf16_to_f32(xr[i]) * r) * bf16_to_f32(w[i]));
}

vqmoe_status launch_rms_norm(const uint16_t *x, const uint16_t *w, int T, int H, float eps, uint16_t *out,
                             cudaStream_t stream) {
    rms_norm_kernel<<<T, 256, 0, stream>>>(x, w, H, eps, out);
    return check_launch("rms_norm_kernel");
}

}  // namespace vqmoe
