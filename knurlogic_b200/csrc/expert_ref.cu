// Routed experts whose VQ weights stay in the reference layout
// (VQMOE_FMT_VQ_REF): the code formats the tiled fast path does not take.
//
// Reference: the VQSwitchLinear contract of
// engine/families/deepseek/heads/deepseek_v4.py:35-42, 111-130 -- codebook
// [K, dim] fp16, vq_scales [E, OUT, IN/group] fp16, codes [E, OUT, IN/dim]
// with one code per entry, uint8 when K <= 256 and uint16 above (the
// reference's own VQ fixture is K 2048, dim 2, group 64). Packed uint32
// codes (pack_bits > 0) are not taken: their bit order is not pinned.
//
// Each CTA owns (active expert, 64 output rows) and runs the expert's pairs
// in passes of up to 64. Per 256-input chunk it dequantises its rows into
// shared memory -- W = fp16(codebook[code][j] * scale), one mul.rn.f16x2 per
// two weights, the same arithmetic as the fast path and vqmoe_dequant --
// while the pairs' fp16 input rows land by cp.async, then 8 warps (16 rows x
// 32 pairs each) multiply with mma.sync m16n8k16 (fp16 products exact,
// float32 sums). The codebooks sit in shared memory when they fit (32 KB a
// matrix: K x dim up to 16384 values) and are read through L1 otherwise.
// Phase 1 (gate and up, SwiGLU / GeGLU) and phase 2 (down, x the routing
// weight) are two launches.
//
// The same kernel serves affine-quantized experts (VQMOE_FMT_AFFINE,
// mlx-lm's QuantizedSwitchLinear, switch_layers.py:24-86): each row of the
// packed uint32 weight is a little-endian bit stream of `bits`-bit values q,
// dequantised as W = bf16(fmaf(scale, q, bias)) with its group's scale and
// bias, and the bf16 activations enter a bf16 mma.sync as they are.
#include <algorithm>

#include "experts.cuh"
#include "stages.cuh"

namespace vqmoe {
namespace rf {

constexpr int kThreads = 256;
constexpr int kRows = 64;                 // output rows per CTA
constexpr int kPairs = 64;                // pairs per pass
constexpr int kChunk = 256;               // inputs per staged chunk
constexpr int kStride = kChunk * 2 + 32;  // bytes per staged row: fragment loads of 8 rows
                                          // cover the 32 banks twice, no conflicts
constexpr int kCbMax = 32768;             // shared-memory codebook budget per matrix
constexpr int kTileBytes = kRows * kStride;

struct Mat {
    const uint8_t *codes;                 // [E][OUT][IN / dim], 1 or 2 bytes per code; AFFINE: packed q words
    const uint16_t *cb;                   // [K][dim] fp16 bits
    const uint16_t *scales;               // [E][OUT][IN / group] fp16 bits (AFFINE: bf16)
    const uint16_t *biases;               // AFFINE: [E][OUT][IN / group] bf16 bits
    int K, dim, group, cbytes, bits;
};

struct Args {
    const int32_t *cnt, *off, *list, *active;
    int E, k, x_per_pair;
    const uint16_t *x;                    // fp16 rows (VQ), bf16 rows (AFFINE)
    int IN, OUT;
    uint16_t *out;                        // [P][OUT]
    int out_f16;
    const float *pair_scale;
    int act;
    Mat m[2];
};

template <int NMAT>
constexpr size_t smem_bytes() {
    return (size_t)NMAT * kCbMax + (size_t)NMAT * kTileBytes + kTileBytes;
}

// the fp16 weights of `dim` inputs from one code, times the scale (half2)
template <int DIM>
__device__ __forceinline__ void dequant_entry(const uint16_t *cbp, uint32_t s2, uint8_t *dst) {
    if (DIM == 2) {
        *reinterpret_cast<uint32_t *>(dst) = hmul2_u32(*reinterpret_cast<const uint32_t *>(cbp), s2);
    } else if (DIM == 4) {
        const uint2 e = *reinterpret_cast<const uint2 *>(cbp);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(hmul2_u32(e.x, s2), hmul2_u32(e.y, s2));
    } else {
        const uint4 e = *reinterpret_cast<const uint4 *>(cbp);
        *reinterpret_cast<uint4 *>(dst) =
            make_uint4(hmul2_u32(e.x, s2), hmul2_u32(e.y, s2), hmul2_u32(e.z, s2), hmul2_u32(e.w, s2));
    }
}

// rows [row0, row0 + 64) x inputs [i0, i0 + 256) of expert e into the tile
// (zeros past OUT and IN)
template <int DIM>
__device__ __forceinline__ void dequant_chunk(const Mat &m, const uint16_t *cb, int e, int row0, int i0, int IN,
                                              int OUT, uint8_t *tile) {
    constexpr int kCodes = kChunk / DIM;             // codes per row per chunk
    const int ncode_row = IN / DIM, ngrp_row = IN / m.group;
    for (int v = threadIdx.x; v < kRows * kCodes; v += kThreads) {
        const int r = v / kCodes, ci = v - r * kCodes;
        const int row = row0 + r, i = i0 + ci * DIM;
        uint8_t *dst = tile + r * kStride + ci * DIM * 2;
        if (row < OUT && i < IN) {
            const size_t rr = (size_t)e * OUT + row;
            const size_t cidx = rr * ncode_row + i / DIM;
            const uint32_t code = m.cbytes == 1 ? (uint32_t)__ldg(m.codes + cidx)
                                                : (uint32_t)__ldg(reinterpret_cast<const uint16_t *>(m.codes) + cidx);
            const uint32_t s = __ldg(m.scales + rr * ngrp_row + i / m.group);
            dequant_entry<DIM>(cb + (size_t)code * DIM, s | (s << 16), dst);
        } else {
            if (DIM == 2) *reinterpret_cast<uint32_t *>(dst) = 0u;
            else if (DIM == 4) *reinterpret_cast<uint2 *>(dst) = make_uint2(0u, 0u);
            else *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

// AFFINE: rows [row0, row0 + 64) x inputs [i0, i0 + 256) of expert e,
// W = bf16(fmaf(scale, q, bias)), 8 inputs (16 output bytes) per thread
__device__ __forceinline__ void dequant_chunk_affine(const Mat &m, int e, int row0, int i0, int IN, int OUT,
                                                     uint8_t *tile) {
    const int words_row = IN * m.bits / 32, ngrp_row = IN / m.group;
    const uint32_t mask = (1u << m.bits) - 1u;
    const uint32_t *wq = reinterpret_cast<const uint32_t *>(m.codes);
    for (int v = threadIdx.x; v < kRows * (kChunk / 8); v += kThreads) {
        const int r = v / (kChunk / 8), j8 = v - r * (kChunk / 8);
        const int row = row0 + r, i = i0 + 8 * j8;
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (row < OUT && i < IN) {
            const size_t rr = (size_t)e * OUT + row;
            // the 8 values' bits: at most 64 bits from the first word they touch
            const long long bit = (long long)i * m.bits;
            const int wi = (int)(bit >> 5), off = (int)(bit & 31);
            const uint32_t *wr = wq + rr * words_row;
            unsigned long long win = __ldg(wr + wi);
            if (off + 8 * m.bits > 32) win |= (unsigned long long)__ldg(wr + wi + 1) << 32;
            win >>= off;
            const size_t gi = rr * ngrp_row + i / m.group;
            const float s = bf16_to_f32(__ldg(m.scales + gi)), b = bf16_to_f32(__ldg(m.biases + gi));
            uint32_t h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                h[j] = f32_to_bf16(__fmaf_rn(s, (float)(uint32_t)((win >> (j * m.bits)) & mask), b));
            o = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
        }
        *reinterpret_cast<uint4 *>(tile + r * kStride + j8 * 16) = o;
    }
}

template <int NMAT, int DIM>
__global__ void __launch_bounds__(kThreads, 1) expert_ref_kernel(const Args a) {
    constexpr bool AFF = DIM == 0;             // affine-quantized weights, bf16 operands
    constexpr bool DUAL = NMAT == 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_pairs[kPairs];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int ai = blockIdx.x;
    const int row0 = blockIdx.y * kRows;
    const uint16_t *cb[NMAT];
    uint8_t *wt[NMAT];
    uint8_t *xt = smem + NMAT * kCbMax + NMAT * kTileBytes;
    // the codebooks (weights) before the routing is ready
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const Mat &M = a.m[m];
        wt[m] = smem + NMAT * kCbMax + m * kTileBytes;
        const int vals = AFF ? 0 : M.K * DIM;
        if (AFF) {
            cb[m] = nullptr;
        } else if (vals * 2 <= kCbMax) {
            uint16_t *dst = reinterpret_cast<uint16_t *>(smem + m * kCbMax);
            for (int i = tid; i < vals / 2; i += kThreads)
                reinterpret_cast<uint32_t *>(dst)[i] = __ldg(reinterpret_cast<const uint32_t *>(M.cb) + i);
            cb[m] = dst;
        } else {
            cb[m] = M.cb;
        }
    }
    pdl_wait();
    if (ai >= a.active[a.E] || row0 >= a.OUT) return;
    const int e = a.active[ai], n = a.cnt[e], base = a.off[e];
    const int IN = a.IN, OUT = a.OUT;
    const int rg = warp & 3, tg = warp >> 2;           // 16 rows, 32 pairs per warp
    for (int tb0 = 0; tb0 < n; tb0 += kPairs) {
        const int np = min(kPairs, n - tb0);
        __syncthreads();                               // the previous pass's epilogue read s_pairs
        if (tid < kPairs) s_pairs[tid] = tid < np ? a.list[base + tb0 + tid] : -1;
        const int nta = max(0, min(4, (np - 32 * tg + 7) >> 3));   // this warp's n-tiles with pairs
        float acc[NMAT][4][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][j][i] = 0.0f;
        for (int i0 = 0; i0 < IN; i0 += kChunk) {
            __syncthreads();                           // s_pairs written; the previous chunk read
            // the pairs' inputs (16 bytes a copy; zeros past IN)
            for (int v = tid; v < np * (kChunk / 8); v += kThreads) {
                const int tk = v / (kChunk / 8), j = v - tk * (kChunk / 8);
                const int p = s_pairs[tk];
                const int xr = a.x_per_pair ? p : p / a.k;
                const int f = i0 + 8 * j;
                const bool ok = f < IN;
                cp_async16(smem_u32(xt + tk * kStride + j * 16), a.x + (size_t)xr * IN + (ok ? f : 0), ok ? 16 : 0);
            }
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                if (AFF) dequant_chunk_affine(a.m[m], e, row0, i0, IN, OUT, wt[m]);
                else dequant_chunk<DIM == 0 ? 2 : DIM>(a.m[m], cb[m], e, row0, i0, IN, OUT, wt[m]);
            }
            cp_async_wait_all();
            __syncthreads();
            if (nta == 0) continue;
            // k-step q covers inputs 16q .. 16q + 15 of the chunk: k-slots
            // {2t, 2t+1, 2t+8, 2t+9} carry inputs 16q + 4t + {0..3} on both
            // operands (the dot product is unchanged), 8-byte loads each
#pragma unroll 4
            for (int q = 0; q < kChunk / 16; ++q) {
                uint2 av[NMAT][2];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint8_t *ar = wt[m] + (16 * rg + g) * kStride + 32 * q + 8 * t;
                    av[m][0] = *reinterpret_cast<const uint2 *>(ar);
                    av[m][1] = *reinterpret_cast<const uint2 *>(ar + 8 * kStride);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < nta) {
                        const uint2 bv = *reinterpret_cast<const uint2 *>(
                            xt + (32 * tg + 8 * j + g) * kStride + 32 * q + 8 * t);
#pragma unroll
                        for (int m = 0; m < NMAT; ++m) {
                            if (AFF) mma_bf16(acc[m][j], av[m][0].x, av[m][1].x, av[m][0].y, av[m][1].y, bv.x, bv.y);
                            else mma_f16(acc[m][j], av[m][0].x, av[m][1].x, av[m][0].y, av[m][1].y, bv.x, bv.y);
                        }
                    }
                }
            }
        }
        // fragment -> (row 16 rg + g (+8), pair 32 tg + 8 j + 2t (+1))
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j >= nta) continue;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int pi = 32 * tg + 8 * j + 2 * t + (i & 1);
                const int row = row0 + 16 * rg + g + (i >> 1) * 8;
                const int p = pi < np ? s_pairs[pi] : -1;
                if (p < 0 || row >= OUT) continue;
                a.out[(size_t)p * OUT + row] =
                    epilogue_value<DUAL>(acc[0][j][i], acc[NMAT - 1][j][i], a.pair_scale, p, a.out_f16, a.act);
            }
        }
    }
}

template <int NMAT, int DIM>
static vqmoe_status launch(const Args &a, cudaStream_t stream) {
    auto fn = expert_ref_kernel<NMAT, DIM>;
    const size_t smem = smem_bytes<NMAT>();
    vqmoe_status s = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), smem, "reference-layout expert kernel");
    if (s != VQMOE_OK) return s;
    const dim3 grid(a.E, (a.OUT + kRows - 1) / kRows);
    if (launch_pdl(fn, grid, dim3(kThreads), smem, stream, a) != cudaSuccess)
        return check_launch("expert_ref_kernel");
    return check_launch("expert_ref_kernel");
}

template <int NMAT>
static vqmoe_status launch_dim(const Args &a, int dim, cudaStream_t stream) {
    if (a.m[0].bits) return launch<NMAT, 0>(a, stream);
    switch (dim) {
        case 2: return launch<NMAT, 2>(a, stream);
        case 4: return launch<NMAT, 4>(a, stream);
        case 8: return launch<NMAT, 8>(a, stream);
        default: return set_error(VQMOE_BAD_FORMAT, "reference-layout VQ: dim %d (2, 4 or 8)", dim);
    }
}

static Mat mat_of(const vqmoe_linear *w) {
    Mat m{};
    m.codes = static_cast<const uint8_t *>(w->codes);
    m.cb = static_cast<const uint16_t *>(w->codebook);
    m.scales = static_cast<const uint16_t *>(w->scales);
    m.K = w->codebook_size;
    m.dim = w->dim;
    m.group = w->group_size;
    m.cbytes = w->codebook_size <= 256 ? 1 : 2;
    if (w->format == VQMOE_FMT_AFFINE) {
        m.codes = static_cast<const uint8_t *>(w->weight);
        m.biases = static_cast<const uint16_t *>(w->biases);
        m.bits = w->bits;
        m.K = m.dim = 0;
    }
    return m;
}

static Args args_of(const RoutedIO &r, const vqmoe_linear *w0, const vqmoe_linear *w1) {
    Args a{};
    a.cnt = r.cnt;
    a.off = r.off;
    a.list = r.list;
    a.active = r.active;
    a.E = r.E;
    a.k = r.k;
    a.x_per_pair = r.x_per_pair;
    a.x = static_cast<const uint16_t *>(r.x);
    a.IN = w0->in_features;
    a.OUT = w0->out_features;
    a.out = static_cast<uint16_t *>(r.out);
    a.out_f16 = r.out_f16;
    a.pair_scale = r.pair_scale;
    a.act = r.act;
    a.m[0] = mat_of(w0);
    a.m[1] = mat_of(w1 ? w1 : w0);
    return a;
}

}  // namespace rf

vqmoe_status launch_experts_ref(const vqmoe_linear *gate, const vqmoe_linear *up, const RoutedIO *r1,
                                const vqmoe_linear *w2, const RoutedIO &r2, cudaStream_t stream) {
    if (r1) {
        vqmoe_status s = rf::launch_dim<2>(rf::args_of(*r1, gate, up), gate->dim, stream);
        if (s != VQMOE_OK) return s;
    }
    return rf::launch_dim<1>(rf::args_of(r2, w2, nullptr), w2->dim, stream);
}

}  // namespace vqmoe
