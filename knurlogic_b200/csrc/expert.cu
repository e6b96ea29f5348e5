// Expert (switch-linear) kernels of the decode / MTP-verify regime on B200.
//
// Reference: SwitchGLU.__call__ / SwitchLinear.__call__
// (glm5_next/_mlx_vlm/models/switch_layers.py:116-125, 172-193) with the
// experts as VQSwitchLinear (codes, codebook, vq_scales; layout from
// engine/families/deepseek/heads/deepseek_v4.py:35-42, 111-130), plus the
// shared expert's dense matmuls (qwen3_5.py:184-185).
//
// One persistent kernel runs both projection stages of the routed experts:
// phase 1 tiles (fused gate/up + SwiGLU: an active expert and 128 output
// rows) and then phase 2 tiles (down, or a single switch linear: an active
// expert and 256 output rows), two CTAs per SM, all taken in order from one
// global counter. A phase 2 tile of expert e starts once every phase 1 tile
// of e has finished (a per-expert count, a bounded wait), so the down tiles
// fill the end of the gate/up phase instead of a second launch.
//
// A CTA stages the tile's token rows (<= 8 at a time, fp16 for VQ) in shared
// memory once; each of its 8 warps then computes 16 (phase 1) or 32
// (phase 2) output rows over the whole K, and writes its results from
// registers (the SwiGLU or the routing weight applied there). No split K,
// no partials.
//
// For a VQ tile each lane
//   * streams its codes and group scales through a ring of four register
//     half-chunk buffers (loads issued three half chunks, ~1 us, ahead);
//   * looks each code up in a shared-memory codebook and feeds the 8-byte
//     entry (4 fp16) straight into mma.sync m16n8k16 as the A operand
//     (fp16 x fp16 -> fp32); B is the tile's token rows from shared memory;
//   * multiplies the entry by its row's 64-input group scale in fp16
//     (mul.rn.f16x2): the weight is fp16(codebook x scale), exactly what
//     vqmoe_dequant and the prefill kernel use.
// Dense tiles (bf16 experts) load A from global memory.
//
// Why mma.sync and registers here rather than tcgen05: at 1-64 tokens the
// layer is bound by HBM and by the shared-memory codebook lookups (8 bytes
// per code, ~16 codes/clk/SM), not by tensor throughput (~4 tokens per
// expert). A register-fed A operand keeps every dequantised weight out of
// shared memory; tcgen05 would need it written to SMEM or TMEM first.
//
// Codebook replication: 16 copies interleaved so that lane L reads only the
// bank pair L % 16; a warp's random 8-byte lookups are then conflict-free
// (2 wavefronts, the minimum for 256 bytes). Entry c of copy b of matrix m
// sits at byte 256*c + 128*m + 8*b (64 KB for gate and up together), so
// one byte permute builds a lookup address: byte 1 = the code, byte 0 =
// the lane's copy offset. Phase 2 restages matrix slot 0 with its codebook.
//
// Device layout (layout.cuh): codes and scales tiled per (expert, 32 rows,
// 256 inputs) in the order the lanes consume them, so a warp's loads are
// contiguous 256-byte requests off one base pointer per matrix. MMA
// sub-step q of a chunk covers inputs [16q, 16q+16); its k-slots
// {2t, 2t+1, 2t+8, 2t+9} carry inputs 16q+4t+{0,1,2,3}, the same
// permutation on A and B, so the dot product is unchanged, and both the
// codebook entry (A) and the activation quad (B) are single 8-byte loads.
#include <algorithm>

#include "experts.cuh"
#include "layout.cuh"
#include "stages.cuh"

namespace vqmoe {

constexpr int kThreads = 256;               // 8 warps per CTA, 2 CTAs per SM
// average pairs per expert from which the routed experts take the tcgen05
// prefill path (expert_prefill.cu) instead of the mma.sync decode path
constexpr int kWarps = kThreads / 32;
constexpr int kRepBytes = 256 * 256;        // replicated codebooks (two matrices), 64 KB
constexpr int kWin = 2048;                  // inputs per staged activation window
constexpr int kXStride = kWin * 2 + 32;     // bytes per staged row: B-fragment
                                            // loads of 4 rows hit 16 bank pairs
constexpr int kXBytes = 8 * kXStride;       // 8 token rows
constexpr int kTR1 = kWarps * 16;           // phase 1 tile: 128 rows (gate and up)
constexpr int kTR2 = kWarps * 32;           // phase 2 tile: 256 rows
constexpr long kWaitLimit = 1L << 21;       // bounded wait for phase 1 tiles (~4 s)

__device__ __forceinline__ uint2 lds2(const uint8_t *base, uint32_t off) {
    return *reinterpret_cast<const uint2 *>(base + off);
}

// Codes and scales of one half chunk (8 MMA sub-steps = 128 inputs) of the
// warp's MT m-tiles: per (matrix, m-tile, row half) 2 code words, 2 scales.
template <int NMAT, int MT>
struct HalfBuf {
    uint32_t cw[NMAT][MT][2][2];   // [m][mt][h][word]
    uint32_t sc[NMAT][MT][2];      // [m][mt][h]: scale groups 2*half, 2*half+1
};

// ct[m]: the warp's first code tile + lane*8 (+ its m-tile's offset);
// st[m]: first scale tile + 2*g. Chunks are 2048 / 128 elements apart.
template <int NMAT, int MT>
__device__ __forceinline__ void load_half(HalfBuf<NMAT, MT> &b, const uint8_t *const (&ct)[NMAT],
                                          const uint16_t *const (&st)[NMAT], int hidx) {
    const int c = hidx >> 1, half = hidx & 1;
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint2 v = ldg_stream_v2(ct[m] + c * 2048 + half * 1024 + (2 * mt + h) * 256);
                b.cw[m][mt][h][0] = v.x;
                b.cw[m][mt][h][1] = v.y;
                b.sc[m][mt][h] = ldg_stream_u32(st[m] + c * 128 + half * 64 + (2 * mt + h) * 16);
            }
}

// 8 sub-steps from a half buffer; xoff: this lane's staged-row offset of
// sub-step 0; lanebyte: this lane's codebook copy offset (lane % 16) * 8.
// Each looked-up codebook entry (4 fp16) is multiplied by its row's group
// scale with one mul.rn.f16x2 per two weights -- W = fp16(codebook * scale),
// the dequantised weight bit for bit (the product of two fp16 values is
// exact before that one rounding) -- and fed to the fp16 MMA, whose
// products are exact and whose sums are float32: the same arithmetic as
// the prefill kernel and vqmoe_dequant.
template <int NMAT, int MT>
__device__ __forceinline__ void compute_half(const HalfBuf<NMAT, MT> &b, float (&acc)[NMAT][MT][4],
                                             const uint8_t *cb, uint32_t lanebyte,
                                             const uint8_t *xs, int xoff) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {          // the half's two scale groups
        // the group's scale of rows g (h = 0) and g + 8 (h = 1), as half2
        uint32_t s2[NMAT][MT][2];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) s2[m][mt][h] = __byte_perm(b.sc[m][mt][h], 0, j ? 0x3232 : 0x1010);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            const int q = 4 * j + qq;
            // address = 256 * code + 8 * copy: code byte qq -> byte 1
            const uint32_t sel = 0x5504u | (qq << 4);
            const uint2 bf = lds2(xs, xoff + q * 32);
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint32_t a0 = __byte_perm(b.cw[m][mt][0][j], lanebyte, sel);
                    const uint32_t a1 = __byte_perm(b.cw[m][mt][1][j], lanebyte, sel);
                    const uint2 e0 = lds2(cb + m * 128, a0);
                    const uint2 e1 = lds2(cb + m * 128, a1);
                    // A fragment: rows g (e0) and g + 8 (e1), k-slots {2t, 2t+1} then {2t+8, 2t+9}
                    mma_f16(acc[m][mt], hmul2_u32(e0.x, s2[m][mt][0]), hmul2_u32(e1.x, s2[m][mt][1]),
                            hmul2_u32(e0.y, s2[m][mt][0]), hmul2_u32(e1.y, s2[m][mt][1]), bf.x, bf.y);
                }
            }
        }
    }
}

// Dense sub-steps [0, nq) of chunk c (A from global: rows r0 and r0 + 8).
template <int NMAT, int MT>
__device__ __forceinline__ void dense_chunk(float (&acc)[NMAT][MT][4], const uint16_t *const (&wr)[NMAT],
                                            int IN, int c, int nq, const uint8_t *xs, int xoff) {
#pragma unroll 4
    for (int q = 0; q < nq; ++q) {
        const uint2 bf = lds2(xs, xoff + q * 32);
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint16_t *wp = wr[m] + (size_t)mt * 16 * IN + (c << 8) + 16 * q;
                const uint2 w0v = ldg_nc_v2(wp);
                const uint2 w1v = ldg_nc_v2(wp + (size_t)8 * IN);
                mma_bf16(acc[m][mt], w0v.x, w1v.x, w0v.y, w1v.y, bf.x, bf.y);
            }
    }
}

// 16 interleaved copies of nmat codebooks: entry c of copy b of matrix m at
// 256c + 128m + 8b (codes >= K read zeros)
__device__ __forceinline__ void stage_codebooks(uint8_t *cb, const LinearDev &w0, const LinearDev &w1,
                                                int nmat) {
    for (int i = threadIdx.x; i < nmat * 4096; i += kThreads) {
        const int m = i >> 12, rr = i & 4095, c = rr >> 4, b = rr & 15;
        const LinearDev &w = m == 0 ? w0 : w1;
        uint2 v = make_uint2(0, 0);
        if (c < w.K) v = ldg_nc_v2(w.codebook + c * 4);
        *reinterpret_cast<uint2 *>(cb + c * 256 + m * 128 + b * 8) = v;
    }
}

// Thread 0: wait until *count >= want (acquire), at most `limit` polls
// (kWaitLimit when 0) with a growing sleep; on running out, store
// kWaitDependency in the call's status word and go on (the tile's results
// are then wrong, and the call reports VQMOE_TIMEOUT, but nothing hangs).
__device__ __noinline__ void wait_count(const uint32_t *count, uint32_t want, uint32_t *err, uint32_t limit) {
    const long polls = limit ? (long)limit : kWaitLimit;
    unsigned ns = 64;
    for (long i = 1;; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(count) : "memory");
        if (v >= want) return;
        if (i >= polls) {
            atomicExch(err, kWaitDependency);
            return;
        }
        __nanosleep(ns);
        if (ns < 2048) ns <<= 1;
    }
}

// One tile of one stage: this CTA's 8 warps over rows [row0, row0 + TR) of
// expert in.e for its in.n pairs, 8 pairs at a time.
template <int NMAT, int MT, bool VQ>
__device__ __forceinline__ void run_tile(const RoutedSet &r, const TileInfo &in, const uint8_t *cb,
                                         uint8_t *xs, int *s_pairs) {
    constexpr bool DUAL = NMAT == 2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t lanebyte = (lane & 15) * 8;
    const int IN = r.IN, OUT = r.OUT;
    const int C = (IN + 255) >> 8;
    const int wrow = in.row0 + warp * 16 * MT;   // this warp's first row
    const bool active = wrow < OUT;
    // every pointer starts at a valid base, whichever branch sets it
    const uint8_t *ct[NMAT];
    const uint16_t *st[NMAT];
    const uint16_t *wr[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const LinearDev &w = m == 0 ? r.w0 : r.w1;
        ct[m] = w.codes;
        st[m] = w.scales;
        wr[m] = w.weight;
    }
    if (VQ) {
        const long long tile0 = ((long long)in.e * ((OUT + 31) >> 5) + (wrow >> 5)) * C;
        const int mt0 = (wrow >> 4) & 1;          // MT == 1: which half of the 32 rows
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const LinearDev &w = m == 0 ? r.w0 : r.w1;
            ct[m] = w.codes + tile0 * 2048 + mt0 * 512 + lane * 8;
            st[m] = w.scales + tile0 * 128 + mt0 * 32 + 2 * g;
        }
    } else {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const LinearDev &w = m == 0 ? r.w0 : r.w1;
            wr[m] = w.weight + (size_t)in.e * OUT * IN + (size_t)(wrow + g) * IN + 4 * t;
        }
    }
    const int span = VQ ? C << 8 : IN;
    for (int tb0 = 0; tb0 < in.n; tb0 += 8) {
        const int nt = min(8, in.n - tb0);
        __syncthreads();                          // the previous block's epilogue read s_pairs
        if (tid < 8) s_pairs[tid] = tid < nt ? r.list[in.base + tb0 + tid] : -1;
        float acc[NMAT][MT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][mt][i] = 0.0f;
        HalfBuf<NMAT, MT> hb[4];
        const int nh = 2 * C;
        if (VQ && active) {
            load_half<NMAT, MT>(hb[0], ct, st, 0);
            if (nh > 1) load_half<NMAT, MT>(hb[1], ct, st, 1);
            if (nh > 2) load_half<NMAT, MT>(hb[2], ct, st, 2);
        }
        for (int w0 = 0; w0 < span; w0 += kWin) {
            const int wend = min(w0 + kWin, span);
            __syncthreads();                      // previous window fully read; s_pairs written
            {
                // stage the pairs' rows (16 bytes per copy; zero past IN). A
                // slot without a pair keeps stale finite data: its B column
                // only feeds outputs that are never written.
                const int nv = (wend - w0) >> 3;
                for (int rr = 0; rr < nt; ++rr) {
                    const int p = s_pairs[rr];
                    const int xr = r.x_per_pair ? p : p / r.k;
                    const uint16_t *row = r.x + (size_t)xr * IN;
                    uint8_t *dst = xs + rr * kXStride;
                    for (int j = tid; j < nv; j += kThreads) {
                        const int f = w0 + 8 * j;
                        const bool ok = f < IN;
                        cp_async16(smem_u32(dst + j * 16), row + (ok ? f : 0), ok ? 16 : 0);
                    }
                }
                cp_async_wait_all();
            }
            __syncthreads();
            if (!active) continue;
            const int c0 = w0 >> 8, c1 = (wend + 255) >> 8;
            if (VQ) {
                // chunks in pairs: halves 2c .. 2c+3 in hb[0..3]; the loads
                // run three halves ahead (a ring of four buffers)
                for (int c = c0; c < c1; c += 2) {
                    const int h0 = 2 * c;
                    const int xoff = g * kXStride + (((c - c0) << 8) + 4 * t) * 2;
                    if (h0 + 3 < nh) load_half<NMAT, MT>(hb[3], ct, st, h0 + 3);
                    compute_half<NMAT, MT>(hb[0], acc, cb, lanebyte, xs, xoff);
                    if (h0 + 4 < nh) load_half<NMAT, MT>(hb[0], ct, st, h0 + 4);
                    compute_half<NMAT, MT>(hb[1], acc, cb, lanebyte, xs, xoff + 256);
                    if (h0 + 2 < nh) {
                        if (h0 + 5 < nh) load_half<NMAT, MT>(hb[1], ct, st, h0 + 5);
                        compute_half<NMAT, MT>(hb[2], acc, cb, lanebyte, xs, xoff + 512);
                        if (h0 + 6 < nh) load_half<NMAT, MT>(hb[2], ct, st, h0 + 6);
                        compute_half<NMAT, MT>(hb[3], acc, cb, lanebyte, xs, xoff + 768);
                    }
                }
            } else {
                for (int c = c0; c < c1; ++c) {
                    const int nq = min(16, (IN - (c << 8)) >> 4);
                    const int xoff = g * kXStride + (((c - c0) << 8) + 4 * t) * 2;
                    dense_chunk<NMAT, MT>(acc, wr, IN, c, nq, xs, xoff);
                }
            }
        }
        // ---- results of this block's pairs for this warp's rows
        if (active) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tk = 2 * t + (i & 1);
                    const int row = wrow + mt * 16 + g + (i >> 1) * 8;
                    const int p = s_pairs[tk];
                    if (p < 0 || row >= OUT) continue;
                    r.out[(size_t)p * OUT + row] = epilogue_value<DUAL>(
                        acc[0][mt][i], acc[NMAT - 1][mt][i], r.pair_scale, p, r.out_f16, r.act);
                }
        }
    }
}

// ----------------------------------------------------------------- kernel
// Tile `tile` of phase 1 (tile < n1) or phase 2: its expert and rows.
__device__ __forceinline__ TileInfo tile_info(const RoutedSet &r, int tile, int n1, int rt1, int rt2) {
    TileInfo in;
    const bool p1 = tile < n1;
    const int u = p1 ? tile : tile - n1;
    const int rt = p1 ? rt1 : rt2;
    in.phase = p1 ? 1 : 2;
    in.ai = u / rt;
    in.e = r.active[in.ai];
    in.n = r.cnt[in.e];
    in.base = r.off[in.e];
    in.row0 = (u - in.ai * rt) * (p1 ? kTR1 : kTR2);
    return in;
}

// VQ1 / VQ2: phase 1 / phase 2 weights are VQ (else dense bf16). A CTA runs
// the phase 1 tiles it takes, then (one codebook restage) phase 2 tiles.
template <bool VQ1, bool VQ2>
__global__ void __launch_bounds__(kThreads, 2) expert_kernel(const PipeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TileInfo s_info;
    __shared__ int s_next;
    __shared__ int s_pairs[8];
    const int tid = threadIdx.x;
    uint8_t *cb = smem;
    uint8_t *xs = smem + ((VQ1 || VQ2) ? kRepBytes : 0);
    // the phase 1 codebooks (weights) before the routing is ready, then the
    // routing kernel's results (launched with programmatic dependence)
    if (VQ1 && a.has1) stage_codebooks(cb, a.s1.w0, a.s1.w1, 2);
    pdl_wait();
    const int nact = a.s2.active[a.s2.E];
    const int rt1 = a.has1 ? (a.s1.OUT + kTR1 - 1) / kTR1 : 0;
    const int rt2 = (a.s2.OUT + kTR2 - 1) / kTR2;
    const int n1 = nact * rt1, n2 = nact * rt2;
    if (tid == 0) s_next = (int)atomicAdd(a.ctl, 1u);
    __syncthreads();
    // ---- phase 1: gate/up + SwiGLU
    if (s_next < n1) {
        for (;;) {
            const int tile = s_next;
            if (tile >= n1) break;
            __syncthreads();                      // everyone has read s_next; codebooks staged
            if (tid == 0) {
                s_info = tile_info(a.s2, tile, n1, rt1, rt2);
                s_next = (int)atomicAdd(a.ctl, 1u);
            }
            __syncthreads();
            const TileInfo in = s_info;
            run_tile<2, 1, VQ1>(a.s1, in, cb, xs, s_pairs);
            __syncthreads();                      // every warp's outputs are stored
            if (tid == 0) {
                __threadfence();
                atomicAdd(a.ctl + 2 + in.ai, 1u);
            }
        }
    }
    // ---- phase 2: down (x routing weight), or the single linear
    if (s_next >= n1 + n2) return;
    __syncthreads();                              // phase 1 done with cb
    if (VQ2) stage_codebooks(cb, a.s2.w0, a.s2.w0, 1);
    for (;;) {
        const int tile = s_next;
        if (tile >= n1 + n2) break;
        __syncthreads();                          // everyone has read s_next; codebook staged
        if (tid == 0) {
            const TileInfo in = tile_info(a.s2, tile, n1, rt1, rt2);
            // phase 2 reads what every phase 1 tile of this expert wrote;
            // those tiles were all taken before this one, by running CTAs
            if (a.has1) wait_count(a.ctl + 2 + in.ai, (uint32_t)rt1, a.err, a.wait_polls);
            s_info = in;
            s_next = (int)atomicAdd(a.ctl, 1u);
        }
        __syncthreads();
        const TileInfo in = s_info;
        run_tile<1, 2, VQ2>(a.s2, in, cb, xs, s_pairs);
        __syncthreads();                          // done with s_pairs / xs before the next tile
    }
}

// ------------------------------------------------------- shared expert
// The shared expert's dense bf16 matmuls (qwen3_5.py:184-185) for up to 64
// tokens per pass. A CTA owns 32 output rows and a K slice: it issues
// cp.async for its whole weight slice and all token rows at once (the
// weights are read exactly once, with the full slice in flight), then its 8
// warps -- one per 8 tokens -- multiply from shared memory. K slices meet in
// a float32 partial buffer; the last CTA of a row block to finish (one
// atomic, no waiting) sums them in slice order and applies the epilogue.
constexpr int kShRows = 32;
constexpr int kShTok = 64;

struct SharedArgs {
    const uint16_t *x;           // [T][IN] bf16
    const uint16_t *w0, *w1;     // [OUT][IN] bf16
    int T, IN, OUT, ks, kslice;  // K slices of kslice inputs (multiple of 16)
    uint16_t *out;               // [T][OUT] bf16
    float *part;                 // [ks][T][NMAT][OUT] (ks > 1)
    uint32_t *sem;               // [OUT / 32]
};

template <int NMAT>
__global__ void __launch_bounds__(256) shared_dense_kernel(const SharedArgs a) {
    constexpr bool DUAL = NMAT == 2;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t s_old;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int rb = blockIdx.x, ksi = blockIdx.y;
    const int row0 = rb * kShRows;
    const int k0 = ksi * a.kslice, kl = min(a.kslice, a.IN - k0);
    const int stride = a.kslice * 2 + 32;            // bytes per staged row
    uint8_t *wa = smem;                              // [NMAT][32][stride]
    uint8_t *xb = smem + NMAT * kShRows * stride;    // [64][stride]
    for (int tp0 = 0; tp0 < a.T; tp0 += kShTok) {
        const int nt = min(kShTok, a.T - tp0);
        __syncthreads();
        const int nv = kl >> 3;
        for (int v = tid; v < (NMAT * kShRows + kShTok) * nv; v += blockDim.x) {
            const int r = v / nv, j = v - r * nv;
            if (r < NMAT * kShRows) {
                const int m = r / kShRows, rr = r - m * kShRows;
                const bool ok = row0 + rr < a.OUT;
                const uint16_t *src = (m == 0 ? a.w0 : a.w1) + (size_t)(ok ? row0 + rr : 0) * a.IN + k0 + 8 * j;
                cp_async16(smem_u32(wa + r * stride + j * 16), src, ok ? 16 : 0);
            } else {
                const int tk = r - NMAT * kShRows;
                const bool ok = tk < nt;
                const uint16_t *src = a.x + (size_t)(ok ? tp0 + tk : 0) * a.IN + k0 + 8 * j;
                cp_async16(smem_u32(xb + tk * stride + j * 16), src, ok ? 16 : 0);
            }
        }
        cp_async_wait_all();
        __syncthreads();
        float acc[NMAT][2][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][mt][i] = 0.0f;
        const uint8_t *xw = xb + (warp * 8 + g) * stride + 8 * t;
#pragma unroll 4
        for (int q = 0; q < (kl >> 4); ++q) {
            const uint2 bf = *reinterpret_cast<const uint2 *>(xw + q * 32);
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    const uint8_t *ar = wa + (m * kShRows + mt * 16 + g) * stride + 8 * t + q * 32;
                    const uint2 a0 = *reinterpret_cast<const uint2 *>(ar);
                    const uint2 a1 = *reinterpret_cast<const uint2 *>(ar + 8 * stride);
                    mma_bf16(acc[m][mt], a0.x, a1.x, a0.y, a1.y, bf.x, bf.y);
                }
        }
        // fragment -> (token tp0 + 8*warp + 2t + (i&1), row row0 + 16mt + g + 8*(i>>1))
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tok = tp0 + warp * 8 + 2 * t + (i & 1);
                const int row = row0 + mt * 16 + g + (i >> 1) * 8;
                if (tok >= a.T || row >= a.OUT) continue;
                if (a.ks == 1) {
                    a.out[(size_t)tok * a.OUT + row] =
                        epilogue_value<DUAL>(acc[0][mt][i], acc[NMAT - 1][mt][i], nullptr, 0, 0);
                } else {
#pragma unroll
                    for (int m = 0; m < NMAT; ++m)
                        a.part[(((size_t)ksi * a.T + tok) * NMAT + m) * a.OUT + row] = acc[m][mt][i];
                }
            }
    }
    if (a.ks == 1) return;
    // the last K slice of this row block sums the slices in slice order
    __threadfence();
    __syncthreads();
    if (tid == 0) s_old = atomicAdd(&a.sem[rb], 1u);
    __syncthreads();
    if (s_old != (uint32_t)(a.ks - 1)) return;
    if (tid == 0) a.sem[rb] = 0u;
    __threadfence();
    for (int o = tid; o < a.T * kShRows; o += blockDim.x) {
        const int tok = o / kShRows, row = row0 + (o - tok * kShRows);
        if (row >= a.OUT) continue;
        float v[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            float pv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                pv[q] = q < a.ks ? __ldcg(&a.part[(((size_t)q * a.T + tok) * NMAT + m) * a.OUT + row]) : 0.0f;
            float sum = pv[0];
#pragma unroll
            for (int q = 1; q < 4; ++q)
                if (q < a.ks) sum += pv[q];
            v[m] = sum;
        }
        a.out[(size_t)tok * a.OUT + row] = epilogue_value<DUAL>(v[0], v[NMAT - 1], nullptr, 0, 0);
    }
}

// K slicing of the shared expert: slices of <= 512 inputs (a multiple of 16)
// so that the grid covers the GPU; plus the shared memory it needs.
void plan_shared_dense(int IN, int OUT, int nmat, int *ks, int *kslice, size_t *smem) {
    const int rbs = (OUT + kShRows - 1) / kShRows;
    int want = std::max(1, (int)((sm_count() + rbs - 1) / rbs));
    want = std::min(want, 4);                    // at most 4 K slices to reduce
    int kl = std::max(16, (IN + want - 1) / want);
    kl = std::min(1024, (kl + 15) / 16 * 16);
    *kslice = kl;
    *ks = (IN + kl - 1) / kl;
    *smem = (size_t)(nmat * kShRows + kShTok) * (kl * 2 + 32);
}

vqmoe_status launch_shared_dense(const void *x, const void *w0, const void *w1, int T, int IN, int OUT,
                                 void *out, float *part, uint32_t *sem, cudaStream_t stream) {
    const int nmat = w1 ? 2 : 1;
    int ks = 1, kl = IN;
    size_t smem = 0;
    plan_shared_dense(IN, OUT, nmat, &ks, &kl, &smem);
    SharedArgs a{};
    a.x = static_cast<const uint16_t *>(x);
    a.w0 = static_cast<const uint16_t *>(w0);
    a.w1 = static_cast<const uint16_t *>(w1 ? w1 : w0);
    a.T = T;
    a.IN = IN;
    a.OUT = OUT;
    a.ks = ks;
    a.kslice = kl;
    a.out = static_cast<uint16_t *>(out);
    a.part = part;
    a.sem = sem;
    dim3 grid((OUT + kShRows - 1) / kShRows, ks);
    auto fn = nmat == 2 ? shared_dense_kernel<2> : shared_dense_kernel<1>;
    vqmoe_status s = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), smem, "shared expert kernel");
    if (s != VQMOE_OK) return s;
    fn<<<grid, 256, smem, stream>>>(a);
    return check_launch("shared_dense_kernel");
}

// ------------------------------------------------------------------ host

template <bool VQ1, bool VQ2>
static vqmoe_status launch_pipe(const PipeArgs &a, size_t smem, cudaStream_t stream) {
    auto fn = expert_kernel<VQ1, VQ2>;
    vqmoe_status s = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), smem, "expert kernel");
    if (s != VQMOE_OK) return s;
    if (launch_pdl(fn, dim3(2 * sm_count()), dim3(kThreads), smem, stream, a) != cudaSuccess)
        return check_launch("expert_kernel");
    return check_launch("expert_kernel");
}

static LinearDev dev_of(const vqmoe_linear *w) {
    LinearDev d{};
    d.codes = static_cast<const uint8_t *>(w->codes);
    d.codebook = static_cast<const uint16_t *>(w->codebook);
    d.scales = static_cast<const uint16_t *>(w->scales);
    d.weight = static_cast<const uint16_t *>(w->weight);
    d.K = w->codebook_size;
    return d;
}

static RoutedSet set_of(const RoutedIO &r, const vqmoe_linear *w0, const vqmoe_linear *w1) {
    RoutedSet s{};
    s.cnt = r.cnt;
    s.off = r.off;
    s.list = r.list;
    s.active = r.active;
    s.E = r.E;
    s.k = r.k;
    s.P = r.P;
    s.x_per_pair = r.x_per_pair;
    s.x = static_cast<const uint16_t *>(r.x);
    s.w0 = dev_of(w0);
    s.w1 = w1 ? dev_of(w1) : s.w0;
    s.IN = w0->in_features;
    s.OUT = w0->out_features;
    s.out = static_cast<uint16_t *>(r.out);
    s.out_f16 = r.out_f16;
    s.pair_scale = r.pair_scale;
    s.act = r.act;
    return s;
}

vqmoe_status launch_experts(const vqmoe_linear *gate, const vqmoe_linear *up, const RoutedIO *r1,
                            const vqmoe_linear *w2, const RoutedIO &r2, uint32_t *ctl, uint32_t *err,
                            uint32_t wait_polls, cudaStream_t stream, cudaEvent_t after_permute) {
    if (is_general(w2->format) || (r1 && is_general(gate->format))) {
        if (after_permute && cudaEventRecord(after_permute, stream) != cudaSuccess) return check_launch("event");
        return launch_experts_ref(gate, up, r1, w2, r2, stream);
    }
    PipeArgs a{};
    a.ctl = ctl;
    a.err = err;
    a.wait_polls = wait_polls;
    a.has1 = r1 != nullptr;
    a.s2 = set_of(r2, w2, nullptr);
    a.s1 = r1 ? set_of(*r1, gate, up) : a.s2;
    const bool vq2 = w2->format == VQMOE_FMT_VQ_U8;
    const bool vq1 = r1 ? gate->format == VQMOE_FMT_VQ_U8 : vq2;
    // many pairs per expert (prefill): the tcgen05 grouped GEMM
    void *xs = r1 ? r1->xs : r2.xs;
    if (prefill_regime(vq1 && vq2, r2.E, r2.P) && xs) return launch_experts_prefill(a, xs, stream, after_permute);
    if (after_permute && cudaEventRecord(after_permute, stream) != cudaSuccess) return check_launch("event");
    const size_t smem = (vq1 || vq2 ? (size_t)kRepBytes : 0) + (size_t)kXBytes;
    if (vq1) return vq2 ? launch_pipe<true, true>(a, smem, stream) : launch_pipe<true, false>(a, smem, stream);
    return vq2 ? launch_pipe<false, true>(a, smem, stream) : launch_pipe<false, false>(a, smem, stream);
}

}  // namespace vqmoe
