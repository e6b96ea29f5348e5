// Routed VQ experts in the prefill regime on the 5th-generation tensor cores
// (tcgen05 + TMEM): a token-permuted grouped GEMM with the VQ dequantisation
// fused into the operand path.
//
// Reference: SwitchGLU.__call__ (glm5_next/_mlx_vlm/models/switch_layers.py:
// 172-193; with many pairs the reference sorts them by expert,
// switch_layers.py:9-21) with VQSwitchLinear experts
// (engine/families/deepseek/heads/deepseek_v4.py:35-42, 111-130) and the
// _SwiGLU activation (qwen3_5.py:108-112).
//
// One persistent CTA of two warpgroups per SM. It takes tiles of (expert, 128
// weight rows, 128 of the expert's pairs) from a global counter -- phase 1
// (gate/up + SwiGLU) tiles first, then phase 2 (down x routing weight, or a
// single switch linear); a phase 2 tile of expert e waits until every phase
// 1 tile of e is done (bounded wait, error flag on expiry).
//
// Per tile, for each 64-input window: the warps gather the pairs' input rows
// (fp16) with cp.async into a 4-stage shared-memory ring, in the canonical
// K-major no-swizzle layout of the MMA's B operand (loaded two windows
// ahead). Each lane owns one weight row and half of each window (the two
// warpgroups take alternate 8-input chunks): it reads the row's codes from
// the tiled VQ layout (layout.cuh), looks each code up in the shared-memory
// codebook, multiplies the 4 fp16 weights by the group scale (one rounding:
// fp16(codebook x scale), the dense dequantisation bit for bit) and stores
// each 64-input window into a TMEM slot, the MMA's A operand. Lane 0 of the
// CTA issues tcgen05.mma M=128 x N=128 x K=16 into TMEM accumulators (gate
// and up: 128 columns each) and commits to the slot's mbarrier (and, after a
// window, to the window's). The epilogue reads the accumulators back
// (tcgen05.ld) and applies the SwiGLU / routing weight.
#include <algorithm>

#include "experts.cuh"
#include "layout.cuh"
#include "stages.cuh"
#include "tcgen05.cuh"

namespace vqmoe {
namespace pf {
using namespace tc;

constexpr int kProducers = 256;               // two warpgroups, each over TMEM lanes 0..127
constexpr int kThreads = kProducers + 32;     // + one warp that issues the MMAs
constexpr int kN = 128;                       // pairs per tile (MMA N)
constexpr int kSlots = 4;                     // A slots per matrix (a 64-input window each)
constexpr int kWin = 64;                      // inputs per x window
constexpr int kStages = 8;                    // x windows in shared memory
constexpr int kAhead = 4;                     // x windows gathered ahead of the one multiplied
constexpr int kStageBytes = kN * kWin * 2;    // 16 KB
constexpr int kLbo = (kN / 8) * 128;          // bytes from one 8-input chunk to the next
constexpr int kCbRegion = 65536;              // the phase's codebooks: gate / up, then down
constexpr size_t kSmem = kCbRegion + (size_t)kStages * kStageBytes;
constexpr int kDCol = 2 * kSlots * 32;        // D of matrix m at kDCol + 128m (all 512 columns)
constexpr int kAllocCols = 512;
constexpr int kMaxE = 512;
constexpr long kSpin = 1L << 22;
// kind::f16, D f32, A f16, B f16, both K-major, N = 128, M = 128
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((128u >> 4) << 24);

// ---------------------------------------------------------------- PTX
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// B operand descriptor, K-major, no swizzle: core matrices of 8 pairs x 8
// inputs (16 bytes a pair); SBO = 128 (the next 8 pairs), LBO = kLbo (the
// next 8 inputs).
__device__ __forceinline__ uint64_t b_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((kLbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)(128u >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ uint2 lds64(uint32_t saddr) {
    uint2 r;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "r"(saddr));
    return r;
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// 16 interleaved copies: entry c of copy b of matrix m at region + 256c + 128m + 8b
__device__ __forceinline__ void stage_codebook(uint8_t *region, const LinearDev &w, int m) {
    for (int i = threadIdx.x; i < 4096; i += kThreads) {
        const int c = i >> 4, b = i & 15;
        uint2 v = make_uint2(0, 0);
        if (c < w.K) v = ldg_nc_v2(w.codebook + c * 4);
        *reinterpret_cast<uint2 *>(region + c * 256 + m * 128 + b * 8) = v;
    }
}

struct Shared {
    uint64_t full[kSlots];                    // an A slot and its window's x stage written
    uint64_t slot[kSlots];                    // MMAs done reading an A slot
    uint64_t stage[kStages];                  // MMAs done reading an x stage
    uint64_t acc;                             // a tile's MMAs done: accumulators final
    TileInfo info;
    int next;
    int pairs[kN];
    float pscale[kN];                         // the pairs' routing weights (phase 2)
    int pre1[kMaxE + 1], pre2[kMaxE + 1];     // tiles before active expert i, per phase
};

// The pipeline state (identical in all threads): batches issued, window
// commits per stage, tile completions.
struct Pipe {
    uint32_t gb;
    uint32_t sw[kStages];
    uint32_t dn;
    bool failed;
};

// ----------------------------------------------------------------- tile
// Two accumulators -> two packed outputs (the first in the low half).
// _SwiGLU (qwen3_5.py:108-112): bf16(bf16(silu(g)) * u) with g and u the
// bf16 outputs of the gate and up matmuls; otherwise bf16(bf16(y) * routing
// weight). Every rounding is the hardware's round-to-nearest-even
// (cvt.rn.bf16x2), the same bits as the software rounding of the other
// kernels for finite values; a bf16 x bf16 product is exact in float32. The
// one approximation: silu's exp and division are the fast forms (ex2 /
// rcp, a few float32 ulp before the bf16 rounding).
template <bool GLU>
__device__ __forceinline__ uint32_t pf_value2(uint32_t g0, uint32_t g1, uint32_t u0, uint32_t u1, bool scaled,
                                              float s0, float s1, int out_f16) {
    const uint32_t gb = cvt_bf16x2(__uint_as_float(g0), __uint_as_float(g1));
    uint32_t v;
    if (GLU) {
        const uint32_t ub = cvt_bf16x2(__uint_as_float(u0), __uint_as_float(u1));
        const uint32_t sb = cvt_bf16x2(silu_fast(bf_lo(gb)), silu_fast(bf_hi(gb)));
        v = cvt_bf16x2(bf_lo(sb) * bf_lo(ub), bf_hi(sb) * bf_hi(ub));
    } else {
        v = scaled ? cvt_bf16x2(bf_lo(gb) * s0, bf_hi(gb) * s1) : gb;
    }
    if (out_f16)
        return cvt_f16x2(fminf(fmaxf(bf_lo(v), -65504.0f), 65504.0f), fminf(fmaxf(bf_hi(v), -65504.0f), 65504.0f));
    return v;
}

// One tile. The producer warps (0..7): thread tid stages, in every window,
// the 16-byte chunk tid % 8 of the 4 pair slots tid / 8 + 32q (q = 0..3),
// with row pointers computed once per tile; each lane dequantises its weight
// row's half of the window into the A slot; one lane per warp then arrives
// on the slot's `full` barrier. The MMA warp (8) waits on `full`, multiplies
// and commits the slot, the x stage and, after the last window, the
// accumulators. One A batch is one 64-input window. Every tile has two A
// operands: gate and up of 128 rows (GLU), or rows row0 .. row0 + 127 and
// row0 + 128 .. row0 + 255 of the one matrix (a switch linear / down).
template <bool GLU>
__device__ __forceinline__ void pf_tile(const RoutedSet &r, const TileInfo &in, uint32_t cb_s, uint8_t *xs,
                                        Shared &sh, uint32_t tmem, Pipe &ps, uint32_t *err) {
    constexpr int NMAT = 2;
    constexpr bool DUAL = GLU;
    const int tid = threadIdx.x, warp = (tid >> 5) & 3, lane = tid & 31;
    const int IN = r.IN, OUT = r.OUT;
    const int C = (IN + 255) >> 8, RB = (OUT + 31) >> 5;
    const int NW = C * 4;                     // 64-input windows
    const uint32_t xs_s = smem_u32(xs);
    if (tid < kN) {
        const int p = tid < in.n ? r.list[in.base + tid] : -1;
        sh.pairs[tid] = p;
        sh.pscale[tid] = (!DUAL && r.pair_scale && p >= 0) ? r.pair_scale[p] : 1.0f;
    }
    __syncthreads();
    if (tid >= kProducers) {
        // ---- the MMA warp
        if (lane == 0) {
            uint32_t gb = ps.gb;
            for (int win = 0; win < NW; ++win, ++gb) {
                const uint32_t slot = gb % kSlots;
                mbar_wait(&sh.full[slot], (gb / kSlots) & 1, err, ps.failed);
                tc_fence_after();
                const int s = win % kStages;
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int k16 = 0; k16 < 4; ++k16)
                        tc_mma(tmem + kDCol + 128 * m, tmem + 32 * (kSlots * m + slot) + 8 * k16,
                               b_desc(xs_s + s * kStageBytes + (2 * k16) * kLbo), win > 0 || k16 > 0);
                tc_commit(&sh.slot[slot]);
                tc_commit(&sh.stage[s]);
            }
            tc_commit(&sh.acc);
        }
        __syncwarp();
        ps.gb += NW;
        tc_fence_before();
        __syncthreads();
        return;
    }
    // ---- the producer warps
    const int wgi = tid >> 7;                 // warpgroup: 8-input chunks 2j + wgi of each window
    const int mt = lane >> 4, hh = (lane >> 3) & 1, g = lane & 7;
    // this lane's row of operand m in the tiled layout: per chunk c, half:
    // codes at tile*2048 + half*1024 + (2mt+h)*256 + 32g (32 bytes), scales
    // at tile*128 + half*64 + (2mt+h)*16 + 2g (2 fp16)
    const uint8_t *cbase[NMAT];
    const uint16_t *sbase[NMAT];
    bool rows_ok[NMAT];
    int row[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const LinearDev &w = (GLU && m == 1) ? r.w1 : r.w0;
        const int rb = (in.row0 >> 5) + warp + (GLU ? 0 : 4 * m);
        rows_ok[m] = rb < RB;
        row[m] = rb * 32 + lane;
        const long long tile0 = ((long long)in.e * RB + (rows_ok[m] ? rb : 0)) * C;
        cbase[m] = w.codes + tile0 * 2048 + (2 * mt + hh) * 256 + 32 * g + 16 * wgi;
        sbase[m] = w.scales + tile0 * 128 + (2 * mt + hh) * 16 + 2 * g;
    }
    const uint32_t lanebyte = (lane & 15) * 8;
    const uint32_t t_warp = tmem + ((uint32_t)(warp * 32) << 16);
    // ---- this thread's staging: input chunk ch of slots n0 + 32q. The MMA's K
    // order within a window is permuted -- input chunk ch sits at K chunk
    // kch(ch) = 4 (ch & 1) + ch / 2 in both operands -- so that warpgroup wgi
    // dequantises the contiguous A columns 16 wgi .. 16 wgi + 15.
    constexpr int kQ = kN * 8 / kProducers;   // slots a thread stages per window
    const int ch = tid & 7, n0 = tid >> 3;
    const int kch = 4 * (ch & 1) + (ch >> 1);
    const uint16_t *src[kQ];
    uint32_t dst0[kQ];
    uint32_t live = 0;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
        const int n = n0 + (kProducers / 8) * q;
        const int p = sh.pairs[n];
        const int xr = p < 0 ? 0 : (r.x_per_pair ? p : p / r.k);
        src[q] = r.x + (size_t)xr * IN + 8 * ch;
        dst0[q] = xs_s + kch * kLbo + (n >> 3) * 128 + (n & 7) * 16;
        live |= (p >= 0 ? 1u : 0u) << q;
    }
#pragma unroll
    for (int w0 = 0; w0 < kAhead; ++w0) {
        if (w0 < NW) {
#pragma unroll
            for (int q = 0; q < kQ; ++q)
                if (live >> q & 1) {
                    const int f = w0 * kWin + 8 * ch;
                    cp_async16(dst0[q] + w0 * kStageBytes, src[q] + w0 * kWin, f < IN ? 16 : 0);
                }
        }
        cp_async_commit();
    }
    // ---- this warpgroup's codes of half chunks (t = 2wgi, 2wgi+1: 16 bytes):
    // cur (windows 2h, 2h+1) and the next two
    uint4 cc[NMAT], nc1[NMAT], nc2[NMAT];
    uint32_t cs[NMAT], ns1[NMAT], ns2[NMAT];
    auto load_half = [&](int hn, int m, uint4 &c, uint32_t &sc) {
        if (rows_ok[m] && hn < 2 * C) {
            c = ldg_stream_v4(cbase[m] + (long long)(hn >> 1) * 2048 + (hn & 1) * 1024);
            sc = ldg_stream_u32(sbase[m] + (long long)(hn >> 1) * 128 + (hn & 1) * 64);
        } else {
            c = make_uint4(0, 0, 0, 0);
            sc = 0u;
        }
    };
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        load_half(0, m, cc[m], cs[m]);
        load_half(1, m, nc1[m], ns1[m]);
        load_half(2, m, nc2[m], ns2[m]);
    }
    for (int hw = 0; hw < NW; hw += 2) {     // two windows = one half chunk
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const int win = hw + ww;
            // refill: window win + kAhead into the stage that window
            // win + kAhead - kStages used (its MMAs must be done)
            if (win + kAhead < NW) {
                const int s2 = (win + kAhead) % kStages;
                if (win >= kStages - kAhead) {
                    warp_wait(&sh.stage[s2], ps.sw[s2] & 1, err, ps.failed);
                    ++ps.sw[s2];
                }
                const int fw = (win + kAhead) * kWin;
#pragma unroll
                for (int q = 0; q < kQ; ++q)
                    if (live >> q & 1)
                        cp_async16(dst0[q] + s2 * kStageBytes, src[q] + fw, fw + 8 * ch < IN ? 16 : 0);
            }
            cp_async_commit();
            // dequantise this lane's 32 inputs of the window (while the copies
            // fly): local quad l = 2j + s is code t = 2wgi + s, b = 4ww + j --
            // byte j of word 2s + ww of this warpgroup's 16 bytes -- and goes to
            // A columns 16wgi + 2l, 2l + 1 (K chunk 4wgi + j = input chunk 2j + wgi)
            const uint32_t slot = ps.gb % kSlots;
            uint32_t a[NMAT][16];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const uint32_t s2v = __byte_perm(cs[m], 0, ww ? 0x3232 : 0x1010);
                const uint32_t words[4] = {cc[m].x, cc[m].y, cc[m].z, cc[m].w};
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    const int j = l >> 1, sb = l & 1;
                    const uint32_t ad = __byte_perm(words[2 * sb + ww], lanebyte, 0x5504u | (j << 4));
                    const uint2 e = lds64(cb_s + (GLU ? m * 128 : 0) + ad);
                    a[m][2 * l] = hmul2_u32(e.x, s2v);
                    a[m][2 * l + 1] = hmul2_u32(e.y, s2v);
                }
            }
            if (ps.gb >= kSlots) warp_wait(&sh.slot[slot], ((ps.gb / kSlots) + 1) & 1, err, ps.failed);
            tc_fence_after();
#pragma unroll
            for (int m = 0; m < NMAT; ++m) tmem_st16(t_warp + 32 * (kSlots * m + slot) + 16 * wgi, a[m]);
            cp_async_wait<kAhead>();          // this thread's copies of window win
            fence_proxy_async();
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.full[slot]);
            ++ps.gb;
        }
        // next half chunk
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            cc[m] = nc1[m];
            cs[m] = ns1[m];
            nc1[m] = nc2[m];
            ns1[m] = ns2[m];
            load_half((hw >> 1) + 3, m, nc2[m], ns2[m]);
        }
    }
    // ---- the tile's MMAs done; then the stage commits the loop did not wait
    // for (windows NW - kStages .. NW - 1), already complete
    warp_wait(&sh.acc, ps.dn & 1, err, ps.failed);
    ++ps.dn;
    for (int win = (NW > kStages ? NW - kStages : 0); win < NW; ++win) {
        const int s2 = win % kStages;
        warp_wait(&sh.stage[s2], ps.sw[s2] & 1, err, ps.failed);
        ++ps.sw[s2];
    }
    tc_fence_after();
    // ---- accumulators -> outputs, 32 pairs at a time; warpgroup wgi takes
    // pairs 64 wgi .. 64 wgi + 63
#pragma unroll 1
    for (int q = 2 * wgi; q < 2 * wgi + 2; ++q) {
        uint32_t dv[NMAT][32];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) tmem_ld32(t_warp + kDCol + 128 * m + 32 * q, dv[m]);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < (GLU ? 1 : NMAT); ++m) {
            if (rows_ok[m] && row[m] < OUT) {
                uint32_t ov[16];
#pragma unroll
                for (int jp = 0; jp < 16; ++jp)
                    ov[jp] = pf_value2<GLU>(dv[m][2 * jp], dv[m][2 * jp + 1], dv[1][2 * jp], dv[1][2 * jp + 1],
                                            r.pair_scale != nullptr, sh.pscale[32 * q + 2 * jp],
                                            sh.pscale[32 * q + 2 * jp + 1], r.out_f16);
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int p = sh.pairs[32 * q + jj];
                    if (p >= 0) r.out[(size_t)p * OUT + row[m]] = (uint16_t)(ov[jj >> 1] >> (16 * (jj & 1)));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
}

// Tiles before active expert i of each phase (pairs in blocks of kN): the
// block counts are read in parallel, then summed in order by one thread.
__device__ __forceinline__ void tile_prefix(const PipeArgs &a, Shared &sh, int nact, int rt1, int rt2) {
    for (int i = threadIdx.x; i < nact; i += kThreads)
        sh.pre2[i] = (a.s2.cnt[a.s2.active[i]] + kN - 1) / kN;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t1 = 0, t2 = 0;
        for (int i = 0; i < nact; ++i) {
            const int nb = sh.pre2[i];
            sh.pre1[i] = t1;
            sh.pre2[i] = t2;
            t1 += nb * rt1;
            t2 += nb * rt2;
        }
        sh.pre1[nact] = t1;
        sh.pre2[nact] = t2;
    }
    __syncthreads();
}

// the active expert holding tile u of a phase: the last i with pre[i] <= u
__device__ __forceinline__ int find_expert(const int *pre, int nact, int u) {
    int lo = 0, hi = nact - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= u) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// --------------------------------------------------------------- kernel
__global__ void __launch_bounds__(kThreads, 1) expert_prefill_kernel(const PipeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ Shared sh;
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x;
    uint8_t *cb = smem, *xs = smem + kCbRegion;
    if (tid == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&sh.full[i], kProducers / 32);
            mbar_init(&sh.slot[i], 1);
        }
        for (int i = 0; i < kStages; ++i) mbar_init(&sh.stage[i], 1);
        mbar_init(&sh.acc, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (tid < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(&s_tmem)),
                     "r"(kAllocCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    uint32_t *err = a.ctl + 1;
    const int nact = min(a.s2.active[a.s2.E], kMaxE);
    const int rt1 = a.has1 ? (a.s1.OUT + 127) / 128 : 0;
    const int rt2 = (a.s2.OUT + 255) / 256;     // phase 2 tiles: 256 rows
    tile_prefix(a, sh, nact, rt1, rt2);
    const int n1 = a.has1 ? sh.pre1[nact] : 0, n2 = sh.pre2[nact];
    Pipe ps{};
    int cb_phase = 0;                         // the phase whose codebooks are staged
    if (tid == 0) sh.next = (int)atomicAdd(a.ctl, 1u);
    __syncthreads();
    for (;;) {
        const int tile = sh.next;
        if (tile >= n1 + n2) break;
        __syncthreads();                      // everyone has read next
        if (tid == 0) {
            TileInfo in;
            const bool p1 = tile < n1;
            const int u = p1 ? tile : tile - n1;
            const int *pre = p1 ? sh.pre1 : sh.pre2;
            const int rt = p1 ? rt1 : rt2;
            in.phase = p1 ? 1 : 2;
            in.ai = find_expert(pre, nact, u);
            in.e = a.s2.active[in.ai];
            const int v = u - pre[in.ai];
            const int blk = v / rt;
            in.row0 = (v - blk * rt) * (p1 ? 128 : 256);
            const int cnt = a.s2.cnt[in.e];
            in.base = a.s2.off[in.e] + blk * kN;
            in.n = min(kN, cnt - blk * kN);
            if (!p1 && a.has1) {
                // every phase 1 tile of this expert (all its blocks) is done;
                // they were all taken before this one, by running CTAs
                const uint32_t want = (uint32_t)(((cnt + kN - 1) / kN) * rt1);
                const uint32_t *c = a.ctl + 2 + in.ai;
                for (long i = 0;; ++i) {
                    uint32_t val;
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(val) : "l"(c) : "memory");
                    if (val >= want) break;
                    if (i >= kSpin) {
                        atomicExch(err, 1u);
                        break;
                    }
                    __nanosleep(256);
                }
            }
            sh.info = in;
            sh.next = (int)atomicAdd(a.ctl, 1u);
        }
        __syncthreads();
        const TileInfo in = sh.info;
        if (in.phase != cb_phase) {
            // a CTA's tiles go phase 1, then phase 2: (re)stage the codebooks
            // once per phase; every lookup of the previous tile is done
            if (in.phase == 1) {
                stage_codebook(cb, a.s1.w0, 0);
                stage_codebook(cb, a.s1.w1, 1);
            } else {
                stage_codebook(cb, a.s2.w0, 0);
            }
            cb_phase = in.phase;
            __syncthreads();
        }
        if (in.phase == 1) {
            pf_tile<true>(a.s1, in, smem_u32(cb), xs, sh, tmem, ps, err);
            if (tid == 0) {
                __threadfence();
                atomicAdd(a.ctl + 2 + in.ai, 1u);
            }
        } else {
            pf_tile<false>(a.s2, in, smem_u32(cb), xs, sh, tmem, ps, err);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid < 32) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(s_tmem),
                     "r"(kAllocCols)
                     : "memory");
    }
}

}  // namespace pf

vqmoe_status launch_experts_prefill(const PipeArgs &a, cudaStream_t stream) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        if (cudaFuncSetAttribute(pf::expert_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pf::kSmem) != cudaSuccess)
            return set_error(VQMOE_LAUNCH_FAILED, "prefill expert kernel: %zu bytes of shared memory",
                             pf::kSmem);
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    pf::expert_prefill_kernel<<<sm_count(), pf::kThreads, pf::kSmem, stream>>>(a);
    return check_launch("expert_prefill_kernel");
}

}  // namespace vqmoe
