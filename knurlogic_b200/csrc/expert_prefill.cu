// Routed VQ experts in the prefill regime on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA): a token-permuted grouped GEMM with the VQ
// dequantisation fused into the operand path.
//
// Reference: SwitchGLU.__call__ (glm5_next/_mlx_vlm/models/switch_layers.py:
// 172-193; with many pairs the reference sorts them by expert,
// switch_layers.py:9-21) with VQSwitchLinear experts
// (engine/families/deepseek/heads/deepseek_v4.py:35-42, 111-130) and the
// _SwiGLU activation (qwen3_5.py:108-112).
//
// Before the kernel, permute_rows_kernel copies the pairs' fp16 input rows
// into expert order (the routing sort's order), so that the 128 pairs of a
// tile are 128 consecutive rows; the gate/up phase writes its SwiGLU
// activations in that order too, so the down phase reads them the same way.
//
// One persistent CTA of ten warps per SM takes tiles of (expert, weight
// rows, 128 of the expert's pairs) from a global counter: phase 1 (gate and
// up, 128 rows each, + SwiGLU) tiles first, then phase 2 (256 rows of down
// x routing weight, or of a single switch linear); a phase 2 tile of expert
// e reads its inputs once every phase 1 tile of e is done (bounded wait,
// error flag on expiry). Every tile has two A operands in TMEM (gate and
// up, or two 128-row halves) and one B operand (the pairs' inputs) in
// shared memory. The roles run decoupled, tile after tile, through
// mbarriers; no block-wide barrier between tiles:
//   warp 9     scheduler + TMA: takes the next tile from the counter and
//              publishes it in a ring of tile descriptors one tile ahead,
//              then copies the current tile's x windows (two 2-D tensor
//              copies of 128 pairs x 64 inputs per 128-input window) into a
//              4-stage ring;
//   warps 0-7  producers, warpgroup g dequantising operand g: each lane owns
//              one weight row, reads its codes from the tiled VQ layout
//              (layout.cuh), looks each code up in the shared-memory
//              codebook, multiplies by the group scale (one rounding:
//              fp16(codebook x scale), the dense dequantisation bit for bit)
//              and stores each 128-input window into a TMEM slot. After a
//              tile's last window they prepare the next tile (its pairs,
//              code prefetch and first two windows), then run this tile's
//              epilogue (tcgen05.ld, SwiGLU / routing weight, stores),
//              releasing the accumulators as soon as they are read;
//   warp 8     MMA: once the previous tile's accumulators are released,
//              tcgen05.mma M=128 x N=128 x K=16, A from TMEM, B from the
//              SW128 stage, into two 128-column accumulators; one barrier
//              wait per 16 MMAs (a wait stalls MMA issue).
#include <algorithm>

#include "experts.cuh"
#include "layout.cuh"
#include "stages.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace vqmoe {
namespace pf {
using namespace tc;

constexpr int kProducers = 256;               // two warpgroups, each over TMEM lanes 0..127
constexpr int kMmaWarp = kProducers / 32;     // 8
constexpr int kTmaWarp = kMmaWarp + 1;        // 9
constexpr int kThreads = kProducers + 64;
constexpr int kN = 128;                       // pairs per tile (MMA N)
constexpr int kSlots = 2;                     // A slots per operand (a 128-input window each: 64 columns)
constexpr int kWin = 128;                     // inputs per window (16 MMAs per barrier wait)
constexpr int kStages = 4;                    // x windows in shared memory
constexpr int kSubBytes = kN * 128;           // one 64-input SW128 sub-tile: 128 pairs x 128 bytes
constexpr int kStageBytes = 2 * kSubBytes;    // 32 KB
constexpr int kCbRegion = 65536;              // the phase's codebooks: gate / up, then down
constexpr size_t kSmem = (size_t)kStages * kStageBytes + kCbRegion + 1024;   // + 1024-byte alignment
constexpr int kDCol = 2 * kSlots * 64;        // D of operand m at kDCol + 128m (all 512 columns)
constexpr int kAllocCols = 512;
constexpr int kMaxE = 512;
constexpr int kRing = 4;                      // tile descriptors published ahead
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
__device__ __forceinline__ uint2 lds64(uint32_t saddr) {
    uint2 r;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "r"(saddr));
    return r;
}

// 16 interleaved copies: entry c of copy b of matrix m at region + 256c + 128m + 8b
// (by threads 0 .. nthreads - 1)
__device__ __forceinline__ void stage_codebook(uint8_t *region, const LinearDev &w, int m, int nthreads) {
    for (int i = threadIdx.x; i < 4096; i += nthreads) {
        const int c = i >> 4, b = i & 15;
        uint2 v = make_uint2(0, 0);
        if (c < w.K) v = ldg_nc_v2(w.codebook + c * 4);
        *reinterpret_cast<uint2 *>(region + c * 256 + m * 128 + b * 8) = v;
    }
}

struct Shared {
    // window gb ready: its A slot written by all producer warps and its x
    // stage landed (TMA transaction count); one wait per window for the MMA
    // thread, whose every wait costs MMA issue time
    uint64_t full[kStages];
    uint64_t slot[kSlots];                    // MMAs done reading an A slot
    uint64_t xempty[kStages];                 // MMAs done reading an x stage
    uint64_t acc;                             // a tile's MMAs done: accumulators final
    uint64_t acc_empty;                       // the epilogue has read the accumulators
    uint64_t ti_full[kRing];                  // tile descriptor published
    uint64_t ti_empty[kRing];                 // tile descriptor read by every consumer
    TileInfo ti[kRing];
    int pairs[2][kN];                         // per tile parity: pair ids, then
    float pscale[2][kN];                      // their routing weights (phase 2)
    int pre1[kMaxE + 1], pre2[kMaxE + 1];     // tiles before active expert i, per phase
};

// ----------------------------------------------------------------- tile
// Two accumulators -> two packed outputs (the first in the low half).
// _SwiGLU (qwen3_5.py:108-112): bf16(bf16(silu(g)) * u) with g and u the
// bf16 outputs of the gate and up matmuls; otherwise bf16(bf16(y) * routing
// weight); with GeGLU (gemma4_text.py:131-135) gelu's tanh form in fp32
// takes silu's place. Every rounding is the hardware's round-to-nearest-even
// (cvt.rn.bf16x2), the same bits as the software rounding of the other
// kernels for finite values; a bf16 x bf16 product is exact in float32. The
// one approximation: silu's exp and division are the fast forms (ex2 /
// rcp, a few float32 ulp before the bf16 rounding).
template <bool GLU>
__device__ __forceinline__ uint32_t pf_value2(uint32_t g0, uint32_t g1, uint32_t u0, uint32_t u1, bool scaled,
                                              float s0, float s1, int out_f16, int act) {
    const uint32_t gb = cvt_bf16x2(__uint_as_float(g0), __uint_as_float(g1));
    uint32_t v;
    if (GLU) {
        const uint32_t ub = cvt_bf16x2(__uint_as_float(u0), __uint_as_float(u1));
        const uint32_t sb = act == VQMOE_ACT_GEGLU
                                ? cvt_bf16x2(gelu_tanh_f32(bf_lo(gb)), gelu_tanh_f32(bf_hi(gb)))
                                : cvt_bf16x2(silu_fast(bf_lo(gb)), silu_fast(bf_hi(gb)));
        v = cvt_bf16x2(bf_lo(sb) * bf_lo(ub), bf_hi(sb) * bf_hi(ub));
    } else {
        v = scaled ? cvt_bf16x2(bf_lo(gb) * s0, bf_hi(gb) * s1) : gb;
    }
    if (out_f16)
        return cvt_f16x2(fminf(fmaxf(bf_lo(v), -65504.0f), 65504.0f), fminf(fmaxf(bf_hi(v), -65504.0f), 65504.0f));
    return v;
}

// A warp's 32 rows (lanes) x 32 pairs of 16-bit outputs, v[j] = pairs 2j,
// 2j + 1 of the lane's row, transposed by three shuffle butterflies (lane
// bits 2, 1, 0 swapped with pair bits 2, 3, 4) so that lane L holds rows 8
// (L >> 3) .. + 7 of pairs 16 (L & 1) + 8 ((L >> 1) & 1) + 4 ((L >> 2) & 1)
// + c, c = 0..3 -- one 16-byte store per pair instead of eight 2-byte ones.
// Afterwards the value of row 8 (L >> 3) + i, pair offset c is half c & 1
// of v[(i & 1) << 3 | ((i >> 1) & 1) << 2 | (i >> 2) << 1 | c >> 1].
__device__ __forceinline__ void transpose_rows8(uint32_t (&v)[16], int lane) {
#pragma unroll
    for (int rd = 0; rd < 3; ++rd) {
        const int lbit = 2 - rd, jbit = 1 + rd;           // lane bit 2 <-> index bit 1, ...
        const bool hi = (lane >> lbit) & 1;
#pragma unroll
        for (int i0 = 0; i0 < 16; ++i0) {
            if (i0 & (1 << jbit)) continue;
            const int i1 = i0 | (1 << jbit);
            const uint32_t send = hi ? v[i0] : v[i1];
            const uint32_t recv = __shfl_xor_sync(0xFFFFFFFFu, send, 1 << lbit);
            if (hi) v[i0] = recv;
            else v[i1] = recv;
        }
    }
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

// ---------------------------------------------------------------- roles
// Tile t of this CTA (t = 0, 1, ...), from the global tile counter value
// `tile`: phase 1 tiles (gate/up, 128 rows each) first, then phase 2 (256
// rows); phase 0 = no tile left.
__device__ __forceinline__ TileInfo make_tile(const PipeArgs &a, const Shared &sh, int tile, int n1, int n2,
                                              int nact, int rt1, int rt2) {
    TileInfo in;
    in.phase = 0;
    in.ai = in.e = in.n = in.base = in.row0 = 0;
    if (tile >= n1 + n2) return in;
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
    return in;
}

__device__ __forceinline__ int tile_windows(const PipeArgs &a, const TileInfo &in) {
    const RoutedSet &r = in.phase == 1 ? a.s1 : a.s2;
    return ((r.IN + 255) >> 8) * 2;
}

// The scheduler + TMA thread (warp 9, lane 0): publishes tile t + 1 in the
// descriptor ring, then (a phase 2 tile: once every phase 1 tile of its
// expert is done) copies tile t's x windows into the stage ring. Publishing
// ahead of the dependency wait keeps the other roles from waiting on it:
// the producers read tile t + 1 before finishing tile t's epilogue.
__device__ __forceinline__ void tma_role(const PipeArgs &a, Shared &sh, const void *map1, const void *map2,
                                         uint32_t xs_s, int n1, int n2, int nact, int rt1, int rt2, uint32_t *err,
                                         bool &failed) {
    uint32_t gb = 0;
    TileInfo cur = make_tile(a, sh, (int)atomicAdd(a.ctl, 1u), n1, n2, nact, rt1, rt2);
    sh.ti[0] = cur;
    mbar_arrive(&sh.ti_full[0]);
    for (int t = 0; cur.phase != 0; ++t) {
        const TileInfo nxt = make_tile(a, sh, (int)atomicAdd(a.ctl, 1u), n1, n2, nact, rt1, rt2);
        const int t1 = t + 1, s1 = t1 % kRing;
        if (t1 >= kRing) mbar_wait(&sh.ti_empty[s1], ((t1 / kRing) + 1) & 1, err, failed);
        sh.ti[s1] = nxt;
        mbar_arrive(&sh.ti_full[s1]);
        const bool p1 = cur.phase == 1;
        if (!p1 && a.has1) {
            // phase 2 reads what every phase 1 tile of this expert wrote;
            // they were all taken before this one, by running CTAs
            const uint32_t want = (uint32_t)(((a.s2.cnt[cur.e] + kN - 1) / kN) * rt1);
            const uint32_t *c = a.ctl + 2 + cur.ai;
            for (long i = 1;; ++i) {
                uint32_t val;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(val) : "l"(c) : "memory");
                if (val >= want) break;
                if (i >= (a.wait_polls ? (long)a.wait_polls : kSpin)) {
                    atomicExch(err, kWaitDependency);
                    break;
                }
                __nanosleep(256);
            }
            // the rows other CTAs wrote, now visible here, before the copies read them
            fence_proxy_async_global();
        }
        const void *map = p1 ? map1 : map2;
        const int NW = tile_windows(a, cur);
        for (int win = 0; win < NW; ++win, ++gb) {
            const int s = gb % kStages;
            if (gb >= (uint32_t)kStages) mbar_wait(&sh.xempty[s], ((gb / kStages) + 1) & 1, err, failed);
            arrive_expect_tx(&sh.full[s], kStageBytes);
            tma_load_2d(xs_s + s * kStageBytes, map, win * kWin, cur.base, &sh.full[s]);
            tma_load_2d(xs_s + s * kStageBytes + kSubBytes, map, win * kWin + 64, cur.base, &sh.full[s]);
        }
        cur = nxt;
    }
}

// The MMA thread (warp 8, lane 0): per tile, once the previous tile's
// accumulators are read out, one barrier wait per window and 16 MMAs
// (operand m: D at kDCol + 128m, A slot kSlots*m + slot).
__device__ __forceinline__ void mma_role(const PipeArgs &a, Shared &sh, uint32_t tmem, uint32_t xs_s,
                                         uint32_t *err, bool &failed) {
    uint32_t gb = 0;
    for (int t = 0;; ++t) {
        const int ts = t % kRing;
        mbar_wait(&sh.ti_full[ts], (t / kRing) & 1, err, failed);
        const TileInfo in = sh.ti[ts];
        mbar_arrive(&sh.ti_empty[ts]);
        if (in.phase == 0) break;
        const int NW = tile_windows(a, in);
        if (t > 0) mbar_wait(&sh.acc_empty, (t - 1) & 1, err, failed);
        for (int win = 0; win < NW; ++win, ++gb) {
            const uint32_t slot = gb % kSlots;
            const int s = gb % kStages;
            mbar_wait(&sh.full[s], (gb / kStages) & 1, err, failed);
            tc_fence_after();
            const uint32_t xb = xs_s + s * kStageBytes;
#pragma unroll
            for (int k16 = 0; k16 < kWin / 16; ++k16)
#pragma unroll
                for (int m = 0; m < 2; ++m)
                    tc_mma(tmem + kDCol + 128 * m, tmem + 64 * (kSlots * m + slot) + 8 * k16,
                           sw128_desc(xb + (k16 >> 2) * kSubBytes + 32 * (k16 & 3)), win > 0 || k16 > 0);
            tc_commit(&sh.slot[slot]);
            tc_commit(&sh.xempty[s]);
        }
        tc_commit(&sh.acc);
    }
}

// A producer lane's view of one tile: its weight row's codes and scales in
// the tiled layout, and its operand's codebook. Warpgroup wg dequantises
// operand wg (gate / up, or down rows 128wg ..); each warp owns 32 rows
// (TMEM lanes 32 (warp & 3) ..), each lane one.
struct ProdTile {
    const uint8_t *cbase;
    const uint16_t *sbase;
    uint32_t cbm;
    int NW;
    bool rows_ok;
};

__device__ __forceinline__ ProdTile prod_tile(const PipeArgs &a, const TileInfo &in, uint32_t cb_s) {
    const int tid = threadIdx.x, lane = tid & 31;
    const bool glu = in.phase == 1;
    const RoutedSet &r = glu ? a.s1 : a.s2;
    const int wg = tid >> 7, warp = (tid >> 5) & 3;
    const int mt = lane >> 4, hh = (lane >> 3) & 1, g = lane & 7;
    const LinearDev &w = (glu && wg == 1) ? r.w1 : r.w0;
    const int C = (r.IN + 255) >> 8, RB = (r.OUT + 31) >> 5;
    const int rb = (in.row0 >> 5) + warp + (glu ? 0 : 4 * wg);
    ProdTile p;
    p.rows_ok = rb < RB;
    p.NW = 2 * C;
    // per chunk c, half: codes at tile*2048 + half*1024 + (2mt+h)*256 + 32g
    // (32 bytes), scales at tile*128 + half*64 + (2mt+h)*16 + 2g (2 fp16)
    const long long tile0 = ((long long)in.e * RB + (p.rows_ok ? rb : 0)) * C;
    p.cbase = w.codes + tile0 * 2048 + (2 * mt + hh) * 256 + 32 * g;
    p.sbase = w.scales + tile0 * 128 + (2 * mt + hh) * 16 + 2 * g;
    p.cbm = cb_s + (glu ? wg * 128 : 0);
    return p;
}

// This row's codes of half chunks (one per window): the current window's and
// the next two.
struct CodeRing {
    uint4 c0[3], c1[3];
    uint32_t sc[3];
};

__device__ __forceinline__ void ring_load(CodeRing &q, const ProdTile &p, int hn, int j) {
    if (p.rows_ok && hn < p.NW) {
        const uint8_t *c = p.cbase + (long long)(hn >> 1) * 2048 + (hn & 1) * 1024;
        q.c0[j] = ldg_stream_v4(c);
        q.c1[j] = ldg_stream_v4(c + 16);
        q.sc[j] = ldg_stream_u32(p.sbase + (long long)(hn >> 1) * 128 + (hn & 1) * 64);
    } else {
        q.c0[j] = q.c1[j] = make_uint4(0, 0, 0, 0);
        q.sc[j] = 0u;
    }
}

__device__ __forceinline__ void ring_start(CodeRing &q, const ProdTile &p) {
    ring_load(q, p, 0, 0);
    ring_load(q, p, 1, 1);
    ring_load(q, p, 2, 2);
}

// Window `win` of the tile: 128 inputs of this lane's row looked up,
// scaled (fp16(codebook x scale)) and stored into the window's A slot
// (columns 64 (kSlots wg + slot) ..); then the ring advances.
__device__ __forceinline__ void produce_window(CodeRing &q, const ProdTile &p, int win, Shared &sh, uint32_t tmem,
                                               uint32_t &gb, uint32_t *err, bool &failed) {
    const int tid = threadIdx.x, lane = tid & 31;
    const int wg = tid >> 7, warp = (tid >> 5) & 3;
    const uint32_t lanebyte = (lane & 15) * 8;
    const uint32_t t_warp = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t slot = gb % kSlots;
    const uint32_t words[8] = {q.c0[0].x, q.c0[0].y, q.c0[0].z, q.c0[0].w,
                               q.c1[0].x, q.c1[0].y, q.c1[0].z, q.c1[0].w};
#pragma unroll
    for (int ww = 0; ww < 2; ++ww) {
        // quad i of 64-input group ww (inputs 64ww + 4i .. + 3): code t =
        // i & 3 of byte b = 4ww + (i >> 2) -- byte i >> 2 of word 2t + ww
        // -- to A columns 32ww + 2i, 32ww + 2i + 1
        const uint32_t s2v = __byte_perm(q.sc[0], 0, ww ? 0x3232 : 0x1010);
        uint32_t av[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int t = i & 3, bq = i >> 2;
            const uint32_t ad = __byte_perm(words[2 * t + ww], lanebyte, 0x5504u | (bq << 4));
            const uint2 e = lds64(p.cbm + ad);
            av[2 * i] = hmul2_u32(e.x, s2v);
            av[2 * i + 1] = hmul2_u32(e.y, s2v);
        }
        if (ww == 0) {
            // the slot's previous window multiplied (its first half computed meanwhile)
            if (gb >= kSlots) warp_wait(&sh.slot[slot], ((gb / kSlots) + 1) & 1, err, failed);
            tc_fence_after();
        }
        tmem_st32(t_warp + 64 * (kSlots * wg + slot) + 32 * ww, av);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh.full[gb % kStages]);
    ++gb;
    q.c0[0] = q.c0[1];
    q.c1[0] = q.c1[1];
    q.sc[0] = q.sc[1];
    q.c0[1] = q.c0[2];
    q.c1[1] = q.c1[2];
    q.sc[1] = q.sc[2];
    ring_load(q, p, win + 3, 2);
}

// Accumulators -> outputs, 32 pairs at a time; warpgroup wg takes pairs
// 64 wg .. 64 wg + 63; output row of pair n: its pair id, or (an
// activation for the next phase) its sorted position base + n. The
// accumulators are released (acc_empty) once every load of them is done.
template <bool GLU>
__device__ __forceinline__ void epilogue(const RoutedSet &r, const TileInfo &in, const int *pairs,
                                         const float *pscale, Shared &sh, uint32_t tmem) {
    constexpr int NMAT = 2;
    const int tid = threadIdx.x, lane = tid & 31;
    const int wg = tid >> 7, warp = (tid >> 5) & 3;
    const int OUT = r.OUT, RB = (OUT + 31) >> 5;
    const uint32_t t_warp = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int q = 2 * wg; q < 2 * wg + 2; ++q) {
        uint32_t dv[NMAT][32];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) tmem_ld32(t_warp + kDCol + 128 * m + 32 * q, dv[m]);
        tmem_wait_ld();
        if (q == 2 * wg + 1) {
            // every accumulator column this warp reads is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.acc_empty);
        }
#pragma unroll
        for (int m = 0; m < (GLU ? 1 : NMAT); ++m) {
            const int rbm = (in.row0 >> 5) + warp + (GLU ? 0 : 4 * m);
            if (rbm < RB) {                   // warp-uniform: OUT is a multiple of 16
                uint32_t ov[16];
#pragma unroll
                for (int jp = 0; jp < 16; ++jp)
                    ov[jp] = pf_value2<GLU>(dv[m][2 * jp], dv[m][2 * jp + 1], dv[1][2 * jp], dv[1][2 * jp + 1],
                                            r.pair_scale != nullptr, pscale[32 * q + 2 * jp],
                                            pscale[32 * q + 2 * jp + 1], r.out_f16, r.act);
                transpose_rows8(ov, lane);
                const int row8 = rbm * 32 + 8 * (lane >> 3);
                const int pb = 16 * (lane & 1) + 8 * ((lane >> 1) & 1) + 4 * ((lane >> 2) & 1);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int n = 32 * q + pb + c, p = pairs[n];
                    uint32_t w4[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int i0 = 2 * k, i1 = 2 * k + 1;
                        const uint32_t va = ov[(i0 & 1) << 3 | ((i0 >> 1) & 1) << 2 | (i0 >> 2) << 1 | (c >> 1)];
                        const uint32_t vb = ov[(i1 & 1) << 3 | ((i1 >> 1) & 1) << 2 | (i1 >> 2) << 1 | (c >> 1)];
                        w4[k] = __byte_perm(va, vb, (c & 1) ? 0x7632 : 0x5410);
                    }
                    if (p >= 0 && row8 < OUT) {
                        const long long orow = r.out_sorted ? (long long)in.base + n : (long long)p;
                        *reinterpret_cast<uint4 *>(r.out + orow * OUT + row8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
            }
        }
    }
}

__device__ __forceinline__ void producers_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kProducers) : "memory"); }

// Tile t's descriptor, read by the whole warp; released by lane 0
__device__ __forceinline__ TileInfo read_tile(Shared &sh, int t, uint32_t *err, bool &failed) {
    const int s = t % kRing;
    warp_wait(&sh.ti_full[s], (t / kRing) & 1, err, failed);
    const TileInfo in = sh.ti[s];
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sh.ti_empty[s]);
    return in;
}

// The routing slots and weights of a tile's pairs (producer threads 0..127)
__device__ __forceinline__ void stage_pairs(const PipeArgs &a, const TileInfo &in, Shared &sh, int buf) {
    const int tid = threadIdx.x;
    if (tid < kN) {
        const RoutedSet &r = in.phase == 1 ? a.s1 : a.s2;
        const int p = tid < in.n ? r.list[in.base + tid] : -1;
        sh.pairs[buf][tid] = p;
        sh.pscale[buf][tid] = (in.phase != 1 && r.pair_scale && p >= 0) ? r.pair_scale[p] : 1.0f;
    }
}

__device__ __forceinline__ void stage_phase_codebooks(const PipeArgs &a, uint8_t *cb, int phase) {
    if (phase == 1) {
        stage_codebook(cb, a.s1.w0, 0, kProducers);
        stage_codebook(cb, a.s1.w1, 1, kProducers);
    } else {
        stage_codebook(cb, a.s2.w0, 0, kProducers);
    }
}

// The producer warps (0-7): tile t's windows; then tile t + 1's
// descriptor, pairs, code ring and first two windows (while the MMA
// finishes tile t); then tile t's epilogue.
__device__ __forceinline__ void producer_role(const PipeArgs &a, Shared &sh, uint8_t *cb, uint32_t tmem,
                                              uint32_t *err, bool &failed) {
    uint32_t gb = 0;
    TileInfo cur = read_tile(sh, 0, err, failed);
    if (cur.phase == 0) return;
    stage_phase_codebooks(a, cb, cur.phase);
    stage_pairs(a, cur, sh, 0);
    producers_sync();
    ProdTile pt = prod_tile(a, cur, smem_u32(cb));
    CodeRing q;
    ring_start(q, pt);
    produce_window(q, pt, 0, sh, tmem, gb, err, failed);
    produce_window(q, pt, 1, sh, tmem, gb, err, failed);
    for (int t = 0;; ++t) {
        for (int win = 2; win < pt.NW; ++win) produce_window(q, pt, win, sh, tmem, gb, err, failed);
        const TileInfo nxt = read_tile(sh, t + 1, err, failed);
        ProdTile pn = pt;
        if (nxt.phase != 0) {
            if (nxt.phase != cur.phase) {
                // a CTA's tiles go phase 1, then phase 2: every lookup of
                // phase 1 done, restage the codebooks once
                producers_sync();
                stage_phase_codebooks(a, cb, nxt.phase);
                producers_sync();
            }
            pn = prod_tile(a, nxt, smem_u32(cb));
            ring_start(q, pn);
            produce_window(q, pn, 0, sh, tmem, gb, err, failed);
            produce_window(q, pn, 1, sh, tmem, gb, err, failed);
            stage_pairs(a, nxt, sh, (t + 1) & 1);
        }
        // ---- tile t's MMAs done: its outputs
        warp_wait(&sh.acc, t & 1, err, failed);
        tc_fence_after();
        if (cur.phase == 1) epilogue<true>(a.s1, cur, sh.pairs[t & 1], sh.pscale[t & 1], sh, tmem);
        else epilogue<false>(a.s2, cur, sh.pairs[t & 1], sh.pscale[t & 1], sh, tmem);
        // every output of tile t stored; tile t + 1's pairs visible
        producers_sync();
        if (cur.phase == 1 && threadIdx.x == 0) {
            __threadfence();
            atomicAdd(a.ctl + 2 + cur.ai, 1u);
        }
        if (nxt.phase == 0) break;
        cur = nxt;
        pt = pn;
    }
}

// --------------------------------------------------------------- kernel
// map1: the phase 1 B rows (the sorted copy of the inputs); map2: phase 2's
// (the sorted SwiGLU activations, or the sorted inputs of a single linear).
__global__ void __launch_bounds__(kThreads, 1)
    expert_prefill_kernel(const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap map2,
                          const PipeArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ Shared sh;
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
    const uint32_t xs_s = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *cb = smem_raw + (xs_s - smem_u32(smem_raw)) + kStages * kStageBytes;
    if (tid == 0) {
        for (int i = 0; i < kSlots; ++i) mbar_init(&sh.slot[i], 1);
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&sh.full[i], kProducers / 32 + 1);   // producer warps + the TMA thread
            mbar_init(&sh.xempty[i], 1);
        }
        mbar_init(&sh.acc, 1);
        mbar_init(&sh.acc_empty, kProducers / 32);
        for (int i = 0; i < kRing; ++i) {
            mbar_init(&sh.ti_full[i], 1);
            mbar_init(&sh.ti_empty[i], kProducers / 32 + 1);   // producer warps + the MMA thread
        }
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
    uint32_t *err = a.err;
    const int nact = min(a.s2.active[a.s2.E], kMaxE);
    const int rt1 = a.has1 ? (a.s1.OUT + 127) / 128 : 0;
    const int rt2 = (a.s2.OUT + 255) / 256;     // phase 2 tiles: 256 rows
    tile_prefix(a, sh, nact, rt1, rt2);
    const int n1 = a.has1 ? sh.pre1[nact] : 0, n2 = sh.pre2[nact];
    bool failed = false;
    if (wid == kTmaWarp) {
        if (lane == 0) tma_role(a, sh, &map1, &map2, xs_s, n1, n2, nact, rt1, rt2, err, failed);
        __syncwarp();
    } else if (wid == kMmaWarp) {
        if (lane == 0) mma_role(a, sh, tmem, xs_s, err, failed);
        __syncwarp();
    } else {
        producer_role(a, sh, cb, tmem, err, failed);
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

// xs[pos][0:IN] = x[row of pair list[pos]][0:IN], 16 bytes per thread
__global__ void permute_rows_kernel(const uint16_t *__restrict__ x, int x_per_pair, int k,
                                    const int32_t *__restrict__ list, int P, int IN, uint16_t *__restrict__ xs) {
    const int v8 = IN / 8;
    const size_t n = (size_t)P * v8;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int pos = (int)(i / v8), v = (int)(i - (size_t)pos * v8);
        const int p = list[pos];
        const size_t row = x_per_pair ? (size_t)p : (size_t)(p / k);
        reinterpret_cast<uint4 *>(xs + (size_t)pos * IN)[v] = reinterpret_cast<const uint4 *>(x + row * IN)[v];
    }
}

}  // namespace pf

vqmoe_status launch_experts_prefill(const PipeArgs &args, void *xs, cudaStream_t stream, cudaEvent_t after_permute) {
    {
        vqmoe_status s = ensure_dynamic_smem(reinterpret_cast<const void *>(pf::expert_prefill_kernel), pf::kSmem,
                                             "prefill expert kernel");
        if (s != VQMOE_OK) return s;
    }
    PipeArgs a = args;
    const RoutedSet &first = a.has1 ? a.s1 : a.s2;
    const int P = first.P, IN = first.IN;
    uint16_t *xs16 = static_cast<uint16_t *>(xs);
    {
        const size_t n = (size_t)P * (IN / 8);
        const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 8);
        pf::permute_rows_kernel<<<grid, 256, 0, stream>>>(first.x, first.x_per_pair, first.k, first.list, P, IN,
                                                          xs16);
        vqmoe_status s = check_launch("permute_rows_kernel");
        if (s != VQMOE_OK) return s;
        if (after_permute && cudaEventRecord(after_permute, stream) != cudaSuccess) return check_launch("event");
    }
    CUtensorMap map1, map2;
    if (!make_tma_map(&map1, xs16, P, IN, pf::kN))
        return set_error(VQMOE_LAUNCH_FAILED, "prefill experts: tensor map of the inputs (P %d, IN %d)", P, IN);
    if (a.has1) {
        // phase 1 writes its activations in sorted order; phase 2 reads them so
        a.s1.out_sorted = 1;
        if (!make_tma_map(&map2, a.s1.out, P, a.s1.OUT, pf::kN))
            return set_error(VQMOE_LAUNCH_FAILED, "prefill experts: tensor map of the activations (P %d, I %d)", P,
                             a.s1.OUT);
    } else {
        map2 = map1;
    }
    pf::expert_prefill_kernel<<<sm_count(), pf::kThreads, pf::kSmem, stream>>>(map1, map2, a);
    return check_launch("expert_prefill_kernel");
}

}  // namespace vqmoe
