// The shared expert's matmuls for many tokens (qwen3_5.py:184-185) on the
// 5th-generation tensor cores: out[T, OUT] = epilogue(x[T, IN] . W^T) with
// bf16 W [OUT, IN] -- two matrices (gate, up) with the fused SwiGLU, or one
// (down).
//
// One persistent CTA of six warps per SM, tiles of 128 weight rows x 128
// tokens taken round robin:
//   warp 0  TMA: per 64-input window, one 2-D tensor copy per operand (128
//           rows x 128 bytes, 128-byte swizzle) into a ring of stages, each
//           with a transaction-count mbarrier;
//   warp 1  MMA: tcgen05.mma kind::f16 (bf16 operands from shared memory,
//           K-major SW128 descriptors) into one of two TMEM accumulators,
//           commits each stage back to the TMA warp and each finished
//           accumulator to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32-lane quarter, SwiGLU or the
//           bf16 rounding, stores; then release the accumulator, so that
//           the epilogue of a tile overlaps the next tile's MMAs.
// Out-of-range rows and tokens of a partial tile are zero-filled by the TMA
// unit and never stored.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "stages.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace vqmoe {
namespace dn {
using namespace tc;

constexpr int kRows = 128;                    // weight rows per tile (MMA M)
constexpr int kTok = 128;                     // tokens per tile (MMA N)
constexpr int kWin = 64;                      // inputs per stage: one 128-byte swizzle row
constexpr int kTileBytes = 128 * 128;         // 128 rows x 128 bytes
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps);
// kind::f16, D f32, A bf16, B bf16, both K-major, N = 128, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTok >> 3) << 17) |
                            ((uint32_t)(kRows >> 4) << 24);

template <int NMAT>
struct Cfg {
    static constexpr int kStageBytes = (NMAT + 1) * kTileBytes;   // A of each matrix, then B
    static constexpr int kStages = NMAT == 2 ? 4 : 6;
    static constexpr int kAccCols = NMAT * kTok;                  // one accumulator buffer
    static constexpr int kAllocCols = NMAT == 2 ? 512 : 256;      // two buffers
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024;   // + 1024-byte alignment
};

struct Args {
    uint16_t *out;               // [T][OUT] bf16
    int T, IN, OUT;
    uint32_t *err;
};

__device__ __forceinline__ void mma_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}
template <int NMAT>
__global__ void __launch_bounds__(kThreads, 1)
    dense_tma_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw0,
                     const __grid_constant__ CUtensorMap tw1, const Args a) {
    using C = Cfg<NMAT>;
    constexpr bool GLU = NMAT == 2;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[C::kStages], empty[C::kStages], acc_full[2], acc_empty[2];
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    if (tid == 0) {
        for (int i = 0; i < C::kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(&s_tmem)),
                     "r"(C::kAllocCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int rt = (a.OUT + kRows - 1) / kRows, nbk = (a.T + kTok - 1) / kTok;
    const int tiles = rt * nbk, NW = a.IN / kWin;
    bool failed = false;
    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int row0 = (tile % rt) * kRows, t0 = (tile / rt) * kTok;
                for (int win = 0; win < NW; ++win, ++it) {
                    const int s = it % C::kStages;
                    if (it >= (uint32_t)C::kStages)
                        mbar_wait(&empty[s], ((it / C::kStages) + 1) & 1, a.err, failed);
                    const uint32_t st = sbase + s * C::kStageBytes;
                    arrive_expect_tx(&full[s], C::kStageBytes);
                    tma_load_2d(st, &tw0, win * kWin, row0, &full[s]);
                    if (GLU) tma_load_2d(st + kTileBytes, &tw1, win * kWin, row0, &full[s]);
                    tma_load_2d(st + NMAT * kTileBytes, &tx, win * kWin, t0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            uint32_t it = 0, tl = 0;
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tl) {
                const uint32_t b = tl & 1;
                if (tl >= 2) mbar_wait(&acc_empty[b], ((tl >> 1) + 1) & 1, a.err, failed);
                tc_fence_after();
                const uint32_t d = tmem + b * C::kAccCols;
                for (int win = 0; win < NW; ++win, ++it) {
                    const int s = it % C::kStages;
                    mbar_wait(&full[s], (it / C::kStages) & 1, a.err, failed);
                    tc_fence_after();
                    const uint32_t st = sbase + s * C::kStageBytes;
#pragma unroll
                    for (int k16 = 0; k16 < kWin / 16; ++k16)
#pragma unroll
                        for (int m = 0; m < NMAT; ++m)
                            mma_ss(d + m * kTok, sw128_desc(st + m * kTileBytes + 32 * k16),
                                   sw128_desc(st + NMAT * kTileBytes + 32 * k16), win > 0 || k16 > 0);
                    tc_commit(&empty[s]);
                }
                tc_commit(&acc_full[b]);
            }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31
        const int q = warp & 3;
        uint32_t tl = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++tl) {
            const int row0 = (tile % rt) * kRows, t0 = (tile / rt) * kTok;
            const uint32_t b = tl & 1;
            warp_wait(&acc_full[b], (tl >> 1) & 1, a.err, failed);
            tc_fence_after();
            const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + b * C::kAccCols;
            const int row = row0 + 32 * q + lane;
#pragma unroll 1
            for (int c = 0; c < kTok / 32; ++c) {
                uint32_t dv[NMAT][32];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) tmem_ld32(tq + m * kTok + 32 * c, dv[m]);
                tmem_wait_ld();
                if (row < a.OUT) {
                    uint32_t ov[16];
#pragma unroll
                    for (int jp = 0; jp < 16; ++jp) {
                        const float g0 = __uint_as_float(dv[0][2 * jp]), g1 = __uint_as_float(dv[0][2 * jp + 1]);
                        const uint32_t gb = cvt_bf16x2(g0, g1);
                        if (GLU) {
                            // _SwiGLU: bf16(bf16(silu(g)) * u), g and u bf16
                            const uint32_t ub = cvt_bf16x2(__uint_as_float(dv[NMAT - 1][2 * jp]),
                                                           __uint_as_float(dv[NMAT - 1][2 * jp + 1]));
                            const uint32_t sb = cvt_bf16x2(silu_fast(bf_lo(gb)), silu_fast(bf_hi(gb)));
                            ov[jp] = cvt_bf16x2(bf_lo(sb) * bf_lo(ub), bf_hi(sb) * bf_hi(ub));
                        } else {
                            ov[jp] = gb;
                        }
                    }
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        const int t = t0 + 32 * c + jj;
                        if (t < a.T) a.out[(size_t)t * a.OUT + row] = (uint16_t)(ov[jj >> 1] >> (16 * (jj & 1)));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(C::kAllocCols)
                     : "memory");
    }
}

// ---------------------------------------------------------------- host
template <int NMAT>
vqmoe_status launch(const void *x, const void *w0, const void *w1, int T, int IN, int OUT, void *out,
                    uint32_t *err, cudaStream_t stream) {
    using C = Cfg<NMAT>;
    static std::once_flag once[64];
    static bool ok[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(VQMOE_LAUNCH_FAILED, "dense prefill: device %d", dev);
    std::call_once(once[dev], [&] {
        ok[dev] = cudaFuncSetAttribute(dense_tma_kernel<NMAT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)C::kSmem) == cudaSuccess;
    });
    if (!ok[dev]) return set_error(VQMOE_LAUNCH_FAILED, "dense prefill kernel: %zu bytes of shared memory", C::kSmem);
    CUtensorMap tx, tw0, tw1;
    if (!make_tma_map(&tx, x, T, IN, kTok) || !make_tma_map(&tw0, w0, OUT, IN, kRows) ||
        !make_tma_map(&tw1, NMAT == 2 ? w1 : w0, OUT, IN, kRows))
        return set_error(VQMOE_LAUNCH_FAILED, "dense prefill: tensor map encoding failed (T %d, IN %d, OUT %d)", T,
                         IN, OUT);
    Args a{static_cast<uint16_t *>(out), T, IN, OUT, err};
    const int tiles = ((OUT + kRows - 1) / kRows) * ((T + kTok - 1) / kTok);
    dense_tma_kernel<NMAT><<<std::min(tiles, sm_count()), kThreads, C::kSmem, stream>>>(tx, tw0, tw1, a);
    return check_launch("dense_tma_kernel");
}

}  // namespace dn

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

bool make_tma_map(CUtensorMap *m, const void *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn || rows <= 0 || cols <= 0 || (cols * 2) % 16 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The shared expert's dense matmul (+ SwiGLU when w1 is set) for many tokens
// on tcgen05 with TMA; IN a multiple of 64, every pointer 16-byte aligned.
vqmoe_status launch_dense_prefill(const void *x, const void *w0, const void *w1, int T, int IN, int OUT,
                                  void *out, uint32_t *err, cudaStream_t stream) {
    if (IN % dn::kWin != 0 || T <= 0 || OUT <= 0)
        return set_error(VQMOE_BAD_SHAPE, "dense prefill: IN %d must be a multiple of %d", IN, dn::kWin);
    return w1 ? dn::launch<2>(x, w0, w1, T, IN, OUT, out, err, stream)
              : dn::launch<1>(x, w0, nullptr, T, IN, OUT, out, err, stream);
}

}  // namespace vqmoe
