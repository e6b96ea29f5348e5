// The tensor-split block's combine and float32 reduction in one kernel,
// over NVLink peer memory.
//
// Reference: under a tensor split every rank runs the whole MoE block on its
// cut and the block output is summed across ranks in float32, then rounded
// once (Reduce, src/knurlogic/engine/split/tensor.py:159-187; the in-model
// all_sum of qwen3_5.py:189-190). Here each rank's kernel
//   A  combines its routed outputs and gated shared expert into its bf16
//      partial (qwen3_5.py:181-187, the same roundings as combine_kernel),
//      written into its part of a buffer every rank can address;
//   B  reduces one column slice of the output: the n ranks' partials of the
//      slice, read over NVLink, summed in float32 in rank order and rounded
//      once to bf16, stored into every rank's result region (two-shot:
//      each partial crosses NVLink once, each result once);
//   C  copies its result region into the caller's output.
// Between the phases the ranks meet at flag barriers: a CTA's writes, a
// system-scope fence, a local counter; the CTA that completes the count
// release-stores the call's epoch into every rank's arrival flag for it,
// and every CTA acquire-spins (bounded) until all n ranks' flags carry the
// epoch. The epoch is each rank's count of finished calls, kept in device
// memory and advanced by the call's last CTA (which also clears the call's
// local counters), so a CUDA graph replays the kernel with the right epoch
// every time; all ranks make the same calls in the same order, so their
// epochs agree. Data other ranks wrote is read with ld.global.cv (fetched
// again, never from a line L1 kept from an earlier call). A wait that runs
// out stores kWaitDependency in the call's status word and the kernel goes
// on (its output is then wrong; nothing hangs).
//
// Each rank's symmetric buffer: kTpFlagBytes of flags and counters, its
// partial [T][H] bf16, its result region [T][H] bf16, then the split
// router's region (tp_gather_kernel: each rank's exact logits of T/n of the
// tokens, or its routing, exchanged the same way before the experts run).
//
// The expert split (ep_reduce_kernel) uses the same flags and barriers over
// another layout: the rank's expert outputs [T*k][H] bf16 (the pairs of the
// experts it owns), then its result region [T][H] bf16.
#include <algorithm>

#include "stages.cuh"

namespace vqmoe {

namespace tp {

// flag words of a rank's buffer
constexpr int kEpoch = 0, kCountA = 1, kCountB = 2, kCountC = 3, kCountG = 4;
constexpr int kArriveA = 8, kArriveB = 8 + kTpMaxRanks, kArriveG = 8 + 2 * kTpMaxRanks;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint4 ld_cv_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.cv.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_cv_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.cv.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t *flags_of(const TpArgs &a, int rank) {
    return reinterpret_cast<uint32_t *>(a.base[rank]);
}

// Thread 0 of every CTA: the CTA's writes so far are done; the last CTA of
// the rank to get here announces the rank to every peer (arrival slot
// `arrive` + rank), then every CTA waits until all ranks have announced.
__device__ void rank_barrier(const TpArgs &a, int count, int arrive, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t *mine = flags_of(a, a.rank);
        __threadfence_system();
        const uint32_t old = atomicAdd(mine + count, 1u);
        if (old == gridDim.x - 1) {
            __threadfence_system();
            for (int q = 0; q < a.n; ++q) st_release_sys(flags_of(a, q) + arrive + a.rank, epoch + 1);
        }
        const long polls = a.wait_polls ? (long)a.wait_polls : (1L << 22);
        for (int q = 0; q < a.n; ++q) {
            unsigned ns = 32;
            for (long i = 1;; ++i) {
                if (ld_acquire_sys(mine + arrive + q) >= epoch + 1) break;
                if (i >= polls) {
                    atomicExch(a.err, kWaitDependency);
                    break;
                }
                __nanosleep(ns);
                if (ns < 1024) ns <<= 1;
            }
        }
    }
    __syncthreads();
}

// The call's last CTA (every CTA has read the epoch and passed the call's
// barriers by then) clears the counters and advances the epoch.
__device__ void finish_call(const TpArgs &a, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t *mine = flags_of(a, a.rank);
        const uint32_t old = atomicAdd(mine + kCountC, 1u);
        if (old == gridDim.x - 1) {
            mine[kCountA] = 0u;
            mine[kCountB] = 0u;
            mine[kCountC] = 0u;
            mine[kCountG] = 0u;
            __threadfence();
            atomicExch(mine + kEpoch, epoch + 1);
        }
    }
}

__global__ void __launch_bounds__(256)
tp_reduce_kernel(const uint16_t *__restrict__ ybuf, int T, int k, int H, const uint16_t *__restrict__ sh,
                 const float *__restrict__ sg, const TpArgs a, uint16_t *__restrict__ out) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t *>(flags_of(a, a.rank) + kEpoch);
    const int vpr = H / 8;
    const size_t nvec = (size_t)T * vpr;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    uint16_t *part = reinterpret_cast<uint16_t *>(a.base[a.rank] + kTpFlagBytes);
    // ---- A: this rank's bf16 partial, as combine_kernel rounds it
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nvec; v += stride) {
        const int tkn = (int)(v / vpr), c8 = (int)(v - (size_t)tkn * vpr);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll 8
        for (int s = 0; s < k; ++s) {
            const uint4 y = __ldg(reinterpret_cast<const uint4 *>(ybuf + ((size_t)tkn * k + s) * H + c8 * 8));
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
            const uint4 sv = *reinterpret_cast<const uint4 *>(sh + (size_t)tkn * H + c8 * 8);
            const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[2 * j] = bf16r(r[2 * j] + bf16r(gate * bf16_to_f32(u[j] & 0xFFFFu)));
                r[2 * j + 1] = bf16r(r[2 * j + 1] + bf16r(gate * bf16_to_f32(u[j] >> 16)));
            }
        }
        uint32_t p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = (uint32_t)f32_to_bf16(r[2 * j]) | ((uint32_t)f32_to_bf16(r[2 * j + 1]) << 16);
        *reinterpret_cast<uint4 *>(part + v * 8) = make_uint4(p[0], p[1], p[2], p[3]);
    }
    rank_barrier(a, kCountA, kArriveA, epoch);
    // ---- B: this rank's column slice, summed over the ranks in rank order
    const size_t part_bytes = (size_t)T * H * 2;
    const int spr = vpr / a.n;                       // vectors of the slice per row
    const size_t nsl = (size_t)T * spr;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nsl; v += stride) {
        const int tkn = (int)(v / spr), c8 = a.rank * spr + (int)(v - (size_t)tkn * spr);
        const size_t off = ((size_t)tkn * vpr + c8) * 16;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        for (int q = 0; q < a.n; ++q) {
            const uint4 pv = ld_cv_v4(a.base[q] + kTpFlagBytes + off);
            const uint32_t u[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] += bf16_to_f32(u[j] & 0xFFFFu);
                acc[2 * j + 1] += bf16_to_f32(u[j] >> 16);
            }
        }
        uint32_t p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = (uint32_t)f32_to_bf16(acc[2 * j]) | ((uint32_t)f32_to_bf16(acc[2 * j + 1]) << 16);
        const uint4 res = make_uint4(p[0], p[1], p[2], p[3]);
        for (int q = 0; q < a.n; ++q)
            *reinterpret_cast<uint4 *>(a.base[q] + kTpFlagBytes + part_bytes + off) = res;
    }
    rank_barrier(a, kCountB, kArriveB, epoch);
    // ---- C: the result into the caller's output
    const uint8_t *red = a.base[a.rank] + kTpFlagBytes + part_bytes;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nvec; v += stride)
        reinterpret_cast<uint4 *>(out)[v] = ld_cv_v4(red + v * 16);
    finish_call(a, epoch);
}

// The expert split's combine and exchange. Every rank holds E / n whole
// experts and wrote, into its own buffer, the outputs y[t, s] of the
// (token, slot) pairs whose expert it owns. After a barrier each rank sums
// one column slice of every token over its k slots in slot order, reading
// each slot from the rank that owns its expert (owner = expert / (E / n)),
// in float32 rounded once, adds the gated shared expert (every rank has
// it), and stores the bf16 result into every rank's result region: the
// unsplit block's combine (qwen3_5.py:181-187) bit for bit. A second barrier,
// then each rank copies its result region into the output.
__global__ void __launch_bounds__(256)
ep_reduce_kernel(const int32_t *__restrict__ inds, int T, int k, int H, int ep_local, const uint16_t *__restrict__ sh,
                 const float *__restrict__ sg, const TpArgs a, uint16_t *__restrict__ out) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t *>(flags_of(a, a.rank) + kEpoch);
    const int vpr = H / 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t ybytes = (size_t)T * k * H * 2;
    rank_barrier(a, kCountA, kArriveA, epoch);          // every rank's expert outputs are in place
    const int spr = vpr / a.n;
    const size_t nsl = (size_t)T * spr;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nsl; v += stride) {
        const int tkn = (int)(v / spr), c8 = a.rank * spr + (int)(v - (size_t)tkn * spr);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        for (int s = 0; s < k; ++s) {
            const int e = inds[(size_t)tkn * k + s];
            const int q = min(e / ep_local, a.n - 1);
            const uint4 y = ld_cv_v4(a.base[q] + kTpFlagBytes + (((size_t)tkn * k + s) * H + c8 * 8) * 2);
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
            const uint4 sv = *reinterpret_cast<const uint4 *>(sh + (size_t)tkn * H + c8 * 8);
            const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[2 * j] = bf16r(r[2 * j] + bf16r(gate * bf16_to_f32(u[j] & 0xFFFFu)));
                r[2 * j + 1] = bf16r(r[2 * j + 1] + bf16r(gate * bf16_to_f32(u[j] >> 16)));
            }
        }
        uint32_t p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) p[j] = (uint32_t)f32_to_bf16(r[2 * j]) | ((uint32_t)f32_to_bf16(r[2 * j + 1]) << 16);
        const uint4 res = make_uint4(p[0], p[1], p[2], p[3]);
        const size_t off = ((size_t)tkn * vpr + c8) * 16;
        for (int q = 0; q < a.n; ++q) *reinterpret_cast<uint4 *>(a.base[q] + kTpFlagBytes + ybytes + off) = res;
    }
    rank_barrier(a, kCountB, kArriveB, epoch);
    const uint8_t *red = a.base[a.rank] + kTpFlagBytes + ybytes;
    for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < (size_t)T * vpr; v += stride)
        reinterpret_cast<uint4 *>(out)[v] = ld_cv_v4(red + v * 16);
    finish_call(a, epoch);
}

// The split router's exchange: this rank computed rows [r0, r1) of up to
// three row-major 32-bit arrays (widths w0..w2; a width 0 or a null array is
// skipped) -- the router's logits, or its expert ids, weights and
// shared-expert gates. Every CTA stores a share of those rows into every
// rank's routing region; the ranks meet at a flag barrier (rank_barrier on
// kCountG / kArriveG, the call's epoch, bounded); then every CTA copies a
// share of all T rows from this rank's region back into the arrays. zero[0
// .. nzero) is cleared on the way (the select kernel's counters). The
// counter is cleared by the call's combine + reduction kernel, which always
// follows.
struct GatherArrays {
    uint32_t *p[3];
    int w[3];
};

__global__ void __launch_bounds__(256)
tp_gather_kernel(GatherArrays g, int T, int r0, int r1, size_t route_off, uint32_t *zero, int nzero,
                 const uint16_t *__restrict__ x, uint16_t *__restrict__ x16, size_t nx8, const TpArgs a) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t *>(flags_of(a, a.rank) + kEpoch);
    const size_t gtid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0u;
    // the VQ experts' fp16 copy of all T tokens (bf16 -> fp16, saturated),
    // while the peers' rows are on their way
    for (size_t v = gtid; v < nx8; v += stride) {
        const uint4 val = reinterpret_cast<const uint4 *>(x)[v];
        uint32_t u[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            u[j] = (uint32_t)bf16_to_f16_sat(u[j] & 0xFFFFu) | ((uint32_t)bf16_to_f16_sat(u[j] >> 16) << 16);
        reinterpret_cast<uint4 *>(x16)[v] = make_uint4(u[0], u[1], u[2], u[3]);
    }
    size_t off = 0;                                     // words of the arrays before m
    for (int m = 0; m < 3; ++m) {
        const int W = g.w[m];
        if (g.p[m] && W) {
            const size_t lo = (size_t)r0 * W, n = (size_t)(r1 - r0) * W;
            for (size_t i = gtid; i < n; i += stride) {
                const uint32_t v = g.p[m][lo + i];
                for (int q = 0; q < a.n; ++q)
                    reinterpret_cast<uint32_t *>(a.base[q] + route_off)[off + lo + i] = v;
            }
        }
        off += (size_t)T * W;
    }
    rank_barrier(a, kCountG, kArriveG, epoch);
    const uint32_t *reg = reinterpret_cast<const uint32_t *>(a.base[a.rank] + route_off);
    off = 0;
    for (int m = 0; m < 3; ++m) {
        const int W = g.w[m];
        if (g.p[m] && W)
            for (size_t i = gtid; i < (size_t)T * W; i += stride) g.p[m][i] = ld_cv_u32(reg + off + i);
        off += (size_t)T * W;
    }
}

}  // namespace tp

size_t tp_route_offset(int T, int H) { return kTpFlagBytes + 2 * (size_t)T * H * sizeof(uint16_t); }

size_t tp_route_bytes(int T) { return (size_t)T * kTpRouteWords * 4; }

vqmoe_status launch_tp_gather(void *const *arrays, const int *widths, int T, int H, int r0, int r1, uint32_t *zero,
                              int nzero, const uint16_t *x, uint16_t *x16, const TpArgs &a, cudaStream_t stream) {
    tp::GatherArrays g{};
    int words = 0;
    for (int m = 0; m < 3; ++m) {
        g.p[m] = static_cast<uint32_t *>(arrays[m]);
        g.w[m] = widths[m];
        words += widths[m];
    }
    if (words > kTpRouteWords) return set_error(VQMOE_BAD_SHAPE, "split router: %d words per token", words);
    // every CTA resident at once (they meet at the barrier): at most one per
    // SM, about eight words per thread
    const size_t nx8 = x16 ? (size_t)T * H / 8 : 0;
    const size_t n = std::max<size_t>((size_t)T * words, nx8);
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((n + 2047) / 2048, (size_t)sm_count()));
    tp::tp_gather_kernel<<<grid, 256, 0, stream>>>(g, T, r0, r1, tp_route_offset(T, H), zero, nzero, x, x16, nx8,
                                                   a);
    return check_launch("tp_gather_kernel");
}

size_t ep_buffer_bytes(int T, int k, int H) { return kTpFlagBytes + ((size_t)T * k + T) * H * sizeof(uint16_t); }

vqmoe_status launch_ep_reduce(const int32_t *inds, int T, int k, int H, int ep_local, const uint16_t *sh,
                              const float *sg, const TpArgs &a, uint16_t *out, cudaStream_t stream) {
    const size_t nvec = (size_t)T * (H / 8);
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((nvec + 255) / 256, (size_t)sm_count()));
    tp::ep_reduce_kernel<<<grid, 256, 0, stream>>>(inds, T, k, H, ep_local, sh, sg, a, out);
    return check_launch("ep_reduce_kernel");
}

vqmoe_status launch_tp_reduce(const uint16_t *ybuf, int T, int k, int H, const uint16_t *sh, const float *sg,
                              const TpArgs &a, uint16_t *out, cudaStream_t stream) {
    // every CTA must be resident at once (they meet at the barriers): one
    // per SM at most, fewer when the work is small
    const size_t nvec = (size_t)T * (H / 8);
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((nvec + 255) / 256, (size_t)sm_count()));
    tp::tp_reduce_kernel<<<grid, 256, 0, stream>>>(ybuf, T, k, H, sh, sg, a, out);
    return check_launch("tp_reduce_kernel");
}

}  // namespace vqmoe
