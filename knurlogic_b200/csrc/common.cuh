// Shared device helpers of libvqmoe: exact rounding, packed loads, the
// mma.sync wrappers the decode kernels use, and host-side error plumbing.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vqmoe.h"

namespace vqmoe {

// Programmatic dependent launch. A kernel launched with launch_pdl may start
// while its predecessor on the stream still runs; it does its
// input-independent prologue, then pdl_wait() returns once the predecessor
// has finished and its writes are visible (a no-op without PDL).
// pdl_trigger() lets this kernel's own dependent launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------- rounding

// float -> bf16 bits, round to nearest even (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16_to_f32(uint32_t b) {
    return __uint_as_float(b << 16);
}

__device__ __forceinline__ float bf16r(float f) {
    return bf16_to_f32(f32_to_bf16(f));
}

// double -> bf16 bits in one rounding (nearest even on the float64
// significand, no float32 step). Values below float32's normal range take
// the float32 route (bf16 rounds at a coarser position there).
__device__ __forceinline__ uint16_t f64_to_bf16(double d) {
    double a = fabs(d);
    if (!(a >= 1.1754943508222875e-38) || !(a <= 3.3895313892515355e38))
        return f32_to_bf16((float)d);
    unsigned long long u = (unsigned long long)__double_as_longlong(d);
    const unsigned long long mask = (1ull << 45) - 1ull;
    unsigned long long low = u & mask;
    unsigned long long odd = (u >> 45) & 1ull;
    unsigned long long r = u & ~mask;
    if (low > (1ull << 44) || (low == (1ull << 44) && odd)) r += (1ull << 45);
    return f32_to_bf16((float)__longlong_as_double((long long)r));
}

// bf16 value -> fp16 bits for the VQ matmul: saturate to +-65504, then
// round to nearest even (exact for |v| in [2^-14, 65504]).
__device__ __forceinline__ uint16_t bf16_to_f16_sat(uint32_t b) {
    float v = bf16_to_f32(b);
    v = fminf(fmaxf(v, -65504.0f), 65504.0f);
    return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float silu_f32(float g) {
    return g / (1.0f + expf(-g));
}

// gelu's tanh form (mlx's gelu_approx, torch's gelu_pytorch_tanh):
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), in fp32
__device__ __forceinline__ float gelu_tanh_f32(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float sigmoid_f32(float g) {
    return 1.0f / (1.0f + expf(-g));
}

// -------------------------------------------------------------- loads
// Global loads through the CUDA intrinsics: the compiler schedules them
// freely but never speculates them past the branch that guards their
// pointer (an asm statement without side effects could be hoisted out of
// its branch and dereference an unset pointer).
__device__ __forceinline__ uint4 ldg_stream_v4(const void *p) {
    return __ldcs(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ uint32_t ldg_stream_u32(const void *p) {
    return __ldcs(reinterpret_cast<const unsigned int *>(p));
}

__device__ __forceinline__ uint2 ldg_nc_v2(const void *p) {
    return __ldg(reinterpret_cast<const uint2 *>(p));
}

__device__ __forceinline__ uint2 ldg_stream_v2(const void *p) {
    return __ldcs(reinterpret_cast<const uint2 *>(p));
}

// 16-byte async copy global -> shared; src_bytes < 16 zero-fills the rest
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}

__device__ __forceinline__ uint16_t ldg_nc_u16(const void *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
}

__device__ __forceinline__ uint2 lds_v2(uint32_t saddr) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(r.x), "=r"(r.y)
                 : "r"(saddr));
    return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// half2 multiply (IEEE, round to nearest even per lane)
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// ---------------------------------------------------------------- mma

// D += A(16x16, row) * B(16x8, col); fp32 accumulate. Not volatile: a pure
// function of its registers, so the compiler may interleave it with loads.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1,
                                        uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B + C with separate C (e.g. a zero quad that starts a sum).
__device__ __forceinline__ void mma_f16_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------ host side

vqmoe_status set_error(vqmoe_status s, const char *fmt, ...);
vqmoe_status check_launch(const char *what);
int sm_count();
// Raises kernel `fn`'s dynamic shared-memory limit on the current device to
// at least `bytes`, once per (kernel, device); safe from several host threads.
vqmoe_status ensure_dynamic_smem(const void *fn, size_t bytes, const char *what);

// Status words at the head of every caller workspace (and of the fixed
// scratch): [0] the routed-expert kernels' bounded waits, [1] the shared
// expert's (side stream). Zeroed at the start of each call; a kernel whose
// wait runs out stores its kind (kWaitDependency, kWaitPipeline) there.
constexpr size_t kStatusBytes = 256;
constexpr uint32_t kWaitDependency = 1;   // a phase 2 tile's wait for its expert's phase 1 tiles
constexpr uint32_t kWaitPipeline = 2;     // an mbarrier wait inside a tcgen05 pipeline
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// a VQ weight format (codebook + codes + scales), either layout
inline bool is_vq(int format) { return format == VQMOE_FMT_VQ_U8 || format == VQMOE_FMT_VQ_REF; }
// a format the general (dequantise-into-shared-memory) expert kernel serves
inline bool is_general(int format) { return format == VQMOE_FMT_VQ_REF || format == VQMOE_FMT_AFFINE; }
inline bool aligned16(const void *p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace vqmoe
