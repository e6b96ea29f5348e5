// The decoder stack's norms around the MoE block (qwen3_5.py:120-130,
// 549-587): the residual add of a DecoderLayer and the RMSNorm that follows
// it, in one pass over the row.
//
// Reference: RMSNorm.__call__ (qwen3_5.py:120-130) normalises in float32
// with the (1 + weight) gain kept in float32 and rounds once, and
// DecoderLayer.__call__ (qwen3_5.py:578-587) adds the attention and MoE
// outputs to the bf16 residual stream (h = x + r, a bf16 add). Here
//   sum  = bf16(x + r)                        (when r is given)
//   norm = bf16(f32(f32(sum) * rs) * w)       rs = 1 / sqrt(ms + eps)
// with ms the mean of the squares: each square of a bf16 value is exact in
// fp64, the sum is accumulated in fp64 and the mean rounded once to float32
// (MLX's fused kernel accumulates in float32: that order is unpinned). The
// same kernel serves the attention's per-head q/k norms (rows = tokens x
// heads, hidden = head_dim). One warp per row up to 1024 columns, a CTA of
// 256 threads per row above.
#include "stages.cuh"

namespace vqmoe {

template <int WARPS_PER_ROW>
__global__ void __launch_bounds__(256)
add_rms_norm_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ r, const float *__restrict__ w,
                    int rows, int H, float eps, uint16_t *__restrict__ sum_out, uint16_t *__restrict__ norm_out) {
    constexpr int kRowsPerCta = 8 / WARPS_PER_ROW;
    __shared__ double s_part[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x * kRowsPerCta + warp / WARPS_PER_ROW;
    const int sub = warp % WARPS_PER_ROW;            // this warp's part of the row
    const int nthr = 32 * WARPS_PER_ROW, t = sub * 32 + lane;
    const bool live = row < rows;
    const size_t base = (size_t)(live ? row : 0) * H;
    double acc = 0.0;
    for (int i = t; i < H && live; i += nthr) {
        float v = bf16_to_f32(x[base + i]);
        if (r) v = bf16r(v + bf16_to_f32(r[base + i]));
        acc += (double)v * (double)v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (WARPS_PER_ROW > 1) {
        if (lane == 0) s_part[warp] = acc;
        __syncthreads();
        acc = 0.0;
        for (int q = 0; q < WARPS_PER_ROW; ++q) acc += s_part[(warp / WARPS_PER_ROW) * WARPS_PER_ROW + q];
    }
    if (!live) return;
    const float ms = (float)(acc / (double)H);
    const float rs = 1.0f / sqrtf(ms + eps);
    for (int i = t; i < H; i += nthr) {
        float v = bf16_to_f32(x[base + i]);
        if (r) {
            v = bf16r(v + bf16_to_f32(r[base + i]));
            if (sum_out) sum_out[base + i] = f32_to_bf16(v);
        }
        norm_out[base + i] = f32_to_bf16((v * rs) * w[i]);
    }
}

vqmoe_status launch_add_rms_norm(const uint16_t *x, const uint16_t *r, const float *w, int rows, int H, float eps,
                                 uint16_t *sum_out, uint16_t *norm_out, cudaStream_t stream) {
    if (H <= 1024) {
        add_rms_norm_kernel<1><<<(rows + 7) / 8, 256, 0, stream>>>(x, r, w, rows, H, eps, sum_out, norm_out);
    } else {
        add_rms_norm_kernel<8><<<rows, 256, 0, stream>>>(x, r, w, rows, H, eps, sum_out, norm_out);
    }
    return check_launch("add_rms_norm_kernel");
}

}  // namespace vqmoe

extern "C" vqmoe_status vqmoe_add_rms_norm(const void *x, const void *residual, const float *weight, int32_t rows,
                                           int32_t hidden, float eps, void *sum_out, void *norm_out, void *stream) {
    using namespace vqmoe;
    if (rows <= 0 || hidden <= 0) return set_error(VQMOE_BAD_SHAPE, "add_rms_norm: rows %d hidden %d", rows, hidden);
    if (!x || !weight || !norm_out) return set_error(VQMOE_BAD_POINTER, "add_rms_norm: x / weight / norm_out null");
    if (!(eps >= 0.0f)) return set_error(VQMOE_BAD_SHAPE, "add_rms_norm: eps %g", (double)eps);
    return launch_add_rms_norm(static_cast<const uint16_t *>(x), static_cast<const uint16_t *>(residual), weight,
                               rows, hidden, eps, static_cast<uint16_t *>(sum_out), static_cast<uint16_t *>(norm_out),
                               static_cast<cudaStream_t>(stream));
}
