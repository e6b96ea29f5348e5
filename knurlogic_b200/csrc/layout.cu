// Loading VQ weights into the device layout (layout.cuh), the inverse, the
// code range check, and the dense fp16 dequantisation of whole experts.
#include <algorithm>

#include "layout.cuh"
#include "stages.cuh"

namespace vqmoe {

// one thread per device byte (codes) or element (scales)
__global__ void prepare_vq_kernel(const uint8_t *__restrict__ codes, const uint16_t *__restrict__ scales,
                                  VqGeom G, uint8_t *__restrict__ dcodes,
                                  uint16_t *__restrict__ dscales) {
    const long long ncode = G.code_bytes(), nscale = G.scale_elems();
    const int NC = G.IN >> 2, NG = G.IN >> 6;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ncode + nscale;
         i += (long long)gridDim.x * blockDim.x) {
        if (i < ncode) {
            const long long tile = i >> 11;
            const int o = (int)(i & 2047);
            const int half = o >> 10, mh = (o >> 8) & 3, lane = (o >> 3) & 31, b = o & 7;
            const int c = (int)(tile % G.chunks());
            const long long er = tile / G.chunks();
            const int rbi = (int)(er % G.rb()), e = (int)(er / G.rb());
            const int row = rbi * 32 + (mh >> 1) * 16 + (mh & 1) * 8 + (lane >> 2);
            const int u = c * 64 + 4 * (half * 8 + b) + (lane & 3);
            dcodes[i] = (row < G.OUT && u < NC) ? codes[((long long)e * G.OUT + row) * NC + u] : 0;
        } else {
            const long long j = i - ncode;
            const long long tile = j >> 7;
            const int o = (int)(j & 127);
            const int half = o >> 6, mh = (o >> 4) & 3, g = (o >> 1) & 7, jj = o & 1;
            const int c = (int)(tile % G.chunks());
            const long long er = tile / G.chunks();
            const int rbi = (int)(er % G.rb()), e = (int)(er / G.rb());
            const int row = rbi * 32 + (mh >> 1) * 16 + (mh & 1) * 8 + g;
            const int grp = c * 4 + half * 2 + jj;
            dscales[j] = (row < G.OUT && grp < NG) ? scales[((long long)e * G.OUT + row) * NG + grp] : 0;
        }
    }
}

__global__ void unprepare_codes_kernel(const uint8_t *__restrict__ dcodes, VqGeom G,
                                       uint8_t *__restrict__ codes) {
    const int NC = G.IN >> 2;
    const long long n = (long long)G.E * G.OUT * NC;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int u = (int)(i % NC);
        const long long er = i / NC;
        const int row = (int)(er % G.OUT), e = (int)(er / G.OUT);
        const int c = u >> 6, uc = u & 63, q = uc >> 2, t = uc & 3;
        const int half = q >> 3, b = q & 7;
        const int rbi = row >> 5, rr = row & 31;
        const int mh = (rr >> 4) * 2 + ((rr >> 3) & 1), g = rr & 7;
        codes[i] = dcodes[G.tile(e, rbi, c) * 2048 + half * 1024 + mh * 256 + (4 * g + t) * 8 + b];
    }
}

// *bad_count += number of codes >= K (the caller zeroes it first)
__global__ void count_bad_codes_kernel(const uint8_t *__restrict__ codes, long long n, int K,
                                       uint32_t *__restrict__ bad_count) {
    uint32_t bad = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        bad += codes[i] >= K;
    for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(bad_count, bad);
}

// W[e][row][i] = fp16(codebook[code][i % 4] * scale) for experts
// [first, first + count), 4 weights per thread
__global__ void dequant_kernel(const uint8_t *__restrict__ dcodes, const uint16_t *__restrict__ cb,
                               const uint16_t *__restrict__ dscales, VqGeom G, int first, int count,
                               uint16_t *__restrict__ out) {
    const int NC = G.IN >> 2;
    const long long n = (long long)count * G.OUT * NC;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int u = (int)(i % NC);
        const long long er = i / NC;
        const int row = (int)(er % G.OUT), e = first + (int)(er / G.OUT);
        const int c = u >> 6, uc = u & 63, q = uc >> 2, t = uc & 3;
        const int half = q >> 3, b = q & 7;
        const int rbi = row >> 5, rr = row & 31;
        const int mh = (rr >> 4) * 2 + ((rr >> 3) & 1), g = rr & 7;
        const long long tile = G.tile(e, rbi, c);
        const uint32_t code = dcodes[tile * 2048 + half * 1024 + mh * 256 + (4 * g + t) * 8 + b];
        const uint16_t s = dscales[tile * 128 + half * 64 + mh * 16 + 2 * g + ((q >> 2) & 1)];
        const uint32_t s2 = (uint32_t)s | ((uint32_t)s << 16);
        const uint2 ev = *reinterpret_cast<const uint2 *>(cb + code * 4);
        *reinterpret_cast<uint2 *>(out + er * G.IN + (long long)u * 4) =
            make_uint2(hmul2_u32(ev.x, s2), hmul2_u32(ev.y, s2));
    }
}

// The same over uint16 codes
__global__ void count_bad_codes_u16_kernel(const uint16_t *__restrict__ codes, long long n, int K,
                                           uint32_t *__restrict__ bad_count) {
    uint32_t bad = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        bad += codes[i] >= K;
    for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(bad_count, bad);
}

// Reference-layout VQ (codes [E][OUT][IN/dim], 1 or 2 bytes per code;
// scales [E][OUT][IN/group]): W = fp16(codebook[code][j] * scale) for
// experts [first, first + count), one code (dim weights) per thread.
__global__ void dequant_ref_kernel(const uint8_t *__restrict__ codes, int cbytes, const uint16_t *__restrict__ cb,
                                   const uint16_t *__restrict__ scales, int OUT, int IN, int dim, int group,
                                   int first, int count, uint16_t *__restrict__ out) {
    const int NC = IN / dim, NG = IN / group;
    const long long n = (long long)count * OUT * NC;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int u = (int)(i % NC);
        const long long er = i / NC;
        const long long src = (long long)first * OUT * NC + i;
        const uint32_t code = cbytes == 1 ? (uint32_t)codes[src] : (uint32_t)reinterpret_cast<const uint16_t *>(codes)[src];
        const uint32_t s = scales[((long long)first * OUT + er) * NG + (u * dim) / group];
        const uint32_t s2 = s | (s << 16);
        const uint32_t *e = reinterpret_cast<const uint32_t *>(cb + (size_t)code * dim);
        uint32_t *o = reinterpret_cast<uint32_t *>(out + er * IN + (long long)u * dim);
        for (int j = 0; j < dim / 2; ++j) o[j] = hmul2_u32(e[j], s2);
    }
}

// AFFINE (weight [E][OUT][IN*bits/32] uint32, each row a little-endian bit
// stream of `bits`-bit values; scales / biases [E][OUT][IN/group] bf16):
// W = bf16(fmaf(scale, q, bias)) for experts [first, first + count), one
// weight per thread
__global__ void dequant_affine_kernel(const uint32_t *__restrict__ wq, const uint16_t *__restrict__ scales,
                                      const uint16_t *__restrict__ biases, int OUT, int IN, int bits, int group,
                                      int first, int count, uint16_t *__restrict__ out) {
    const int words_row = IN * bits / 32, NG = IN / group;
    const long long n = (long long)count * OUT * IN;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int u = (int)(i % IN);
        const long long er = i / IN;
        const long long row = (long long)first * OUT + er;
        const long long bit = (long long)u * bits;
        const uint32_t *wr = wq + row * words_row;
        unsigned long long win = wr[bit >> 5];
        if ((int)(bit & 31) + bits > 32) win |= (unsigned long long)wr[(bit >> 5) + 1] << 32;
        const uint32_t q = (uint32_t)(win >> (bit & 31)) & ((1u << bits) - 1u);
        const float s = bf16_to_f32(scales[row * NG + u / group]), b = bf16_to_f32(biases[row * NG + u / group]);
        out[i] = f32_to_bf16(__fmaf_rn(s, (float)q, b));
    }
}

static int grid_for(long long n) {
    return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sm_count() * 16));
}

static vqmoe_status check_geom(int E, int OUT, int IN) {
    if (E <= 0 || OUT <= 0 || IN <= 0 || IN % 64 || OUT % 16)
        return set_error(VQMOE_BAD_SHAPE, "VQ geometry E %d OUT %d IN %d (IN %% 64, OUT %% 16)", E, OUT, IN);
    return VQMOE_OK;
}

}  // namespace vqmoe

using namespace vqmoe;

extern "C" {

vqmoe_status vqmoe_vq_layout_bytes(int32_t num_experts, int32_t out_features, int32_t in_features,
                                   int64_t *code_bytes, int64_t *scale_bytes) {
    vqmoe_status s = check_geom(num_experts, out_features, in_features);
    if (s != VQMOE_OK) return s;
    if (!code_bytes || !scale_bytes) return set_error(VQMOE_BAD_POINTER, "layout_bytes: outputs");
    VqGeom G{num_experts, out_features, in_features};
    *code_bytes = G.code_bytes();
    *scale_bytes = G.scale_elems() * 2;
    return VQMOE_OK;
}

vqmoe_status vqmoe_prepare_vq(const uint8_t *codes, const void *scales, int32_t num_experts,
                              int32_t out_features, int32_t in_features, uint8_t *codes_dev,
                              void *scales_dev, void *stream) {
    vqmoe_status s = check_geom(num_experts, out_features, in_features);
    if (s != VQMOE_OK) return s;
    if (!codes || !scales || !aligned16(codes_dev) || !aligned16(scales_dev))
        return set_error(VQMOE_BAD_POINTER, "prepare_vq: pointers (device outputs 16-byte aligned)");
    VqGeom G{num_experts, out_features, in_features};
    const long long n = G.code_bytes() + G.scale_elems();
    prepare_vq_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        codes, static_cast<const uint16_t *>(scales), G, codes_dev, static_cast<uint16_t *>(scales_dev));
    return check_launch("prepare_vq_kernel");
}

vqmoe_status vqmoe_unprepare_codes(const uint8_t *codes_dev, int32_t num_experts, int32_t out_features,
                                   int32_t in_features, uint8_t *codes, void *stream) {
    vqmoe_status s = check_geom(num_experts, out_features, in_features);
    if (s != VQMOE_OK) return s;
    if (!codes_dev || !codes) return set_error(VQMOE_BAD_POINTER, "unprepare_codes: pointers");
    VqGeom G{num_experts, out_features, in_features};
    const long long n = (long long)num_experts * out_features * (in_features / 4);
    unprepare_codes_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(codes_dev, G, codes);
    return check_launch("unprepare_codes_kernel");
}

vqmoe_status vqmoe_count_bad_codes(const uint8_t *codes, int64_t count, int32_t codebook_size,
                                   uint32_t *bad_count, void *stream) {
    if (!codes || !bad_count || count <= 0)
        return set_error(VQMOE_BAD_POINTER, "count_bad_codes: pointers / count");
    if (codebook_size <= 0 || codebook_size > 256)
        return set_error(VQMOE_BAD_FORMAT, "codebook_size %d (1..256)", codebook_size);
    count_bad_codes_kernel<<<grid_for(count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        codes, count, codebook_size, bad_count);
    return check_launch("count_bad_codes_kernel");
}

vqmoe_status vqmoe_count_bad_codes_u16(const uint16_t *codes, int64_t count, int32_t codebook_size,
                                       uint32_t *bad_count, void *stream) {
    if (!codes || !bad_count || count <= 0)
        return set_error(VQMOE_BAD_POINTER, "count_bad_codes_u16: pointers / count");
    if (codebook_size <= 0 || codebook_size > 65536)
        return set_error(VQMOE_BAD_FORMAT, "codebook_size %d (1..65536)", codebook_size);
    count_bad_codes_u16_kernel<<<grid_for(count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        codes, count, codebook_size, bad_count);
    return check_launch("count_bad_codes_u16_kernel");
}

vqmoe_status vqmoe_dequant(const vqmoe_linear *w, int32_t first, int32_t count, void *out,
                           void *stream) {
    if (w && w->format == VQMOE_FMT_AFFINE) {
        const int b = w->bits;
        if (w->num_experts <= 0 || w->out_features <= 0 || w->in_features <= 0 ||
            (b != 2 && b != 3 && b != 4 && b != 5 && b != 6 && b != 8) || w->group_size <= 0 ||
            w->in_features % w->group_size || (w->in_features * b) % 32)
            return set_error(VQMOE_BAD_FORMAT, "dequant: affine geometry");
        if (first < 0 || count <= 0 || first + count > w->num_experts)
            return set_error(VQMOE_BAD_SHAPE, "dequant: experts [%d, %d) of %d", first, first + count,
                             w->num_experts);
        if (!w->weight || !w->scales || !w->biases || !out) return set_error(VQMOE_BAD_POINTER, "dequant: pointers");
        const long long n = (long long)count * w->out_features * w->in_features;
        dequant_affine_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint32_t *>(w->weight), static_cast<const uint16_t *>(w->scales),
            static_cast<const uint16_t *>(w->biases), w->out_features, w->in_features, b, w->group_size, first,
            count, static_cast<uint16_t *>(out));
        return check_launch("dequant_affine_kernel");
    }
    if (w && w->format == VQMOE_FMT_VQ_REF) {
        if (w->num_experts <= 0 || w->out_features <= 0 || w->in_features <= 0 ||
            (w->dim != 2 && w->dim != 4 && w->dim != 8) || w->group_size <= 0 || w->group_size % w->dim ||
            w->in_features % w->group_size || w->codebook_size <= 0 || w->codebook_size > 65536)
            return set_error(VQMOE_BAD_FORMAT, "dequant: reference-layout VQ geometry");
        if (first < 0 || count <= 0 || first + count > w->num_experts)
            return set_error(VQMOE_BAD_SHAPE, "dequant: experts [%d, %d) of %d", first, first + count,
                             w->num_experts);
        if (!w->codes || !w->codebook || !w->scales || !aligned16(out) || !aligned16(w->codebook))
            return set_error(VQMOE_BAD_POINTER, "dequant: pointers");
        const long long n = (long long)count * w->out_features * (w->in_features / w->dim);
        dequant_ref_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t *>(w->codes), w->codebook_size <= 256 ? 1 : 2,
            static_cast<const uint16_t *>(w->codebook), static_cast<const uint16_t *>(w->scales), w->out_features,
            w->in_features, w->dim, w->group_size, first, count, static_cast<uint16_t *>(out));
        return check_launch("dequant_ref_kernel");
    }
    if (!w || w->format != VQMOE_FMT_VQ_U8) return set_error(VQMOE_BAD_FORMAT, "dequant: not a VQ linear");
    vqmoe_status s = check_geom(w->num_experts, w->out_features, w->in_features);
    if (s != VQMOE_OK) return s;
    if (w->dim != 4 || w->group_size != 64)
        return set_error(VQMOE_BAD_FORMAT, "dequant: dim %d group %d (4, 64)", w->dim, w->group_size);
    if (first < 0 || count <= 0 || first + count > w->num_experts)
        return set_error(VQMOE_BAD_SHAPE, "dequant: experts [%d, %d) of %d", first, first + count,
                         w->num_experts);
    if (!w->codes || !w->codebook || !w->scales || !aligned16(out))
        return set_error(VQMOE_BAD_POINTER, "dequant: pointers");
    VqGeom G{w->num_experts, w->out_features, w->in_features};
    const long long n = (long long)count * w->out_features * (w->in_features / 4);
    dequant_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(w->codes), static_cast<const uint16_t *>(w->codebook),
        static_cast<const uint16_t *>(w->scales), G, first, count, static_cast<uint16_t *>(out));
    return check_launch("dequant_kernel");
}

}  // extern "C"
