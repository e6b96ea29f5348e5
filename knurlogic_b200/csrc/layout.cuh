// Device layout of a VQ switch linear's codes and scales.
//
// The reference layout (deepseek_v4.py:35-42, 111-130) is codes
// [E, OUT, IN/4] uint8 (dim-4 codes, one per entry) and vq_scales
// [E, OUT, IN/64] fp16. The kernels read a tiled copy instead, made once at
// load (vqmoe_prepare_vq): rows padded to OUTP = 32*ceil(OUT/32), inputs to
// INP = 256*ceil(IN/256) (padding codes 0, padding scales 0, so padded
// weights are exactly 0), cut into tiles of 32 rows x 256 inputs.
//
// Inside a code tile (2048 bytes) the byte for row r = 16*mt + 8*h + g and
// chunk-local code u = 4*(8*half + b) + t sits at
//     half*1024 + (2*mt + h)*256 + (4*g + t)*8 + b.
// Lane 4g+t of a warp computing MMA sub-step q = 8*half + b (inputs
// [16q, 16q+16) of the chunk) needs exactly these codes: each warp load of
// one (half, mt, h) is a contiguous 256-byte request, and a warp's codes
// for a whole unit are one contiguous run of tiles.
// A scale tile (128 fp16) holds scale group 4*c + 2*half + jj of row r at
//     half*64 + (2*mt + h)*16 + 2*g + jj.
#pragma once

#include <stdint.h>

namespace vqmoe {

struct VqGeom {
    int E, OUT, IN;
    __host__ __device__ int rb() const { return (OUT + 31) >> 5; }
    __host__ __device__ int chunks() const { return (IN + 255) >> 8; }
    __host__ __device__ long long tiles() const { return (long long)E * rb() * chunks(); }
    __host__ __device__ long long code_bytes() const { return tiles() * 2048; }
    __host__ __device__ long long scale_elems() const { return tiles() * 128; }
    __host__ __device__ long long tile(int e, int rbi, int c) const {
        return ((long long)e * rb() + rbi) * chunks() + c;
    }
};

}  // namespace vqmoe
