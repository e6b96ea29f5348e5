// Expert (switch-linear) kernels of the decode / MTP-verify regime on B200.
//
// Reference: SwitchGLU.__call__ / SwitchLinear.__call__
// (glm5_next/_mlx_vlm/models/switch_layers.py:116-125, 172-193) with the
// experts as VQSwitchLinear (codes, codebook, vq_scales; layout from
// engine/families/deepseek/heads/deepseek_v4.py:35-42, 111-130).
//
// One persistent kernel family computes, for every (token, slot) pair routed
// to an expert, out[pair] = x_row(pair) @ W[expert]^T with the weights
// dequantised in registers:
//   * VQ: each 8-byte codebook entry (4 fp16) is read from a shared-memory
//     copy and multiplied by its fp16 group scale in one mul.rn.f16x2 -- the
//     product IS the dequantised fp16 weight -- and those registers are the
//     A operand of mma.sync m16n8k16 (fp16 x fp16 -> fp32). B is the
//     expert's (<= 8) token rows, staged in shared memory as fp16.
//   * dense bf16 experts and the shared expert: A is loaded from HBM as is
//     (bf16 x bf16 -> fp32).
// Why mma.sync and registers rather than tcgen05 here: at 1-64 tokens the
// layer is bound by HBM and by the shared-memory codebook lookups (8 bytes
// per code, ~16 codes/clk/SM), not by tensor throughput (~4 tokens per
// expert). A register-fed A operand keeps every dequantised weight out of
// shared memory; tcgen05 would need it written to SMEM or TMEM first.
//
// Codebook replication: 16 copies interleaved so that lane L reads only the
// bank pair L % 16; a warp's random 8-byte lookups are then conflict-free
// (2 wavefronts, the minimum for 256 bytes). 32 KB per codebook.
//
// Device code layout (vqmoe_prepare_codes): each row's codes in chunks of
// 64 (256 inputs); inside a chunk of 4*nq codes, code 4q+t sits at t*nq+q,
// so thread t of an MMA quad loads its nq codes with one 16-byte load and
// sub-step q covers inputs [16q, 16q+16) of the chunk in natural order.
// MMA k-slots {2t, 2t+1, 2t+8, 2t+9} carry inputs 16q+4t+{0,1,2,3}: the same
// permutation on A and B, so the dot product is unchanged, and both the
// codebook entry (A) and the activation quad (B) are single 8-byte loads.
#include "common.cuh"

namespace vqmoe {

constexpr int kThreads = 256;          // 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kTokBlk = 8;             // tokens per pass (MMA N)
constexpr int kRepBytes = 256 * 16 * 8;  // replicated codebook, 32 KB

struct LinearDev {
    const uint8_t *codes;      // VQ device layout [E][OUT][IN/4]
    const uint16_t *codebook;  // [K][4] fp16 bits
    const uint16_t *scales;    // [E][OUT][IN/64] fp16 bits
    const uint16_t *weight;    // dense [E][OUT][IN] bf16 bits
    int K;
};

struct ExpertArgs {
    const int32_t *inds;  // [P] expert of each pair; nullptr: every row is a
                          // pair of expert 0 (the shared expert)
    int P;                // pairs (routed) or rows (identity)
    int k;                // slots per token
    int E;                // experts
    const uint16_t *x;    // bf16 input rows
    int x_per_pair;       // 1: x row = pair; 0: x row = pair / k
    LinearDev w0, w1;     // w1 only for the fused gate/up (DUAL) kernel
    int IN, OUT;
    uint16_t *out;        // bf16 [P][OUT]
    const float *pair_scale;  // optional [P]: out = bf16(bf16(acc) * s)
    int ks;               // K split across warps (1, 2, 4)
    int rows_per_tile;    // 32 * (kWarps / ks)
    int row_blocks;
    int ntiles;
    int list_cap;
    int xs_stride;        // bytes per staged token row
    int xs_bytes;         // max(staging, reduction) bytes
};

template <int FMT, bool DUAL>
__global__ void __launch_bounds__(kThreads, 2) expert_kernel(const ExpertArgs a) {
    constexpr int NMAT = DUAL ? 2 : 1;
    constexpr bool VQ = FMT == VQMOE_FMT_VQ_U8;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_cnt[kWarps];
    uint8_t *cbrep = smem;
    int32_t *s_list = reinterpret_cast<int32_t *>(smem + (VQ ? NMAT * kRepBytes : 0));
    uint8_t *xs = reinterpret_cast<uint8_t *>(s_list + a.list_cap);
    float *red = reinterpret_cast<float *>(xs);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kq = warp % a.ks, rq = warp / a.ks;
    const int IN = a.IN, OUT = a.OUT, S = a.xs_stride;
    const int C = (IN + 255) / 256;

    if (VQ) {
        // 16 interleaved copies: entry c of copy b at byte c*128 + b*8
        for (int i = tid; i < NMAT * 256 * 16; i += kThreads) {
            int m = i / 4096, r = i - m * 4096, c = r >> 4, b = r & 15;
            const LinearDev &w = m == 0 ? a.w0 : a.w1;
            uint2 v = make_uint2(0, 0);
            if (c < w.K) v = *reinterpret_cast<const uint2 *>(w.codebook + c * 4);
            *reinterpret_cast<uint2 *>(cbrep + m * kRepBytes + c * 128 + b * 8) = v;
        }
    }
    const uint32_t cb_s = smem_u32(cbrep) + (lane & 15) * 8;
    const uint32_t xs_s = smem_u32(xs);

    for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
        const int e = tile / a.row_blocks, rb = tile - e * a.row_blocks;
        int cursor = 0;  // next pair id to scan
      for (;;) {
        // ---- the next (at most list_cap) pairs of expert e, ascending pair
        // id (a stable sort by expert); a scan step adds <= kThreads entries
        // and only runs while they fit, so s_list never overflows
        int n = 0;
        if (a.inds) {
            while (cursor < a.P && n + kThreads <= a.list_cap) {
                int p = cursor + tid;
                bool hit = p < a.P && a.inds[p] == e;
                unsigned bal = __ballot_sync(0xffffffffu, hit);
                if (lane == 0) s_cnt[warp] = __popc(bal);
                __syncthreads();
                int off = n, tot = 0;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    int c = s_cnt[w];
                    off += w < warp ? c : 0;
                    tot += c;
                }
                if (hit) s_list[off + __popc(bal & ((1u << lane) - 1u))] = p;
                n += tot;
                cursor += kThreads;
                __syncthreads();
            }
        } else {
            n = a.P;       // identity routing: pairs 0 .. P-1, no list
            cursor = a.P;
        }
        if (n == 0) break;
        const int row_base = rb * a.rows_per_tile + rq * 32;
        const bool mt_ok0 = row_base < OUT, mt_ok1 = row_base + 16 < OUT;

        for (int tb0 = 0; tb0 < n; tb0 += kTokBlk) {
            const int nt = min(kTokBlk, n - tb0);
            __syncthreads();  // previous pass's epilogue is done with xs / red
            // ---- stage up to 8 input rows (fp16 for VQ, bf16 for dense)
            {
                const int vpr = IN / 8;
                for (int v = tid; v < kTokBlk * vpr; v += kThreads) {
                    int r = v / vpr, c8 = v - r * vpr;
                    uint4 val = make_uint4(0, 0, 0, 0);
                    if (r < nt) {
                        int pair = a.inds ? s_list[tb0 + r] : tb0 + r;
                        int xr = a.x_per_pair ? pair : pair / a.k;
                        val = *reinterpret_cast<const uint4 *>(a.x + (size_t)xr * IN + c8 * 8);
                        if (VQ) {
                            uint32_t u[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                u[j] = (uint32_t)bf16_to_f16_sat(u[j] & 0xFFFFu) |
                                       ((uint32_t)bf16_to_f16_sat(u[j] >> 16) << 16);
                            val = make_uint4(u[0], u[1], u[2], u[3]);
                        }
                    }
                    *reinterpret_cast<uint4 *>(xs + r * S + c8 * 16) = val;
                }
            }
            __syncthreads();

            float acc[NMAT][2][4];
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[m][mt][i] = 0.0f;

            if (mt_ok0) {
                for (int c = kq; c < C; c += a.ks) {
                    const int feat0 = c * 256;
                    const int nq = min(16, (IN - feat0) >> 4);
                    const uint32_t xb = xs_s + g * S + (feat0 + 4 * t) * 2;
                    if (VQ) {
                        uint32_t cw[NMAT][2][2][4];
                        uint32_t sc[NMAT][2][2][4];
#pragma unroll
                        for (int m = 0; m < NMAT; ++m) {
                            const LinearDev &w = m == 0 ? a.w0 : a.w1;
#pragma unroll
                            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const int row = row_base + mt * 16 + h * 8 + g;
                                    const bool ok = mt == 0 || mt_ok1;
                                    const size_t rix = (size_t)e * OUT + row;
                                    const uint8_t *cp = w.codes + rix * (IN / 4) + c * 64 + t * nq;
                                    const uint16_t *sp = w.scales + rix * (IN / 64) + c * 4;
                                    if (ok && nq == 16) {
                                        uint4 v = ldg_stream_v4(cp);
                                        cw[m][mt][h][0] = v.x;
                                        cw[m][mt][h][1] = v.y;
                                        cw[m][mt][h][2] = v.z;
                                        cw[m][mt][h][3] = v.w;
                                    } else {
#pragma unroll
                                        for (int j = 0; j < 4; ++j)
                                            cw[m][mt][h][j] = (ok && 4 * j < nq) ? ldg_stream_u32(cp + 4 * j) : 0u;
                                    }
#pragma unroll
                                    for (int j = 0; j < 4; ++j) {
                                        uint32_t s = (ok && 4 * j < nq) ? ldg_nc_u16(sp + j) : 0u;
                                        sc[m][mt][h][j] = s | (s << 16);
                                    }
                                }
                        }
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            if (q < nq) {
                                const int j = q >> 2, sh = (q & 3) * 8;
                                const uint2 bf = lds_v2(xb + q * 32);
#pragma unroll
                                for (int m = 0; m < NMAT; ++m) {
                                    const uint32_t cbm = cb_s + m * kRepBytes;
#pragma unroll
                                    for (int mt = 0; mt < 2; ++mt) {
                                        if (mt == 0 || mt_ok1) {
                                            const uint32_t c0 = (cw[m][mt][0][j] >> sh) & 0xFFu;
                                            const uint32_t c1 = (cw[m][mt][1][j] >> sh) & 0xFFu;
                                            const uint2 e0 = lds_v2(cbm + c0 * 128);
                                            const uint2 e1 = lds_v2(cbm + c1 * 128);
                                            const uint32_t s0 = sc[m][mt][0][j], s1 = sc[m][mt][1][j];
                                            mma_f16(acc[m][mt], hmul2_u32(e0.x, s0), hmul2_u32(e1.x, s1),
                                                    hmul2_u32(e0.y, s0), hmul2_u32(e1.y, s1), bf.x, bf.y);
                                        }
                                    }
                                }
                            }
                        }
                    } else {
#pragma unroll 4
                        for (int q = 0; q < nq; ++q) {
                            const uint2 bf = lds_v2(xb + q * 32);
#pragma unroll
                            for (int m = 0; m < NMAT; ++m) {
                                const LinearDev &w = m == 0 ? a.w0 : a.w1;
#pragma unroll
                                for (int mt = 0; mt < 2; ++mt) {
                                    if (mt == 0 || mt_ok1) {
                                        const size_t r0 = (size_t)e * OUT + row_base + mt * 16 + g;
                                        const uint16_t *wp = w.weight + r0 * IN + feat0 + 16 * q + 4 * t;
                                        const uint2 w0 = ldg_nc_v2(wp);
                                        const uint2 w1 = ldg_nc_v2(wp + (size_t)8 * IN);
                                        mma_bf16(acc[m][mt], w0.x, w1.x, w0.y, w1.y, bf.x, bf.y);
                                    }
                                }
                            }
                        }
                    }
                }
            }
            __syncthreads();  // all warps done reading xs: reuse it for partials
            {
                const int R = a.rows_per_tile;
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const int rl = rq * 32 + mt * 16 + g;
                        float *base = red + ((size_t)(kq * NMAT + m) * R) * kTokBlk;
                        base[rl * kTokBlk + 2 * t] = acc[m][mt][0];
                        base[rl * kTokBlk + 2 * t + 1] = acc[m][mt][1];
                        base[(rl + 8) * kTokBlk + 2 * t] = acc[m][mt][2];
                        base[(rl + 8) * kTokBlk + 2 * t + 1] = acc[m][mt][3];
                    }
            }
            __syncthreads();
            {
                const int R = a.rows_per_tile;
                for (int o = tid; o < R * kTokBlk; o += kThreads) {
                    const int tok = o / R, rl = o - tok * R;
                    const int row = rb * R + rl;
                    if (tok >= nt || row >= OUT) continue;
                    float s[NMAT];
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        float v = 0.0f;
                        for (int q = 0; q < a.ks; ++q)
                            v += red[((size_t)(q * NMAT + m) * R + rl) * kTokBlk + tok];
                        s[m] = v;
                    }
                    const int pair = a.inds ? s_list[tb0 + tok] : tb0 + tok;
                    uint16_t res;
                    if (DUAL) {
                        // _SwiGLU (qwen3_5.py:108-112): bf16(bf16(silu(g)) * u)
                        const float gv = bf16r(s[0]), uv = bf16r(s[NMAT - 1]);
                        res = f32_to_bf16(bf16r(silu_f32(gv)) * uv);
                    } else {
                        float y = bf16r(s[0]);
                        if (a.pair_scale) y = y * a.pair_scale[pair];
                        res = f32_to_bf16(y);
                    }
                    a.out[(size_t)pair * OUT + row] = res;
                }
            }
        }
        if (cursor >= a.P) break;
      }
    }
}

// ------------------------------------------------------------------ host

template <int FMT, bool DUAL>
static vqmoe_status launch_one(const ExpertArgs &a, size_t smem, int grid,
                               cudaStream_t stream) {
    static size_t configured[64] = {0};   // per device
    int dev = 0;
    cudaGetDevice(&dev);
    auto fn = expert_kernel<FMT, DUAL>;
    if (dev < 0 || dev >= 64 || smem > configured[dev]) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return set_error(VQMOE_LAUNCH_FAILED, "expert kernel: %zu bytes of shared memory", smem);
        if (dev >= 0 && dev < 64) configured[dev] = smem;
    }
    fn<<<grid, kThreads, smem, stream>>>(a);
    return check_launch("expert_kernel");
}

static int pick_ks(int chunks) {
    if (chunks % 4 == 0) return 4;
    if (chunks % 2 == 0) return 2;
    return 1;
}

// Shared by vqmoe_switch_linear / switch_glu / sparse_moe_block.
// inds == nullptr: identity routing (rows 0..P-1 all use expert 0).
vqmoe_status launch_expert(const vqmoe_linear *w0, const vqmoe_linear *w1,
                           const int32_t *inds, int P, int k, const void *x,
                           int x_per_pair, void *out, const float *pair_scale,
                           int list_cap, cudaStream_t stream) {
    const bool dual = w1 != nullptr;
    ExpertArgs a{};
    a.inds = inds;
    a.P = P;
    a.k = k;
    a.E = inds ? w0->num_experts : 1;
    a.x = static_cast<const uint16_t *>(x);
    a.x_per_pair = x_per_pair;
    a.IN = w0->in_features;
    a.OUT = w0->out_features;
    auto dev = [](const vqmoe_linear *w) {
        LinearDev d{};
        d.codes = static_cast<const uint8_t *>(w->codes);
        d.codebook = static_cast<const uint16_t *>(w->codebook);
        d.scales = static_cast<const uint16_t *>(w->scales);
        d.weight = static_cast<const uint16_t *>(w->weight);
        d.K = w->codebook_size;
        return d;
    };
    a.w0 = dev(w0);
    a.w1 = dual ? dev(w1) : a.w0;
    a.out = static_cast<uint16_t *>(out);
    a.pair_scale = pair_scale;
    const int chunks = (a.IN + 255) / 256;
    a.ks = pick_ks(chunks);
    a.rows_per_tile = 32 * (kWarps / a.ks);
    a.row_blocks = (a.OUT + a.rows_per_tile - 1) / a.rows_per_tile;
    a.ntiles = a.E * a.row_blocks;
    // pair-list capacity: >= one scan step (kThreads); more only saves re-scans
    a.list_cap = inds ? (int)std::min<size_t>(2048, std::max<size_t>(kThreads, align_up((size_t)list_cap, 32))) : 0;
    a.xs_stride = (int)align_up((size_t)a.IN * 2, 128) + 32;
    const int nmat = dual ? 2 : 1;
    const size_t stage = (size_t)kTokBlk * a.xs_stride;
    const size_t redb = (size_t)a.ks * nmat * a.rows_per_tile * kTokBlk * sizeof(float);
    a.xs_bytes = (int)std::max(stage, redb);
    const bool vq = w0->format == VQMOE_FMT_VQ_U8;
    const size_t smem = (vq ? nmat * (size_t)kRepBytes : 0) + (size_t)a.list_cap * 4 + a.xs_bytes;
    if (smem > 227 * 1024)
        return set_error(VQMOE_BAD_SHAPE, "expert kernel needs %zu bytes of shared memory", smem);
    const int grid = std::min(a.ntiles, 2 * sm_count());
    if (vq)
        return dual ? launch_one<VQMOE_FMT_VQ_U8, true>(a, smem, grid, stream)
                    : launch_one<VQMOE_FMT_VQ_U8, false>(a, smem, grid, stream);
    return dual ? launch_one<VQMOE_FMT_DENSE_BF16, true>(a, smem, grid, stream)
                : launch_one<VQMOE_FMT_DENSE_BF16, false>(a, smem, grid, stream);
}

}  // namespace vqmoe
