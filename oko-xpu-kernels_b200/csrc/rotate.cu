// The ConvRot rotation family on sm_100a: one kernel template covers
//
//   mode 0  bf16 [M,K] (or [M,2K] for a paired activation) -> act -> rotate ->
//           per-row int8 [M,K] + fp32 scale [M]
//           (reference: launch_convrot_quant_warp<ACT>, src/xpuint8.cpp:450-502)
//   mode 1  int32 acc [M,2K] / [M,K] -> dequant -> act -> rotate -> int8 + scale
//           (reference: launch_dequant_act_quant_warp<ACT>, src/xpuint8.cpp:517-573)
//   mode 2  bf16 [M,K] -> rotate -> bf16 [M,K]
//           (reference: launch_rotate_bf16<G>, src/xpuint8.cpp:588-635)
//   mode 3  int8 [N,K] * fp32 [N] -> bf16 round -> rotate -> bf16 [N,K]
//           (reference: dequant_weight_torch, python/xpu_kernels/int8/ops.py:169-191)
//
// Work decomposition.  A 256-element group is owned by a half-warp ("slot"):
// lane l loads elements [16l, 16l+16) with two 16-byte loads, so a half-warp
// reads 512 contiguous bytes.  With element i = 16w + q the digits are
// i0 = q&3, i1 = q>>2 (inside a lane) and i2 = w&3, i3 = w>>2 (across lanes),
// w = l.  Axes 0 and 1 run in registers (accumulation-chain association, as the
// reference's `inreg`), then a swizzled 1 KB shared-memory transpose gives lane
// l the elements 16w + l, w = 0..15, so axes 2 and 3 also run in registers
// (butterfly association, as the reference's `bfly_xor`).  This keeps the
// cross-lane traffic at one smem write + one read per element instead of four
// warp shuffles.  The arithmetic and its association are the reference's, with
// the per-stage 1/2 factors applied once as 1/16 (exact).
//
// A row's groups are spread over `spr` slots of one CTA (a slot may own up to
// GPL groups); the rotated values stay in registers while the CTA reduces the
// row abs-max through shared memory, and only then are quantized.  Output
// bytes are staged back through the slot's tile so every global store is a
// contiguous 16-byte store.
#include "act.cuh"
#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

constexpr int kTileFloats = 272;  // 16x16 floats + 16 floats of skew between slots


struct RotParams {
    const void *in;
    const float *w_scale;  // mode 1: [K or 2K]; mode 3: [N] row scale
    const float *x_scale;  // mode 1: [M]
    void *out;
    float *scale;          // modes 0, 1: [M]
    int64_t M, K, in_stride;
    int G, spr, R;
};

template <int MODE, int ACT>
__device__ __forceinline__ void load_group(const RotParams &p, int64_t row, int g, int l,
                                           float (&v)[16]) {
    const int64_t off = static_cast<int64_t>(g) * kGroup + l * 16;
    if constexpr (MODE == 0 || MODE == 2) {
        const uint16_t *x = static_cast<const uint16_t *>(p.in) + row * p.in_stride + off;
        const uint4 *xa = reinterpret_cast<const uint4 *>(x);
        unpack16_bf16(__ldcs(xa), __ldcs(xa + 1), v);
        if constexpr (MODE == 0 && act_paired(ACT)) {
            const uint4 *xb = reinterpret_cast<const uint4 *>(x + p.K);
            float u[16];
            unpack16_bf16(__ldcs(xb), __ldcs(xb + 1), u);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], u[t]);
        } else if constexpr (MODE == 0 && ACT != 0) {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], 0.f);
        }
    } else if constexpr (MODE == 1) {
        const int32_t *a = static_cast<const int32_t *>(p.in) + row * p.in_stride + off;
        const float xs = __ldg(p.x_scale + row);
        const int4 *ah = reinterpret_cast<const int4 *>(a);
        const float4 *wh = reinterpret_cast<const float4 *>(p.w_scale + off);
        float h[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int4 ai = __ldcs(ah + j);
            const float4 wi = __ldg(wh + j);
            // dequant then the bf16 round of the unfused store (src/xpuint8.cpp:246-248)
            h[4 * j + 0] = round_bf16(__fmul_rn(static_cast<float>(ai.x), __fmul_rn(wi.x, xs)));
            h[4 * j + 1] = round_bf16(__fmul_rn(static_cast<float>(ai.y), __fmul_rn(wi.y, xs)));
            h[4 * j + 2] = round_bf16(__fmul_rn(static_cast<float>(ai.z), __fmul_rn(wi.z, xs)));
            h[4 * j + 3] = round_bf16(__fmul_rn(static_cast<float>(ai.w), __fmul_rn(wi.w, xs)));
        }
        if constexpr (ACT == 5) {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<5>(h[t], 0.f);
        } else {
            const int4 *ag = reinterpret_cast<const int4 *>(a + p.K);
            const float4 *wg = reinterpret_cast<const float4 *>(p.w_scale + p.K + off);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int4 ai = __ldcs(ag + j);
                const float4 wi = __ldg(wg + j);
                const float gq[4] = {
                    round_bf16(__fmul_rn(static_cast<float>(ai.x), __fmul_rn(wi.x, xs))),
                    round_bf16(__fmul_rn(static_cast<float>(ai.y), __fmul_rn(wi.y, xs))),
                    round_bf16(__fmul_rn(static_cast<float>(ai.z), __fmul_rn(wi.z, xs))),
                    round_bf16(__fmul_rn(static_cast<float>(ai.w), __fmul_rn(wi.w, xs)))};
#pragma unroll
                for (int t = 0; t < 4; ++t) v[4 * j + t] = activate<ACT>(h[4 * j + t], gq[t]);
            }
        }
    } else {  // MODE 3: int8 weight row * scale, rounded to bf16 before the rotation
        const int8_t *w = static_cast<const int8_t *>(p.in) + row * p.in_stride + off;
        const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(w));
        const float s = __ldg(p.w_scale + row);
        const uint32_t words[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float q = static_cast<float>(static_cast<int8_t>((words[j] >> (8 * t)) & 0xFF));
                v[4 * j + t] = round_bf16(__fmul_rn(q, s));
            }
        }
    }
}

// Axes 0..3 of one group; `tile` is the slot's private swizzled 16x16 tile.
// On entry lane l holds elements 16l + q; on exit it holds 16w + l (w = 0..15),
// unscaled (x16).
__device__ __forceinline__ void rotate_group(float (&v)[16], float *tile, int l) {
    // axis 0: stride 1 inside the lane's 16 values; axis 1: stride 4
#pragma unroll
    for (int j = 0; j < 4; ++j) axis_seq(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) axis_seq(v[j], v[j + 4], v[j + 8], v[j + 12]);
    // transpose: lane l writes row l, reads column l
    const int sw = (l >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4 *>(tile + l * 16 + ((c ^ sw) << 2)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    __syncwarp();
#pragma unroll
    for (int w = 0; w < 16; ++w) v[w] = tile[w * 16 + ((((l >> 2) ^ (w >> 1)) & 3) << 2) + (l & 3)];
    __syncwarp();
    // axis 2: registers 4g..4g+3; axis 3: registers c, c+4, c+8, c+12
#pragma unroll
    for (int j = 0; j < 4; ++j) axis_bfly(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) axis_bfly(v[j], v[j + 4], v[j + 8], v[j + 12]);
}

template <int MODE, int ACT, int GPL>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const RotParams p) {
    extern __shared__ __align__(16) float smem[];
    constexpr bool QUANT = (MODE == 0 || MODE == 1);
    const int slot = threadIdx.x >> 4, l = threadIdx.x & 15;
    const int nslots = blockDim.x >> 4;
    float *tile = smem + slot * kTileFloats;
    unsigned int *row_amax = reinterpret_cast<unsigned int *>(smem + nslots * kTileFloats);

    const int rib = slot / p.spr, sidx = slot - rib * p.spr;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * p.R + rib;
    const bool active = rib < p.R && row < p.M;

    if constexpr (QUANT) {
        if (threadIdx.x < p.R) row_amax[threadIdx.x] = 0u;
        __syncthreads();
    }

    float vals[GPL][16];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
        const int g = sidx + p.spr * j;
        const bool on = active && g < p.G;
        if (on) {
            load_group<MODE, ACT>(p, row, g, l, vals[j]);
        } else {
#pragma unroll
            for (int t = 0; t < 16; ++t) vals[j][t] = 0.f;
        }
        rotate_group(vals[j], tile, l);  // every lane takes part: it syncs the warp
        if constexpr (QUANT) {
#pragma unroll
            for (int t = 0; t < 16; ++t) amax = fmaxf(amax, fabsf(vals[j][t]));
        }
    }

    float inv16 = 0.f;
    if constexpr (QUANT) {
        // half-warp reduce (xor < 16 stays inside the slot), then per row in smem
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        if (active && l == 0) atomicMax(row_amax + rib, __float_as_uint(amax));
        __syncthreads();
        // No early exit for idle slots: the staging below syncs whole warps.
        if (active) {
            // rowmax of the per-stage-scaled values is the unscaled max / 16 (exact)
            const float rowmax = __fmul_rn(__uint_as_float(row_amax[rib]), 0.0625f);
            const float s = fmaxf(__fdiv_rn(rowmax, 127.0f), 1e-30f);
            if (sidx == 0 && l == 0) p.scale[row] = s;
            inv16 = __fmul_rn(__frcp_rn(s), 0.0625f);  // 1/s then the deferred 1/16, exact
        }
    }

#pragma unroll
    for (int j = 0; j < GPL; ++j) {
        const int g = sidx + p.spr * j;
        const bool on = active && g < p.G;
        const int64_t off = row * p.K + static_cast<int64_t>(g) * kGroup;
        if constexpr (QUANT) {
            unsigned char *tb = reinterpret_cast<unsigned char *>(tile);
#pragma unroll
            for (int w = 0; w < 16; ++w) {
                // rint(v * (1/s)) with the round-to-nearest-even of an fp32 add:
                // r + 1.5*2^23 lands the integer in the low mantissa bits
                const float r = __fmul_rn(vals[j][w], inv16);
                const float m = __fadd_rn(r, 12582912.0f);
                int qi = static_cast<int>(__float_as_uint(m) & 0xFFu) ^ 0x80;
                qi -= 0x80;  // low byte as a signed value
                qi = max(-127, min(127, qi));
                tb[16 * w + l] = static_cast<unsigned char>(qi);
            }
            __syncwarp();
            const uint4 o = *reinterpret_cast<const uint4 *>(tb + 16 * l);
            __syncwarp();
            if (on) __stcs(reinterpret_cast<uint4 *>(static_cast<int8_t *>(p.out) + off) + l, o);
        } else {
            uint16_t *tb = reinterpret_cast<uint16_t *>(tile);
#pragma unroll
            for (int w = 0; w < 16; ++w)
                tb[16 * w + l] = static_cast<uint16_t>(f32_to_bf16_bits(__fmul_rn(vals[j][w], 0.0625f)));
            __syncwarp();
            const uint4 o0 = *reinterpret_cast<const uint4 *>(tb + 16 * l);
            const uint4 o1 = *reinterpret_cast<const uint4 *>(tb + 16 * l + 8);
            __syncwarp();
            if (on) {
                uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + off + 16 * l);
                __stcs(dst, o0);
                __stcs(dst + 1, o1);
            }
        }
    }
}

template <int MODE, int ACT>
int dispatch_gpl(cudaStream_t s, RotParams p, int gpl, int threads, size_t smem, int64_t blocks) {
#define XPU_ROT_CASE(N)                                                                    \
    case N:                                                                                \
        rotate_rows_kernel<MODE, ACT, N><<<static_cast<unsigned>(blocks), threads, smem, s>>>(p); \
        break;
    switch (gpl) {
        XPU_ROT_CASE(1)
        XPU_ROT_CASE(2)
        XPU_ROT_CASE(3)
        XPU_ROT_CASE(4)
        XPU_ROT_CASE(6)
        XPU_ROT_CASE(8)
        default:
            set_error("unsupported group count per slot");
            return 4;
    }
#undef XPU_ROT_CASE
    return launch_status("rotate");
}

}  // namespace

int launch_rotate_rows(cudaStream_t s, int mode, int act, const void *in, const float *w_scale,
                       const float *x_scale, void *out, float *scale, int64_t M, int64_t K) {
    {
        // the streaming kernels (rotate_bulk.cu) cover every shape they fit
        const int rc = mode == 1 ? launch_rotate_bulk(s, 1, act, in, x_scale, w_scale, out, scale, M, K)
                                 : launch_rotate_bulk(s, mode, act, in, w_scale, nullptr, out, scale, M, K);
        if (rc >= 0) return rc;
    }
    const int64_t G = K / kGroup;
    // groups per slot: the smallest of {1,2,3,4,6,8} that fits the row into 16
    // slots (one 256-thread CTA), so K <= 32768
    int gpl = 1;
    const int cand[] = {1, 2, 3, 4, 6, 8};
    bool fit = false;
    for (int c : cand) {
        if ((G + c - 1) / c <= 16) { gpl = c; fit = true; break; }
    }
    if (!fit) {
        set_error("K is too large for the rotation kernels (at most 32768)");
        return 4;
    }
    const int spr = static_cast<int>((G + gpl - 1) / gpl);   // slots per row
    const int R = spr <= 16 ? 16 / spr : 1;                  // rows per CTA
    int threads = ((R * spr * 16 + 31) / 32) * 32;
    RotParams p{};
    p.in = in; p.w_scale = w_scale; p.x_scale = x_scale; p.out = out; p.scale = scale;
    p.M = M; p.K = K; p.G = static_cast<int>(G); p.spr = spr; p.R = R;
    const bool paired = act_paired(act);
    p.in_stride = (mode <= 1 && paired) ? 2 * K : K;
    const int nslots = threads / 16;
    const size_t smem = static_cast<size_t>(nslots) * kTileFloats * sizeof(float) + 64 * sizeof(unsigned);
    const int64_t blocks = (M + R - 1) / R;
    if (blocks > 0x7FFFFFFF) {
        set_error("M is too large");
        return 2;
    }
    if (mode == 0) {
        switch (act) {
            case 0: return dispatch_gpl<0, 0>(s, p, gpl, threads, smem, blocks);
            case 1: return dispatch_gpl<0, 1>(s, p, gpl, threads, smem, blocks);
            case 2: return dispatch_gpl<0, 2>(s, p, gpl, threads, smem, blocks);
            case 3: return dispatch_gpl<0, 3>(s, p, gpl, threads, smem, blocks);
            case 4: return dispatch_gpl<0, 4>(s, p, gpl, threads, smem, blocks);
            case 5: return dispatch_gpl<0, 5>(s, p, gpl, threads, smem, blocks);
            default: break;
        }
    } else if (mode == 1) {
        switch (act) {
            case 3: return dispatch_gpl<1, 3>(s, p, gpl, threads, smem, blocks);
            case 4: return dispatch_gpl<1, 4>(s, p, gpl, threads, smem, blocks);
            case 5: return dispatch_gpl<1, 5>(s, p, gpl, threads, smem, blocks);
            default: break;
        }
    } else if (mode == 2) {
        return dispatch_gpl<2, 0>(s, p, gpl, threads, smem, blocks);
    } else if (mode == 3) {
        return dispatch_gpl<3, 0>(s, p, gpl, threads, smem, blocks);
    }
    set_error("internal: bad rotation mode/activation");
    return 6;
}

}  // namespace xpuint8
