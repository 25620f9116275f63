// RMS norm + rotary position embedding of attention heads, reading either the
// bf16 q / k projections or the INT8 GEMM's int32 accumulator directly.
//
// This is the consumer the reference feeds its fused qkv accumulator into
// (python/xpu_kernels/triton/rope.py:378-408 `_rows_dq`, :643-652
// `rms_rope_split_half_dequant`; the bf16 form :360-376 `_rows`; the chain it
// restates, python/xpu_kernels/triton/reference.py:63-98).  Per (row, head) of
// D elements:
//
//   x_d   = bf16(float(acc[d]) * (w_scale[h*D + d] * x_scale[row]))   (int32 input)
//         = in[d]                                                     (bf16 input)
//   inv   = rsqrt(sum_d x_d^2 / D + eps)
//   y_d   = bf16((x_d * inv) * weight[d])
//   out_i = bf16(f00 * y_a + f01 * y_b),  out_j = bf16(f10 * y_a + f11 * y_b)
//
// over the pairs (a, b) = (i, i + D/2) (split half) or (2i, 2i + 1)
// (interleaved), with [[f00, f01], [f10, f11]] the rotation of pair i at this
// row's (batch, position) in freqs [fb, fs, D/2, 2, 2] (fb, fs: 1 broadcasts).
// The int32 form's x_d is exactly the dequant epilogue's output, so
// rms_rope(int32 accumulator) equals rms_rope(linear_split output) bit for bit.
//
// One warp per (row, head): lane l owns pairs l, l + 32, ..; the sum of squares
// is a per-lane sum then a butterfly over the warp (the reference's Triton
// kernel sums in its own block order, so the two agree to the last bit of the
// sum, not always bit for bit).  Memory-bound: each element is read once and
// written once; freqs rows are shared by every head of a row (L1/L2 hits).
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

struct RopeArgs {
    const void *in;
    int64_t ld_in;        // elements between rows of the input
    const float *x_scale;  // [rows] (int32 input)
    const float *w_scale;  // [H*D] (int32 input)
    const float *weight;   // [D] the RMS norm's scale
    const float *freqs;    // [fb, fs, D/2, 2, 2]
    int64_t fb, fs;
    uint16_t *out;
    int64_t ld_out;       // elements between rows of the output
    int64_t rows, S, H;
    int D;
    float eps;
};

__device__ __forceinline__ float bf16_at(const uint16_t *p) {
    return __uint_as_float(static_cast<uint32_t>(*p) << 16);
}

template <bool I32, bool SPLIT, int PPL>
__global__ void __launch_bounds__(256) rms_rope_kernel(const RopeArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);  // (row, head)
    if (item >= a.rows * a.H) return;
    const int64_t row = item / a.H;
    const int h = static_cast<int>(item - row * a.H);
    const int D = a.D, half = D / 2;
    const int64_t b = row / a.S, s = row - b * a.S;
    const float *f = a.freqs + ((((a.fb == 1) ? 0 : b) * a.fs + ((a.fs == 1) ? 0 : s)) * half) * 4;
    float x0[PPL], x1[PPL];
    const float xs = I32 ? __ldg(a.x_scale + row) : 0.f;
#pragma unroll
    for (int j = 0; j < PPL; ++j) {
        const int i = lane + 32 * j;                 // this lane's pair
        const int d0 = SPLIT ? i : 2 * i, d1 = SPLIT ? i + half : 2 * i + 1;
        if constexpr (I32) {
            const int32_t *src = static_cast<const int32_t *>(a.in) + row * a.ld_in + static_cast<int64_t>(h) * D;
            const float *ws = a.w_scale + static_cast<int64_t>(h) * D;
            x0[j] = round_bf16(__fmul_rn(static_cast<float>(__ldg(src + d0)), __fmul_rn(__ldg(ws + d0), xs)));
            x1[j] = round_bf16(__fmul_rn(static_cast<float>(__ldg(src + d1)), __fmul_rn(__ldg(ws + d1), xs)));
        } else {
            const uint16_t *src = static_cast<const uint16_t *>(a.in) + row * a.ld_in + static_cast<int64_t>(h) * D;
            x0[j] = bf16_at(src + d0);
            x1[j] = bf16_at(src + d1);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PPL; ++j) ss = __fadd_rn(__fadd_rn(ss, __fmul_rn(x0[j], x0[j])), __fmul_rn(x1[j], x1[j]));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xFFFFFFFFu, ss, m));
    // D is a power of two: the division by D is exact
    const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), a.eps));
    uint16_t *dst = a.out + row * a.ld_out + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int j = 0; j < PPL; ++j) {
        const int i = lane + 32 * j;
        const int d0 = SPLIT ? i : 2 * i, d1 = SPLIT ? i + half : 2 * i + 1;
        const float y0 = round_bf16(__fmul_rn(__fmul_rn(x0[j], inv), __ldg(a.weight + d0)));
        const float y1 = round_bf16(__fmul_rn(__fmul_rn(x1[j], inv), __ldg(a.weight + d1)));
        const float4 r = __ldg(reinterpret_cast<const float4 *>(f) + i);  // f00, f01, f10, f11
        const float o0 = __fadd_rn(__fmul_rn(r.x, y0), __fmul_rn(r.y, y1));
        const float o1 = __fadd_rn(__fmul_rn(r.z, y0), __fmul_rn(r.w, y1));
        dst[d0] = static_cast<uint16_t>(f32_to_bf16_bits(o0));
        dst[d1] = static_cast<uint16_t>(f32_to_bf16_bits(o1));
    }
}

template <bool I32, bool SPLIT>
int launch_pp(cudaStream_t s, const RopeArgs &a) {
    const int64_t items = a.rows * a.H;
    const int64_t blocks = (items + 7) / 8;
    if (blocks > 0x7FFFFFFF) {
        set_error("rms_rope: too many rows x heads");
        return 2;
    }
    switch (a.D) {
        case 64: rms_rope_kernel<I32, SPLIT, 1><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a); break;
        case 128: rms_rope_kernel<I32, SPLIT, 2><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a); break;
        case 256: rms_rope_kernel<I32, SPLIT, 4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a); break;
        default:
            set_error("rms_rope: the head dim must be 64, 128 or 256");
            return 2;
    }
    return launch_status("rms_rope");
}

}  // namespace

int launch_rms_rope(cudaStream_t s, const void *in, bool in_int32, int64_t ld_in, const float *x_scale,
                    const float *w_scale, const float *weight, const float *freqs, int64_t fb,
                    int64_t fs, void *out, int64_t ld_out, int64_t B, int64_t S, int64_t H, int64_t D,
                    float eps, bool split_half) {
    RopeArgs a{};
    a.in = in; a.ld_in = ld_in;
    a.x_scale = x_scale; a.w_scale = w_scale; a.weight = weight;
    a.freqs = freqs; a.fb = fb; a.fs = fs;
    a.out = static_cast<uint16_t *>(out); a.ld_out = ld_out;
    a.rows = B * S; a.S = S; a.H = H; a.D = static_cast<int>(D);
    a.eps = eps;
    if (in_int32) return split_half ? launch_pp<true, true>(s, a) : launch_pp<true, false>(s, a);
    return split_half ? launch_pp<false, true>(s, a) : launch_pp<false, false>(s, a);
}

}  // namespace xpuint8
