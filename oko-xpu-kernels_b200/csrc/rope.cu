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
// D / 8 lanes per (row, head), eight elements per lane; the sum of squares is a
// per-lane sum then a butterfly over the head's lanes (the reference's Triton
// kernel sums in its own block order, so the two agree to the last bit of the
// sum, not always bit for bit).  Memory-bound: each element is read once and
// written once; freqs rows are shared by every head of a row (L1/L2 hits).
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

// n / d for 0 <= n < 2^31 by one high multiply, an add and a shift: the
// invariant-divisor method of Granlund & Montgomery ("Division by Invariant
// Integers using Multiplication", PLDI 1994, section 4) with l = ceil(log2 d)
// and m = floor(2^32 (2^l - d) / d) + 1; n < 2^31 keeps umulhi(n, m) + n below
// 2^32.
struct DivU32 {
    uint32_t d, m, l;
};

DivU32 make_div(uint32_t d) {
    uint32_t l = 0;
    while ((uint64_t{1} << l) < d) ++l;
    const uint64_t m = ((uint64_t{1} << 32) * ((uint64_t{1} << l) - d)) / d + 1;
    return DivU32{d, static_cast<uint32_t>(m), l};
}

__device__ __forceinline__ uint32_t div_u32(uint32_t n, const DivU32 &v) {
    return (__umulhi(n, v.m) + n) >> v.l;
}

// bf16 bits of two floats, round to nearest even by the hardware conversion,
// with a NaN written as 0x7FC0 (the hardware's canonical NaN is 0x7FFF, which
// no finite or infinite input produces)
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
    uint32_t p;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
    if ((p & 0xFFFFu) == 0x7FFFu) p = (p & 0xFFFF0000u) | 0x7FC0u;
    if ((p >> 16) == 0x7FFFu) p = (p & 0xFFFFu) | 0x7FC00000u;
    return p;
}

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
    uint32_t tasks;       // rows x chunks per row, below 2^31
    uint32_t H, chunk;    // heads per row; heads per warp task
    DivU32 chunks, S;     // chunks per row; positions per batch
    float eps;
};

constexpr int kIters = 4;  // head passes per warp task: freqs and weight loads amortise over them

// One warp task = one row's run of `chunk` heads.  8 elements (four pairs) per
// lane, D / 8 lanes per head, HPW = 32 / (D / 8) heads per pass: split half,
// lane q owns elements 4q..4q+3 and their partners D/2 on; interleaved,
// elements 8q..8q+7.  Every global access is 8 or 16 bytes.  The row's freqs
// (64 bytes per lane, which touch eight cache lines per warp load) and the
// norm weight are loaded once per task; the next pass's input is loaded before
// this pass's arithmetic.
template <bool I32, bool SPLIT, int D>
__global__ void __launch_bounds__(256) rms_rope_kernel(const RopeArgs a) {
    constexpr int LPH = D / 8;  // lanes per head
    constexpr int HALF = D / 2;
    constexpr int HPW = 32 / LPH;
    const int lane = threadIdx.x & 31;
    const int q = lane % LPH;   // this lane's block of four pairs within the head
    const uint32_t slot = lane / LPH;
    const uint32_t task = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (task >= a.tasks) return;  // whole warps only
    const uint32_t row = div_u32(task, a.chunks);
    const uint32_t h0 = (task - row * a.chunks.d) * a.chunk;
    const uint32_t h_end = min(h0 + a.chunk, a.H);
    const int passes = static_cast<int>((h_end - h0 + HPW - 1) / HPW);
    const int e0 = SPLIT ? 4 * q : 8 * q;  // element offsets of this lane's two runs of four
    const int e1 = SPLIT ? 4 * q + HALF : 8 * q + 4;

    const uint32_t b = div_u32(row, a.S);
    const uint32_t s = row - b * a.S.d;
    const int64_t frow = ((a.fb == 1) ? 0 : static_cast<int64_t>(b)) * a.fs + ((a.fs == 1) ? 0 : s);
    const float4 *f4 = reinterpret_cast<const float4 *>(a.freqs + frow * HALF * 4) + 4 * q;  // pairs 4q .. 4q+3
    float4 fr[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) fr[t] = __ldg(f4 + t);  // f00, f01, f10, f11 of pair 4q + t
    const float4 wa = __ldg(reinterpret_cast<const float4 *>(a.weight + e0));
    const float4 wb = __ldg(reinterpret_cast<const float4 *>(a.weight + e1));
    const float wt[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    const float xs = I32 ? __ldg(a.x_scale + row) : 0.f;
    const char *in_row = static_cast<const char *>(a.in) + row * a.ld_in * (I32 ? 4 : 2);
    uint16_t *out_row = a.out + row * a.ld_out;

    // raw input of one pass: int32 -> u, v (16 bytes each) + w_scale; bf16 -> u.x/y, v.x/y
    auto load = [&](int pass, int4 &u, int4 &v, float4 &wu, float4 &wv) {
        const uint32_t h = h0 + pass * HPW + slot;
        const uint32_t hc = h < h_end ? h : h0;  // lanes past the run reload a live head
        if constexpr (I32) {
            const int32_t *src = reinterpret_cast<const int32_t *>(in_row) + hc * D;
            u = __ldcs(reinterpret_cast<const int4 *>(src + e0));
            v = __ldcs(reinterpret_cast<const int4 *>(src + e1));
            const float *ws = a.w_scale + hc * D;
            wu = __ldg(reinterpret_cast<const float4 *>(ws + e0));
            wv = __ldg(reinterpret_cast<const float4 *>(ws + e1));
        } else {
            const uint16_t *src = reinterpret_cast<const uint16_t *>(in_row) + hc * D;
            const uint2 x0 = __ldcs(reinterpret_cast<const uint2 *>(src + e0));
            const uint2 x1 = __ldcs(reinterpret_cast<const uint2 *>(src + e1));
            u = make_int4(static_cast<int>(x0.x), static_cast<int>(x0.y), 0, 0);
            v = make_int4(static_cast<int>(x1.x), static_cast<int>(x1.y), 0, 0);
        }
    };
    int4 u, v, un, vn;
    float4 wu, wv, wun, wvn;
    load(0, u, v, wu, wv);
    for (int pass = 0; pass < passes; ++pass) {
        if (pass + 1 < passes) load(pass + 1, un, vn, wun, wvn);
        float x[8];
        if constexpr (I32) {
            // the dequant epilogue's value: bf16(float(acc) * (w_scale * x_scale))
            const int iv[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
            const float sc[8] = {wu.x, wu.y, wu.z, wu.w, wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) x[t] = __fmul_rn(static_cast<float>(iv[t]), __fmul_rn(sc[t], xs));
#pragma unroll
            for (int t = 0; t < 8; t += 2) round_bf16x2(x[t], x[t + 1]);
        } else {
            const uint32_t w[4] = {static_cast<uint32_t>(u.x), static_cast<uint32_t>(u.y),
                                   static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y)};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                x[2 * t] = bf16_lo(w[t]);
                x[2 * t + 1] = bf16_hi(w[t]);
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int t = 0; t < 8; ++t) ss = __fadd_rn(ss, __fmul_rn(x[t], x[t]));
#pragma unroll
        for (int m = LPH / 2; m >= 1; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xFFFFFFFFu, ss, m));
        // D is a power of two, so ss * (1 / D) is the correctly rounded ss / D
        const float inv = __frsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / D), a.eps));
        float y[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) y[t] = __fmul_rn(__fmul_rn(x[t], inv), wt[t]);
#pragma unroll
        for (int t = 0; t < 8; t += 2) round_bf16x2(y[t], y[t + 1]);
        float o[8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            // split: pair t is (y[t], y[4 + t]); interleaved: (y[2t], y[2t + 1])
            const int ia = SPLIT ? t : 2 * t, ib = SPLIT ? 4 + t : 2 * t + 1;
            o[ia] = __fadd_rn(__fmul_rn(fr[t].x, y[ia]), __fmul_rn(fr[t].y, y[ib]));
            o[ib] = __fadd_rn(__fmul_rn(fr[t].z, y[ia]), __fmul_rn(fr[t].w, y[ib]));
        }
        const uint32_t h = h0 + pass * HPW + slot;
        if (h < h_end) {
            uint16_t *dst = out_row + h * D;
            __stcs(reinterpret_cast<uint2 *>(dst + e0),
                   make_uint2(pack_bf16x2_rn(o[0], o[1]), pack_bf16x2_rn(o[2], o[3])));
            __stcs(reinterpret_cast<uint2 *>(dst + e1),
                   make_uint2(pack_bf16x2_rn(o[4], o[5]), pack_bf16x2_rn(o[6], o[7])));
        }
        u = un; v = vn; wu = wun; wv = wvn;
    }
}

template <bool I32, bool SPLIT>
int launch_pp(cudaStream_t s, const RopeArgs &a, int D) {
    const uint32_t blocks = (a.tasks + 7) / 8;  // eight warp tasks per block
    switch (D) {
        case 64: rms_rope_kernel<I32, SPLIT, 64><<<blocks, 256, 0, s>>>(a); break;
        case 128: rms_rope_kernel<I32, SPLIT, 128><<<blocks, 256, 0, s>>>(a); break;
        case 256: rms_rope_kernel<I32, SPLIT, 256><<<blocks, 256, 0, s>>>(a); break;
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
    if (B * S * H >= (int64_t{1} << 31) || S < 1 || H < 1) {
        set_error("rms_rope: rows x heads must be below 2^31");
        return 2;
    }
    RopeArgs a{};
    a.in = in; a.ld_in = ld_in;
    a.x_scale = x_scale; a.w_scale = w_scale; a.weight = weight;
    a.freqs = freqs; a.fb = fb; a.fs = fs;
    a.out = static_cast<uint16_t *>(out); a.ld_out = ld_out;
    // a task is kIters passes of 32 / (D / 8) heads, or the row's heads split
    // into equal runs of whole passes
    const int64_t hpw = 32 / (D / 8);
    const int64_t chunks = (H + hpw * kIters - 1) / (hpw * kIters);
    const int64_t chunk = ((H + chunks - 1) / chunks + hpw - 1) / hpw * hpw;
    a.H = static_cast<uint32_t>(H);
    a.chunk = static_cast<uint32_t>(chunk);
    a.chunks = make_div(static_cast<uint32_t>((H + chunk - 1) / chunk));
    a.tasks = static_cast<uint32_t>(B * S * a.chunks.d);
    a.S = make_div(static_cast<uint32_t>(S));
    a.eps = eps;
    const int d = static_cast<int>(D);
    if (in_int32) return split_half ? launch_pp<true, true>(s, a, d) : launch_pp<true, false>(s, a, d);
    return split_half ? launch_pp<false, true>(s, a, d) : launch_pp<false, false>(s, a, d);
}

}  // namespace xpuint8
