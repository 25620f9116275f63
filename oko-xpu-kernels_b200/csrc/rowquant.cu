// Quantizers without a rotation, for the gradient paths.
//
// quantize_row: per-row symmetric int8 of bf16 [M,K] (optionally of
//   bf16(x[m,k] * bf16(col_scale[k])), the column-scaled gradient of
//   linear_dx_int8).  The arithmetic is the torch chain quantize_row_torch
//   (python/xpu_kernels/int8/ops.py:320-330): scale = max(amax / 127, 1e-30),
//   q = clamp(rint(x / scale), +-127), both true IEEE divisions; the column
//   scale product follows ops.py:365 (bf16 * bf16 -> bf16).
//   For K <= 8192 a 128-thread CTA holds a row in registers (one read of the
//   input, the next row's loads in flight while this one is quantized, one
//   barrier per row); longer rows are read twice (the second read hits L2).
//
// colquant: the operand of the int8 weight gradient.  g[m,n] = dy[m,n]*xs[m]
//   (fp32), per-column tg[n] = max(amax_m |g| / 127, 1e-30),
//   gq[m,n] = clamp(rint(g / tg[n]), +-127).  Three launches over tiles of
//   128 rows x 256 columns: column abs-max (reduced per tile in shared memory,
//   then one atomicMax per column on the bit pattern of a non-negative
//   float), scale, quantize.
//
// Division.  Every x / s is RN(x / s) computed as Markstein's correction of
// the product with the correctly rounded reciprocal y = RN(1 / s) (Markstein,
// IBM J. Res. Dev. 34(1), 1990): q0 = RN(x y), r = x - s q0 (exact in one
// FMA), RN(q0 + r y).  For the row quantizer the operands are bf16 values and
// RN(bf16 / 127) divisors, 2^31 pairs in all, and xpuint8_check_scale_math
// compares every one of them with the IEEE division; the column quantizer's
// quotients are checked against it on pseudo-random pairs.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

// the code rint(x / s) given y = RN(1 / s), for |x| <= the maximum s was made
// from (so |x / s| <= 127 + ulps): the low byte of RN(x / s) + 1.5 * 2^23
// (round to nearest even by the fp32 add, no conversion instruction)
__device__ __forceinline__ uint32_t q_div(float x, float s, float y) {
    return __float_as_uint(__fadd_rn(div_by_rcp(x, s, y), 12582912.0f)) & 0xFFu;
}

template <bool COLSCALE>
__device__ __forceinline__ void load8(const uint16_t *x, const float *cs, int64_t k, float (&v)[8]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(x + k);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf16_lo(u[j]);
        v[2 * j + 1] = bf16_hi(u[j]);
    }
    if constexpr (COLSCALE) {
        const float4 c0 = __ldg(reinterpret_cast<const float4 *>(cs + k));
        const float4 c1 = __ldg(reinterpret_cast<const float4 *>(cs + k) + 1);
        const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = round_bf16(__fmul_rn(v[t], round_bf16(c[t])));
    }
}

template <bool COLSCALE>
__global__ void __launch_bounds__(256) quantize_row_kernel(const uint16_t *__restrict__ x,
                                                           const float *__restrict__ cs,
                                                           int8_t *__restrict__ q,
                                                           float *__restrict__ scale, int64_t K) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    const uint16_t *xr = x + row * K;
    int8_t *qr = q + row * K;
    const int64_t kv = K & ~static_cast<int64_t>(7);
    float amax = 0.f;
    for (int64_t k = threadIdx.x * 8; k < kv; k += blockDim.x * 8) {
        float v[8];
        load8<COLSCALE>(xr, cs, k, v);
#pragma unroll
        for (int t = 0; t < 8; ++t) amax = fmaxf(amax, fabsf(v[t]));
    }
    for (int64_t k = kv + threadIdx.x; k < K; k += blockDim.x) {
        float v = bf16_bits_to_f32(xr[k]);
        if constexpr (COLSCALE) v = round_bf16(__fmul_rn(v, round_bf16(cs[k])));
        amax = fmaxf(amax, fabsf(v));
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float rm = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) rm = fmaxf(rm, red[w]);
    float s;
    const float y = row_scale_inv(rm, s);
    if (threadIdx.x == 0) scale[row] = s;
    for (int64_t k = threadIdx.x * 8; k < kv; k += blockDim.x * 8) {
        float v[8];
        load8<COLSCALE>(xr, cs, k, v);
        uint2 o;
        uint32_t b[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) b[t] = q_div(v[t], s, y);
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
        *reinterpret_cast<uint2 *>(qr + k) = o;
    }
    for (int64_t k = kv + threadIdx.x; k < K; k += blockDim.x) {
        float v = bf16_bits_to_f32(xr[k]);
        if constexpr (COLSCALE) v = round_bf16(__fmul_rn(v, round_bf16(cs[k])));
        qr[k] = static_cast<int8_t>(q_div(v, s, y));
    }
}

// Register-resident form for K <= 8192: a 128-thread CTA per row at a time
// (persistent over rows); thread t owns the 8-element chunks t, t + 128, ...
// (CH of them).  The next row's loads are issued before this row is
// quantized; one barrier per row (double-buffered warp maxima).
template <bool COLSCALE, int CH>
__global__ void __launch_bounds__(128) quantize_row_reg_kernel(const uint16_t *__restrict__ x,
                                                               const float *__restrict__ cs,
                                                               int8_t *__restrict__ q,
                                                               float *__restrict__ scale,
                                                               int64_t M, int64_t K) {
    __shared__ float red[2][4];
    const int t = threadIdx.x;
    const int nch = static_cast<int>(K >> 3);
    uint32_t csb[COLSCALE ? CH * 4 : 1];  // bf16(col_scale) of this thread's columns, in pairs
    if constexpr (COLSCALE) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int ch = t + 128 * c;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                csb[4 * c + j] = ch < nch ? pack_bf16x2(__ldg(cs + 8 * ch + 2 * j), __ldg(cs + 8 * ch + 2 * j + 1)) : 0u;
        }
    }
    auto load = [&](int64_t row, uint4 (&raw)[CH]) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + row * K);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int ch = t + 128 * c;
            raw[c] = (row < M && ch < nch) ? __ldcs(src + ch) : make_uint4(0, 0, 0, 0);
        }
    };
    uint4 raw[CH];
    load(blockIdx.x, raw);
    int k = 0;
    for (int64_t row = blockIdx.x; row < M; row += gridDim.x, ++k) {
        float v[CH * 8];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const uint32_t u[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[8 * c + 2 * j] = bf16_lo(u[j]);
                v[8 * c + 2 * j + 1] = bf16_hi(u[j]);
            }
        }
        if constexpr (COLSCALE) {
#pragma unroll
            for (int i = 0; i < CH * 4; ++i) {
                v[2 * i] = round_bf16(__fmul_rn(v[2 * i], bf16_lo(csb[i])));
                v[2 * i + 1] = round_bf16(__fmul_rn(v[2 * i + 1], bf16_hi(csb[i])));
            }
        }
        load(row + gridDim.x, raw);  // the next row's loads fly meanwhile
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < CH * 8; i += 2) amax = max3_abs(amax, v[i], v[i + 1]);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        if ((t & 31) == 0) red[k & 1][t >> 5] = amax;
        __syncthreads();
        const float rm = fmaxf(fmaxf(red[k & 1][0], red[k & 1][1]), fmaxf(red[k & 1][2], red[k & 1][3]));
        float s;
        const float y = row_scale_inv(rm, s);
        if (t == 0) scale[row] = s;
        int8_t *qr = q + row * K;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int ch = t + 128 * c;
            if (ch < nch) {
                uint32_t b[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    b[j] = q_div(v[8 * c + j], s, y);
                }
                uint2 o;
                o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
                o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
                __stcs(reinterpret_cast<uint2 *>(qr + 8 * ch), o);
            }
        }
    }
}

// Column quantizer tiles: a 256-thread CTA covers kColRows rows x 256
// columns; thread (ty, tx) = (threadIdx.x / 32, threadIdx.x % 32) owns the 8
// columns 8 tx .. 8 tx + 7 of the tile and the rows ty, ty + 8, ... of it, so
// a warp reads 512 contiguous bytes of a row and keeps four loads in flight.
constexpr int kColRows = 128;

// column abs-max of g = dy * xs: a CTA reduces its tile over rows in shared
// memory and posts one atomicMax per column (on the bit pattern of a
// non-negative float).  dy is read with the normal L2 policy: the second pass
// (colquant_kernel) reads it again, from L2 when it fits (the C4 gradient,
// 42 MB, does), and streams it out of the cache there.
__global__ void __launch_bounds__(256) colamax_kernel(const uint16_t *__restrict__ dy,
                                                      const float *__restrict__ xs,
                                                      unsigned int *__restrict__ amax,
                                                      int64_t M, int64_t N) {
    __shared__ float red[8][256];
    pdl_wait();
    pdl_trigger();
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 256 + 8 * tx;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kColRows;
    const int64_t m1 = min(M, m0 + kColRows);
    float mx[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (n < N) {
#pragma unroll 8
        for (int64_t m = m0 + ty; m < m1; m += 8) {
            const float x = __ldg(xs + m);
            const uint4 w = __ldcg(reinterpret_cast<const uint4 *>(dy + m * N + n));
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                mx[2 * j] = fmaxf(mx[2 * j], fabsf(__fmul_rn(bf16_lo(u[j]), x)));
                mx[2 * j + 1] = fmaxf(mx[2 * j + 1], fabsf(__fmul_rn(bf16_hi(u[j]), x)));
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) red[ty][8 * tx + t] = mx[t];
    __syncthreads();
    const int64_t c = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (c < N) {
        float v = red[0][threadIdx.x];
#pragma unroll
        for (int r = 1; r < 8; ++r) v = fmaxf(v, red[r][threadIdx.x]);
        atomicMax(amax + c, __float_as_uint(v));
    }
}

__global__ void colscale_kernel(float *tg, int64_t N) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n < N) {
        float s;
        row_scale_inv(tg[n], s);
        tg[n] = s;
    }
}

// gq = clamp(rint(g / tg[n]), +-127), g = dy * xs; each thread's 8 column
// reciprocals are computed once
__global__ void __launch_bounds__(256) colquant_kernel(const uint16_t *__restrict__ dy,
                                                       const float *__restrict__ xs,
                                                       const float *__restrict__ tg,
                                                       int8_t *__restrict__ gq, int64_t M,
                                                       int64_t N) {
    pdl_wait();
    pdl_trigger();
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 256 + 8 * tx;
    if (n >= N) return;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kColRows;
    const int64_t m1 = min(M, m0 + kColRows);
    float t[8], y[8];
    {
        const float4 t0 = __ldg(reinterpret_cast<const float4 *>(tg + n));
        const float4 t1 = __ldg(reinterpret_cast<const float4 *>(tg + n) + 1);
        t[0] = t0.x; t[1] = t0.y; t[2] = t0.z; t[3] = t0.w;
        t[4] = t1.x; t[5] = t1.y; t[6] = t1.z; t[7] = t1.w;
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = rcp_rn(t[j]);
    }
#pragma unroll 4
    for (int64_t m = m0 + ty; m < m1; m += 8) {
        const float x = __ldg(xs + m);
        const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(dy + m * N + n));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        uint32_t b[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            b[2 * j] = q_div(__fmul_rn(bf16_lo(u[j]), x), t[2 * j], y[2 * j]);
            b[2 * j + 1] = q_div(__fmul_rn(bf16_hi(u[j]), x), t[2 * j + 1], y[2 * j + 1]);
        }
        uint2 o;
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
        __stcs(reinterpret_cast<uint2 *>(gq + m * N + n), o);
    }
}

}  // namespace

namespace {
// resident CTAs per SM of a kernel (no dynamic shared memory), cached per kernel
template <typename Kern>
int resident_per_sm(Kern kern, int threads) {
    struct Entry {
        const void *fn;
        int per;
    };
    static Entry cache[32] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    const void *fn = reinterpret_cast<const void *>(kern);
    int i = 0;
    for (; i < 32 && cache[i].fn; ++i)
        if (cache[i].fn == fn) return cache[i].per;
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, threads, 0) != cudaSuccess || per < 1) per = 1;
    if (i < 32) cache[i] = {fn, per};
    return per;
}
}  // namespace

int launch_quantize_row(cudaStream_t s, const void *x, const float *col_scale, int8_t *q,
                        float *scale, int64_t M, int64_t K) {
    if (M > 0x7FFFFFFF) {
        set_error("M is too large");
        return 2;
    }
    const bool vec_ok = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                        (reinterpret_cast<uintptr_t>(q) & 7u) == 0 && (K & 7) == 0 &&
                        (!col_scale || (reinterpret_cast<uintptr_t>(col_scale) & 15u) == 0);
    if (!vec_ok) {
        set_error("quantize_row needs 16-byte aligned rows (K % 8 == 0 and aligned pointers)");
        return 2;
    }
    const uint16_t *xb = static_cast<const uint16_t *>(x);
    const int64_t nch = K / 8;
    const int ch = static_cast<int>((nch + 127) / 128);
    if (ch <= 8) {
        // persistent CTAs: as many as are resident at once, at most one per row
        auto go = [&](auto kern, const float *c) {
            const int per = resident_per_sm(kern, 128);
            const int64_t grid = std::min<int64_t>(M, static_cast<int64_t>(num_sms()) * per);
            kern<<<static_cast<unsigned>(grid), 128, 0, s>>>(xb, c, q, scale, M, K);
        };
#define XPU_RQ_CASE(C)                                                     \
    case C:                                                                \
        if (col_scale) go(quantize_row_reg_kernel<true, C>, col_scale);    \
        else go(quantize_row_reg_kernel<false, C>, nullptr);               \
        break;
        switch (ch) {
            XPU_RQ_CASE(1)
            XPU_RQ_CASE(2)
            XPU_RQ_CASE(3)
            XPU_RQ_CASE(4)
            XPU_RQ_CASE(5)
            XPU_RQ_CASE(6)
            XPU_RQ_CASE(7)
            XPU_RQ_CASE(8)
            default: break;
        }
#undef XPU_RQ_CASE
        return launch_status("quantize_row");
    }
    if (col_scale)
        quantize_row_kernel<true><<<static_cast<unsigned>(M), 256, 0, s>>>(xb, col_scale, q, scale, K);
    else
        quantize_row_kernel<false><<<static_cast<unsigned>(M), 256, 0, s>>>(xb, nullptr, q, scale, K);
    return launch_status("quantize_row");
}

int launch_colquant(cudaStream_t s, const void *dy, const float *x_scale, int8_t *gq, float *tg,
                    int64_t M, int64_t N) {
    const uint16_t *d = static_cast<const uint16_t *>(dy);
    if ((M + kColRows - 1) / kColRows > 65535) {
        set_error("M is too large for the column quantizer");
        return 2;
    }
    if (cudaMemsetAsync(tg, 0, static_cast<size_t>(N) * sizeof(float), s) != cudaSuccess)
        return launch_status("colquant memset");
    const dim3 grid(static_cast<unsigned>((N + 255) / 256), static_cast<unsigned>((M + kColRows - 1) / kColRows));
    // the three kernels launch with programmatic serialization (each waits
    // for the one before it before touching memory)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(256);
    cfg.gridDim = grid;
    unsigned int *amax = reinterpret_cast<unsigned int *>(tg);
    if (cudaLaunchKernelEx(&cfg, colamax_kernel, d, x_scale, amax, M, N) != cudaSuccess)
        return launch_status("colquant (column maxima)");
    cfg.gridDim = dim3(static_cast<unsigned>((N + 255) / 256));
    if (cudaLaunchKernelEx(&cfg, colscale_kernel, tg, N) != cudaSuccess)
        return launch_status("colquant (scales)");
    cfg.gridDim = grid;
    if (cudaLaunchKernelEx(&cfg, colquant_kernel, d, x_scale, static_cast<const float *>(tg), gq, M, N) !=
        cudaSuccess)
        return launch_status("colquant");
    return launch_status("colquant");
}

}  // namespace xpuint8
