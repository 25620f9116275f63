// Quantizers without a rotation, for the gradient paths.
//
// quantize_row: per-row symmetric int8 of bf16 [M,K] (optionally of
//   bf16(x[m,k] * bf16(col_scale[k])), the column-scaled gradient of
//   linear_dx_int8).  The arithmetic is the torch chain quantize_row_torch
//   (python/xpu_kernels/int8/ops.py:320-330): scale = max(amax / 127, 1e-30),
//   q = clamp(rint(x / scale), +-127), both true IEEE divisions; the column
//   scale product follows ops.py:365 (bf16 * bf16 -> bf16).
//   One CTA per row; the row is read twice (the second read hits L2).
//
// colquant: the operand of the int8 weight gradient.  g[m,n] = dy[m,n]*xs[m]
//   (fp32), per-column tg[n] = max(amax_m |g| / 127, 1e-30),
//   gq[m,n] = clamp(rint(g / tg[n]), +-127).  Three launches: column abs-max
//   (atomicMax on the bit pattern of a non-negative float), scale, quantize.
#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

__device__ __forceinline__ int8_t q_div(float x, float s) {
    const float r = rintf(__fdiv_rn(x, s));
    return static_cast<int8_t>(fmaxf(-127.f, fminf(127.f, r)));
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
    const float s = fmaxf(__fdiv_rn(rm, 127.0f), 1e-30f);
    if (threadIdx.x == 0) scale[row] = s;
    for (int64_t k = threadIdx.x * 8; k < kv; k += blockDim.x * 8) {
        float v[8];
        load8<COLSCALE>(xr, cs, k, v);
        uint2 o;
        uint32_t b[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) b[t] = static_cast<uint8_t>(q_div(v[t], s));
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
        *reinterpret_cast<uint2 *>(qr + k) = o;
    }
    for (int64_t k = kv + threadIdx.x; k < K; k += blockDim.x) {
        float v = bf16_bits_to_f32(xr[k]);
        if constexpr (COLSCALE) v = round_bf16(__fmul_rn(v, round_bf16(cs[k])));
        qr[k] = q_div(v, s);
    }
}

// column abs-max of g = dy * xs over a strip of rows; 8 columns per thread
__global__ void __launch_bounds__(256) colamax_kernel(const uint16_t *__restrict__ dy,
                                                      const float *__restrict__ xs,
                                                      unsigned int *__restrict__ amax,
                                                      int64_t M, int64_t N, int rows_per_cta) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (n >= N) return;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * rows_per_cta;
    const int64_t m1 = min(M, m0 + rows_per_cta);
    float mx[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t m = m0; m < m1; ++m) {
        const float x = __ldg(xs + m);
        const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(dy + m * N + n));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            mx[2 * j] = fmaxf(mx[2 * j], fabsf(__fmul_rn(bf16_lo(u[j]), x)));
            mx[2 * j + 1] = fmaxf(mx[2 * j + 1], fabsf(__fmul_rn(bf16_hi(u[j]), x)));
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) atomicMax(amax + n + t, __float_as_uint(mx[t]));
}

__global__ void colscale_kernel(float *tg, int64_t N) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n < N) tg[n] = fmaxf(__fdiv_rn(tg[n], 127.0f), 1e-30f);
}

__global__ void __launch_bounds__(256) colquant_kernel(const uint16_t *__restrict__ dy,
                                                       const float *__restrict__ xs,
                                                       const float *__restrict__ tg,
                                                       int8_t *__restrict__ gq, int64_t M,
                                                       int64_t N) {
    const int64_t chunks = N >> 3;
    const int64_t total = M * chunks;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / chunks;
        const int64_t n = (i - m * chunks) << 3;
        const float x = __ldg(xs + m);
        const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(dy + m * N + n));
        const float4 t0 = __ldg(reinterpret_cast<const float4 *>(tg + n));
        const float4 t1 = __ldg(reinterpret_cast<const float4 *>(tg + n) + 1);
        const float t[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        uint32_t b[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            b[2 * j] = static_cast<uint8_t>(q_div(__fmul_rn(bf16_lo(u[j]), x), t[2 * j]));
            b[2 * j + 1] = static_cast<uint8_t>(q_div(__fmul_rn(bf16_hi(u[j]), x), t[2 * j + 1]));
        }
        uint2 o;
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
        __stcs(reinterpret_cast<uint2 *>(gq + m * N + n), o);
    }
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
    if (col_scale)
        quantize_row_kernel<true><<<static_cast<unsigned>(M), 256, 0, s>>>(xb, col_scale, q, scale, K);
    else
        quantize_row_kernel<false><<<static_cast<unsigned>(M), 256, 0, s>>>(xb, nullptr, q, scale, K);
    return launch_status("quantize_row");
}

int launch_colquant(cudaStream_t s, const void *dy, const float *x_scale, int8_t *gq, float *tg,
                    int64_t M, int64_t N) {
    const uint16_t *d = static_cast<const uint16_t *>(dy);
    if (cudaMemsetAsync(tg, 0, static_cast<size_t>(N) * sizeof(float), s) != cudaSuccess)
        return launch_status("colquant memset");
    const int rows_per_cta = 64;
    dim3 grid1(static_cast<unsigned>((N / 8 + 255) / 256),
               static_cast<unsigned>((M + rows_per_cta - 1) / rows_per_cta));
    colamax_kernel<<<grid1, 256, 0, s>>>(d, x_scale, reinterpret_cast<unsigned int *>(tg), M, N,
                                          rows_per_cta);
    colscale_kernel<<<static_cast<unsigned>((N + 255) / 256), 256, 0, s>>>(tg, N);
    const int64_t total = M * (N >> 3);
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > cap) blocks = cap;
    colquant_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, x_scale, tg, gq, M, N);
    return launch_status("colquant");
}

}  // namespace xpuint8
