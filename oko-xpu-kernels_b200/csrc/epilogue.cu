// Standalone dequant epilogue: int32 [M,N] (row stride acc_row_stride) ->
// bf16 [M,N], out = bf16(float(acc) * (w_scale[n] * x_scale[m]) + bias[n]).
// Reference: launch_dequant_epilogue, src/xpuint8.cpp:692-710 (and the
// row-strided entry :1038-1077).  The product and the bias add round
// separately in fp32, then one round-to-nearest-even to bf16.
//
// HBM-bound (4 B in + 2 B out per element).  Each thread handles 8 consecutive
// columns: two 16-byte accumulator loads, one 16-byte bf16 store.  A
// grid-stride loop over (row, 8-column chunk) sized to the SM count.
#include "common.cuh"
#include "internal.h"

namespace xpuint8 {
namespace {

__device__ __forceinline__ float deq(int32_t a, float ws, float xs) {
    return __fmul_rn(static_cast<float>(a), __fmul_rn(ws, xs));
}

template <bool BIAS, bool VEC>
__global__ void __launch_bounds__(256) dequant_epilogue_kernel(
    const int32_t *__restrict__ acc, uint16_t *__restrict__ out, const float *__restrict__ xs,
    const float *__restrict__ ws, const float *__restrict__ bias, int64_t M, int64_t N,
    int64_t lda) {
    const int64_t chunks = N >> 3;  // N % 16 == 0
    const int64_t total = M * chunks;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / chunks;
        const int64_t n = (i - m * chunks) << 3;
        const float x = __ldg(xs + m);
        int32_t a[8];
        if constexpr (VEC) {
            const int4 *src = reinterpret_cast<const int4 *>(acc + m * lda + n);
            const int4 a0 = __ldcs(src), a1 = __ldcs(src + 1);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) a[t] = __ldcs(acc + m * lda + n + t);
        }
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(ws + n));
        const float4 w1 = __ldg(reinterpret_cast<const float4 *>(ws + n) + 1);
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = deq(a[t], w[t], x);
        if constexpr (BIAS) {
            const float4 b0 = __ldg(reinterpret_cast<const float4 *>(bias + n));
            const float4 b1 = __ldg(reinterpret_cast<const float4 *>(bias + n) + 1);
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = __fadd_rn(v[t], b[t]);
        }
        uint4 o;
        o.x = pack_bf16x2(v[0], v[1]);
        o.y = pack_bf16x2(v[2], v[3]);
        o.z = pack_bf16x2(v[4], v[5]);
        o.w = pack_bf16x2(v[6], v[7]);
        __stcs(reinterpret_cast<uint4 *>(out + m * N + n), o);
    }
}

}  // namespace

int launch_dequant_epilogue(cudaStream_t s, const int32_t *acc, void *out, const float *x_scale,
                            const float *w_scale, const float *bias, int64_t M, int64_t N,
                            int64_t lda) {
    const int64_t total = M * (N >> 3);
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > cap) blocks = cap;
    // 16-byte vector loads need a 16-byte aligned base and a row stride that
    // keeps every row 16-byte aligned; a strided slice may not
    const bool vec = (reinterpret_cast<uintptr_t>(acc) & 15u) == 0 && (lda & 3) == 0;
    uint16_t *o = static_cast<uint16_t *>(out);
    if (bias) {
        if (vec) dequant_epilogue_kernel<true, true><<<blocks, threads, 0, s>>>(acc, o, x_scale, w_scale, bias, M, N, lda);
        else dequant_epilogue_kernel<true, false><<<blocks, threads, 0, s>>>(acc, o, x_scale, w_scale, bias, M, N, lda);
    } else {
        if (vec) dequant_epilogue_kernel<false, true><<<blocks, threads, 0, s>>>(acc, o, x_scale, w_scale, bias, M, N, lda);
        else dequant_epilogue_kernel<false, false><<<blocks, threads, 0, s>>>(acc, o, x_scale, w_scale, bias, M, N, lda);
    }
    return launch_status("dequant_epilogue");
}

}  // namespace xpuint8
