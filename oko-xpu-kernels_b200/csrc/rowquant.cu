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
//   gq[m,n] = clamp(rint(g / tg[n]), +-127).  Launches over tiles of 512
//   columns x a run of rows: zero the maxima, column abs-max (reduced per
//   tile in shared memory, then one atomicMax per column on the bit pattern
//   of a non-negative float), scale (unless pass 2 makes them), quantize.
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

// q_div on a pair of values, as packed fp32x2 operations (each lane of a
// packed operation rounds as the scalar one): the two codes in the low bytes
// of the halves.  The final add is an FMA with a unit product, because ptxas
// contracts a packed multiply feeding a packed add into one rounding.
// ns = -s, so that the exact remainder x - s q0 is one FMA.
__device__ __forceinline__ f2 q_div2(f2 x, f2 ns, f2 y) {
    const f2 q0 = mul2(x, y);
    const f2 r = fma2(q0, ns, x);  // x - s q0, exact
    return fma2(fma2(r, y, q0), mk2(1.0f, 1.0f), mk2(12582912.0f, 12582912.0f));
}

// the low bytes of four words (the codes q_div / q_div2 leave there) as one
// word, c0 in the lowest byte: three byte permutes
__device__ __forceinline__ uint32_t pack_codes4(float c0, float c1, float c2, float c3) {
    const uint32_t lo = __byte_perm(__float_as_uint(c0), __float_as_uint(c1), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(c2), __float_as_uint(c3), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
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
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();  // the consumer (a GEMM) may set up while the rows are quantized
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
            // bf16(x * bf16(col_scale)): a packed product and one conversion per pair
#pragma unroll
            for (int i = 0; i < CH * 4; ++i) {
                float a, b;
                un2(mul2(mk2(v[2 * i], v[2 * i + 1]), mk2(bf16_lo(csb[i]), bf16_hi(csb[i]))), a, b);
                round_bf16x2(a, b);
                v[2 * i] = a;
                v[2 * i + 1] = b;
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
        const f2 ns2 = mk2(-s, -s), y2 = mk2(y, y);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int ch = t + 128 * c;
            if (ch < nch) {
                float b[8];
#pragma unroll
                for (int j = 0; j < 8; j += 2)
                    un2(q_div2(mk2(v[8 * c + j], v[8 * c + j + 1]), ns2, y2), b[j], b[j + 1]);
                uint2 o;
                o.x = pack_codes4(b[0], b[1], b[2], b[3]);
                o.y = pack_codes4(b[4], b[5], b[6], b[7]);
                __stcs(reinterpret_cast<uint2 *>(qr + 8 * ch), o);
            }
        }
    }
}

// Column quantizer tiles: a 256-thread CTA covers a run of rows x 512
// columns; lane l of warp w owns the 16 columns 16 l .. 16 l + 15 of the
// tile (32 bytes of a row: a warp reads 1 KB contiguous) and the rows
// w, w + 8, ... of the run, keeping four rows of loads in flight.
constexpr int kColW = 512;     // columns per tile
constexpr int kColLanes = 8;   // rows read at once (one per warp)

// the 16 fp32 values g = dy * x of a lane's 16 columns of one row, as 8
// pairs, from the row's 32 bytes (a, b)
__device__ __forceinline__ void g16(uint4 a, uint4 b, float x, f2 (&g)[8]) {
    const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const f2 x2 = mk2(x, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = mul2(mk2(bf16_lo(u[j]), bf16_hi(u[j])), x2);
}
__device__ __forceinline__ void load_g16(const uint16_t *p, float x, f2 (&g)[8]) {
    g16(__ldcg(reinterpret_cast<const uint4 *>(p)), __ldcg(reinterpret_cast<const uint4 *>(p) + 1), x, g);
}

// Pass 1: column abs-maxima of g = dy * xs over a run of rows, reduced over
// the CTA's row lanes in shared memory and posted with one atomicMax per
// column on the bit pattern of a non-negative float into amax (zeroed
// before).  dy is read with the normal L2 policy, so that the second pass
// finds it in L2 when it fits (config C4's 42 MB does).
__global__ void __launch_bounds__(256) colamax_kernel(const uint16_t *__restrict__ dy,
                                                      const float *__restrict__ xs,
                                                      unsigned int *__restrict__ amax, int64_t M,
                                                      int64_t N, int64_t rows) {
    __shared__ float red[kColLanes][kColW];
    pdl_wait();
    pdl_trigger();
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * kColW + 16 * l;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * rows;
    const int64_t m1 = min(M, m0 + rows);
    float mx[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) mx[t] = 0.f;
    if (n < N) {
#pragma unroll 4
        for (int64_t m = m0 + w; m < m1; m += kColLanes) {
            f2 g[8];
            load_g16(dy + m * N + n, __ldg(xs + m), g);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float a, b;
                un2(g[j], a, b);
                mx[2 * j] = fmaxf(mx[2 * j], fabsf(a));
                mx[2 * j + 1] = fmaxf(mx[2 * j + 1], fabsf(b));
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 16; t += 4)
        *reinterpret_cast<float4 *>(&red[w][16 * l + t]) = make_float4(mx[t], mx[t + 1], mx[t + 2], mx[t + 3]);
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kColW / 256; ++h) {
        const int c = threadIdx.x + 256 * h;
        const int64_t col = static_cast<int64_t>(blockIdx.x) * kColW + c;
        if (col < N) {
            float v = red[0][c];
#pragma unroll
            for (int r = 1; r < kColLanes; ++r) v = fmaxf(v, red[r][c]);
            atomicMax(amax + col, __float_as_uint(v));
        }
    }
}

// the column maxima zeroed before pass 1 (a kernel rather than a memset node,
// so that pass 1 may launch while it runs)
__global__ void colzero_kernel(unsigned int *amax, int64_t N) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n < N) amax[n] = 0u;
}

// tg[n] = max(amax[n] / 127, 1e-30) in place (after the atomic form of pass 1)
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

// Pass 2: gq = clamp(rint(g / tg[n]), +-127) over a run of rows, 16 codes
// per lane and row in one 16-byte store.  FROM_AMAX: the CTA makes the scales
// of its 512 columns from the column maxima of pass 1 (amax; the CTAs of the
// first run also write them to tg); otherwise it reads them from tg.  Each
// column's reciprocal is made once per CTA, and the first four rows of each
// lane are loaded before that, so that their latency covers it.
template <bool FROM_AMAX>
__global__ void __launch_bounds__(256, 3) colquant_kernel(const uint16_t *__restrict__ dy,
                                                       const float *__restrict__ xs,
                                                       const unsigned int *__restrict__ amax,
                                                       float *__restrict__ tg, int8_t *__restrict__ gq,
                                                       int64_t M, int64_t N, int64_t rows) {
    constexpr int kAhead = 4;
    __shared__ float s_t[kColW], s_y[kColW];
    pdl_wait();
    pdl_trigger();
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * kColW + 16 * l;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * rows;
    const int64_t m1 = min(M, m0 + rows);
    uint4 pa[kAhead], pb[kAhead];
    float px[kAhead];
#pragma unroll
    for (int i = 0; i < kAhead; ++i) {
        const int64_t m = m0 + w + kColLanes * i;
        pa[i] = pb[i] = make_uint4(0u, 0u, 0u, 0u);
        px[i] = 0.f;
        if (n < N && m < m1) {
            const uint4 *p = reinterpret_cast<const uint4 *>(dy + m * N + n);
            pa[i] = __ldcg(p);
            pb[i] = __ldcg(p + 1);
            px[i] = __ldg(xs + m);
        }
    }
#pragma unroll
    for (int h = 0; h < kColW / 256; ++h) {
        const int c = threadIdx.x + 256 * h;
        const int64_t col = static_cast<int64_t>(blockIdx.x) * kColW + c;
        float t = 1.f, y = 1.f;
        if (col < N) {
            if constexpr (FROM_AMAX) {
                row_scale_inv(__uint_as_float(amax[col]), t);  // t as colscale_kernel makes it
                if (blockIdx.y == 0) tg[col] = t;
            } else {
                t = tg[col];
            }
            y = rcp_rn(t);
        }
        s_t[c] = t;
        s_y[c] = y;
    }
    __syncthreads();
    if (n >= N) return;
    f2 nt2[8], y2[8];  // -t (the remainder below is one FMA) and RN(1 / t), in pairs
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        nt2[j] = mk2(-s_t[16 * l + 2 * j], -s_t[16 * l + 2 * j + 1]);
        y2[j] = mk2(s_y[16 * l + 2 * j], s_y[16 * l + 2 * j + 1]);
    }
    const f2 one = mk2(1.0f, 1.0f), magic = mk2(12582912.0f, 12582912.0f);
    auto quant_row = [&](int64_t m, const f2 (&g)[8]) {
        float c[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            // RN(g / t) by Markstein's correction of RN(g * y), then
            // RN(q + 1.5 * 2^23), whose low byte is the code (the sum as an
            // FMA with a unit product: a packed multiply feeding a packed add
            // would be contracted into one rounding)
            const f2 q0 = mul2(g[j], y2[j]);
            const f2 r = fma2(q0, nt2[j], g[j]);  // g - q0 * t, exact
            un2(fma2(fma2(r, y2[j], q0), one, magic), c[2 * j], c[2 * j + 1]);
        }
        uint4 o;
        o.x = pack_codes4(c[0], c[1], c[2], c[3]);
        o.y = pack_codes4(c[4], c[5], c[6], c[7]);
        o.z = pack_codes4(c[8], c[9], c[10], c[11]);
        o.w = pack_codes4(c[12], c[13], c[14], c[15]);
        __stcs(reinterpret_cast<uint4 *>(gq + m * N + n), o);
    };
#pragma unroll
    for (int i = 0; i < kAhead; ++i) {
        const int64_t m = m0 + w + kColLanes * i;
        if (m < m1) {
            f2 g[8];
            g16(pa[i], pb[i], px[i], g);
            quant_row(m, g);
        }
    }
#pragma unroll 4
    for (int64_t m = m0 + w + kColLanes * kAhead; m < m1; m += kColLanes) {
        f2 g[8];
        load_g16(dy + m * N + n, __ldg(xs + m), g);
        quant_row(m, g);
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
    // programmatic serialization: the kernels wait for the one before them
    // before their first global access, and let the next one launch at once
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (ch <= 8) {
        // persistent CTAs: as many as are resident at once, at most one per row
        auto go = [&](auto kern, const float *c) {
            const int per = resident_per_sm(kern, 128);
            const int64_t grid = std::min<int64_t>(M, static_cast<int64_t>(num_sms()) * per);
            cfg.gridDim = dim3(static_cast<unsigned>(grid));
            cfg.blockDim = dim3(128);
            cudaLaunchKernelEx(&cfg, kern, xb, c, q, scale, M, K);
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
    cfg.gridDim = dim3(static_cast<unsigned>(M));
    cfg.blockDim = dim3(256);
    if (col_scale)
        cudaLaunchKernelEx(&cfg, quantize_row_kernel<true>, xb, col_scale, q, scale, K);
    else
        cudaLaunchKernelEx(&cfg, quantize_row_kernel<false>, xb, static_cast<const float *>(nullptr), q, scale, K);
    return launch_status("quantize_row");
}

int launch_colquant(cudaStream_t s, const void *dy, const float *x_scale, int8_t *gq, float *tg,
                    int64_t M, int64_t N, unsigned int *amax_ws) {
    const uint16_t *d = static_cast<const uint16_t *>(dy);
    const int64_t blocks = (N + kColW - 1) / kColW;
    // runs of rows (a multiple of the row lanes) so that each pass is about
    // one wave of resident CTAs
    auto split = [&](int per, int64_t &runs, int64_t &rows) {
        const int64_t want = std::max<int64_t>(1, static_cast<int64_t>(num_sms()) * per / blocks);
        rows = (M + want - 1) / want;
        rows = (rows + kColLanes - 1) / kColLanes * kColLanes;
        runs = (M + rows - 1) / rows;
    };
    int64_t runs_a, rows_a, runs_q, rows_q;
    split(resident_per_sm(colamax_kernel, 256), runs_a, rows_a);
    split(amax_ws ? resident_per_sm(colquant_kernel<true>, 256) : resident_per_sm(colquant_kernel<false>, 256),
          runs_q, rows_q);
    if (runs_a > 65535 || runs_q > 65535 || blocks > 0x7FFFFFFF) {
        set_error("the gradient is too large for the column quantizer");
        return 2;
    }
    unsigned int *amax = amax_ws ? amax_ws : reinterpret_cast<unsigned int *>(tg);
    // the kernels launch with programmatic serialization (each waits for the
    // one before it before touching memory)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(256);
    cfg.gridDim = dim3(static_cast<unsigned>((N + 255) / 256));
    if (cudaLaunchKernelEx(&cfg, colzero_kernel, amax, N) != cudaSuccess)
        return launch_status("colquant (zero the maxima)");
    cfg.gridDim = dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(runs_a));
    if (cudaLaunchKernelEx(&cfg, colamax_kernel, d, x_scale, amax, M, N, rows_a) != cudaSuccess)
        return launch_status("colquant (column maxima)");
    if (!amax_ws) {
        cfg.gridDim = dim3(static_cast<unsigned>((N + 255) / 256));
        if (cudaLaunchKernelEx(&cfg, colscale_kernel, tg, N) != cudaSuccess)
            return launch_status("colquant (scales)");
    }
    cfg.gridDim = dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(runs_q));
    const unsigned int *ca = amax;
    const cudaError_t e = amax_ws
        ? cudaLaunchKernelEx(&cfg, colquant_kernel<true>, d, x_scale, ca, tg, gq, M, N, rows_q)
        : cudaLaunchKernelEx(&cfg, colquant_kernel<false>, d, x_scale, ca, tg, gq, M, N, rows_q);
    if (e != cudaSuccess) return launch_status("colquant");
    return launch_status("colquant");
}

}  // namespace xpuint8
