// The rotation family, streaming form (modes 0, 2, 3 of rotate.cu):
//
//   mode 0  bf16 [M,K] ([M,2K] paired) -> act -> rotate -> int8 [M,K] + scale [M]
//           (reference: launch_convrot_quant_warp<ACT>, src/xpuint8.cpp:450-502)
//   mode 2  bf16 [M,K] -> rotate -> bf16 [M,K]  (launch_rotate_bf16, :588-635)
//   mode 3  int8 [N,K] * scale [N] -> bf16 -> rotate -> bf16 [N,K]
//           (dequant_weight_torch, python/xpu_kernels/int8/ops.py:169-191)
//
// Three kernels.  rotate_quant4_kernel is the quantizer without activation for
// K a multiple of 1024 up to 8192 (four groups per half-warp);
// rotate_direct_kernel (K <= 8192) every other mode, activation and row width
// the linear entries meet; both are described above them.  rotate_bulk_kernel serves longer rows
// (K up to 32768 in slots of 1, 2 or 4 pairs of groups): persistent CTAs walk
// "batches" of R consecutive rows, load each group straight from global memory
// into registers, and stage the result in shared memory in its final order, so
// that a batch leaves with one bulk store (cp.async.bulk) per CTA.
//
// Arithmetic: a half-warp ("slot") owns PAIRS of 256-groups and processes the
// two groups of a pair together as packed fp32x2 values, so every butterfly
// step is one add/sub.f32x2 for two elements.  Lane l first holds elements
// 16l..16l+15 of both groups (digits i0, i1 in registers: axes 0 and 1 in the
// accumulation-chain association of the reference's `inreg`), a swizzled
// 2 KB shared-memory transpose then gives it elements 16w + l, w = 0..15
// (digits i2, i3 in registers: axes 2 and 3 in the butterfly association of
// `bfly_xor`).  Same association and rounding as rotate.cu, so the two kernels
// produce the same bits; the per-stage 1/2 factors are applied once as 1/16.
//
// Row abs-max: per-group maxima go through shared-memory atomics into a
// triple-buffered per-row array; quantization (reciprocal multiply, RNE by an
// fp32 magic add) happens after one CTA barrier.  Neither kernel waits on an
// mbarrier or on another CTA: every barrier is a CTA barrier.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <string>

#include "act.cuh"
#include "common.cuh"
#include "internal.h"

namespace xpuint8 {

namespace {

constexpr int kSlots = 16;             // half-warps per 256-thread CTA
constexpr int kCacheDevices = 64;      // devices whose occupancy is cached
constexpr int kTileBytes = 16 * 128;   // 16 rows x 16 fp32x2 per slot

struct BulkParams {
    const uint8_t *in;
    const float *row_scale;  // mode 3: the weight's per-row scale; mode 1: x_scale [M]
    const float *col_scale;  // mode 1: the weight scale [K] or [2K]
    uint8_t *out;
    float *scale;            // mode 0: per-row output scale
    int64_t M, K;
    int G, R, nbatch, os;    // os: output stages (1 or 2)
    uint32_t in_row_bytes, out_row_bytes;
    uint32_t out_stage_bytes;
};


// the 16 values lane l owns of one group, loaded from global memory (row = absolute row)
template <int MODE, int ACT>
__device__ __forceinline__ void load16_global(const BulkParams &p, int64_t row, int g, int l,
                                              float (&v)[16]) {
    if constexpr (MODE == 3) {
        const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(p.in + row * p.in_row_bytes + g * 256 + l * 16));
        const float s = __ldg(p.row_scale + row);
        const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int t = 0; t < 4; ++t)
                v[4 * j + t] = round_bf16(
                    __fmul_rn(static_cast<float>(static_cast<int8_t>((w[j] >> (8 * t)) & 0xFF)), s));
    } else {
        const uint4 *base = reinterpret_cast<const uint4 *>(p.in + row * p.in_row_bytes + (g * 256 + l * 16) * 2);
        const uint4 a0 = __ldcs(base), a1 = __ldcs(base + 1);
        unpack16_bf16(a0, a1, v);
        if constexpr (MODE == 0 && act_paired(ACT)) {
            const uint4 *hb = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(base) + p.K * 2);
            const uint4 b0 = __ldcs(hb), b1 = __ldcs(hb + 1);
            float u[16];
            unpack16_bf16(b0, b1, u);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], u[t]);
        } else if constexpr (MODE == 0 && ACT != 0) {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], 0.f);
        }
    }
}

// accumulation-chain radix-4 butterfly (unscaled) on fp32x2 lanes
__device__ __forceinline__ void seq2(f2 &a0, f2 &a1, f2 &a2, f2 &a3) {
    const f2 p = add2(a0, a1), m = sub2(a0, a1);
    const f2 o0 = sub2(add2(p, a2), a3);
    const f2 o1 = add2(sub2(p, a2), a3);
    const f2 o2 = add2(add2(m, a2), a3);
    const f2 o3 = add2(sub2(a2, m), a3);
    a0 = o0; a1 = o1; a2 = o2; a3 = o3;
}
// butterfly-association radix-4 butterfly (unscaled) on fp32x2 lanes
__device__ __forceinline__ void bfly2(f2 &a0, f2 &a1, f2 &a2, f2 &a3) {
    const f2 p = add2(a0, a1), m = sub2(a0, a1);
    const f2 q = add2(a2, a3), n = sub2(a2, a3);
    a0 = add2(p, n); a1 = sub2(p, n); a2 = add2(m, q); a3 = sub2(q, m);
}

// Rotate a pair of groups.  In: P[q] = (A[16l+q], B[16l+q]).  Out: P[w] =
// (A[16w+l], B[16w+l]), unscaled (x16).  `tile` is the slot's 2 KB tile.
__device__ __forceinline__ void rotate_pair(f2 (&P)[16], uint32_t tile, int l) {
#pragma unroll
    for (int j = 0; j < 4; ++j) seq2(P[4 * j], P[4 * j + 1], P[4 * j + 2], P[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) seq2(P[j], P[j + 4], P[j + 8], P[j + 12]);
    // row l <- P (128 bytes, 16-byte chunk c at c ^ (l & 7)); then read column l
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float a0, b0, a1, b1;
        un2(P[2 * c], a0, b0);
        un2(P[2 * c + 1], a1, b1);
        st_shared_v4(tile + l * 128 + ((c ^ (l & 7)) << 4), __float_as_uint(a0), __float_as_uint(b0),
                     __float_as_uint(a1), __float_as_uint(b1));
    }
    __syncwarp();
#pragma unroll
    for (int w = 0; w < 16; ++w) {
        const uint32_t addr = tile + w * 128 + ((((l >> 1) ^ w) & 7) << 4) + ((l & 1) << 3);
        asm volatile("ld.shared.b64 %0, [%1];" : "=l"(P[w].v) : "r"(addr));
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly2(P[4 * j], P[4 * j + 1], P[4 * j + 2], P[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly2(P[j], P[j + 4], P[j + 8], P[j + 12]);
}

// max over the 16 lanes of this thread's half-warp.  The mask names only that
// half: the two slots of a warp may take different paths (a pair inside one
// row reduces once, a pair across two rows twice), and a full-warp mask would
// make them wait for each other's shuffles forever.
__device__ __forceinline__ float halfwarp_max(float v) {
    const unsigned mask = 0xFFFFu << (threadIdx.x & 16u);
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(mask, v, m));
    return v;
}

template <int MODE, int ACT, int PPS>
__global__ void __launch_bounds__(256, (PPS == 1 ? 4 : 1)) rotate_bulk_kernel(const BulkParams p) {
    constexpr bool QUANT = (MODE == 0);
    extern __shared__ __align__(128) uint8_t smem[];
    // shared memory: the output stages, the slots' transpose tiles, the row maxima
    const uint32_t out_base = smem_u32(smem);
    const uint32_t tile_base = out_base + p.os * p.out_stage_bytes;
    unsigned int *row_amax =
        reinterpret_cast<unsigned int *>(smem + p.os * p.out_stage_bytes + kSlots * kTileBytes);

    const int slot = threadIdx.x >> 4, l = threadIdx.x & 15;
    const uint32_t tile = tile_base + slot * kTileBytes;
    const int groups = p.R * p.G;

    if (threadIdx.x < 3 * 32) row_amax[threadIdx.x] = 0u;
    __syncthreads();

    auto batch_rows = [&](int b) -> int {
        const int64_t r0 = static_cast<int64_t>(b) * p.R;
        const int64_t left = p.M - r0;
        return static_cast<int>(left < p.R ? left : p.R);
    };

    int k = 0;
    for (int b = blockIdx.x; b < p.nbatch; b += gridDim.x, ++k) {
        const int rows = batch_rows(b);
        const int64_t row0 = static_cast<int64_t>(b) * p.R;
        unsigned int *amax_now = row_amax + 32 * (k % 3);

        f2 vals[PPS][16];
#pragma unroll
        for (int j = 0; j < PPS; ++j) {
            const int f0 = 2 * (slot + kSlots * j), f1 = f0 + 1;
            const int r0 = f0 / p.G, g0 = f0 - r0 * p.G;
            const int r1 = f1 / p.G, g1 = f1 - r1 * p.G;
            const bool v0 = f0 < groups && r0 < rows, v1 = f1 < groups && r1 < rows;
            float a[16], c[16];
            if (v0) {
                load16_global<MODE, ACT>(p, row0 + r0, g0, l, a);
            } else {
#pragma unroll
                for (int t = 0; t < 16; ++t) a[t] = 0.f;
            }
            if (v1) {
                load16_global<MODE, ACT>(p, row0 + r1, g1, l, c);
            } else {
#pragma unroll
                for (int t = 0; t < 16; ++t) c[t] = 0.f;
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) vals[j][t] = mk2(a[t], c[t]);
            rotate_pair(vals[j], tile, l);
            if constexpr (QUANT) {
                float m0 = 0.f, m1 = 0.f;
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    float x0, x1;
                    un2(vals[j][t], x0, x1);
                    m0 = fmaxf(m0, fabsf(x0));
                    m1 = fmaxf(m1, fabsf(x1));
                }
                m0 = halfwarp_max(m0);
                m1 = halfwarp_max(m1);
                if (l == 0) {
                    if (v0) atomicMax(amax_now + r0, __float_as_uint(m0));
                    if (v1) atomicMax(amax_now + r1, __float_as_uint(m1));
                }
            }
        }
        if constexpr (QUANT) {
            if (threadIdx.x < 32) row_amax[32 * ((k + 1) % 3) + threadIdx.x] = 0u;
        }
        // the output stage this batch fills has been read by its last store
        if (threadIdx.x == 0) {
            if (p.os == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
        }
        __syncthreads();

        const uint32_t ostage = out_base + (k % p.os) * p.out_stage_bytes;
#pragma unroll
        for (int j = 0; j < PPS; ++j) {
            const int f0 = 2 * (slot + kSlots * j), f1 = f0 + 1;
            const int r0 = f0 / p.G, g0 = f0 - r0 * p.G;
            const int r1 = f1 / p.G, g1 = f1 - r1 * p.G;
            const bool v0 = f0 < groups && r0 < rows, v1 = f1 < groups && r1 < rows;
            if constexpr (QUANT) {
                float inv0 = 0.f, inv1 = 0.f;
                if (v0) {
                    const float s = fmaxf(__fdiv_rn(__fmul_rn(__uint_as_float(amax_now[r0]), 0.0625f), 127.0f), 1e-30f);
                    inv0 = __fmul_rn(__frcp_rn(s), 0.0625f);
                    if (g0 == 0 && l == 0) p.scale[row0 + r0] = s;
                }
                if (v1) {
                    const float s = fmaxf(__fdiv_rn(__fmul_rn(__uint_as_float(amax_now[r1]), 0.0625f), 127.0f), 1e-30f);
                    inv1 = __fmul_rn(__frcp_rn(s), 0.0625f);
                    if (g1 == 0 && l == 0) p.scale[row0 + r1] = s;
                }
                const f2 magic = mk2(12582912.0f, 12582912.0f);
                // an invalid group of a pair writes into the slot's transpose
                // tile (free at this point, rewritten before its next read),
                // so the loop has no per-element branch
                const uint32_t o0 = v0 ? ostage + r0 * p.out_row_bytes + g0 * 256 + l : tile + l;
                const uint32_t o1 = v1 ? ostage + r1 * p.out_row_bytes + g1 * 256 + l : tile + l;
#pragma unroll
                for (int w = 0; w < 16; ++w) {
                    // rint(v * (1/s)): |v/s| <= 127 (+ulps), so the low byte of
                    // (v/s + 1.5*2^23) is the two's-complement code.  The
                    // products are scalar __fmul_rn: ptxas contracts a packed
                    // f32x2 multiply feeding a packed add into one FFMA2, which
                    // would round v*(1/s) + 1.5*2^23 once instead of twice.
                    float x0, x1, q0, q1;
                    un2(vals[j][w], x0, x1);
                    un2(add2(mk2(__fmul_rn(x0, inv0), __fmul_rn(x1, inv1)), magic), q0, q1);
                    asm volatile("st.shared.u8 [%0], %1;" ::"r"(o0 + 16 * w), "r"(__float_as_uint(q0)) : "memory");
                    asm volatile("st.shared.u8 [%0], %1;" ::"r"(o1 + 16 * w), "r"(__float_as_uint(q1)) : "memory");
                }
            } else {
                const f2 sixteenth = mk2(0.0625f, 0.0625f);
                const uint32_t o0 = v0 ? ostage + r0 * p.out_row_bytes + (g0 * 256 + l) * 2 : tile + 2 * l;
                const uint32_t o1 = v1 ? ostage + r1 * p.out_row_bytes + (g1 * 256 + l) * 2 : tile + 2 * l;
#pragma unroll
                for (int w = 0; w < 16; ++w) {
                    float x0, x1;
                    un2(mul2(vals[j][w], sixteenth), x0, x1);
                    const uint32_t hb = cvt_bf16x2(x0, x1);
                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(o0 + 32 * w), "r"(hb & 0xFFFFu) : "memory");
                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(o1 + 32 * w), "r"(hb >> 16) : "memory");
                }
            }
        }
        fence_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            bulk_store(p.out + row0 * p.out_row_bytes, ostage, rows * p.out_row_bytes);
            bulk_commit();
        }
    }
    if (threadIdx.x == 0) bulk_wait<0>();
    __syncthreads();
}

// The hot form of the family for K <= 8192: one pair of groups per slot, the
// batch's R rows laid out over the 16 slots once per CTA (no per-batch index
// arithmetic), global loads straight into registers one batch ahead (the
// next batch's loads are in flight while this one is transformed).
//
// Per slot, shared memory holds the transpose tile (16 rows of 128 bytes at a
// 144-byte pitch, so every access is a base register plus an immediate and a
// half-warp's row writes and column reads are conflict-free), two output
// buffers of one pair of groups, and 32 bytes of skew that put the two slots
// of a warp on different banks.  A batch's groups are consecutive in the
// dense output, so each slot writes its pair back with its own bulk copy from
// its own buffer: the CTA synchronises once per batch, for the row abs-max.
// Lane l's input of one group: 16 elements, as bf16 (modes 0, 2), int8 (mode
// 3) or int32 accumulators (mode 1); paired activations also carry the
// second half (the gate, or SwiGLU's up).
template <int MODE, int ACT>
struct GroupIn {
    static constexpr int kPaired = (MODE <= 1 && act_paired(ACT)) ? 2 : 1;
    static constexpr int kVec = MODE == 3 ? 1 : (MODE == 1 ? 4 : 2);  // uint4 per half
    uint4 v[kPaired * kVec];
};
template <int MODE, int ACT>
struct RawPair {
    GroupIn<MODE, ACT> a, b;  // the slot's two groups
};

constexpr int kPitch = 144;                 // transpose tile row pitch (128 data + 16 skew)
constexpr int kTileP = 16 * kPitch;         // 2304 bytes
__host__ __device__ constexpr int group_out_bytes(int mode) { return mode <= 1 ? 256 : 512; }
__host__ __device__ constexpr int slot_bytes(int mode) {
    return kTileP + 4 * group_out_bytes(mode) + 32;
}

// lane l's 16 elements of a group at p (and, paired, at p + half bytes)
template <int MODE, int ACT>
__device__ __forceinline__ void load_group(const uint8_t *p, bool valid, uint32_t half,
                                           GroupIn<MODE, ACT> &g) {
    using G = GroupIn<MODE, ACT>;
    if (!valid) return;
    const uint4 *s = reinterpret_cast<const uint4 *>(p);
#pragma unroll
    for (int i = 0; i < G::kVec; ++i) g.v[i] = __ldcs(s + i);
    if constexpr (G::kPaired == 2) {
        const uint4 *h = reinterpret_cast<const uint4 *>(p + half);
#pragma unroll
        for (int i = 0; i < G::kVec; ++i) g.v[G::kVec + i] = __ldcs(h + i);
    }
}

// dequant of 4 accumulators: bf16(float(acc) * (w * xs)), the unfused chain's
// rounding (src/xpuint8.cpp:246-248)
__device__ __forceinline__ void dequant4(const uint4 &a, const float4 &w, float xs, float *h) {
    h[0] = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(a.x)), __fmul_rn(w.x, xs)));
    h[1] = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(a.y)), __fmul_rn(w.y, xs)));
    h[2] = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(a.z)), __fmul_rn(w.z, xs)));
    h[3] = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(a.w)), __fmul_rn(w.w, xs)));
}

// The 16 fp32 values lane l feeds the rotation.  s: mode 3's row scale, mode
// 1's x_scale; ws: mode 1's weight scales of the group's 16 (hidden) columns,
// ws + K those of the gate columns.
template <int MODE, int ACT>
__device__ __forceinline__ void decode(const GroupIn<MODE, ACT> &g, float s, const float *ws,
                                       int64_t K, float (&v)[16]) {
    if constexpr (MODE == 3) {
        const uint32_t w[4] = {g.v[0].x, g.v[0].y, g.v[0].z, g.v[0].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int t = 0; t < 4; ++t)
                v[4 * j + t] = round_bf16(
                    __fmul_rn(static_cast<float>(static_cast<int8_t>((w[j] >> (8 * t)) & 0xFF)), s));
    } else if constexpr (MODE == 1) {
        const float4 *wh = reinterpret_cast<const float4 *>(ws);
        float h[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) dequant4(g.v[j], __ldg(wh + j), s, h + 4 * j);
        if constexpr (act_paired(ACT)) {
            const float4 *wg = reinterpret_cast<const float4 *>(ws + K);
            float q[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) dequant4(g.v[4 + j], __ldg(wg + j), s, q + 4 * j);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(h[t], q[t]);
        } else {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(h[t], 0.f);
        }
    } else {
        unpack16_bf16(g.v[0], g.v[1], v);
        if constexpr (MODE == 0 && act_paired(ACT)) {
            float u[16];
            unpack16_bf16(g.v[2], g.v[3], u);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], u[t]);
        } else if constexpr (MODE == 0 && ACT != 0) {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = activate<ACT>(v[t], 0.f);
        }
    }
}

// rotate_pair over the padded tile: P[q] = (A[16l+q], B[16l+q]) in,
// P[w] = (A[16w+l], B[16w+l]) out (unscaled, x16)
__device__ __forceinline__ void rotate_pair_padded(f2 (&P)[16], uint32_t tile, int l) {
#pragma unroll
    for (int j = 0; j < 4; ++j) seq2(P[4 * j], P[4 * j + 1], P[4 * j + 2], P[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) seq2(P[j], P[j + 4], P[j + 8], P[j + 12]);
    const uint32_t wrow = tile + l * kPitch;  // row l: P[0..15], 8 bytes each
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float a0, b0, a1, b1;
        un2(P[2 * c], a0, b0);
        un2(P[2 * c + 1], a1, b1);
        st_shared_v4(wrow + 16 * c, __float_as_uint(a0), __float_as_uint(b0), __float_as_uint(a1),
                     __float_as_uint(b1));
    }
    __syncwarp();
    const uint32_t rcol = tile + l * 8;       // column l of rows 0..15
#pragma unroll
    for (int w = 0; w < 16; ++w)
        asm volatile("ld.shared.b64 %0, [%1];" : "=l"(P[w].v) : "r"(rcol + w * kPitch));
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly2(P[4 * j], P[4 * j + 1], P[4 * j + 2], P[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) bfly2(P[j], P[j + 4], P[j + 8], P[j + 12]);
}

// Batches of loads in flight per thread.  Two (a ring of two register
// buffers, the loop unrolled by two) for the rotations without quantization;
// one for the quantizer, whose per-batch row-max barrier makes more resident
// CTAs (8 of 64 registers a thread) worth more than a deeper prefetch
// (measured at M = 65536, K = 4096: 4.0 TB/s against 3.7-3.9 TB/s).
#ifndef XPUINT8_QUANT_DEPTH
#define XPUINT8_QUANT_DEPTH 1
#endif
__host__ __device__ constexpr int direct_depth(int mode, int act) {
    return mode == 1 ? 1 : (mode == 0 ? ((act == 0 || act == 1 || act == 5) ? XPUINT8_QUANT_DEPTH : 1) : 2);
}
// resident 128-thread CTAs per SM the register budget is fitted to:
// XPUINT8_QUANT_CTAS (72 registers a thread) for the quantizer,
// XPUINT8_DIRECT_CTAS (96) for the two-deep rotations, 4 (128) for paired
// inputs and for mode 1's int32 accumulators (64 registers of loads in flight)
#ifndef XPUINT8_DIRECT_CTAS
#define XPUINT8_DIRECT_CTAS 5
#endif
#ifndef XPUINT8_QUANT_CTAS
#define XPUINT8_QUANT_CTAS 7
#endif
constexpr int direct_min_ctas128(int mode, int act) {
    return ((mode == 0 && act_paired(act)) || mode == 1) ? 4
           : mode == 0                                   ? XPUINT8_QUANT_CTAS
                                                         : XPUINT8_DIRECT_CTAS;
}

// SLOTS half-warps per CTA (8, 10, 12 or 16): a batch is the R rows whose
// groups fill the slots (R * G <= 2 * SLOTS), so the row abs-max barrier spans
// one CTA of the size the row width suits (K = 1280: 10 slots, 4 rows;
// K = 4096: 8 slots, one row; K = 5120: 10 slots, one row)
template <int MODE, int ACT, int SLOTS>
__global__ void __launch_bounds__(SLOTS * 16, direct_min_ctas128(MODE, ACT) * 8 / SLOTS)
    rotate_direct_kernel(const BulkParams p) {
    constexpr int DEPTH = direct_depth(MODE, ACT);
    constexpr bool QUANT = (MODE <= 1);
    constexpr int GOB = group_out_bytes(MODE);  // output bytes of one group
    constexpr int IEB = MODE == 3 ? 1 : (MODE == 1 ? 4 : 2);  // input bytes per element
    extern __shared__ __align__(128) uint8_t smem[];
    const int slot = threadIdx.x >> 4, l = threadIdx.x & 15;
    const uint32_t tile = smem_u32(smem) + slot * slot_bytes(MODE);
    const uint32_t obuf = tile + kTileP;  // two buffers of one pair's output
    unsigned int *row_amax = reinterpret_cast<unsigned int *>(smem + SLOTS * slot_bytes(MODE));

    // this slot's pair of groups within a batch (the same for every batch)
    const int f0 = 2 * slot, f1 = f0 + 1;
    const int r0 = f0 / p.G, g0 = f0 - r0 * p.G;
    const int r1 = f1 / p.G, g1 = f1 - r1 * p.G;
    const bool in0 = f0 < p.R * p.G, in1 = f1 < p.R * p.G;
    const bool same_row = r0 == r1;
    // byte offsets inside a batch (a batch is at most 32 rows of at most 32 KB)
    const uint32_t off0 = r0 * p.in_row_bytes + (g0 * 256 + l * 16) * IEB;
    const uint32_t off1 = r1 * p.in_row_bytes + (g1 * 256 + l * 16) * IEB;
    // a paired input's second half, in bytes
    const uint32_t half = static_cast<uint32_t>(IEB) * static_cast<uint32_t>(p.K);
    // mode 1: the weight scales of each group's columns
    const float *ws0 = MODE == 1 ? p.col_scale + g0 * 256 + l * 16 : nullptr;
    const float *ws1 = MODE == 1 ? p.col_scale + g1 * 256 + l * 16 : nullptr;

    if (threadIdx.x < 3 * 32) row_amax[threadIdx.x] = 0u;
    __syncthreads();
    // launched with programmatic serialization: the input and the outputs are
    // touched only once the previous kernel of the stream has completed; the
    // next kernel (the GEMM that reads the codes) may start its prologue now
    pdl_wait();
    pdl_trigger();

    auto batch_rows = [&](int b) -> int {
        const int64_t left = p.M - static_cast<int64_t>(b) * p.R;
        return static_cast<int>(left < p.R ? left : p.R);
    };
    // load batch b (when it exists) into r
    // (an invalid group -- a row past the end of a partial last batch, or the
    // odd slot of an odd group count -- loads the batch's first bytes, which
    // are in bounds: no branch around the loads or the decode)
    auto fetch = [&](int b, RawPair<MODE, ACT> &r) {
        if (b < p.nbatch) {
            const int rows = batch_rows(b);
            const uint8_t *src = p.in + static_cast<int64_t>(b) * p.R * p.in_row_bytes;
            load_group<MODE, ACT>((in0 && r0 < rows) ? src + off0 : src, true, half, r.a);
            load_group<MODE, ACT>((in1 && r1 < rows) ? src + off1 : src, true, half, r.b);
        }
    };
    // transform batch b (k-th of this CTA) from raw, whose registers then take
    // the load of batch b + DEPTH * gridDim.x
    auto batch = [&](int b, int k, RawPair<MODE, ACT> &raw) {
        const int rows = batch_rows(b);
        const int64_t row0 = static_cast<int64_t>(b) * p.R;
        const bool v0 = in0 && r0 < rows, v1 = in1 && r1 < rows;
        unsigned int *amax_now = row_amax + 32 * (k % 3);

        // An invalid group's values stay in its own half of the packed
        // arithmetic: it posts no maximum, no scale and no stored byte.
        float a[16], c[16];
        const float s0 = (MODE == 3 || MODE == 1) ? __ldg(p.row_scale + row0 + (v0 ? r0 : 0)) : 0.f;
        const float s1 = (MODE == 3 || MODE == 1) ? __ldg(p.row_scale + row0 + (v1 ? r1 : 0)) : 0.f;
        decode<MODE, ACT>(raw.a, s0, ws0, p.K, a);
        decode<MODE, ACT>(raw.b, s1, ws1, p.K, c);
        // the loads of DEPTH batches on fly while this one is transformed
        fetch(b + DEPTH * static_cast<int>(gridDim.x), raw);
        f2 vals[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) vals[t] = mk2(a[t], c[t]);
        rotate_pair_padded(vals, tile, l);

        float inv0 = 0.f, inv1 = 0.f;
        if constexpr (QUANT) {
            // per-group maxima of |v| over the slot's half-warp, three-input
            // maxima over pairs of values
            float m0 = 0.f, m1 = 0.f;
#pragma unroll
            for (int t = 0; t < 16; t += 2) {
                float a0, b0, a1, b1;
                un2(vals[t], a0, b0);
                un2(vals[t + 1], a1, b1);
                m0 = max3_abs(m0, a0, a1);
                m1 = max3_abs(m1, b0, b1);
            }
            if (same_row) {
                m0 = halfwarp_max(fmaxf(m0, m1));
                if (l == 0 && v0) atomicMax(amax_now + r0, __float_as_uint(m0));
            } else {
                m0 = halfwarp_max(m0);
                m1 = halfwarp_max(m1);
                if (l == 0) {
                    if (v0) atomicMax(amax_now + r0, __float_as_uint(m0));
                    if (v1) atomicMax(amax_now + r1, __float_as_uint(m1));
                }
            }
            // the buffer two batches on was last read before the previous barrier
            if (threadIdx.x < 32) row_amax[32 * ((k + 1) % 3) + threadIdx.x] = 0u;
            __syncthreads();  // every slot's contribution to this batch's row maxima
            float s0 = 1.f, s1 = 1.f;
            // the maxima are of x16 values: the scale is of max/16, the code v/16 * (1/s)
            if (v0) inv0 = __fmul_rn(row_scale_inv(__fmul_rn(__uint_as_float(amax_now[r0]), 0.0625f), s0), 0.0625f);
            if (same_row) {
                inv1 = inv0;
                s1 = s0;
            } else if (v1) {
                inv1 = __fmul_rn(row_scale_inv(__fmul_rn(__uint_as_float(amax_now[r1]), 0.0625f), s1), 0.0625f);
            }
            if (l == 0) {
                if (v0 && g0 == 0) p.scale[row0 + r0] = s0;
                if (v1 && g1 == 0) p.scale[row0 + r1] = s1;
            }
        }
        // this slot's output buffer k&1: its bulk store of two batches ago has
        // finished reading it
        const uint32_t ob = obuf + (k & 1) * (2 * GOB);
        if (l == 0) bulk_wait_read<1>();
        __syncwarp();
        if constexpr (QUANT) {
            // rint(v * (1/s)), |v/s| <= 127 (+ulps); group A's codes at
            // ob + 16w + l, group B's 256 bytes on
            const uint32_t o = ob + l;
#pragma unroll
            for (int w = 0; w < 16; ++w) {
                float q0, q1;
                un2(quant_magic2(vals[w], inv0, inv1), q0, q1);
                asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 16 * w), "r"(__float_as_uint(q0)) : "memory");
                asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 256 + 16 * w), "r"(__float_as_uint(q1)) : "memory");
            }
        } else {
            const f2 sixteenth = mk2(0.0625f, 0.0625f);
            const uint32_t o = ob + 2 * l;
#pragma unroll
            for (int w = 0; w < 16; ++w) {
                float x0, x1;
                un2(mul2(vals[w], sixteenth), x0, x1);
                const uint32_t hb = cvt_bf16x2(x0, x1);
                asm volatile("st.shared.u16 [%0], %1;" ::"r"(o + 32 * w), "r"(hb & 0xFFFFu) : "memory");
                asm volatile("st.shared.u16 [%0], %1;" ::"r"(o + 512 + 32 * w), "r"(hb >> 16) : "memory");
            }
        }
        fence_async_smem();
        __syncwarp();
        // the batch's groups are consecutive in the dense output: group f starts f * GOB bytes in
        if (l == 0 && v0) {
            bulk_store(p.out + row0 * p.out_row_bytes + f0 * GOB, ob, (v1 ? 2 : 1) * GOB);
            bulk_commit();
        }
    };
    RawPair<MODE, ACT> ra{}, rb{};
    fetch(blockIdx.x, ra);
    if constexpr (DEPTH == 2) fetch(blockIdx.x + gridDim.x, rb);
    int k = 0;
    for (int b = blockIdx.x; b < p.nbatch;) {
        batch(b, k, ra);
        b += gridDim.x;
        ++k;
        if constexpr (DEPTH == 2) {
            if (b >= p.nbatch) break;
            batch(b, k, rb);
            b += gridDim.x;
            ++k;
        }
    }
    if (l == 0) bulk_wait<0>();
    __syncwarp();
}

// ---------------------------------------------------------------------------
// The quantizer (mode 0, no activation) for rows of a multiple of four groups
// (K % 1024 == 0, K <= 8192): each half-warp slot owns four consecutive groups
// of a row -- two pairs, each rotated as fp32x2 like rotate_direct_kernel's
// one pair -- so the per-batch work (addresses, the row maximum, the scale,
// the barrier, one 1 KB bulk store per slot) is spread over twice the
// elements.  SLOTS slots per CTA, R = 4 * SLOTS / G rows per batch.
//
// Measured on B200 at M = 65536, K = 4096 (config C5): 164 us (4.9 TB/s) with
// 64-thread CTAs of 128 registers, against 182 us for rotate_direct_kernel's
// one pair per slot; 128-thread CTAs 167 us.  The row's scale needs every slot
// of its row, so a batch holds whole rows: SLOTS is the smallest even team
// size whose 4 * SLOTS groups are whole rows.
constexpr int kQ4SlotBytes = kTileP + 2 * 1024 + 32;  // transpose tile, two 1 KB code buffers, skew
template <int SLOTS>
__global__ void __launch_bounds__(SLOTS * 16, (512 / (SLOTS * 16)) > 0 ? 512 / (SLOTS * 16) : 1)
    rotate_quant4_kernel(const BulkParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int slot = threadIdx.x >> 4, l = threadIdx.x & 15;
    const uint32_t tile = smem_u32(smem) + slot * kQ4SlotBytes;
    const uint32_t obuf = tile + kTileP;  // two buffers of the slot's four groups' codes
    unsigned int *row_amax = reinterpret_cast<unsigned int *>(smem + SLOTS * kQ4SlotBytes);
    const int f = 4 * slot;  // the slot's first group within a batch
    const int r = f / p.G, g = f - r * p.G;
    const uint32_t off = r * p.in_row_bytes + (g * 256 + l * 16) * 2;
    if (threadIdx.x < 3 * 32) row_amax[threadIdx.x] = 0u;
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    auto batch_rows = [&](int b) -> int {
        const int64_t left = p.M - static_cast<int64_t>(b) * p.R;
        return static_cast<int>(left < p.R ? left : p.R);
    };
    struct Raw {
        uint4 v[8];  // four groups x this lane's 16 bf16
    };
    // (a row past the end of a partial last batch loads the batch's first
    // bytes, in bounds; its results are never stored)
    auto fetch = [&](int b, Raw &raw) {
        if (b < p.nbatch) {
            const uint8_t *src = p.in + static_cast<int64_t>(b) * p.R * p.in_row_bytes;
            const uint4 *q = reinterpret_cast<const uint4 *>(r < batch_rows(b) ? src + off : src);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                raw.v[2 * i] = __ldcs(q + 32 * i);
                raw.v[2 * i + 1] = __ldcs(q + 32 * i + 1);
            }
        }
    };
    auto batch = [&](int b, int k, Raw &raw) {
        const int64_t row0 = static_cast<int64_t>(b) * p.R;
        const bool valid = r < batch_rows(b);
        unsigned int *amax_now = row_amax + 32 * (k % 3);
        f2 va[16], vb[16];
        {
            float a[16], c[16];
            unpack16_bf16(raw.v[0], raw.v[1], a);
            unpack16_bf16(raw.v[2], raw.v[3], c);
#pragma unroll
            for (int t = 0; t < 16; ++t) va[t] = mk2(a[t], c[t]);
            unpack16_bf16(raw.v[4], raw.v[5], a);
            unpack16_bf16(raw.v[6], raw.v[7], c);
#pragma unroll
            for (int t = 0; t < 16; ++t) vb[t] = mk2(a[t], c[t]);
        }
        fetch(b + static_cast<int>(gridDim.x), raw);
        rotate_pair_padded(va, tile, l);
        rotate_pair_padded(vb, tile, l);
        float m = 0.f;
#pragma unroll
        for (int t = 0; t < 16; t += 2) {
            float a0, b0, a1, b1;
            un2(va[t], a0, b0);
            un2(va[t + 1], a1, b1);
            m = max3_abs(m, a0, a1);
            m = max3_abs(m, b0, b1);
            un2(vb[t], a0, b0);
            un2(vb[t + 1], a1, b1);
            m = max3_abs(m, a0, a1);
            m = max3_abs(m, b0, b1);
        }
        m = halfwarp_max(m);
        if (l == 0 && valid) atomicMax(amax_now + r, __float_as_uint(m));
        if (threadIdx.x < 32) row_amax[32 * ((k + 1) % 3) + threadIdx.x] = 0u;
        __syncthreads();
        float s = 1.f, inv = 0.f;
        if (valid) inv = __fmul_rn(row_scale_inv(__fmul_rn(__uint_as_float(amax_now[r]), 0.0625f), s), 0.0625f);
        if (l == 0 && valid && g == 0) p.scale[row0 + r] = s;
        const uint32_t ob = obuf + (k & 1) * 1024;
        if (l == 0) bulk_wait_read<1>();
        __syncwarp();
        const uint32_t o = ob + l;
#pragma unroll
        for (int w = 0; w < 16; ++w) {
            float q0, q1, q2, q3;
            un2(quant_magic2(va[w], inv, inv), q0, q1);
            un2(quant_magic2(vb[w], inv, inv), q2, q3);
            asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 16 * w), "r"(__float_as_uint(q0)) : "memory");
            asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 256 + 16 * w), "r"(__float_as_uint(q1)) : "memory");
            asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 512 + 16 * w), "r"(__float_as_uint(q2)) : "memory");
            asm volatile("st.shared.u8 [%0], %1;" ::"r"(o + 768 + 16 * w), "r"(__float_as_uint(q3)) : "memory");
        }
        fence_async_smem();
        __syncwarp();
        if (l == 0 && valid) {
            bulk_store(p.out + row0 * p.out_row_bytes + f * 256, ob, 1024);
            bulk_commit();
        }
    };
    Raw ra;
    fetch(blockIdx.x, ra);
    int k = 0;
    for (int b = blockIdx.x; b < p.nbatch; b += gridDim.x, ++k) batch(b, k, ra);
    if (l == 0) bulk_wait<0>();
    __syncwarp();
}

template <int SLOTS>
int launch_quant4(cudaStream_t s, BulkParams p) {
    auto kern = rotate_quant4_kernel<SLOTS>;
    p.R = 4 * SLOTS / p.G;
    const int64_t nb = (p.M + p.R - 1) / p.R;
    if (nb > 0x7FFFFFFF) return -1;
    p.nbatch = static_cast<int>(nb);
    const size_t smem = static_cast<size_t>(SLOTS) * kQ4SlotBytes + 3 * 32 * 4;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return launch_status("rotate (shared memory attribute)");
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, SLOTS * 16, smem) != cudaSuccess) per = 1;
    const int64_t grid = std::min<int64_t>(p.nbatch, static_cast<int64_t>(num_sms()) * std::max(1, per));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(SLOTS * 16);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return launch_status("rotate");
    return launch_status("rotate");
}

template <int MODE, int ACT, int SLOTS>
int launch_direct(cudaStream_t s, const BulkParams &p) {
    auto kern = rotate_direct_kernel<MODE, ACT, SLOTS>;
    const size_t smem = static_cast<size_t>(SLOTS) * slot_bytes(MODE) + 3 * 32 * 4;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return launch_status("rotate (shared memory attribute)");
    // resident CTAs per SM, cached per device (atomic: first calls from
    // several host threads may race to fill it, with the same value)
    static std::atomic<int> cached_per_sm[kCacheDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = (dev >= 0 && dev < kCacheDevices) ? cached_per_sm[dev].load(std::memory_order_relaxed) : 0;
    if (per_sm == 0) {
        int per = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, SLOTS * 16, smem) != cudaSuccess)
            per = 1;
        per_sm = std::max(1, per);
        if (dev >= 0 && dev < kCacheDevices) cached_per_sm[dev].store(per_sm, std::memory_order_relaxed);
    }
    const int64_t grid = std::min<int64_t>(p.nbatch, static_cast<int64_t>(num_sms()) * per_sm);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(SLOTS * 16);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return launch_status("rotate");
    return launch_status("rotate");
}
template <int MODE, int ACT>
int launch_direct(cudaStream_t s, const BulkParams &p, int slots) {
    switch (slots) {
        case 8: return launch_direct<MODE, ACT, 8>(s, p);
        case 10: return launch_direct<MODE, ACT, 10>(s, p);
        case 12: return launch_direct<MODE, ACT, 12>(s, p);
        default: return launch_direct<MODE, ACT, 16>(s, p);
    }
}

// The kernel for longer rows.  Its shared memory depends on the batch (R
// rows), so the occupancy is computed per launch (a host-side calculation);
// it sizes the persistent grid only.
template <int MODE, int ACT, int PPS>
int launch_bulk(cudaStream_t s, const BulkParams &p, size_t smem) {
    auto kern = rotate_bulk_kernel<MODE, ACT, PPS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return launch_status("rotate (shared memory attribute)");
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, 256, smem) != cudaSuccess) per = 1;
    const int64_t grid = std::min<int64_t>(p.nbatch, static_cast<int64_t>(num_sms()) * std::max(1, per));
    kern<<<static_cast<unsigned>(grid), 256, smem, s>>>(p);
    return launch_status("rotate");
}
template <int MODE, int ACT>
int launch_pps(cudaStream_t s, const BulkParams &p, int pps, size_t smem) {
    switch (pps) {
        case 1: return launch_bulk<MODE, ACT, 1>(s, p, smem);
        case 2: return launch_bulk<MODE, ACT, 2>(s, p, smem);
        case 4: return launch_bulk<MODE, ACT, 4>(s, p, smem);
        default: break;
    }
    set_error("unsupported group count per slot");
    return 4;
}

}  // namespace

// Returns -1 when the shape does not fit the streaming kernel (the caller then
// uses the register-staged kernel of rotate.cu).
int launch_rotate_bulk(cudaStream_t s, int mode, int act, const void *in, const float *row_scale,
                       const float *col_scale, void *out, float *scale, int64_t M, int64_t K) {
    const int64_t G = K / kGroup;
    int pps = 0, R = 0;
    double best = -1;
    for (int c : {1, 2, 4}) {
        if (G > 2 * kSlots * c) continue;
        const int r = static_cast<int>((2 * kSlots * c) / G);
        const double util = static_cast<double>(r * G) / (2 * kSlots * c);
        if (util >= 0.85) { pps = c; R = r; break; }
        if (util > best) { best = util; pps = c; R = r; }
    }
    if (G > 32 && (pps == 0 || R < 1)) return -1;
    if (R > 32) R = 32;
    if (R < 1) R = 1;
    BulkParams p{};
    p.in = static_cast<const uint8_t *>(in);
    p.row_scale = row_scale;
    p.col_scale = col_scale;
    p.out = static_cast<uint8_t *>(out);
    p.scale = scale;
    p.M = M; p.K = K; p.G = static_cast<int>(G); p.R = R;
    const bool paired = mode <= 1 && act_paired(act);
    const int64_t in_elem = mode == 3 ? 1 : (mode == 1 ? 4 : 2);
    p.in_row_bytes = static_cast<uint32_t>(in_elem * K * (paired ? 2 : 1));
    p.out_row_bytes = static_cast<uint32_t>(mode <= 1 ? K : 2 * K);
    p.out_stage_bytes = (R * p.out_row_bytes + 127u) & ~127u;
    const int64_t nb = (M + R - 1) / R;
    if (nb > 0x7FFFFFFF) return -1;
    p.nbatch = static_cast<int>(nb);
    // rotate_bulk_kernel's output stages: double-buffered unless single
    // buffering fits more CTAs per SM (228 KB of shared memory, 1 KB reserved
    // per CTA)
    auto total = [&](int os) {
        return static_cast<size_t>(os) * p.out_stage_bytes + kSlots * kTileBytes + 3 * 32 * 4;
    };
    int best_ctas = 0;
    for (int os : {2, 1}) {
        const int ctas = static_cast<int>((228 * 1024) / (total(os) + 1024));
        if (ctas > best_ctas) { best_ctas = ctas; p.os = os; }
    }
    if (best_ctas == 0) return -1;
    const size_t smem = total(p.os);
    if (G <= 32) {
        // one batch per CTA-sized team of half-warps: the team size whose
        // batches fill the most slots, the smallest of equals
        int slots = 16;
        double best_fill = -1.0;
        for (int c : {8, 10, 12, 16}) {
            if (G > 2 * c) continue;
            const int64_t r = std::min<int64_t>(32, (2 * c) / G);
            const double fill = static_cast<double>(r * G) / (2 * c);
            if (fill > best_fill + 1e-9) { best_fill = fill; slots = c; }
        }
        p.R = static_cast<int>(std::min<int64_t>(32, (2 * slots) / G));
        const int64_t nbd = (M + p.R - 1) / p.R;
        if (nbd > 0x7FFFFFFF) return -1;
        p.nbatch = static_cast<int>(nbd);
        if (mode == 0 && act == 0 && G % 4 == 0) {
            // four groups per slot, whole rows per batch (K = 1024 .. 8192 in steps of 1024)
            for (int t : {4, 6, 8, 10, 12, 14, 16}) {
                if ((4 * t) % G != 0) continue;
                switch (t) {
                    case 4: return launch_quant4<4>(s, p);
                    case 6: return launch_quant4<6>(s, p);
                    case 8: return launch_quant4<8>(s, p);
                    case 10: return launch_quant4<10>(s, p);
                    case 12: return launch_quant4<12>(s, p);
                    case 14: return launch_quant4<14>(s, p);
                    default: return launch_quant4<16>(s, p);
                }
            }
        }
        if (mode == 0) {
            switch (act) {
                case 0: return launch_direct<0, 0>(s, p, slots);
                case 1: return launch_direct<0, 1>(s, p, slots);
                case 2: return launch_direct<0, 2>(s, p, slots);
                case 3: return launch_direct<0, 3>(s, p, slots);
                case 4: return launch_direct<0, 4>(s, p, slots);
                case 5: return launch_direct<0, 5>(s, p, slots);
                default: return -1;
            }
        }
        if (mode == 1) {
            switch (act) {
                case 3: return launch_direct<1, 3>(s, p, slots);
                case 4: return launch_direct<1, 4>(s, p, slots);
                case 5: return launch_direct<1, 5>(s, p, slots);
                default: return -1;
            }
        }
        if (mode == 2) return launch_direct<2, 0>(s, p, slots);
        if (mode == 3) return launch_direct<3, 0>(s, p, slots);
        return -1;
    }
    if (mode == 0) {
        switch (act) {
            case 0: return launch_pps<0, 0>(s, p, pps, smem);
            case 1: return launch_pps<0, 1>(s, p, pps, smem);
            case 2: return launch_pps<0, 2>(s, p, pps, smem);
            case 3: return launch_pps<0, 3>(s, p, pps, smem);
            case 4: return launch_pps<0, 4>(s, p, pps, smem);
            case 5: return launch_pps<0, 5>(s, p, pps, smem);
            default: return -1;
        }
    }
    if (mode == 2) return launch_pps<2, 0>(s, p, pps, smem);
    if (mode == 3) return launch_pps<3, 0>(s, p, pps, smem);
    return -1;
}

// ---------------------------------------------------------------------------
// Self-check of the quantizers' scale arithmetic (xpuint8_check_scale_math):
// [0] row_scale_inv against its library-call definition on every
//     non-negative float and +inf;
// [1] the code computation quant_magic2 against the scalar IEEE operations on
//     2^31 pseudo-random (value, reciprocal) pairs whose products fall in the
//     code range, so that a contraction of the two roundings into one shows;
// [2] the row quantizer's code rint(div_by_rcp(x, s, 1/s)) against
//     rint(x / s) with the IEEE division, for every bf16 x and every bf16 row
//     maximum amax >= |x| (s the row scale of amax): all the pairs that
//     quantizer can meet;
// [3] the same for the column quantizer on 2^31 pseudo-random fp32 pairs.
// ---------------------------------------------------------------------------
__device__ unsigned long long g_scale_math_bad[4];

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7FEB352Du;
    x ^= x >> 15; x *= 0x846CA68Bu;
    x ^= x >> 16;
    return x;
}

// the int8 code of a quotient: clamp(rint(q), +-127)
__device__ __forceinline__ int code_of(float q) {
    return static_cast<int>(fmaxf(-127.f, fminf(127.f, rintf(q))));
}

__global__ void check_scale_math_kernel() {
    const uint64_t n = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    unsigned long long bad_scale = 0, bad_quant = 0, bad_rowdiv = 0, bad_coldiv = 0;
    for (uint64_t u = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u <= 0x7F800000ull;
         u += n) {
        const float a = __uint_as_float(static_cast<uint32_t>(u));
        float s1, s2;
        const float i1 = row_scale_inv(a, s1);
        const float i2 = row_scale_inv_lib(a, s2);
        bad_scale += (__float_as_uint(s1) != __float_as_uint(s2) || __float_as_uint(i1) != __float_as_uint(i2));
        // v = +-1.m1 * 2^e1, inv = 1.m2 * 2^e2 with e1 + e2 in [-4, 5]: |v * inv| < 128
        const uint32_t h1 = mix32(static_cast<uint32_t>(u) * 2u + 1u), h2 = mix32(h1 ^ 0x9E3779B9u);
        const int e1 = static_cast<int>(h2 & 31u) - 16, e2 = static_cast<int>((h2 >> 5) % 10u) - 4 - e1;
        const float v = __uint_as_float(((h1 & 1u) << 31) | static_cast<uint32_t>(127 + e1) << 23 | (h1 >> 9));
        const float iv = __uint_as_float(static_cast<uint32_t>(127 + e2) << 23 | (h2 >> 9));
        float p0, p1;
        un2(quant_magic2(mk2(v, -v), iv, iv), p0, p1);
        const float q = __fadd_rn(__fmul_rn(v, iv), 12582912.0f);
        const float qn = __fadd_rn(__fmul_rn(-v, iv), 12582912.0f);
        bad_quant += (__float_as_uint(p0) != __float_as_uint(q) || __float_as_uint(p1) != __float_as_uint(qn));
        // [2] bf16 x over bf16 amax >= |x|
        const uint32_t ab = static_cast<uint32_t>(u >> 16), xb = static_cast<uint32_t>(u & 0xFFFFu);
        const float am = bf16_bits_to_f32(ab), xv = bf16_bits_to_f32(xb);
        if (ab < 0x7F80u && (xb & 0x7FFFu) <= ab) {
            float s;
            const float y = row_scale_inv(am, s);
            bad_rowdiv += code_of(div_by_rcp(xv, s, y)) != code_of(__fdiv_rn(xv, s));
        }
        // [3] fp32 g over a column maximum >= |g|
        {
            const uint32_t h3 = mix32(h2 + 0x632BE5ABu), h4 = mix32(h3 ^ 0x85EBCA6Bu);
            const float g = __uint_as_float((h3 & 0x80000000u) | (static_cast<uint32_t>(64 + (h3 >> 1) % 128u) << 23) |
                                            (h4 >> 9));
            const float cm = __fmul_rn(fabsf(g), __uint_as_float(0x3F800000u | (mix32(h4) >> 9)));
            float s;
            const float y = row_scale_inv(cm, s);
            bad_coldiv += code_of(div_by_rcp(g, s, y)) != code_of(__fdiv_rn(g, s));
        }
    }
    if (bad_scale) atomicAdd(&g_scale_math_bad[0], bad_scale);
    if (bad_quant) atomicAdd(&g_scale_math_bad[1], bad_quant);
    if (bad_rowdiv) atomicAdd(&g_scale_math_bad[2], bad_rowdiv);
    if (bad_coldiv) atomicAdd(&g_scale_math_bad[3], bad_coldiv);
}

int check_scale_math(int64_t *bad_scale, int64_t *bad_quant) {
    const unsigned long long zero[4] = {0, 0, 0, 0};
    if (cudaMemcpyToSymbol(g_scale_math_bad, zero, sizeof(zero)) != cudaSuccess)
        return launch_status("scale-math check (reset)");
    check_scale_math_kernel<<<num_sms() * 8, 256>>>();
    if (const int rc = launch_status("scale-math check")) return rc;
    unsigned long long got[4] = {0, 0, 0, 0};
    if (cudaMemcpyFromSymbol(got, g_scale_math_bad, sizeof(got)) != cudaSuccess)
        return launch_status("scale-math check (read)");
    // the scale counts; the code and division counts together
    *bad_scale = static_cast<int64_t>(got[0]);
    *bad_quant = static_cast<int64_t>(got[1] + got[2] + got[3]);
    if (got[1] || got[2] || got[3])
        set_error("scale-math check: code " + std::to_string(got[1]) + ", row division " +
                  std::to_string(got[2]) + ", column division " + std::to_string(got[3]) +
                  " mismatches");
    return 0;
}

}  // namespace xpuint8
