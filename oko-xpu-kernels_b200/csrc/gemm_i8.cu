// int8 x int8 -> int32 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::i8) with TMEM accumulators, fed by TMA, and fused epilogues.
//
// This replaces the reference's `torch._int_mm` call sites
// (python/xpu_kernels/int8/ops.py:587, :634, :714, :716, :371) and fuses the
// dequant epilogue (src/xpuint8.cpp:692-710) and the GEGLU activation
// (src/xpuint8.cpp:204-212) into the GEMM's TMEM drain.
//
//   D[M,N] = A * B^T, A: [M,K] (K-major) or [K,M] (MN-major),
//                     B: [N,K] (K-major) or [K,N] (MN-major)
//
// Epilogues:
//   raw     int32 D (bit-exact; the _int_mm replacement)
//   dequant bf16(float(D) * (col_scale[n] * row_scale[m]) + bias[n])
//   geglu   B holds [hidden | gate] rows; a CTA loads hidden rows [n, n+128)
//           and gate rows [N+n, N+n+128) into one 256-wide B tile, and writes
//           y = bf16(h * bf16(gelu_erf(g))) with h, g the bf16-rounded dequants
//   situ    the same tiles, y = MossImage's situ of h and g (act.cuh)
//   gelu    the dequant epilogue, then y = bf16(gelu_erf(bf16(dequant)))
//   split   the dequant epilogue with the output's columns cut into parts that
//           land in separate buffers (q, k, v of one projection GEMM)
//
// Structure: persistent CTA pairs (clusters of 2 on neighbouring SMs, one CTA
// per SM, 320 threads each) walk 256 x bn output tiles; the pair's MMAs are
// tcgen05.mma.cta_group::2 (M = 256, N = bn <= 256, K = 32), which read each
// operand half from the CTA that holds it.  Per k-block of 128 a CTA loads only
// its 128 rows of A and bn/2 rows of B (32 KB, where a single-SM 128 x 256
// tile needs 48 KB), which is what keeps the tensor pipe fed at short K.
//   warp 0     TMA producer (one thread per CTA): 6-stage ring
//              (128-byte swizzle); the bytes of both CTAs complete on the
//              leader's FULL barrier
//   warp 1     TMEM allocation in both CTAs; in the leader (rank 0) the MMA
//              issuer: 4 MMAs per k-block, a commit to both CTAs' EMPTY
//              barriers to free the slot, and per tile to both TFULL barriers
//   warps 2-9  epilogue in both CTAs: tcgen05.ld 32 columns at a time (warp w
//              drains TMEM lanes 32*(w%4)..+31, i.e. one output row per thread,
//              and half of the tile's columns), scale, convert, stage in shared
//              memory and TMA-store; each warp then arrives on the leader's
//              TEMPTY barrier
// TMEM holds two 128 x 256 int32 accumulators per CTA (512 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// No load here uses cluster multicast: every CTA fetches its own operand
// halves, so the kernel is safe to run with any operand in any GPU's memory.
//
// Every mbarrier wait is bounded (common.cuh: mbar_wait); on a timeout the
// kernel records the wait site in g_gemm_fault, drains its own TMA loads and
// MMAs (again with a bound), frees its TMEM and returns.
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "act.cuh"
#include "common.cuh"
#include "internal.h"

namespace xpuint8 {

__device__ int g_gemm_fault = 0;

namespace {

// A CTA pair computes a 256 x bn output tile (bn <= 256): each CTA holds 128
// rows of A and bn/2 rows of B per k-block, and 128 accumulator rows.
constexpr int BM = 128, BN = 256, BK = 128;
constexpr int A_BYTES = BM * BK, B_BYTES = (BN / 2) * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kTmemCols = 2 * BN;  // two accumulators of up to 256 columns
constexpr int GROUP_M = 16;

struct GemmArgs {
    void *out;
    int64_t ldo;
    const float *row_scale;
    const float *col_scale;
    const float *bias;
    int M, N, K;
    int num_m, num_n, num_k;
    int bn;  // output columns per tile (multiple of 32, 128..256); GEGLU: 128
    // num_m counts 256-row pair tiles
    int b_early;  // B, the column scales and the bias may be read before the
                  // wait for the previous kernel (it does not write them)
    int split_n;  // > 0: output column n goes to destination n / split_n, column
                  // n % split_n (the split projection: q, k, v from one GEMM)
};

// The output's tensor maps: one per destination.  Either every output tile is
// stored to each of them (the N-sharded linear's all-gather: this rank's
// column block into every rank's output, peers' buffers mapped by CUDA IPC
// and written over NVLink by the TMA unit, tile by tile as the tiles finish),
// or (split_n > 0) the output's columns are cut into consecutive parts of
// split_n columns and each part goes to its own destination (the q, k and v
// projections from one GEMM over the concatenated weight).
constexpr int kMaxOut = 8;
struct OutMaps {
    CUtensorMap m[kMaxOut];
    int n;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int &mb, int &nb) {
    const int per_group = GROUP_M * num_n;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int gsz = min(GROUP_M, num_m - first_m);
    const int local = tile - group * per_group;
    mb = first_m + local % gsz;
    nb = local / gsz;
}

// bounded wait that ignores other threads' faults: used only to drain our own
// asynchronous work before the CTA releases its shared memory and TMEM
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0; it < kWaitMaxIters; ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 255u) == 0u && global_timer_ns() - t0 > kWaitTimeoutNs) break;
    }
    atomicCAS(&g_gemm_fault, 0, 99);
}

// Epilogue staging.  Each epilogue warp owns two 2 KB buffers of 32 rows x 64
// bytes (64-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ ((r>>1)&3),
// the pattern the TMA store unswizzles).  A 32-column chunk of the warp's 32
// rows (bf16; int32 uses 16-column chunks) is converted in registers, written
// to one buffer and handed to a TMA bulk-tensor store, which also clips the
// M/N tails; the next buffers are filled meanwhile.
constexpr int kStageBufs = 2;                                  // per epilogue warp
// a staging buffer: 32 rows of 64 bytes, or of 128 bytes (128-byte swizzle:
// chunk c of row r at c ^ (r & 7)) for the wide-store epilogue
template <int EPI>
constexpr int stage_bytes() { return EPI == kEpiDequantWide ? 32 * 128 : 32 * 64; }

// Per-epilogue configuration.  The epilogue warps come in groups of four, one
// per TMEM lane quarter (warp w reads lanes 32*(w%4)..+31), each group draining
// its share of the tile's columns.  Two groups for the dequant epilogues: a
// third or fourth group drains the last tile sooner but costs a ring stage of
// shared memory and slows the main loop more than it gains (measured at
// M=2048, N=10240, K=1280).  Four groups for the activation epilogues, whose
// drain is the slower side.  The ring takes what shared memory the staging
// buffers leave (227 KB per CTA).
#ifndef XPU_ACT_EPI_WARPS
#define XPU_ACT_EPI_WARPS 16
#endif
template <int EPI>
struct Cfg {
    // the activation epilogues evaluate a transcendental per output, so their
    // drain is slower than the main loop: more warps drain each tile
    static constexpr bool kHeavy = EPI == kEpiSituBf16 || EPI == kEpiGeluBf16 || EPI == kEpiGegluBf16;
    static constexpr int kEpiWarps = kHeavy ? XPU_ACT_EPI_WARPS : 8;
    static constexpr int kGroups = kEpiWarps / 4;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
    static constexpr int kStages = (EPI == kEpiDequantWide || (kHeavy && kEpiWarps > 8)) ? 5 : 6;
    static constexpr int kEpiSmem = kEpiWarps * kStageBufs * stage_bytes<EPI>();
    static constexpr size_t kSmemBytes =
        static_cast<size_t>(kStages) * STAGE_BYTES + kEpiSmem + 2 * BN * 4 + 256;
    static_assert(kSmemBytes <= 232448, "over the 227 KB shared-memory limit of a CTA");
};

__device__ __forceinline__ uint32_t stage_chunk_addr(uint32_t buf, int row, int c) {
    return buf + row * 64 + ((c ^ ((row >> 1) & 3)) << 4);
}
__device__ __forceinline__ uint32_t stage_chunk_addr_wide(uint32_t buf, int row, int c) {
    return buf + row * 128 + ((c ^ (row & 7)) << 4);
}
// 32 bf16 results of this row into half h (columns 32h..32h+31) of a wide buffer
__device__ __forceinline__ void stage_bf16_32_wide(uint32_t buf, int lane, int h, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        st_shared_v4(stage_chunk_addr_wide(buf, lane, 4 * h + c), cvt_bf16x2(v[8 * c], v[8 * c + 1]),
                     cvt_bf16x2(v[8 * c + 2], v[8 * c + 3]), cvt_bf16x2(v[8 * c + 4], v[8 * c + 5]),
                     cvt_bf16x2(v[8 * c + 6], v[8 * c + 7]));
}

// one 32-column chunk of bf16 output: v[0..31] are the fp32 results of this row
__device__ __forceinline__ void stage_bf16_32(uint32_t buf, int lane, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        st_shared_v4(stage_chunk_addr(buf, lane, c), cvt_bf16x2(v[8 * c], v[8 * c + 1]),
                     cvt_bf16x2(v[8 * c + 2], v[8 * c + 3]), cvt_bf16x2(v[8 * c + 4], v[8 * c + 5]),
                     cvt_bf16x2(v[8 * c + 6], v[8 * c + 7]));
}

// hand a filled buffer to the TMA unit (one lane: a store per destination, or
// to the one destination of its part when split_n > 0; one bulk group), then
// flip buffers.  A split part is a multiple of the chunk width, so a chunk
// never straddles two parts.
__device__ __forceinline__ void stage_flush(const OutMaps &om, uint32_t buf, int lane, int x, int y,
                                            int split_n) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (split_n > 0) {
            const int part = x / split_n;
            tma_store_2d(&om.m[part], buf, x - part * split_n, y);
        } else {
            tma_store_2d(&om.m[0], buf, x, y);
#pragma unroll
            for (int i = 1; i < kMaxOut; ++i)
                if (i < om.n) tma_store_2d(&om.m[i], buf, x, y);
        }
        bulk_commit();
    }
}
// before refilling a buffer: its previous store (kStageBufs stores ago) must
// have read it
__device__ __forceinline__ void stage_reserve(int lane) {
    if (lane == 0) bulk_wait_read<kStageBufs - 1>();
    __syncwarp();
}

// dequant of 32 accumulators of one row: float(acc) * (w_scale[n] * x_scale[m])
// (+ bias[n]), each operation rounded.  The product feeding the bias add is a
// scalar __fmul_rn: ptxas contracts a packed f32x2 multiply followed by a
// packed add into one FFMA2.
__device__ __forceinline__ void dequant32(const uint32_t (&r)[32], const float *ws, const float *bs,
                                          f2 xs2, bool bias, float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 w = *reinterpret_cast<const float4 *>(ws + j);
        float s[4];
        un2(mul2(mk2(w.x, w.y), xs2), s[0], s[1]);
        un2(mul2(mk2(w.z, w.w), xs2), s[2], s[3]);
#pragma unroll
        for (int t = 0; t < 4; ++t)
            v[j + t] = __fmul_rn(static_cast<float>(static_cast<int32_t>(r[j + t])), s[t]);
        if (bias) {
            const float4 b = *reinterpret_cast<const float4 *>(bs + j);
            f2 p01 = add2(mk2(v[j], v[j + 1]), mk2(b.x, b.y));
            f2 p23 = add2(mk2(v[j + 2], v[j + 3]), mk2(b.z, b.w));
            un2(p01, v[j], v[j + 1]);
            un2(p23, v[j + 2], v[j + 3]);
        }
    }
}

// y = bf16(h * bf16(gelu_erf(g))) from the hidden and gate accumulators
__device__ __forceinline__ void geglu32(const uint32_t (&rh)[32], const uint32_t (&rg)[32],
                                        const float *wsh, const float *wsg, f2 xs2, float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const float2 wh = *reinterpret_cast<const float2 *>(wsh + j);
        const float2 wg = *reinterpret_cast<const float2 *>(wsg + j);
        float h0, h1, g0, g1;
        un2(mul2(mk2(static_cast<float>(static_cast<int32_t>(rh[j])),
                     static_cast<float>(static_cast<int32_t>(rh[j + 1]))),
                 mul2(mk2(wh.x, wh.y), xs2)), h0, h1);
        un2(mul2(mk2(static_cast<float>(static_cast<int32_t>(rg[j])),
                     static_cast<float>(static_cast<int32_t>(rg[j + 1]))),
                 mul2(mk2(wg.x, wg.y), xs2)), g0, g1);
        // h, g rounded to bf16 (the unfused chain stores them), then
        // y = bf16(h * bf16(0.5 g (1 + erf(g / sqrt 2))))
        round_bf16x2(h0, h1);
        round_bf16x2(g0, g1);
        float e0 = __fmul_rn(__fmul_rn(0.5f, g0),
                             __fadd_rn(1.0f, erff(__fmul_rn(g0, 0.7071067811865476f))));
        float e1 = __fmul_rn(__fmul_rn(0.5f, g1),
                             __fadd_rn(1.0f, erff(__fmul_rn(g1, 0.7071067811865476f))));
        round_bf16x2(e0, e1);
        v[j] = __fmul_rn(h0, e0);
        v[j + 1] = __fmul_rn(h1, e1);
    }
}

// y = bf16(situ(h, g)) from the hidden and gate accumulators: h, g the
// bf16-rounded dequants, then the gate's and the hidden half's factors
// (act.cuh; the reference's situ_reg, src/xpuint8.cpp:142-160) multiplied
__device__ __forceinline__ void situ32(const uint32_t (&rh)[32], const uint32_t (&rg)[32],
                                       const float *wsh, const float *wsg, f2 xs2, float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const float2 wh = *reinterpret_cast<const float2 *>(wsh + j);
        const float2 wg = *reinterpret_cast<const float2 *>(wsg + j);
        float h0, h1, g0, g1;
        un2(mul2(mk2(static_cast<float>(static_cast<int32_t>(rh[j])),
                     static_cast<float>(static_cast<int32_t>(rh[j + 1]))),
                 mul2(mk2(wh.x, wh.y), xs2)), h0, h1);
        un2(mul2(mk2(static_cast<float>(static_cast<int32_t>(rg[j])),
                     static_cast<float>(static_cast<int32_t>(rg[j + 1]))),
                 mul2(mk2(wg.x, wg.y), xs2)), g0, g1);
        round_bf16x2(h0, h1);
        round_bf16x2(g0, g1);
        v[j] = __fmul_rn(piece_situ_gate(g0), piece_situ_hidden(h0));
        v[j + 1] = __fmul_rn(piece_situ_gate(g1), piece_situ_hidden(h1));
    }
}

// Drain this warp's share of one accumulator tile: 32 rows (its TMEM lane
// quarter) x columns [c0, c1), 32 columns at a time.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs &a, const OutMaps &tmOut, uint32_t taddr,
                                              int m0, int n0, int quarter, int c0, int c1, int lane,
                                              float xs, const float *s_ws, const float *s_b,
                                              uint32_t bufs, int &bsel) {
    const int y = m0 + quarter * 32;
    const f2 xs2 = mk2(xs, xs);
    const bool bias = a.bias != nullptr;
    constexpr int kStageBytes = stage_bytes<EPI>();
    if constexpr (EPI == kEpiDequantWide) {
        // 64 columns per store (the tile width is a multiple of 64)
#pragma unroll 1
        for (int c = c0; c < c1; c += 64) {
            if (n0 + c >= a.N) break;
            uint32_t r0[32], r1[32];
            tmem_ld32(taddr + c, r0);
            tmem_ld32(taddr + c + 32, r1);
            stage_reserve(lane);
            const uint32_t buf = bufs + bsel * kStageBytes;
            float v[32];
            tmem_wait_ld(r0);
            dequant32(r0, s_ws + c, s_b + c, xs2, bias, v);
            stage_bf16_32_wide(buf, lane, 0, v);
            tmem_wait_ld(r1);
            dequant32(r1, s_ws + c + 32, s_b + c + 32, xs2, bias, v);
            stage_bf16_32_wide(buf, lane, 1, v);
            stage_flush(tmOut, buf, lane, n0 + c, y, a.split_n);
            bsel ^= 1;
        }
    } else {
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
        if (n0 + c >= a.N) break;
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        if constexpr (EPI == kEpiRawI32) {
            tmem_wait_ld(r);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                stage_reserve(lane);
                const uint32_t buf = bufs + bsel * kStageBytes;
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    st_shared_v4(stage_chunk_addr(buf, lane, q), r[16 * h + 4 * q],
                                 r[16 * h + 4 * q + 1], r[16 * h + 4 * q + 2], r[16 * h + 4 * q + 3]);
                stage_flush(tmOut, buf, lane, n0 + c + 16 * h, y, a.split_n);
                bsel ^= 1;
            }
        } else {
            float v[32];
            if constexpr (EPI == kEpiDequantBf16 || EPI == kEpiGeluBf16) {
                tmem_wait_ld(r);
                dequant32(r, s_ws + c, s_b + c, xs2, bias, v);
                if constexpr (EPI == kEpiGeluBf16) {
#pragma unroll
                    for (int t = 0; t < 32; ++t) v[t] = piece_gelu_erf(round_bf16(v[t]));
                }
            } else {
                uint32_t rg[32];
                tmem_ld32(taddr + 128 + c, rg);
                tmem_wait_ld(r);
                tmem_wait_ld(rg);
                if constexpr (EPI == kEpiSituBf16) situ32(r, rg, s_ws + c, s_ws + 128 + c, xs2, v);
                else geglu32(r, rg, s_ws + c, s_ws + 128 + c, xs2, v);
            }
            stage_reserve(lane);
            const uint32_t buf = bufs + bsel * kStageBytes;
            stage_bf16_32(buf, lane, v);
            stage_flush(tmOut, buf, lane, n0 + c, y, a.split_n);
            bsel ^= 1;
        }
    }
    }
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(Cfg<EPI>::kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ OutMaps tmOut, const GemmArgs args) {
    constexpr int STAGES = Cfg<EPI>::kStages;
    constexpr int kEpiWarps = Cfg<EPI>::kEpiWarps;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw;
    if (smem_u32(smem) & 1023u) {  // the 128-byte swizzle needs 1024-byte aligned tiles
        // (the same layout in both CTAs of the pair: both leave here)
        if (threadIdx.x == 0) atomicCAS(&g_gemm_fault, 0, 98);
        return;
    }
    const uint32_t sA = smem_u32(smem);
    const uint32_t sB = sA + STAGES * A_BYTES;
    const uint32_t sEpi = sA + STAGES * STAGE_BYTES;  // 2 staging buffers per epilogue warp
    float *s_ws = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES + Cfg<EPI>::kEpiSmem);
    float *s_b = s_ws + BN;
    uint64_t *bars = reinterpret_cast<uint64_t *>(s_b + BN);
    const uint32_t bar0 = smem_u32(bars);
    const uint32_t final_bar = bar0 + 8 * (2 * STAGES + 4);
    const uint32_t epi_bar = bar0 + 8 * (2 * STAGES + 5);  // the epilogue threads
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 6);
#define FULL(s) (bar0 + 8u * (s))
#define EMPTY(s) (bar0 + 8u * (STAGES + (s)))
#define TFULL(a) (bar0 + 8u * (2 * STAGES + (a)))
#define TEMPTY(a) (bar0 + 8u * (2 * STAGES + 2 + (a)))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *fault = &g_gemm_fault;
    const uint32_t rank = cluster_rank();  // 0: the leader, which issues the pair's MMAs
    const bool leader = rank == 0;
    const int pair = static_cast<int>(cluster_index());
    const int npairs = static_cast<int>(cluster_count());

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(FULL(s), 1);   // leader: its producer's expect_tx + both CTAs' bytes
            mbar_init(EMPTY(s), 1);  // the leader's MMA commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(TFULL(a), 1);                // the leader's MMA commit
            mbar_init(TEMPTY(a), 2 * kEpiWarps);   // leader: every epilogue warp of both CTAs
        }
        mbar_init(final_bar, 1);
        mbar_init(epi_bar, 32 * kEpiWarps);
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        for (int i = 0; i < tmOut.n; ++i) prefetch_tmap(&tmOut.m[i]);
    }
    // both CTAs' barriers exist before either CTA arrives on the other's
    cluster_sync();
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above overlaps the previous kernel of the stream.  Each role
    // waits for that kernel (pdl_wait) before its first global access that may
    // depend on it: A, the row scales and the output always; B, the column
    // scales and the bias too unless args.b_early (the linear entries, where
    // the previous kernel is the activation quantizer).

    const int num_tiles = args.num_m * args.num_n;
    // the paired epilogues: B tiles of 128 hidden + 128 gate rows
    constexpr bool GEGLU = (EPI == kEpiGegluBf16 || EPI == kEpiSituBf16);
    const int BN_OUT = GEGLU ? 128 : args.bn;
    const int B_ROWS = GEGLU ? BN : args.bn;  // MMA N: rows of B per pair tile
    const int B_HALF = B_ROWS / 2;            // rows of B this CTA loads

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer (both CTAs)
            // Each CTA loads its own 128 rows of A and its half of B; the
            // completion bytes of both count on the leader's FULL barrier, on
            // which the leader's producer posted the pair's byte total.
            int stage = 0;
            uint32_t ph = 0;
            uint32_t issued = 0;  // k-blocks issued by this CTA
            const uint32_t pair_tx = static_cast<uint32_t>(2 * (A_BYTES + B_HALF * BK));
            // this CTA's half of B for k-block kb of output-column block nb into slot st
            auto load_b = [&](int st, int nb, int kb) {
                const uint32_t fb = peer_smem(FULL(st), 0);
                const uint32_t dB = sB + st * B_BYTES;
                if constexpr (B_MN) {
                    tma_load_2d_pair(dB, &tmB, fb, nb * BN + static_cast<int>(rank) * 128, kb * BK);
                } else if constexpr (GEGLU) {
                    // leader: hidden rows [n, n+128); follower: gate rows [N+n, N+n+128)
                    tma_load_2d_pair(dB, &tmB, fb, kb * BK, (leader ? 0 : args.N) + nb * 128);
                } else {
                    tma_load_2d_pair(dB, &tmB, fb, kb * BK, nb * args.bn + static_cast<int>(rank) * B_HALF);
                }
            };
            // b_early: the B halves of the first pass over the ring load before
            // the wait (their bytes complete on FULL ahead of the leader's
            // expect_tx, which the barrier's transaction count allows)
            uint32_t pre = 0;
            if (args.b_early) {
                int tile = pair, kb = 0;
                for (; pre < static_cast<uint32_t>(STAGES) && tile < num_tiles; ++pre) {
                    int mb, nb;
                    tile_coords(tile, args.num_m, args.num_n, mb, nb);
                    load_b(static_cast<int>(pre), nb, kb);
                    if (++kb == args.num_k) { kb = 0; tile += npairs; }
                }
            }
            pdl_wait();
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
                int mb, nb;
                tile_coords(tile, args.num_m, args.num_n, mb, nb);
                const int arow = mb * (2 * BM) + static_cast<int>(rank) * BM;
                for (int kb = 0; kb < args.num_k; ++kb) {
                    if (!mbar_wait(EMPTY(stage), ph ^ 1u, fault, 1)) { ok = false; break; }
                    if (leader) mbar_expect_tx(FULL(stage), pair_tx);
                    const uint32_t fb = peer_smem(FULL(stage), 0);
                    const uint32_t dA = sA + stage * A_BYTES;
                    if constexpr (A_MN) tma_load_2d_pair(dA, &tmA, fb, arow, kb * BK);
                    else tma_load_2d_pair(dA, &tmA, fb, kb * BK, arow);
                    if (issued >= pre) load_b(stage, nb, kb);
                    ++issued;
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
            }
            pdl_trigger();  // every load is issued: the next kernel may begin launching
            // every load has landed once the MMAs that read it have completed:
            // the last k-block issued into slot s (number i, i % STAGES == s)
            // frees the slot in phase i / STAGES
            for (uint32_t s = 0; s < STAGES && s < issued; ++s) {
                const uint32_t last = s + ((issued - 1 - s) / STAGES) * STAGES;
                drain_wait(EMPTY(s), (last / STAGES) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ------------------------------------------------ MMA issuer (leader only)
            const uint32_t idesc = umma_idesc_i8(2 * BM, B_ROWS, A_MN, B_MN);
            int stage = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t aph = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
                if (!mbar_wait(TEMPTY(acc), aph ^ 1u, fault, 2)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < args.num_k; ++kb) {
                    if (!mbar_wait(FULL(stage), ph, fault, 3)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = sA + stage * A_BYTES, b0 = sB + stage * B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; ++kk) {
                        // K-major: a 32-byte step inside the swizzled 128-byte row;
                        // MN-major: 32 rows of 128 bytes
                        const uint64_t ad = A_MN ? umma_sdesc_sw128(a0 + kk * 4096, BK * 128, 1024)
                                                 : umma_sdesc_sw128(a0 + kk * 32, 16, 1024);
                        const uint64_t bd = B_MN ? umma_sdesc_sw128(b0 + kk * 4096, BK * 128, 1024)
                                                 : umma_sdesc_sw128(b0 + kk * 32, 16, 1024);
                        umma_i8_pair(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    // the slot is free in both CTAs once these MMAs have read it
                    umma_commit_pair(EMPTY(stage));
                    umma_commit_pair(peer_smem(EMPTY(stage), 1));
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit_pair(TFULL(acc));
                umma_commit_pair(peer_smem(TFULL(acc), 1));
                acc ^= 1;
                if (acc == 0) aph ^= 1u;
            }
            // every MMA this thread issued has completed once this barrier flips
            umma_commit_pair(final_bar);
            drain_wait(final_bar, 0);
        }
    } else {
        // ---------------------------------------------------------- epilogue (both CTAs)
        const int quarter = warp & 3;         // TMEM lanes 32*quarter .. +31
        const int group = (warp - 2) >> 2;    // which share of the tile's columns
        // paired: 128 / groups output columns per group; otherwise BN / groups columns of
        // the accumulator per group, clipped to the tile's bn
        constexpr int kCols = GEGLU ? 128 / Cfg<EPI>::kGroups : BN / Cfg<EPI>::kGroups;
        const int col0 = kCols * group;
        const int col1 = GEGLU ? col0 + kCols : min(col0 + kCols, args.bn);
        const int et = threadIdx.x - 64;      // index among the epilogue threads; the
                                              // first 256 stage the tile's column scales
        const uint32_t bufs = sEpi + (warp - 2) * kStageBufs * stage_bytes<EPI>();
        const uint32_t tempty_leader0 = peer_smem(TEMPTY(0), 0);
        int bsel = 0;
        int acc = 0;
        uint32_t aph = 0;
        uint32_t epi_phase = 0;
        // a barrier of the epilogue threads whose wait is bounded like every other
        auto epi_sync = [&](int site) {
            mbar_arrive(epi_bar);
            const bool ok = mbar_wait(epi_bar, epi_phase & 1u, fault, site);
            ++epi_phase;
            return ok;
        };
        // column et's scale and bias of a tile, read ahead of the tile (registers)
        auto fetch = [&](int tile, float &w, float &b) {
            int mb, nb;
            tile_coords(tile, args.num_m, args.num_n, mb, nb);
            const int n0 = nb * BN_OUT;
            int n;
            if constexpr (GEGLU) n = (et < 128) ? n0 + et : args.N + n0 + (et - 128);
            else n = n0 + et;
            const bool in = GEGLU ? (n0 + (et & 127)) < args.N : (et < BN_OUT && n0 + et < args.N);
            w = (in && args.col_scale) ? __ldg(args.col_scale + n) : 1.f;
            b = (in && args.bias) ? __ldg(args.bias + n) : 0.f;
        };
        float pre_w = 1.f, pre_b = 0.f;
        const bool stager = et < 2 * BM;
        if (!args.b_early) pdl_wait();
        if (stager && pair < num_tiles) fetch(pair, pre_w, pre_b);
        if (args.b_early) pdl_wait();
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            int mb, nb;
            tile_coords(tile, args.num_m, args.num_n, mb, nb);
            const int n0 = nb * BN_OUT;
            const int m0 = mb * (2 * BM) + static_cast<int>(rank) * BM;
            if (!epi_sync(5)) break;  // everyone is done with the previous tile's scales
            if (stager) {
                s_ws[et] = pre_w;
                s_b[et] = pre_b;
            }
            if (!epi_sync(6)) break;
            if (stager && tile + npairs < num_tiles) fetch(tile + npairs, pre_w, pre_b);
            const int row = m0 + quarter * 32 + lane;
            const float xs = (row < args.M && args.row_scale) ? __ldg(args.row_scale + row) : 1.f;
            if (!mbar_wait(TFULL(acc), aph, fault, 4)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
            epilogue_tile<EPI>(args, tmOut, taddr, m0, n0, quarter, col0, col1, lane, xs, s_ws,
                               s_b, bufs, bsel);
            // hand the accumulator back to the leader's MMA issuer (one arrival per warp)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) mbar_arrive(TEMPTY(acc));
                else mbar_arrive_cluster(tempty_leader0 + 8u * acc);
            }
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
        // the stores must have left shared memory before the CTA exits
        if (lane == 0) bulk_wait<0>();
        __syncwarp();
    }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
    // neither CTA leaves while the other may still arrive on its barriers or
    // (leader) read its shared memory and write its TMEM
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// -------------------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D tensor map: `inner` contiguous elements per row, `outer` rows, row
// stride `ld` bytes, swizzled boxes of box_inner x box_outer elements
bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint64_t ld,
              uint32_t box_inner, uint32_t box_outer,
              CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {ld};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(m, dtype, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (error " + std::to_string(static_cast<int>(r)) +
                  "): operands need 16-byte aligned bases and row strides");
        return false;
    }
    return true;
}

// CTA pairs that can be resident at once for this kernel (cached per device;
// launch_inst sets the shared-memory attribute on every launch, so a device
// reset, which clears it, cannot leave a launch without it)
template <int EPI, bool A_MN, bool B_MN>
int resident_pairs(int dev) {
    auto kern = gemm_i8_kernel<EPI, A_MN, B_MN>;
    // atomic: first calls from several host threads may race to fill it (same value)
    static std::atomic<int> cached[32] = {};
    if (dev >= 0 && dev < 32) {
        const int c = cached[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Cfg<EPI>::kSmemBytes)) != cudaSuccess)
        return -1;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * num_sms());
    cfg.blockDim = dim3(Cfg<EPI>::kThreads);
    cfg.dynamicSmemBytes = Cfg<EPI>::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) return -1;
    if (dev >= 0 && dev < 32) cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

template <int EPI, bool A_MN, bool B_MN>
int launch_inst(cudaStream_t s, const CUtensorMap &ma, const CUtensorMap &mb, const OutMaps &mo,
                const GemmArgs &a, int pairs) {
    auto kern = gemm_i8_kernel<EPI, A_MN, B_MN>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Cfg<EPI>::kSmemBytes)) != cudaSuccess)
        return launch_status("gemm (shared memory attribute)");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // the prologue may overlap the previous kernel (the kernel waits for it
    // before its first global access)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(Cfg<EPI>::kThreads);
    cfg.dynamicSmemBytes = Cfg<EPI>::kSmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, ma, mb, mo, a) != cudaSuccess) return launch_status("gemm");
    return launch_status("gemm");
}

template <int EPI, bool A_MN, bool B_MN>
int launch_sized(cudaStream_t s, const CUtensorMap &ma, const CUtensorMap &mb,
                 const OutMaps &mo, const GemmArgs &a, int64_t tiles) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int resident = resident_pairs<EPI, A_MN, B_MN>(dev);
    if (resident <= 0) {
        set_error("no CTA pair of the GEMM fits on the device");
        return 5;
    }
    const int pairs = static_cast<int>(tiles < resident ? tiles : resident);
    return launch_inst<EPI, A_MN, B_MN>(s, ma, mb, mo, a, pairs);
}

}  // namespace

int launch_gemm(cudaStream_t s, const GemmCall &c) {
    if (c.M <= 0 || c.N <= 0 || c.K <= 0) {
        set_error("M, N and K must be positive");
        return 2;
    }
    if (c.M > 0x7FFFFF00 || c.N > 0x7FFFFF00 || c.K > 0x7FFFFF00) {
        set_error("M, N and K must fit in 31 bits");
        return 2;
    }
    if (c.N % 16) {
        set_error("N must be a multiple of 16");
        return 2;
    }
    // the paired epilogues (GEGLU, situ): B holds [hidden | gate] rows
    const bool geglu = c.epilogue == kEpiGegluBf16 || c.epilogue == kEpiSituBf16;
    if ((geglu || c.epilogue == kEpiGeluBf16) && (c.a_mn || c.b_mn)) {
        set_error("the activation epilogues need K-major operands");
        return 2;
    }
    if (c.split_n > 0) {
        // the split projection: N / split_n parts, each its own [M, split_n] output
        if (c.epilogue != kEpiDequantBf16 || c.a_mn || c.b_mn || !c.outs ||
            c.split_n % 32 != 0 || c.N % c.split_n != 0 || c.nout != c.N / c.split_n) {
            set_error("split output: the dequant epilogue with K-major operands, parts of a "
                      "multiple of 32 columns, one output buffer per part");
            return 2;
        }
    }
    const uintptr_t oa = reinterpret_cast<uintptr_t>(c.outs ? c.outs[0] : c.out);
    if ((oa & 15u) || (c.ldo % 8)) {
        set_error("the output needs a 16-byte aligned base and a row stride multiple of 8");
        return 2;
    }
    if ((c.col_scale && (reinterpret_cast<uintptr_t>(c.col_scale) & 15u)) ||
        (c.bias && (reinterpret_cast<uintptr_t>(c.bias) & 15u))) {
        set_error("scales and bias need 16-byte aligned bases");
        return 2;
    }
    // Output columns per tile.  Tiles (256 rows x bn) are spread over the CTA
    // pairs in waves (a persistent pair takes every P-th tile, P = pairs on
    // the device), so the critical path is ceil(tiles / P) tiles; a narrower
    // tile can finish sooner when it fills the last wave better (N = 10240 at
    // M = 2048: 320 tiles of 256 columns take 5 waves of 74 pairs, 368 tiles
    // of 224 columns also 5 waves of 7/8 the work).  Each tile also costs a
    // fixed drain and hand-over, counted as 32 columns.  Only a K-major B is
    // narrowed: an MN-major B tile is loaded as two 128-column boxes.
    int bn = BN;
    const bool wide = c.epilogue == kEpiDequantWide;
    const int step = wide ? 64 : 32;  // the wide epilogue stores 64 columns at a time
    // XPUINT8_GEMM_BN=<128..256, multiple of 32> fixes the width (tests, tuning)
    const char *force = std::getenv("XPUINT8_GEMM_BN");
    const int forced = force ? std::atoi(force) : 0;
    if (!geglu && !c.b_mn && forced >= 128 && forced <= BN && forced % step == 0) {
        bn = forced;
    } else if (!geglu && !c.b_mn) {
        const int64_t sms = num_sms() / 2;  // CTA pairs
        const int64_t num_m = (c.M + 2 * BM - 1) / (2 * BM);
        int64_t best = -1;
        for (int cand = BN; cand >= 128; cand -= step) {
            const int64_t tiles = num_m * ((c.N + cand - 1) / cand);
            const int64_t cost = ((tiles + sms - 1) / sms) * (cand + 32);
            if (best < 0 || cost < best) {
                best = cost;
                bn = cand;
            }
        }
    }
    CUtensorMap ma, mb;
    // A: K-major [M rows, K bytes]; MN-major [K rows, M bytes]
    if (!c.a_mn) {
        if (!make_map(&ma, c.a, c.K, c.M, c.lda, BK, BM)) return 2;
    } else {
        if (!make_map(&ma, c.a, c.M, c.K, c.lda, BM, BK)) return 2;
    }
    const int64_t b_rows = geglu ? 2 * c.N : c.N;
    if (!c.b_mn) {
        // each CTA of a pair loads half of the pair's B rows
        if (!make_map(&mb, c.b, c.K, b_rows, c.ldb, BK, geglu ? 128 : bn / 2)) return 2;
    } else {
        if (!make_map(&mb, c.b, c.N, c.K, c.ldb, 128, BK)) return 2;
    }
    // output: 32-row boxes, 64-byte rows (16 int32 or 32 bf16 columns), 64-byte
    // swizzle; one map per destination (c.out, or the c.nout buffers of c.outs)
    OutMaps mo{};
    const int nout = c.outs ? c.nout : 1;
    if (nout < 1 || nout > kMaxOut) {
        set_error("between 1 and 8 output buffers");
        return 2;
    }
    mo.n = nout;
    for (int i = 0; i < nout; ++i) {
        void *base = c.outs ? c.outs[i] : c.out;
        if (!base || (reinterpret_cast<uintptr_t>(base) & 15u)) {
            set_error("every output buffer needs a 16-byte aligned base");
            return 2;
        }
        if (c.epilogue == kEpiRawI32) {
            if (!make_map(&mo.m[i], base, c.N, c.M, c.ldo * 4, 16, 32, CU_TENSOR_MAP_DATA_TYPE_INT32,
                          CU_TENSOR_MAP_SWIZZLE_64B))
                return 2;
        } else if (wide) {
            if (!make_map(&mo.m[i], base, c.N, c.M, c.ldo * 2, 64, 32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          CU_TENSOR_MAP_SWIZZLE_128B))
                return 2;
        } else {
            const int64_t cols = c.split_n > 0 ? c.split_n : c.N;
            if (!make_map(&mo.m[i], base, cols, c.M, c.ldo * 2, 32, 32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          CU_TENSOR_MAP_SWIZZLE_64B))
                return 2;
        }
    }
    GemmArgs a{};
    a.out = c.out; a.ldo = c.ldo;
    a.row_scale = c.row_scale; a.col_scale = c.col_scale; a.bias = c.bias;
    a.M = static_cast<int>(c.M); a.N = static_cast<int>(c.N); a.K = static_cast<int>(c.K);
    a.b_early = c.b_early ? 1 : 0;
    a.split_n = c.split_n > 0 ? static_cast<int>(c.split_n) : 0;
    a.num_m = static_cast<int>((c.M + 2 * BM - 1) / (2 * BM));
    a.bn = geglu ? 128 : bn;
    a.num_n = static_cast<int>((c.N + a.bn - 1) / a.bn);
    a.num_k = static_cast<int>((c.K + BK - 1) / BK);
    const int64_t tiles = static_cast<int64_t>(a.num_m) * a.num_n;
    if (tiles > 0x7FFFFFFF) {
        set_error("too many output tiles");
        return 2;
    }
    switch (c.epilogue) {
        case kEpiRawI32:
            if (!c.a_mn && !c.b_mn) return launch_sized<kEpiRawI32, false, false>(s, ma, mb, mo, a, tiles);
            if (!c.a_mn && c.b_mn) return launch_sized<kEpiRawI32, false, true>(s, ma, mb, mo, a, tiles);
            if (c.a_mn && c.b_mn) return launch_sized<kEpiRawI32, true, true>(s, ma, mb, mo, a, tiles);
            break;
        case kEpiDequantBf16:
            if (!c.a_mn && !c.b_mn) return launch_sized<kEpiDequantBf16, false, false>(s, ma, mb, mo, a, tiles);
            if (!c.a_mn && c.b_mn) return launch_sized<kEpiDequantBf16, false, true>(s, ma, mb, mo, a, tiles);
            if (c.a_mn && c.b_mn) return launch_sized<kEpiDequantBf16, true, true>(s, ma, mb, mo, a, tiles);
            break;
        case kEpiGegluBf16:
            return launch_sized<kEpiGegluBf16, false, false>(s, ma, mb, mo, a, tiles);
        case kEpiSituBf16:
            return launch_sized<kEpiSituBf16, false, false>(s, ma, mb, mo, a, tiles);
        case kEpiGeluBf16:
            return launch_sized<kEpiGeluBf16, false, false>(s, ma, mb, mo, a, tiles);
        case kEpiDequantWide:
            if (!c.a_mn && !c.b_mn) return launch_sized<kEpiDequantWide, false, false>(s, ma, mb, mo, a, tiles);
            break;
        default:
            break;
    }
    set_error("unsupported operand layout combination");
    return 2;
}

int gemm_fault_status(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_fault, sizeof(int)) != cudaSuccess) {
        set_error("could not read the GEMM fault word");
        return -1;
    }
    if (reset && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_gemm_fault, &zero, sizeof(int));
    }
    return v;
}

}  // namespace xpuint8
