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
//
// Structure (one CTA per SM, persistent over output tiles, 192 threads):
//   warp 0     TMA producer (one thread): A 128x128 and B 256x128 int8 tiles per
//              k-block into a 4-stage shared-memory ring (128-byte swizzle)
//   warp 1     TMEM allocator and MMA issuer (one thread): 4 x
//              tcgen05.mma.kind::i8 (128x256x32) per k-block, tcgen05.commit to
//              free the ring slot and, per tile, to hand the accumulator over
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time (warp w drains TMEM
//              lanes 32*(w%4)..+31, i.e. one output row per thread), scale,
//              convert and store
// TMEM holds two 128x256 int32 accumulators (512 columns), so the epilogue of
// tile i overlaps the MMAs of tile i+1.
//
// No load here uses cluster multicast: every CTA fetches its own tiles, so the
// kernel is safe to run with any operand in any GPU's memory.
//
// Every mbarrier wait is bounded (common.cuh: mbar_wait); on a timeout the
// kernel records the wait site in g_gemm_fault, drains its own TMA loads and
// MMAs (again with a bound), frees its TMEM and returns.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace xpuint8 {

__device__ int g_gemm_fault = 0;

namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kThreads = 192;
constexpr int kTmemCols = 2 * BN;
constexpr int GROUP_M = 16;
constexpr size_t kSmemBytes = static_cast<size_t>(STAGES) * STAGE_BYTES + 1024 + 256;

struct GemmArgs {
    void *out;
    int64_t ldo;
    const float *row_scale;
    const float *col_scale;
    const float *bias;
    int M, N, K;
    int num_m, num_n, num_k;
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

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs &a, uint32_t taddr, int row,
                                               int col0, float xs, bool row_ok) {
    uint32_t r[32];
    tmem_ld32(taddr, r);
    if constexpr (EPI == kEpiGegluBf16) {
        uint32_t gt[32];
        tmem_ld32(taddr + 128, gt);
        tmem_wait_ld();
        if (!row_ok || col0 >= a.N) return;
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 wh = __ldg(reinterpret_cast<const float4 *>(a.col_scale + col0 + j));
            const float4 wg = __ldg(reinterpret_cast<const float4 *>(a.col_scale + a.N + col0 + j));
            const float whv[4] = {wh.x, wh.y, wh.z, wh.w};
            const float wgv[4] = {wg.x, wg.y, wg.z, wg.w};
            float y[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float h = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(r[j + t])),
                                                     __fmul_rn(whv[t], xs)));
                const float g = round_bf16(__fmul_rn(static_cast<float>(static_cast<int32_t>(gt[j + t])),
                                                     __fmul_rn(wgv[t], xs)));
                const float ge = __fmul_rn(__fmul_rn(0.5f, g),
                                           __fadd_rn(1.0f, erff(__fmul_rn(g, 0.7071067811865476f))));
                y[t] = __fmul_rn(h, round_bf16(ge));
            }
            packed[j / 2] = pack_bf16x2(y[0], y[1]);
            packed[j / 2 + 1] = pack_bf16x2(y[2], y[3]);
        }
        uint16_t *dst = static_cast<uint16_t *>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
        uint4 *d4 = reinterpret_cast<uint4 *>(dst);
        d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        if (col0 + 16 < a.N) {
            d4[2] = make_uint4(packed[8], packed[9], packed[10], packed[11]);
            d4[3] = make_uint4(packed[12], packed[13], packed[14], packed[15]);
        }
    } else {
        tmem_wait_ld();
        if (!row_ok || col0 >= a.N) return;
        if constexpr (EPI == kEpiRawI32) {
            int32_t *dst = static_cast<int32_t *>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
            int4 *d4 = reinterpret_cast<int4 *>(dst);
            const int nv = (col0 + 16 < a.N) ? 8 : 4;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < nv)
                    d4[j] = make_int4(static_cast<int>(r[4 * j]), static_cast<int>(r[4 * j + 1]),
                                      static_cast<int>(r[4 * j + 2]), static_cast<int>(r[4 * j + 3]));
        } else {  // dequant -> bf16
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float w[4] = {1.f, 1.f, 1.f, 1.f};
                if (a.col_scale) {
                    const float4 wv = __ldg(reinterpret_cast<const float4 *>(a.col_scale + col0 + j));
                    w[0] = wv.x; w[1] = wv.y; w[2] = wv.z; w[3] = wv.w;
                }
                float v[4];
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    v[t] = __fmul_rn(static_cast<float>(static_cast<int32_t>(r[j + t])), __fmul_rn(w[t], xs));
                if (a.bias) {
                    const float4 bv = __ldg(reinterpret_cast<const float4 *>(a.bias + col0 + j));
                    v[0] = __fadd_rn(v[0], bv.x); v[1] = __fadd_rn(v[1], bv.y);
                    v[2] = __fadd_rn(v[2], bv.z); v[3] = __fadd_rn(v[3], bv.w);
                }
                packed[j / 2] = pack_bf16x2(v[0], v[1]);
                packed[j / 2 + 1] = pack_bf16x2(v[2], v[3]);
            }
            uint16_t *dst = static_cast<uint16_t *>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
            d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
            if (col0 + 16 < a.N) {
                d4[2] = make_uint4(packed[8], packed[9], packed[10], packed[11]);
                d4[3] = make_uint4(packed[12], packed[13], packed[14], packed[15]);
            }
        }
    }
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sA = smem_u32(smem);
    const uint32_t sB = sA + STAGES * A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    const uint32_t bar0 = smem_u32(bars);
    const uint32_t final_bar = bar0 + 8 * (2 * STAGES + 4);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
#define FULL(s) (bar0 + 8u * (s))
#define EMPTY(s) (bar0 + 8u * (STAGES + (s)))
#define TFULL(a) (bar0 + 8u * (2 * STAGES + (a)))
#define TEMPTY(a) (bar0 + 8u * (2 * STAGES + 2 + (a)))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *fault = &g_gemm_fault;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(TFULL(a), 1);
            mbar_init(TEMPTY(a), 128);
        }
        mbar_init(final_bar, 1);
        fence_mbar_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_tiles = args.num_m * args.num_n;
    constexpr bool GEGLU = (EPI == kEpiGegluBf16);
    constexpr int BN_OUT = GEGLU ? 128 : BN;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ TMA producer
            int stage = 0;
            uint32_t ph = 0;
            uint32_t last_ph[STAGES];
            bool used[STAGES];
            for (int s = 0; s < STAGES; ++s) { used[s] = false; last_ph[s] = 0; }
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                int mb, nb;
                tile_coords(tile, args.num_m, args.num_n, mb, nb);
                for (int kb = 0; kb < args.num_k; ++kb) {
                    if (!mbar_wait(EMPTY(stage), ph ^ 1u, fault, 1)) { ok = false; break; }
                    mbar_expect_tx(FULL(stage), STAGE_BYTES);
                    const uint32_t dA = sA + stage * A_BYTES, dB = sB + stage * B_BYTES;
                    if constexpr (A_MN) tma_load_2d(dA, &tmA, FULL(stage), mb * BM, kb * BK);
                    else tma_load_2d(dA, &tmA, FULL(stage), kb * BK, mb * BM);
                    if constexpr (B_MN) {
                        tma_load_2d(dB, &tmB, FULL(stage), nb * BN, kb * BK);
                        tma_load_2d(dB + B_BYTES / 2, &tmB, FULL(stage), nb * BN + 128, kb * BK);
                    } else if constexpr (GEGLU) {
                        tma_load_2d(dB, &tmB, FULL(stage), kb * BK, nb * 128);
                        tma_load_2d(dB + B_BYTES / 2, &tmB, FULL(stage), kb * BK, args.N + nb * 128);
                    } else {
                        tma_load_2d(dB, &tmB, FULL(stage), kb * BK, nb * BN);
                    }
                    used[stage] = true;
                    last_ph[stage] = ph;
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
            }
            // our loads must have landed before the CTA can leave
            for (int s = 0; s < STAGES; ++s)
                if (used[s]) drain_wait(FULL(s), last_ph[s]);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t IDESC = umma_idesc_i8(BM, BN, A_MN, B_MN);
            int stage = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t aph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
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
                        umma_i8(d, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(EMPTY(stage));
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit(TFULL(acc));
                acc ^= 1;
                if (acc == 0) aph ^= 1u;
            }
            // every MMA this thread issued has completed once this barrier flips
            umma_commit(final_bar);
            drain_wait(final_bar, 0);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
        int acc = 0;
        uint32_t aph = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int mb, nb;
            tile_coords(tile, args.num_m, args.num_n, mb, nb);
            if (!mbar_wait(TFULL(acc), aph, fault, 4)) break;
            tc_fence_after();
            const int row = mb * BM + quarter * 32 + lane;
            const bool row_ok = row < args.M;
            const float xs = (row_ok && args.row_scale) ? __ldg(args.row_scale + row) : 1.f;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN_OUT / 32; ++c)
                epilogue_chunk<EPI>(args, taddr + c * 32, row, nb * BN_OUT + c * 32, xs, row_ok);
            tc_fence_before();
            mbar_arrive(TEMPTY(acc));
            acc ^= 1;
            if (acc == 0) aph ^= 1u;
        }
    }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
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

// 2-D int8 tensor map: `inner` contiguous elements per row, `outer` rows, row
// stride `ld` bytes, 128-byte swizzled boxes of box_inner x box_outer
bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint64_t ld,
              uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {ld};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                           strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (error " + std::to_string(static_cast<int>(r)) +
                  "): operands need 16-byte aligned bases and row strides");
        return false;
    }
    return true;
}

template <int EPI, bool A_MN, bool B_MN>
int launch_inst(cudaStream_t s, const CUtensorMap &ma, const CUtensorMap &mb, const GemmArgs &a,
                int grid) {
    auto kern = gemm_i8_kernel<EPI, A_MN, B_MN>;
    static int configured_mask = 0;  // one bit per device ordinal (< 32)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !(configured_mask & (1 << dev))) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemBytes)) != cudaSuccess)
            return launch_status("gemm (shared memory attribute)");
        if (dev < 32) configured_mask |= (1 << dev);
    }
    kern<<<grid, kThreads, kSmemBytes, s>>>(ma, mb, a);
    return launch_status("gemm");
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
    const bool geglu = c.epilogue == kEpiGegluBf16;
    if (geglu && (c.a_mn || c.b_mn)) {
        set_error("the GEGLU epilogue needs K-major operands");
        return 2;
    }
    const uintptr_t oa = reinterpret_cast<uintptr_t>(c.out);
    if ((oa & 15u) || (c.ldo % 8)) {
        set_error("the output needs a 16-byte aligned base and a row stride multiple of 8");
        return 2;
    }
    if ((c.col_scale && (reinterpret_cast<uintptr_t>(c.col_scale) & 15u)) ||
        (c.bias && (reinterpret_cast<uintptr_t>(c.bias) & 15u))) {
        set_error("scales and bias need 16-byte aligned bases");
        return 2;
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
        if (!make_map(&mb, c.b, c.K, b_rows, c.ldb, BK, geglu ? 128 : BN)) return 2;
    } else {
        if (!make_map(&mb, c.b, c.N, c.K, c.ldb, 128, BK)) return 2;
    }
    GemmArgs a{};
    a.out = c.out; a.ldo = c.ldo;
    a.row_scale = c.row_scale; a.col_scale = c.col_scale; a.bias = c.bias;
    a.M = static_cast<int>(c.M); a.N = static_cast<int>(c.N); a.K = static_cast<int>(c.K);
    a.num_m = static_cast<int>((c.M + BM - 1) / BM);
    a.num_n = static_cast<int>((c.N + (geglu ? 128 : BN) - 1) / (geglu ? 128 : BN));
    a.num_k = static_cast<int>((c.K + BK - 1) / BK);
    const int64_t tiles = static_cast<int64_t>(a.num_m) * a.num_n;
    if (tiles > 0x7FFFFFFF) {
        set_error("too many output tiles");
        return 2;
    }
    const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
    switch (c.epilogue) {
        case kEpiRawI32:
            if (!c.a_mn && !c.b_mn) return launch_inst<kEpiRawI32, false, false>(s, ma, mb, a, grid);
            if (!c.a_mn && c.b_mn) return launch_inst<kEpiRawI32, false, true>(s, ma, mb, a, grid);
            if (c.a_mn && c.b_mn) return launch_inst<kEpiRawI32, true, true>(s, ma, mb, a, grid);
            break;
        case kEpiDequantBf16:
            if (!c.a_mn && !c.b_mn) return launch_inst<kEpiDequantBf16, false, false>(s, ma, mb, a, grid);
            if (!c.a_mn && c.b_mn) return launch_inst<kEpiDequantBf16, false, true>(s, ma, mb, a, grid);
            if (c.a_mn && c.b_mn) return launch_inst<kEpiDequantBf16, true, true>(s, ma, mb, a, grid);
            break;
        case kEpiGegluBf16:
            return launch_inst<kEpiGegluBf16, false, false>(s, ma, mb, a, grid);
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
