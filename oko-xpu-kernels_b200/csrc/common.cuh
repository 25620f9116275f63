// Shared device helpers for libxpuint8 (sm_100a): bf16 conversions, the
// radix-4 ConvRot butterflies, and thin inline-PTX wrappers for mbarrier,
// TMA (cp.async.bulk.tensor) and the tcgen05 tensor-core / TMEM instructions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xpuint8 {

constexpr int kGroup = 256;  // ConvRot group size (a power of 4; 4 radix-4 digits)

// ---------------------------------------------------------------------------
// bf16 <-> fp32 (bit-level: exact widening, round-to-nearest-even narrowing)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// round-to-nearest-even fp32 -> bf16 bits; NaN -> canonical quiet NaN
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return u >> 16;
}
// fp32 -> bf16 -> fp32 through the hardware round-to-nearest-even conversion:
// the bits of f32_to_bf16_bits for every non-NaN value (a NaN stays a NaN)
__device__ __forceinline__ float round_bf16(float f) {
    uint16_t h;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f));
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
// the same for two values with one conversion
__device__ __forceinline__ void round_bf16x2(float &lo, float &hi) {
    uint32_t p;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
    lo = __uint_as_float(p << 16);
    hi = __uint_as_float(p & 0xFFFF0000u);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return f32_to_bf16_bits(lo) | (f32_to_bf16_bits(hi) << 16);
}

// 16 packed bf16 (two 16-byte words) -> 16 fp32
__device__ __forceinline__ void unpack16_bf16(const uint4 &a, const uint4 &b, float (&v)[16]) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[2 * j] = bf16_lo(w[j]);
        v[2 * j + 1] = bf16_hi(w[j]);
    }
}

// ---------------------------------------------------------------------------
// The radix-4 ConvRot butterflies, without the 1/2 factor of each stage.
//
// H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]; one stage is H4/2.  The
// 1/2 of the four stages is applied once at the end (x 1/16): a power-of-two
// scaling commutes with fp32 rounding, so the result carries exactly the bits
// of the per-stage form for every normal-range value.
//
// axis_seq: the accumulation-chain association, out_r = ((h0 a0 + h1 a1) + h2
//   a2) + h3 a3.  The shared first partial sums give 2.5 adds per element.
// axis_bfly: the butterfly association, p=a0+a1, m=a0-a1, q=a2+a3, n=a2-a3,
//   out = (p+n, p-n, m+q, q-m).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void axis_seq(float &a0, float &a1, float &a2, float &a3) {
    const float p = __fadd_rn(a0, a1), m = __fsub_rn(a0, a1);
    const float o0 = __fsub_rn(__fadd_rn(p, a2), a3);
    const float o1 = __fadd_rn(__fsub_rn(p, a2), a3);
    const float o2 = __fadd_rn(__fadd_rn(m, a2), a3);
    const float o3 = __fadd_rn(__fsub_rn(a2, m), a3);
    a0 = o0; a1 = o1; a2 = o2; a3 = o3;
}
__device__ __forceinline__ void axis_bfly(float &a0, float &a1, float &a2, float &a3) {
    const float p = __fadd_rn(a0, a1), m = __fsub_rn(a0, a1);
    const float q = __fadd_rn(a2, a3), n = __fsub_rn(a2, a3);
    a0 = __fadd_rn(p, n); a1 = __fsub_rn(p, n); a2 = __fadd_rn(m, q); a3 = __fsub_rn(q, m);
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// A wait that always ends.  It gives up after timeout_ns of wall time (2 s
// unless given; or kWaitMaxIters polls), records `site` in *fault (first
// writer wins) and returns false; it also returns false as soon as another
// thread has recorded a fault, so every role of every CTA leaves its loop
// within a bounded time.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s
constexpr uint32_t kWaitMaxIters = 1u << 28;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *fault, int site,
                                          uint64_t timeout_ns = kWaitTimeoutNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1; it < kWaitMaxIters; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0u) {
            if (*reinterpret_cast<volatile int *>(fault) != 0) return false;
            if (global_timer_ns() - t0 > timeout_ns) break;
        }
    }
    atomicCAS(fault, 0, site);
    return false;
}

// TMA: 2-D tiled bulk tensor load into this CTA's shared memory, completing
// `bytes` on the mbarrier.  x is the innermost coordinate (elements).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, uint32_t bar, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start (prologue, barrier set-up, TMEM
// allocation) while the kernel before it in the stream is still running.
// pdl_wait() returns once every prerequisite grid has completed and its memory
// operations are visible (a no-op for a kernel launched without the
// attribute); pdl_trigger() lets the next such kernel begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// tcgen05: TMEM allocation (one full warp), MMA issue and commit (one thread),
// TMEM -> register loads (one warp per 32-lane quarter).
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tcgen05.wait::ld that also "redefines" the 32 registers of a pending
// tcgen05.ld, so the compiler cannot move their uses above the wait
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
          "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
          "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
          "+r"(r[31])
        :
        : "memory");
}
// 32 TMEM lanes x 32-bit, 32 consecutive columns: thread t of the warp gets
// lane (base_lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// ---------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs on neighbouring SMs): the tensor-core MMA
// with .cta_group::2 spans both SMs.  Rank 0 (the leader) issues the MMAs; each
// CTA holds half of every operand tile at the same shared-memory offset and
// half of the accumulator rows in its own TMEM.  Every tcgen05 instruction of
// such a kernel uses .cta_group::2.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// the shared::cluster address of `addr` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t peer_smem(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// all threads of both CTAs; orders each thread's earlier memory operations
// (remote mbarrier arrivals included) before the peer's later ones
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (`bar` is a shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, uint32_t bar, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.cta_group::2"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T (M = 256 over the pair)
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on an mbarrier of either CTA (shared::cluster address) once every
// pair MMA this thread issued has completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// TMA: 2-D tiled bulk tensor store from this CTA's shared memory (bulk group)
__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA)
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completing on an mbarrier
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}
// 1-D bulk copy shared -> global (bulk group)
__device__ __forceinline__ void bulk_store(void *dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                     reinterpret_cast<uint64_t>(dst)),
                 "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Packed fp32x2 arithmetic (sm_100): two independent IEEE round-to-nearest
// operations per instruction; the bits are those of the scalar operations.
struct f2 {
    uint64_t v;
};
__device__ __forceinline__ f2 mk2(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void un2(f2 x, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x.v));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
// two fp32 -> packed bf16x2 (round to nearest even), lo in the low half
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---------------------------------------------------------------------------
// The quantizers' per-row scale s = max(amax / 127, 1e-30) and its reciprocal,
// both IEEE round-to-nearest, without the library divide / reciprocal calls
// (each is a subroutine with a slow-path branch, and every warp of a
// quantizer evaluates them once per row).
//
// div127_rn: division by the constant 127 with one FMA correction (Markstein,
//   IBM J. Res. Dev. 34(1), 1990; Brisebarre, Muller and Raina, "Accelerating
//   correctly rounded floating-point division when the divisor is known in
//   advance", IEEE Trans. Computers 53(8), 2004):
//   c = RN(1/127), q = RN(a c), r = a - 127 q (exact in one FMA), RN(q + r c).
// rcp_rn: the hardware reciprocal estimate refined by two Newton-Raphson steps
//   in FMA form, y' = RN(y + y RN(1 - s y)); the second is Markstein's
//   correctly rounding iteration for an estimate within one ulp of 1/s.
// row_scale_inv uses them for every finite amax and the library calls for
// NaN and the few values above 3e38.  xpuint8_check_scale_math compares it with
// the library-call form on every non-negative float, bit for bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float div127_rn(float a) {
    const float c = __uint_as_float(0x3C010204u);  // RN(1/127)
    const float q = __fmul_rn(a, c);
    const float r = __fmaf_rn(-q, 127.0f, a);
    return __fmaf_rn(r, c, q);
}
__device__ __forceinline__ float rcp_rn(float s) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
    float e = __fmaf_rn(-s, y, 1.0f);
    y = __fmaf_rn(y, e, y);
    e = __fmaf_rn(-s, y, 1.0f);
    return __fmaf_rn(y, e, y);
}
// s = max(amax / 127, 1e-30) and 1 / s
__device__ __forceinline__ float row_scale_inv(float amax, float &s) {
    if (amax <= 3.0e38f) {
        s = fmaxf(div127_rn(amax), 1e-30f);
        return rcp_rn(s);
    }
    s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    return __frcp_rn(s);
}
// RN(x / s) given y = RN(1 / s): Markstein's correction of the product with
// the reciprocal, q0 = RN(x y), r = x - s q0 (exact in one FMA), RN(q0 + r y)
__device__ __forceinline__ float div_by_rcp(float x, float s, float y) {
    const float q0 = __fmul_rn(x, y);
    const float r = __fmaf_rn(-q0, s, x);
    return __fmaf_rn(r, y, q0);
}
// the same with the library calls (the definition the fast form is checked against)
__device__ __forceinline__ float row_scale_inv_lib(float amax, float &s) {
    s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
    return __frcp_rn(s);
}

__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return r;
}
// rint(v * inv) for |v * inv| < 2^22, as fp32 bits whose low byte is the
// two's-complement int8 code: p = RN(v * inv), then RN(p * 1 + 1.5*2^23).
// The sum is written as an FMA with an exact unit product because ptxas
// contracts a packed multiply feeding a packed add into one FFMA2 even
// without -fmad (rounding v*inv + 1.5*2^23 once instead of twice); an FMA's
// multiplicand cannot absorb another multiply.  xpuint8_check_scale_math
// checks the result against the scalar operations.
__device__ __forceinline__ f2 quant_magic2(f2 v, float inv0, float inv1) {
    return fma2(mul2(v, mk2(inv0, inv1)), mk2(1.0f, 1.0f), mk2(12582912.0f, 12582912.0f));
}
// max(m, |a|, |b|) in one three-input maximum
__device__ __forceinline__ float max3_abs(float m, float a, float b) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
    return r;
}

// UMMA shared-memory matrix descriptor, 128-byte swizzle (sm100 version 1).
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  version (1)
//   bits 61-63  layout (2 = SWIZZLE_128B)
__device__ __forceinline__ uint64_t umma_sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// UMMA instruction descriptor for kind::i8 (signed x signed -> s32).
//   bits 4-5 D format (2 = S32), 7-9 A format (1 = S8), 10-12 B format (1 = S8),
//   bit 15/16 A/B major (0 = K, 1 = MN), 17-22 N>>3, 24-28 M>>4
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N, bool a_mn, bool b_mn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace xpuint8
