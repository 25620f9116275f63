// Self-test of the library's device-side failure detection: a kernel whose
// bounded wait runs out on purpose.
//
// Every mbarrier wait of the GEMM goes through mbar_wait (common.cuh): after
// its time limit it records a site number in a device fault word and returns
// false, and the kernel then drains its own asynchronous work and exits, so a
// lost arrival becomes an error status the host can read instead of a hung
// GPU.  xpuint8_wait_probe exercises that path without a fault: one CTA
// initialises a shared-memory mbarrier that nothing will ever arrive on and
// waits on it through the same mbar_wait, with a short limit.  The wait gives
// up, the site lands in g_probe_fault (reported by xpuint8_fault_status and
// cleared by its reset), and the kernel returns normally.  No TMA, no tensor
// core, no trap: the only thing that "fails" is the wait.
//
// The probe has its own fault word, so a probe result left uncleared never
// makes a later GEMM give up early (the GEMM's waits watch g_gemm_fault).
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"
#include "internal.h"

namespace xpuint8 {

__device__ int g_probe_fault = 0;
__device__ unsigned long long g_probe_elapsed_ns = 0;

namespace {

__global__ void wait_probe_kernel(uint64_t limit_ns, int site) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);  // one arrival completes the phase; none will come
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_timer_ns();
        const bool ok = mbar_wait(b, 0, &g_probe_fault, site, limit_ns);
        g_probe_elapsed_ns = ok ? 0ull : global_timer_ns() - t0;
        asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(b) : "memory");
    }
    __syncthreads();
}

}  // namespace

int launch_wait_probe(int64_t limit_ns, int site, int64_t *elapsed_ns) {
    // at least 1 us, at most the library's own 2 s limit
    const uint64_t lim = static_cast<uint64_t>(
        limit_ns < 1000 ? 1000 : (limit_ns > static_cast<int64_t>(kWaitTimeoutNs)
                                      ? static_cast<int64_t>(kWaitTimeoutNs)
                                      : limit_ns));
    wait_probe_kernel<<<1, 32>>>(lim, site);
    if (const int rc = launch_status("wait probe")) return rc;
    const cudaError_t e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) {
        set_error(std::string("wait probe: ") + cudaGetErrorString(e));
        return 5;
    }
    unsigned long long el = 0;
    if (cudaMemcpyFromSymbol(&el, g_probe_elapsed_ns, sizeof(el)) != cudaSuccess)
        return launch_status("wait probe (read)");
    if (elapsed_ns) *elapsed_ns = static_cast<int64_t>(el);
    return 0;
}

int probe_fault_status(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_probe_fault, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_probe_fault, &zero, sizeof(int));
    }
    return v;
}

}  // namespace xpuint8
