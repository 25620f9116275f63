// The INT8 linear for callers that cannot allocate device memory.
//
// xpuint8_linear_stream needs two scratch buffers between its kernels: the
// rotated int8 activation (M x K bytes) and its per-row scales (M floats).
// Some callers have no way to provide them: a plugin loaded into an
// application that owns every byte of the GPU's memory through its own pool
// and forbids side allocations, a C caller without a device allocator of its
// own, or code on a path where calling cudaMalloc would synchronise the
// device.  xpuint8_linear_noalloc_stream takes only the inputs and the output
// and keeps its scratch in a fixed array compiled into this library, so it
// allocates nothing.
//
// The array's cost and limits:
//   * every GPU that loads the library holds kNoAllocQBytes + 4 * kNoAllocRows
//     bytes (8 MiB + 64 KiB) until the process exits;
//   * a call accepts at most kNoAllocRows rows and M * K <= kNoAllocQBytes;
//     larger calls return 2 with a message and launch nothing;
//   * all calls on a device share the one array: two calls whose work
//     overlaps on the GPU (different streams without ordering between them)
//     race on it.  Calls on one stream, or otherwise ordered, are safe.
//
// Set-up: the first call in each CUDA context (for the runtime's primary
// context: the first call on each device) looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and keeps it, keyed by the
// context's unique id; that first call may also load this library's device
// code.  Make it before any stream capture on that device.  A device reset, or
// a host application that makes another context current, gives a new id and
// the address is looked up again: a kept address is never used in a context
// other than the one it was resolved in.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "internal.h"
#include "xpu_kernels/convrot.h"

namespace xpuint8 {
namespace {

constexpr int64_t kNoAllocQBytes = int64_t(8) << 20;  // int8 activations, 8 MiB
constexpr int64_t kNoAllocRows = 16384;                 // fp32 row scales, 64 KiB

// The scratch itself.  In host code these names are host-side stand-ins, not
// device addresses: only the addresses resolved below may be handed to a kernel.
static __device__ __align__(256) int8_t g_noalloc_q[kNoAllocQBytes];
static __device__ __align__(256) float g_noalloc_scale[kNoAllocRows];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

// the driver's cuCtxGetCurrent / cuCtxGetId (looked up once)
struct CtxFns {
    CtxGetCurrentFn current = nullptr;
    CtxGetIdFn id = nullptr;
};
const CtxFns &ctx_fns() {
    static CtxFns fns;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fns.current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fns.id = reinterpret_cast<CtxGetIdFn>(p);
    });
    return fns;
}

// the unique id of the context current on this thread (0 = none yet)
unsigned long long current_ctx_id() {
    const CtxFns &f = ctx_fns();
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!f.current || !f.id || f.current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (f.id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// resolved addresses, one entry per context seen (oldest replaced when full)
constexpr int kMaxContexts = 64;
struct Resolved {
    unsigned long long ctx_id;
    int8_t *q;
    float *scale;
};
std::mutex g_mutex;
Resolved g_resolved[kMaxContexts];
int g_next = 0;

// device addresses of the scratch in the current context (looked up once per context)
int resolve_scratch(int8_t **q, float **scale) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        set_error("linear_noalloc: no usable current device");
        return 1;
    }
    unsigned long long id = current_ctx_id();
    void *pq = nullptr, *ps = nullptr;
    if (id == 0) {
        // no context is current yet: the lookup makes the runtime's primary
        // context of `dev` current, and the addresses belong to it
        cudaError_t e = cudaGetSymbolAddress(&pq, g_noalloc_q);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&ps, g_noalloc_scale);
        if (e != cudaSuccess) {
            set_error(std::string("linear_noalloc: cannot resolve the built-in scratch: ") +
                      cudaGetErrorString(e));
            return 5;
        }
        id = current_ctx_id();
        if (id == 0) {
            set_error("linear_noalloc: no CUDA context is current after the symbol lookup");
            return 5;
        }
    }
    std::lock_guard<std::mutex> lock(g_mutex);
    for (const Resolved &r : g_resolved) {
        if (r.ctx_id == id) {
            *q = r.q;
            *scale = r.scale;
            return 0;
        }
    }
    if (!pq) {
        cudaError_t e = cudaGetSymbolAddress(&pq, g_noalloc_q);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&ps, g_noalloc_scale);
        if (e != cudaSuccess) {
            set_error(std::string("linear_noalloc: cannot resolve the built-in scratch: ") +
                      cudaGetErrorString(e));
            return 5;
        }
    }
    Resolved &slot = g_resolved[g_next];
    g_next = (g_next + 1) % kMaxContexts;
    slot.ctx_id = id;
    slot.q = static_cast<int8_t *>(pq);
    slot.scale = static_cast<float *>(ps);
    *q = slot.q;
    *scale = slot.scale;
    return 0;
}

}  // namespace
}  // namespace xpuint8

using namespace xpuint8;

extern "C" int xpuint8_linear_noalloc_stream(const void *stream, const void *x, const int8_t *w8,
                                             const float *w_scale, const float *bias, void *out,
                                             int64_t M, int64_t N, int64_t K, int32_t activation) {
    if (M <= 0 || K <= 0) {
        set_error("M and K must be positive");
        return 2;
    }
    if (M > kNoAllocRows || K > kNoAllocQBytes || M * K > kNoAllocQBytes) {
        set_error("linear_noalloc: M=" + std::to_string(M) + ", K=" + std::to_string(K) +
                  " exceeds the built-in scratch (at most " + std::to_string(kNoAllocRows) +
                  " rows and M*K <= " + std::to_string(kNoAllocQBytes) +
                  "); use xpuint8_linear_stream with caller-provided scratch");
        return 2;
    }
    int8_t *q = nullptr;
    float *scale = nullptr;
    if (int rc = resolve_scratch(&q, &scale)) return rc;
    return xpuint8_linear_stream(stream, x, w8, w_scale, bias, out, q, scale, M, N, K, activation);
}
