// The C ABI of libxpuint8 (include/xpu_kernels/convrot.h): argument checks,
// return codes, error text, and dispatch to the sm_100a kernels.
//
// Return codes follow the reference library (src/xpuint8.cpp:730-1081):
//   0 ok; 1 no usable device; 2 bad size / pointer / alignment; 3 K not a
//   multiple of 256; 4 unsupported group count; 5 launch failure; 6 bad
//   activation id.
// Stream semantics: `stream` is a cudaStream_t (the reference's `sycl_queue`
// argument).  NULL is the legacy default stream -- torch's default stream has
// handle 0 -- which is a deliberate difference from the reference, where a
// null queue is an error.  `_stream` entries enqueue and return; the entries
// without a stream run on the legacy default stream and wait for completion,
// as the reference's blocking entries do.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"
#include "xpu_kernels/convrot.h"

namespace xpuint8 {

namespace {
thread_local std::string g_error;
std::mutex g_init_mutex;
int g_init_rc = -1;
constexpr int kMaxDevices = 64;
std::string g_names[kMaxDevices];
int g_sms[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return 0;
    return d < kMaxDevices ? d : 0;
}
void fill_device(int d) {
    std::call_once(g_dev_once[d], [d] {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, d) == cudaSuccess) {
            g_names[d] = prop.name;
            g_sms[d] = prop.multiProcessorCount;
        } else {
            g_sms[d] = 148;
        }
    });
}
}  // namespace

void set_error(const std::string &msg) { g_error = msg; }

int launch_status(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return 0;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return 5;
}

int num_sms() {
    const int d = current_device();
    fill_device(d);
    return g_sms[d] > 0 ? g_sms[d] : 148;
}

}  // namespace xpuint8

using namespace xpuint8;

namespace {

cudaStream_t as_stream(const void *s) { return static_cast<cudaStream_t>(const_cast<void *>(s)); }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_mk(int64_t M, int64_t K) {
    if (M <= 0 || K <= 0) {
        set_error("M and K must be positive");
        return 2;
    }
    if (K % 256 != 0) {
        set_error("K must be divisible by the ConvRot group size (256)");
        return 3;
    }
    return 0;
}

int check_ptrs(std::initializer_list<const void *> ptrs) {
    for (const void *p : ptrs) {
        if (!p) {
            set_error("a required pointer is null");
            return 2;
        }
        if (!aligned16(p)) {
            set_error("device pointers must be 16-byte aligned");
            return 2;
        }
    }
    return 0;
}

// the blocking entries: run on the legacy default stream and wait
int finish_blocking(int rc, const char *what) {
    if (rc != 0) return rc;
    const cudaError_t e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) {
        set_error(std::string(what) + ": " + cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int convrot_quantize(cudaStream_t s, const void *x, int8_t *q, float *scale, int64_t M,
                     int64_t K, int act) {
    if (int rc = check_mk(M, K)) return rc;
    if (act < 0 || act > 5) {
        set_error("activation must be 1 (GELU-tanh), 2 (SwiGLU), 3 (situ), 4 (GEGLU) "
                  "or 5 (GELU-erf)");
        return 6;
    }
    if (int rc = check_ptrs({x, q, scale})) return rc;
    return launch_rotate_rows(s, 0, act, x, nullptr, nullptr, q, scale, M, K);
}

int dequant_act_quantize(cudaStream_t s, const void *acc, int8_t *q, float *scale,
                         const float *x_scale, const float *w_scale, int64_t M, int64_t K,
                         int32_t act) {
    if (int rc = check_mk(M, K)) return rc;
    if (act != 3 && act != 4 && act != 5) {
        set_error("dequant_act_quantize supports activation 3 (situ), 4 (GEGLU) or 5 (GELU-erf)");
        return 6;
    }
    if (int rc = check_ptrs({acc, q, w_scale})) return rc;
    if (!x_scale || !scale) {
        set_error("a required pointer is null");
        return 2;
    }
    return launch_rotate_rows(s, 1, act, acc, w_scale, x_scale, q, scale, M, K);
}

int rotate_bf16(cudaStream_t s, const void *x, void *xr, int64_t M, int64_t K) {
    if (int rc = check_mk(M, K)) return rc;
    if (int rc = check_ptrs({x, xr})) return rc;
    return launch_rotate_rows(s, 2, 0, x, nullptr, nullptr, xr, nullptr, M, K);
}

int dequant_weight(cudaStream_t s, const void *w8, const float *w_scale, void *out, int64_t N,
                   int64_t K) {
    if (N <= 0 || K <= 0) {
        set_error("N and K must be positive");
        return 2;
    }
    if (K % 256 != 0) {
        set_error("K must be divisible by the ConvRot group size (256)");
        return 3;
    }
    if (int rc = check_ptrs({w8, out})) return rc;
    if (!w_scale) {
        set_error("a required pointer is null");
        return 2;
    }
    return launch_rotate_rows(s, 3, 0, w8, w_scale, nullptr, out, nullptr, N, K);
}

int dequant_epilogue(cudaStream_t s, const int32_t *acc, void *out, const float *x_scale,
                     const float *w_scale, const float *bias, int64_t M, int64_t N,
                     int64_t stride, bool slice) {
    if (M <= 0 || N <= 0 || N % 16 != 0 || stride < N) {
        set_error(slice ? "M, N must be positive, N a multiple of 16, acc_row_stride >= N"
                        : "M, N must be positive and N must be a multiple of 16");
        return 2;
    }
    if (!acc || !out || !x_scale || !w_scale) {
        set_error("a required pointer is null");
        return 2;
    }
    if (!aligned16(out) || !aligned16(w_scale) || (bias && !aligned16(bias)) ||
        (reinterpret_cast<uintptr_t>(acc) & 3u)) {
        set_error("out, w_scale and bias must be 16-byte aligned");
        return 2;
    }
    return launch_dequant_epilogue(s, acc, out, x_scale, w_scale, bias, M, N, stride);
}

// layout: 0 = a [M,K], b [N,K] (a @ b^T); 1 = a [M,K], b [K,N] (a @ b);
//         2 = a [K,M], b [K,N] (a^T @ b)
// b_early: the kernel launched just before on `s` is this library's activation
// quantizer (or does not write b, col_scale, bias), so the GEMM may load those
// before it completes
int int_mm_common(cudaStream_t s, int epi, const int8_t *a, const int8_t *b, void *out,
                  const float *row_scale, const float *col_scale, const float *bias, int64_t M,
                  int64_t N, int64_t K, int32_t layout, int64_t ldo, bool b_early = false) {
    if (M <= 0 || N <= 0 || K <= 0) {
        set_error("M, N and K must be positive");
        return 2;
    }
    if (layout < 0 || layout > 2) {
        set_error("layout must be 0 (a @ b.T), 1 (a @ b) or 2 (a.T @ b)");
        return 2;
    }
    if (!a || !b || !out) {
        set_error("a required pointer is null");
        return 2;
    }
    if (ldo < N) {
        set_error("the output row stride must be >= N");
        return 2;
    }
    GemmCall c;
    c.epilogue = epi;
    c.a = a; c.b = b; c.out = out; c.ldo = ldo;
    c.row_scale = row_scale; c.col_scale = col_scale; c.bias = bias;
    c.M = M; c.N = N; c.K = K;
    c.b_early = b_early;
    c.a_mn = layout == 2;
    c.b_mn = layout >= 1;
    c.lda = c.a_mn ? M : K;
    c.ldb = c.b_mn ? N : K;
    if ((c.lda % 16) || (c.ldb % 16) || !aligned16(a) || !aligned16(b)) {
        set_error("int8 operands need 16-byte aligned bases and row lengths that are "
                  "multiples of 16");
        return 2;
    }
    return launch_gemm(s, c);
}

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

struct FfnLayout {
    size_t xq, xs, mid, q2, xs2, total;
};
FfnLayout ffn_layout(int64_t M, int64_t K, int64_t inner, int act) {
    FfnLayout L{};
    size_t off = 0;
    L.xq = off; off += align256(static_cast<size_t>(M) * K);
    L.xs = off; off += align256(static_cast<size_t>(M) * 4);
    (void)act;  // every activation's intermediate is the bf16 y
    L.mid = off; off += align256(static_cast<size_t>(M) * inner * 2);
    L.q2 = off; off += align256(static_cast<size_t>(M) * inner);
    L.xs2 = off; off += align256(static_cast<size_t>(M) * 4);
    L.total = off;
    return L;
}

}  // namespace

extern "C" {

int xpuint8_init(void) {
    std::lock_guard<std::mutex> lock(g_init_mutex);
    if (g_init_rc >= 0) return g_init_rc;
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        set_error(std::string("no CUDA device: ") +
                  (e != cudaSuccess ? cudaGetErrorString(e) : "device count is 0"));
        g_init_rc = 1;
        return 1;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major != 10 || prop.minor != 0) {
        set_error("libxpuint8 is built for sm_100a (B200); the current device is not compute "
                  "capability 10.0");
        g_init_rc = 1;
        return 1;
    }
    g_init_rc = 0;
    return 0;
}

const char *xpuint8_device_name(void) {
    if (xpuint8_init() != 0) return nullptr;
    const int d = current_device();
    fill_device(d);
    return g_names[d].c_str();
}

int xpuint8_convrot_groupsize(void) { return 256; }

const char *xpuint8_last_error(void) { return g_error.c_str(); }

int xpuint8_convrot_quantize(const void *x, int8_t *q, float *scale, int64_t M, int64_t K) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(convrot_quantize(0, x, q, scale, M, K, 0), "convrot_quantize");
}

int xpuint8_convrot_quantize_stream(const void *stream, const void *x, int8_t *q, float *scale,
                                    int64_t M, int64_t K) {
    return convrot_quantize(as_stream(stream), x, q, scale, M, K, 0);
}

int xpuint8_convrot_quantize_act(const void *x, int8_t *q, float *scale, int64_t M, int64_t K,
                                 int32_t activation) {
    if (xpuint8_init() != 0) return 1;
    if (activation < 1 || activation > 5) {
        set_error("activation must be 1 (GELU-tanh), 2 (SwiGLU), 3 (situ), 4 (GEGLU) "
                  "or 5 (GELU-erf)");
        return 6;
    }
    return finish_blocking(convrot_quantize(0, x, q, scale, M, K, activation),
                           "convrot_quantize_act");
}

int xpuint8_convrot_quantize_act_stream(const void *stream, const void *x, int8_t *q, float *scale,
                                        int64_t M, int64_t K, int32_t activation) {
    if (activation < 1 || activation > 5) {
        set_error("activation must be 1 (GELU-tanh), 2 (SwiGLU), 3 (situ), 4 (GEGLU) "
                  "or 5 (GELU-erf)");
        return 6;
    }
    return convrot_quantize(as_stream(stream), x, q, scale, M, K, activation);
}

int xpuint8_dequant_weight(const void *w8, const float *w_scale, void *out, int64_t N, int64_t K) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(dequant_weight(0, w8, w_scale, out, N, K), "dequant_weight");
}

int xpuint8_dequant_weight_stream(const void *stream, const void *w8, const float *w_scale,
                                  void *out, int64_t N, int64_t K) {
    return dequant_weight(as_stream(stream), w8, w_scale, out, N, K);
}

int xpuint8_convrot_rotate_bf16(const void *x, void *xr, int64_t M, int64_t K) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(rotate_bf16(0, x, xr, M, K), "convrot_rotate_bf16");
}

int xpuint8_convrot_rotate_bf16_stream(const void *stream, const void *x, void *xr, int64_t M,
                                       int64_t K) {
    return rotate_bf16(as_stream(stream), x, xr, M, K);
}

int xpuint8_dequant_epilogue(const int32_t *acc, void *out, const float *x_scale,
                             const float *w_scale, const float *bias, int64_t M, int64_t N) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(dequant_epilogue(0, acc, out, x_scale, w_scale, bias, M, N, N, false),
                           "dequant_epilogue");
}

int xpuint8_dequant_epilogue_stream(const void *stream, const int32_t *acc, void *out,
                                    const float *x_scale, const float *w_scale, const float *bias,
                                    int64_t M, int64_t N) {
    return dequant_epilogue(as_stream(stream), acc, out, x_scale, w_scale, bias, M, N, N, false);
}

int xpuint8_dequant_epilogue_slice(const int32_t *acc, void *out, const float *x_scale,
                                   const float *w_scale, const float *bias, int64_t M, int64_t N,
                                   int64_t acc_row_stride) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(dequant_epilogue(0, acc, out, x_scale, w_scale, bias, M, N,
                                            acc_row_stride, true),
                           "dequant_epilogue_slice");
}

int xpuint8_dequant_epilogue_slice_stream(const void *stream, const int32_t *acc, void *out,
                                          const float *x_scale, const float *w_scale,
                                          const float *bias, int64_t M, int64_t N,
                                          int64_t acc_row_stride) {
    return dequant_epilogue(as_stream(stream), acc, out, x_scale, w_scale, bias, M, N,
                            acc_row_stride, true);
}

int xpuint8_dequant_act_quantize(const void *acc, int8_t *q, float *scale, const float *x_scale,
                                 const float *w_scale, int64_t M, int64_t K, int32_t activation) {
    if (xpuint8_init() != 0) return 1;
    return finish_blocking(dequant_act_quantize(0, acc, q, scale, x_scale, w_scale, M, K, activation),
                           "dequant_act_quantize");
}

int xpuint8_dequant_act_quantize_stream(const void *stream, const void *acc, int8_t *q,
                                        float *scale, const float *x_scale, const float *w_scale,
                                        int64_t M, int64_t K, int32_t activation) {
    return dequant_act_quantize(as_stream(stream), acc, q, scale, x_scale, w_scale, M, K,
                                activation);
}

// ---------------------------------------------------------------- new entries

int xpuint8_int_mm_stream(const void *stream, const int8_t *a, const int8_t *b, int32_t *c,
                          int64_t M, int64_t N, int64_t K, int32_t layout, int64_t ldc) {
    return int_mm_common(as_stream(stream), kEpiRawI32, a, b, c, nullptr, nullptr, nullptr, M, N,
                         K, layout, ldc);
}

int xpuint8_int_mm_dequant_stream(const void *stream, const int8_t *a, const int8_t *b, void *out,
                                  const float *row_scale, const float *col_scale,
                                  const float *bias, int64_t M, int64_t N, int64_t K,
                                  int32_t layout, int64_t ldo) {
    if (!row_scale) {
        set_error("row_scale must not be null");
        return 2;
    }
    return int_mm_common(as_stream(stream), kEpiDequantBf16, a, b, out, row_scale, col_scale, bias,
                         M, N, K, layout, ldo);
}

int xpuint8_int_mm_geglu_stream(const void *stream, const int8_t *a, const int8_t *up_w8, void *y,
                                const float *x_scale, const float *up_scale, int64_t M,
                                int64_t inner, int64_t K) {
    if (!x_scale || !up_scale) {
        set_error("x_scale and up_scale must not be null");
        return 2;
    }
    return int_mm_common(as_stream(stream), kEpiGegluBf16, a, up_w8, y, x_scale, up_scale, nullptr,
                         M, inner, K, 0, inner);
}

int xpuint8_linear_stream(const void *stream, const void *x, const int8_t *w8,
                          const float *w_scale, const float *bias, void *out, int8_t *xq,
                          float *xs, int64_t M, int64_t N, int64_t K, int32_t activation) {
    if (N <= 0 || N % 16 != 0) {
        set_error("N must be a positive multiple of 16");
        return 2;
    }
    if (int rc = convrot_quantize(as_stream(stream), x, xq, xs, M, K, activation)) return rc;
    return int_mm_common(as_stream(stream), kEpiDequantBf16, xq, w8, out, xs, w_scale, bias, M, N,
                         K, 0, N, true);
}

int xpuint8_linear_split_stream(const void *stream, const void *x, const int8_t *w8,
                                const float *w_scale, const float *bias, void *const *outs,
                                int32_t nparts, int8_t *xq, float *xs, int64_t M, int64_t N,
                                int64_t K, int32_t activation) {
    if (N <= 0 || N % 32 != 0) {
        set_error("linear_split: each part's width N must be a positive multiple of 32");
        return 2;
    }
    if (!outs || nparts < 1 || nparts > 8) {
        set_error("linear_split: 1 <= nparts <= 8 and an output table are required");
        return 2;
    }
    for (int i = 0; i < nparts; ++i) {
        if (!outs[i] || !aligned16(outs[i])) {
            set_error("linear_split: every output buffer needs a 16-byte aligned base");
            return 2;
        }
    }
    if (!w8 || !w_scale || !aligned16(w8) || !aligned16(w_scale) || (bias && !aligned16(bias))) {
        set_error("linear_split: w8, w_scale (and bias) must be non-null and 16-byte aligned");
        return 2;
    }
    if (int rc = convrot_quantize(as_stream(stream), x, xq, xs, M, K, activation)) return rc;
    GemmCall c;
    c.epilogue = kEpiDequantBf16;
    c.a = xq; c.b = w8; c.lda = K; c.ldb = K;
    c.outs = outs; c.nout = nparts; c.ldo = N; c.split_n = N;
    c.row_scale = xs; c.col_scale = w_scale; c.bias = bias;
    c.M = M; c.N = static_cast<int64_t>(nparts) * N; c.K = K;
    c.b_early = true;  // the quantizer above is the kernel just before
    return launch_gemm(as_stream(stream), c);
}

int64_t xpuint8_ffn_workspace_bytes(int64_t M, int64_t K, int64_t inner, int32_t activation) {
    if (M <= 0 || K <= 0 || inner <= 0) return -1;
    return static_cast<int64_t>(ffn_layout(M, K, inner, activation).total);
}

int xpuint8_ffn_stream(const void *stream, const void *x, const int8_t *up_w8,
                       const float *up_scale, const int8_t *down_w8, const float *down_scale,
                       const float *down_bias, void *out, void *workspace, int64_t M, int64_t K,
                       int64_t inner, int32_t activation) {
    cudaStream_t s = as_stream(stream);
    if (activation != 3 && activation != 4 && activation != 5) {
        set_error("the fused FFN supports activation 3 (situ), 4 (GEGLU) or 5 (GELU-erf)");
        return 6;
    }
    if (int rc = check_mk(M, K)) return rc;
    if (inner <= 0 || inner % 256 != 0) {
        set_error("the FFN's inner width must be a positive multiple of 256");
        return 3;
    }
    if (!workspace || !aligned16(workspace)) {
        set_error("the FFN workspace must be a 16-byte aligned buffer");
        return 2;
    }
    const FfnLayout L = ffn_layout(M, K, inner, activation);
    char *ws = static_cast<char *>(workspace);
    int8_t *xq = reinterpret_cast<int8_t *>(ws + L.xq);
    float *xs = reinterpret_cast<float *>(ws + L.xs);
    int8_t *q2 = reinterpret_cast<int8_t *>(ws + L.q2);
    float *xs2 = reinterpret_cast<float *>(ws + L.xs2);
    if (int rc = convrot_quantize(s, x, xq, xs, M, K, 0)) return rc;
    // the up-projection's epilogue dequantizes, applies the activation and
    // stores y bf16 [M, inner]; y's rotate+quantize is then the reference's
    // dequant_act_quantize of the int32 accumulator (which rounds the dequant
    // and the activation to bf16 at the same points)
    void *y = ws + L.mid;
    const int epi = activation == 4 ? kEpiGegluBf16 : (activation == 3 ? kEpiSituBf16 : kEpiGeluBf16);
    if (int rc = int_mm_common(s, epi, xq, up_w8, y, xs, up_scale, nullptr, M, inner, K, 0, inner, true))
        return rc;
    if (int rc = convrot_quantize(s, y, q2, xs2, M, inner, 0)) return rc;
    return int_mm_common(s, kEpiDequantBf16, q2, down_w8, out, xs2, down_scale, down_bias, M, K,
                         inner, 0, K, true);
}

// ------------------------------------------------------------ fused backward
namespace {
struct DxLayout {
    size_t q, a, dxr, total;
};
DxLayout dx_layout(int64_t M, int64_t N, int64_t K) {
    DxLayout L{};
    size_t off = 0;
    L.q = off; off += align256(static_cast<size_t>(M) * N);       // int8 row-quantized dy
    L.a = off; off += align256(static_cast<size_t>(M) * 4);       // its row scales
    L.dxr = off; off += align256(static_cast<size_t>(M) * K * 2);  // dx before the rotation
    L.total = off;
    return L;
}
struct DwLayout {
    size_t gq, tg, amax, dwr, total;
};
DwLayout dw_layout(int64_t M, int64_t N, int64_t K) {
    DwLayout L{};
    size_t off = 0;
    L.gq = off; off += align256(static_cast<size_t>(M) * N);       // column-quantized dy * xs
    L.tg = off; off += align256(static_cast<size_t>(N) * 4);       // its column scales
    L.amax = off; off += align256(static_cast<size_t>(N) * 4);     // its column maxima
    L.dwr = off; off += align256(static_cast<size_t>(N) * K * 2);  // dW before the rotation
    L.total = off;
    return L;
}
int check_workspace(const void *ws) {
    if (!ws || !aligned16(ws)) {
        set_error("the workspace must be a 16-byte aligned buffer");
        return 2;
    }
    return 0;
}
}  // namespace

int64_t xpuint8_linear_dx_int8_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return -1;
    return static_cast<int64_t>(dx_layout(M, N, K).total);
}

int xpuint8_linear_dx_int8_stream(const void *stream, const void *dy, const int8_t *w8,
                                  const float *w_scale, void *dx, void *workspace, int64_t M,
                                  int64_t N, int64_t K) {
    cudaStream_t s = as_stream(stream);
    if (int rc = check_mk(M, K)) return rc;
    if (N <= 0 || N % 16 != 0) {
        set_error("linear_dx_int8: N must be a positive multiple of 16");
        return 2;
    }
    if (int rc = check_ptrs({dy, w8, w_scale, dx})) return rc;
    if (int rc = check_workspace(workspace)) return rc;
    const DxLayout L = dx_layout(M, N, K);
    char *ws = static_cast<char *>(workspace);
    int8_t *q = reinterpret_cast<int8_t *>(ws + L.q);
    float *a = reinterpret_cast<float *>(ws + L.a);
    void *dxr = ws + L.dxr;
    // d = bf16(dy * bf16(w_scale)) row-quantized in one pass
    if (int rc = launch_quantize_row(s, dy, w_scale, q, a, M, N)) return rc;
    // dxr = bf16(float(q @ w8) * a[m]): w8 [N, K] read as stored (MN-major B)
    if (int rc = int_mm_common(s, kEpiDequantBf16, q, w8, dxr, a, nullptr, nullptr, M, K, N, 1, K,
                               true))
        return rc;
    // the rotation undone along K
    return launch_rotate_rows(s, 2, 0, dxr, nullptr, nullptr, dx, nullptr, M, K);
}

int64_t xpuint8_linear_dw_int8_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return -1;
    return static_cast<int64_t>(dw_layout(M, N, K).total);
}

int xpuint8_linear_dw_int8_stream(const void *stream, const void *dy, const int8_t *xq,
                                  const float *x_scale, void *dw, void *workspace, int64_t M,
                                  int64_t N, int64_t K) {
    cudaStream_t s = as_stream(stream);
    if (int rc = check_mk(M, K)) return rc;
    if (N <= 0 || N % 16 != 0) {
        set_error("linear_dw_int8: N must be a positive multiple of 16");
        return 2;
    }
    if (int rc = check_ptrs({dy, xq, dw})) return rc;
    if (!x_scale) {
        set_error("a required pointer is null");
        return 2;
    }
    if (int rc = check_workspace(workspace)) return rc;
    const DwLayout L = dw_layout(M, N, K);
    char *ws = static_cast<char *>(workspace);
    int8_t *gq = reinterpret_cast<int8_t *>(ws + L.gq);
    float *tg = reinterpret_cast<float *>(ws + L.tg);
    void *dwr = ws + L.dwr;
    // g = dy * xs[m] quantized per column n (over the tokens m)
    if (int rc = launch_colquant(s, dy, x_scale, gq, tg, M, N,
                                 reinterpret_cast<unsigned int *>(ws + L.amax)))
        return rc;
    // dwr [N, K] = bf16(float(gq^T @ xq) * tg[n]): both operands MN-major
    if (int rc = int_mm_common(s, kEpiDequantBf16, gq, xq, dwr, tg, nullptr, nullptr, N, K, M, 2, K,
                               true))
        return rc;
    return launch_rotate_rows(s, 2, 0, dwr, nullptr, nullptr, dw, nullptr, N, K);
}

int xpuint8_quantize_row_stream(const void *stream, const void *x, const float *col_scale,
                                int8_t *q, float *scale, int64_t M, int64_t K) {
    if (M <= 0 || K <= 0) {
        set_error("M and K must be positive");
        return 2;
    }
    if (!x || !q || !scale) {
        set_error("a required pointer is null");
        return 2;
    }
    return launch_quantize_row(as_stream(stream), x, col_scale, q, scale, M, K);
}

int xpuint8_colquant_stream(const void *stream, const void *dy, const float *x_scale, int8_t *gq,
                            float *tg, int64_t M, int64_t N) {
    if (M <= 0 || N <= 0 || N % 16 != 0) {
        set_error("M, N must be positive and N must be a multiple of 16");
        return 2;
    }
    if (int rc = check_ptrs({dy, gq, tg})) return rc;
    if (!x_scale) {
        set_error("a required pointer is null");
        return 2;
    }
    return launch_colquant(as_stream(stream), dy, x_scale, gq, tg, M, N);
}

int xpuint8_rms_rope_stream(const void *stream, const void *x, int32_t x_is_int32, int64_t ldx,
                            const float *x_scale, const float *w_scale, const float *weight,
                            const float *freqs, int64_t freqs_batch, int64_t freqs_seq, void *out,
                            int64_t ldo, int64_t B, int64_t S, int64_t H, int64_t D, float eps,
                            int32_t split_half) {
    if (B <= 0 || S <= 0 || H <= 0) {
        set_error("rms_rope: B, S and H must be positive");
        return 2;
    }
    if (D != 64 && D != 128 && D != 256) {
        set_error("rms_rope: the head dim must be 64, 128 or 256");
        return 2;
    }
    if (ldx < H * D || ldo < H * D) {
        set_error("rms_rope: row strides must be at least H * D elements");
        return 2;
    }
    if ((freqs_batch != 1 && freqs_batch != B) || (freqs_seq != 1 && freqs_seq != S)) {
        set_error("rms_rope: freqs must be [1 or B, 1 or S, D/2, 2, 2]");
        return 2;
    }
    if (!x || !weight || !freqs || !out || (x_is_int32 && (!x_scale || !w_scale))) {
        set_error("a required pointer is null");
        return 2;
    }
    // 16-byte (int32) or 8-byte (bf16) accesses of four elements per head run
    const uintptr_t xa = reinterpret_cast<uintptr_t>(x);
    if (!aligned16(freqs) || !aligned16(weight) || (x_is_int32 && (!aligned16(w_scale) || (xa & 15u) || (ldx % 4))) ||
        (!x_is_int32 && ((xa & 7u) || (ldx % 4))) || (reinterpret_cast<uintptr_t>(out) & 7u) || (ldo % 4)) {
        set_error("rms_rope: freqs, weight (and w_scale) need 16-byte aligned bases; x (16 bytes "
                  "for int32, 8 for bf16) and out (8 bytes) aligned, row strides multiples of 4");
        return 2;
    }
    return launch_rms_rope(as_stream(stream), x, x_is_int32 != 0, ldx, x_scale, w_scale, weight, freqs,
                           freqs_batch, freqs_seq, out, ldo, B, S, H, D, eps, split_half != 0);
}

int xpuint8_fault_status(int32_t reset) {
    const int g = gemm_fault_status(reset);
    const int r = probe_fault_status(reset);
    if (g < 0 || r < 0) return -1;
    return g != 0 ? g : r;
}

int xpuint8_wait_probe(int64_t limit_ns, int32_t site, int64_t *elapsed_ns) {
    if (xpuint8_init() != 0) return 1;
    if (site == 0) {
        set_error("wait_probe: the site must be non-zero");
        return 2;
    }
    return launch_wait_probe(limit_ns, site, elapsed_ns);
}

// ---------------------------------------------------------------- peer buffers
int xpuint8_ipc_alloc(int64_t bytes, void **ptr, void *handle) {
    if (bytes <= 0 || !ptr || !handle) {
        set_error("ipc_alloc: a positive size and non-null ptr / handle are required");
        return 2;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (e != cudaSuccess) {
        set_error(std::string("ipc_alloc: cudaMalloc: ") + cudaGetErrorString(e));
        return 5;
    }
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error(std::string("ipc_alloc: cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
        return 5;
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return 0;
}

int xpuint8_ipc_open(const void *handle, void **ptr) {
    if (!handle || !ptr) {
        set_error("ipc_open: handle and ptr must not be null");
        return 2;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_error(std::string("ipc_open: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        return 5;
    }
    *ptr = p;
    return 0;
}

int xpuint8_ipc_close(void *ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) {
        set_error(std::string("ipc_close: ") + cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int xpuint8_ipc_free(void *ptr) {
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) {
        set_error(std::string("ipc_free: ") + cudaGetErrorString(e));
        return 5;
    }
    return 0;
}

int xpuint8_linear_allgather_cols_stream(const void *stream, const void *x, const int8_t *w8,
                                         const float *w_scale, const float *bias,
                                         void *const *outs, int32_t nranks, int64_t col_offset,
                                         int64_t n_total, int8_t *xq, float *xs, int64_t M,
                                         int64_t N, int64_t K, int32_t activation) {
    if (N <= 0 || N % 16 != 0) {
        set_error("N (this rank's columns) must be a positive multiple of 16");
        return 2;
    }
    if (!outs || nranks < 1 || nranks > 8) {
        set_error("allgather: 1 <= nranks <= 8 and an output table are required");
        return 2;
    }
    if (n_total % 16 != 0 || col_offset < 0 || col_offset % 16 != 0 || col_offset + N > n_total) {
        set_error("allgather: the column block [col_offset, col_offset + N) must lie inside the "
                  "n_total output columns, with col_offset and n_total multiples of 16");
        return 2;
    }
    void *dst[8];
    for (int r = 0; r < nranks; ++r) {
        if (!outs[r] || !aligned16(outs[r])) {
            set_error("allgather: every output buffer needs a 16-byte aligned base");
            return 2;
        }
        // this rank's column block of rank r's [M, n_total] output
        dst[r] = static_cast<char *>(outs[r]) + col_offset * 2;
    }
    if (!w8 || !w_scale || !aligned16(w8)) {
        set_error("a required pointer is null or misaligned");
        return 2;
    }
    if (int rc = convrot_quantize(as_stream(stream), x, xq, xs, M, K, activation)) return rc;
    GemmCall c;
    // 128-byte row segments per store: the tiles cross NVLink in larger writes
    c.epilogue = kEpiDequantWide;
    c.a = xq; c.b = w8; c.lda = K; c.ldb = K;
    c.outs = dst; c.nout = nranks; c.ldo = n_total;
    c.row_scale = xs; c.col_scale = w_scale; c.bias = bias;
    c.M = M; c.N = N; c.K = K;
    c.b_early = true;  // the quantizer above is the kernel just before
    return launch_gemm(as_stream(stream), c);
}

int xpuint8_linear_allgather_stream(const void *stream, const void *x, const int8_t *w8,
                                    const float *w_scale, const float *bias, void *const *outs,
                                    int32_t nranks, int32_t rank, int8_t *xq, float *xs, int64_t M,
                                    int64_t N, int64_t K, int32_t activation) {
    if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) {
        set_error("allgather: 1 <= nranks <= 8 and 0 <= rank < nranks are required");
        return 2;
    }
    return xpuint8_linear_allgather_cols_stream(stream, x, w8, w_scale, bias, outs, nranks,
                                                static_cast<int64_t>(rank) * N,
                                                static_cast<int64_t>(nranks) * N, xq, xs, M, N, K,
                                                activation);
}

int xpuint8_check_scale_math(int64_t *bad_scale, int64_t *bad_quant) {
    if (!bad_scale || !bad_quant) {
        set_error("a required pointer is null");
        return 2;
    }
    return check_scale_math(bad_scale, bad_quant);
}

}  // extern "C"
