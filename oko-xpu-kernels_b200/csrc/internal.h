// Host-side declarations shared between the translation units of libxpuint8.
// Every launcher validates nothing the C entry points already validated; it
// enqueues on `stream` and returns 0, or 5 with the error recorded.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace xpuint8 {

// error reporting (abi.cu): thread-local message read by xpuint8_last_error
void set_error(const std::string &msg);
int launch_status(const char *what);  // cudaGetLastError -> 0 or 5 (+ message)
int num_sms();                        // SM count of the current device

// rotation family (rotate.cu)
//   mode: 0 = activation bf16 -> int8 (act 0..5), 1 = dequant+act int32 -> int8 (act 3,4,5),
//         2 = rotate bf16 -> bf16, 3 = dequant_weight int8 -> bf16
int launch_rotate_rows(cudaStream_t s, int mode, int act, const void *in, const float *w_scale,
                       const float *x_scale, void *out, float *scale, int64_t M, int64_t K);

// streaming rotation (rotate_bulk.cu); -1 = shape not covered.  row_scale:
// mode 3's weight scale, mode 1's x_scale; col_scale: mode 1's w_scale
int launch_rotate_bulk(cudaStream_t s, int mode, int act, const void *in, const float *row_scale,
                       const float *col_scale, void *out, float *scale, int64_t M, int64_t K);
// self-check of the quantizers' scale arithmetic (rotate_bulk.cu); counts mismatches
int check_scale_math(int64_t *bad_scale, int64_t *bad_quant);

// dequant epilogue (epilogue.cu)
int launch_dequant_epilogue(cudaStream_t s, const int32_t *acc, void *out, const float *x_scale,
                            const float *w_scale, const float *bias, int64_t M, int64_t N,
                            int64_t acc_row_stride);

// row / column quantizers (rowquant.cu)
int launch_quantize_row(cudaStream_t s, const void *x, const float *col_scale, int8_t *q,
                        float *scale, int64_t M, int64_t K);
// amax_ws: N words of scratch for the column maxima (the scales are then
// made inside the quantizing pass); NULL: tg holds them (one launch more)
int launch_colquant(cudaStream_t s, const void *dy, const float *x_scale, int8_t *gq, float *tg,
                    int64_t M, int64_t N, unsigned int *amax_ws = nullptr);

// tcgen05 int8 GEMM (gemm_i8.cu)
// kEpiDequantWide: the dequant epilogue storing 32 rows x 64 columns (128-byte
// row segments) per TMA store instead of 32 x 32, one ring stage fewer: for
// outputs written over NVLink, where small writes waste link bandwidth
// kEpiSituBf16: the GEGLU tile layout ([hidden | gate] rows) with MossImage's
// situ; kEpiGeluBf16: the dequant epilogue followed by the erf-GELU (each the
// activation of the fused FFN's up-projection, stored as bf16)
enum GemmEpilogue {
    kEpiRawI32 = 0,
    kEpiDequantBf16 = 1,
    kEpiGegluBf16 = 2,
    kEpiDequantWide = 3,
    kEpiSituBf16 = 4,
    kEpiGeluBf16 = 5
};
struct GemmCall {
    int epilogue = kEpiRawI32;
    const int8_t *a = nullptr;  // [M,K] (a_mn=0) or [K,M] (a_mn=1), row stride lda
    const int8_t *b = nullptr;  // [N,K] (b_mn=0) or [K,N] (b_mn=1), row stride ldb
    bool a_mn = false, b_mn = false;
    int64_t lda = 0, ldb = 0;
    void *out = nullptr;        // int32 or bf16 [M, N], row stride ldo (elements)
    int64_t ldo = 0;
    void *const *outs = nullptr;  // instead of out: nout destinations, each tile stored to all
    int nout = 0;
    // > 0 (with outs): the output's columns in consecutive parts of split_n,
    // part i stored to outs[i] as its own [M, split_n] (row stride ldo)
    int64_t split_n = 0;
    const float *row_scale = nullptr;  // [M]  (x_scale)
    const float *col_scale = nullptr;  // [N]  (w_scale) or null = 1; GEGLU: [2N]
    const float *bias = nullptr;       // [N]  or null
    int64_t M = 0, N = 0, K = 0;       // GEGLU: N = output width (half of B's rows)
    // B, col_scale and bias are not written by the kernel launched just before
    // this GEMM on the stream (the linear entries: that kernel is the
    // activation quantizer), so the GEMM may load them before waiting for it
    bool b_early = false;
};
int launch_gemm(cudaStream_t s, const GemmCall &c);
int gemm_fault_status(int reset);  // device fault word of the GEMM waits

// RMS norm + rotary embedding of attention heads (rope.cu), from bf16 heads or
// from the int32 accumulator with its dequant
int launch_rms_rope(cudaStream_t s, const void *in, bool in_int32, int64_t ld_in, const float *x_scale,
                    const float *w_scale, const float *weight, const float *freqs, int64_t fb,
                    int64_t fs, void *out, int64_t ld_out, int64_t B, int64_t S, int64_t H, int64_t D,
                    float eps, bool split_half);

// the bounded-wait self-test (waitprobe.cu): one CTA waits on an mbarrier that
// nothing arrives on, gives up after limit_ns and records `site`
int launch_wait_probe(int64_t limit_ns, int site, int64_t *elapsed_ns);
int probe_fault_status(int reset);  // its fault word

}  // namespace xpuint8
