/* libxpuint8 for NVIDIA B200 (sm_100a): fused ConvRot INT8 primitives.
 *
 * A drop-in for the reference library's C ABI (okolenmi/oko-xpu-kernels,
 * include/xpu_kernels/convrot.h): the same symbols, argument meanings and
 * return codes, implemented with hand-written CUDA kernels.  Each declaration
 * below cites the reference declaration it replaces.  The entries after the
 * marked line are new: the reference obtained the GEMM from torch._int_mm and
 * the row quantizer from Triton, so it has no C symbol for them.
 *
 * Pointers are caller-owned device pointers (16-byte aligned); nothing is
 * allocated per call.  Scales and bias are fp32; activations and outputs bf16.
 *
 * Streams: `stream` is a cudaStream_t passed as `const void *` (the
 * reference's `const void *sycl_queue`).  NULL selects the legacy default
 * stream (torch's default stream has handle 0), where the reference returned
 * an error for a null queue.  `_stream` entries enqueue asynchronously and
 * never synchronise; the entries without a stream run on the legacy default
 * stream and block until the work is done.
 *
 * Return codes: 0 ok; 1 no usable device; 2 bad size, null pointer or
 * misalignment; 3 K (or the FFN inner width) not a multiple of 256; 4
 * unsupported group count (K > 32768); 5 kernel launch failure; 6 bad
 * activation id.  The message is in xpuint8_last_error() (per thread).
 */
#ifndef XPU_INT8_H
#define XPU_INT8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Checks that a compute capability 10.0 device is present.
 * Replaces convrot.h:30 xpuint8_init. */
int xpuint8_init(void);

/* Name of the current device, or NULL without one.
 * Replaces convrot.h:33 xpuint8_device_name. */
const char *xpuint8_device_name(void);

/* The ConvRot group size, 256.  Replaces convrot.h:37 xpuint8_convrot_groupsize. */
int xpuint8_convrot_groupsize(void);

/* Rotate + quantize: x bf16 [M,K] -> q int8 [M,K] + scale fp32 [M].
 * Replaces convrot.h:41-42 xpuint8_convrot_quantize and :46-47 _stream. */
int xpuint8_convrot_quantize(const void *x, int8_t *q, float *scale, int64_t M, int64_t K);
int xpuint8_convrot_quantize_stream(const void *stream, const void *x, int8_t *q, float *scale,
                                    int64_t M, int64_t K);

/* Activation fused before rotation and quantization: 1 GELU-tanh [M,K];
 * 2 SwiGLU [M,2K] as [gate, up]; 3 situ [M,2K] as [hidden, gate]; 4 GEGLU
 * (erf) [M,2K] as [hidden, gate]; 5 GELU-erf [M,K].  Output int8 [M,K].
 * Replaces convrot.h:58-62 xpuint8_convrot_quantize_act and _stream. */
int xpuint8_convrot_quantize_act(const void *x, int8_t *q, float *scale, int64_t M, int64_t K,
                                 int32_t activation);
int xpuint8_convrot_quantize_act_stream(const void *stream, const void *x, int8_t *q,
                                        float *scale, int64_t M, int64_t K, int32_t activation);

/* int8 [N,K] + fp32 [N] -> bf16 [N,K]: bf16(w8 * s) then the rotation undone.
 * Replaces convrot.h:67-70 xpuint8_dequant_weight and _stream. */
int xpuint8_dequant_weight(const void *w8, const float *w_scale, void *out, int64_t N,
                           int64_t K);
int xpuint8_dequant_weight_stream(const void *stream, const void *w8, const float *w_scale,
                                  void *out, int64_t N, int64_t K);

/* Rotation only, bf16 [M,K] -> bf16 [M,K].
 * Replaces convrot.h:72-74 xpuint8_convrot_rotate_bf16 and _stream. */
int xpuint8_convrot_rotate_bf16(const void *x, void *xr, int64_t M, int64_t K);
int xpuint8_convrot_rotate_bf16_stream(const void *stream, const void *x, void *xr, int64_t M,
                                       int64_t K);

/* out bf16 [M,N] = bf16(float(acc) * (w_scale[n] * x_scale[m]) + bias[n]);
 * bias may be NULL; N % 16 == 0.
 * Replaces convrot.h:78-85 xpuint8_dequant_epilogue and _stream. */
int xpuint8_dequant_epilogue(const int32_t *acc, void *out, const float *x_scale,
                             const float *w_scale, const float *bias, int64_t M, int64_t N);
int xpuint8_dequant_epilogue_stream(const void *stream, const int32_t *acc, void *out,
                                    const float *x_scale, const float *w_scale,
                                    const float *bias, int64_t M, int64_t N);

/* As above for a [M,N] column slice of a [M, acc_row_stride] accumulator.
 * Replaces convrot.h:90-96 xpuint8_dequant_epilogue_slice and _stream. */
int xpuint8_dequant_epilogue_slice(const int32_t *acc, void *out, const float *x_scale,
                                   const float *w_scale, const float *bias, int64_t M, int64_t N,
                                   int64_t acc_row_stride);
int xpuint8_dequant_epilogue_slice_stream(const void *stream, const int32_t *acc, void *out,
                                          const float *x_scale, const float *w_scale,
                                          const float *bias, int64_t M, int64_t N,
                                          int64_t acc_row_stride);

/* Dequant + activation (3 situ, 4 GEGLU, 5 GELU-erf) + rotate + quantize of an
 * up-projection accumulator: acc int32 [M,2K] (paired) or [M,K]; w_scale
 * [2K] or [K]; q int8 [M,K] + scale [M].
 * Replaces convrot.h:106-112 xpuint8_dequant_act_quantize and _stream. */
int xpuint8_dequant_act_quantize(const void *acc, int8_t *q, float *scale, const float *x_scale,
                                 const float *w_scale, int64_t M, int64_t K, int32_t activation);
int xpuint8_dequant_act_quantize_stream(const void *stream, const void *acc, int8_t *q,
                                        float *scale, const float *x_scale,
                                        const float *w_scale, int64_t M, int64_t K,
                                        int32_t activation);

/* Message of the last failure on this thread.  Replaces convrot.h:114. */
const char *xpuint8_last_error(void);

/* ---------------- new entries (no C symbol in the reference) ---------------- */

/* int8 GEMM on the tensor cores, exact int32 result c [M,N] (row stride ldc).
 * layout 0: a [M,K], b [N,K] -> a @ b^T  (torch._int_mm(a, b.t()), ops.py:587,634,714,716)
 * layout 1: a [M,K], b [K,N] -> a @ b    (torch._int_mm(a, b), ops.py:371)
 * layout 2: a [K,M], b [K,N] -> a^T @ b  (the int8 weight gradient)
 * Row lengths of a and b must be multiples of 16 bytes; N % 16 == 0. */
int xpuint8_int_mm_stream(const void *stream, const int8_t *a, const int8_t *b, int32_t *c,
                          int64_t M, int64_t N, int64_t K, int32_t layout, int64_t ldc);

/* The GEMM with the dequant epilogue fused into the accumulator drain:
 * out bf16 [M,N] = bf16(float(a*b) * (col_scale[n] * row_scale[m]) + bias[n]).
 * col_scale NULL means 1; bias may be NULL.  Replaces the pair
 * torch._int_mm + xpuint8_dequant_epilogue (ops.py:634 + :479-497). */
int xpuint8_int_mm_dequant_stream(const void *stream, const int8_t *a, const int8_t *b,
                                  void *out, const float *row_scale, const float *col_scale,
                                  const float *bias, int64_t M, int64_t N, int64_t K,
                                  int32_t layout, int64_t ldo);

/* Up-projection GEMM with the GEGLU epilogue: up_w8 [2*inner, K] as [hidden;
 * gate], up_scale [2*inner]; y bf16 [M, inner] = bf16(h * bf16(gelu_erf(g)))
 * with h, g the bf16 dequants.  Replaces torch._int_mm + the dequant and
 * GEGLU of xpuint8_dequant_act_quantize (ops.py:714-715). */
int xpuint8_int_mm_geglu_stream(const void *stream, const int8_t *a, const int8_t *up_w8,
                                void *y, const float *x_scale, const float *up_scale, int64_t M,
                                int64_t inner, int64_t K);

/* The whole INT8 linear: rotate+quantize x (activation 0..5 as in
 * _quantize_act), then the GEMM with the fused dequant epilogue.  xq int8
 * [M,K] and xs fp32 [M] are caller-provided scratch.  Replaces
 * python/xpu_kernels/int8/ops.py:591-646 (linear) in one C call. */
int xpuint8_linear_stream(const void *stream, const void *x, const int8_t *w8,
                          const float *w_scale, const float *bias, void *out, int8_t *xq,
                          float *xs, int64_t M, int64_t N, int64_t K, int32_t activation);

/* The INT8 linear against a weight of `nparts` concatenated projections
 * (q, k, v: w8 [nparts*N, K] = cat(Wq, Wk, Wv), w_scale [nparts*N], bias
 * [nparts*N] or NULL) in one GEMM whose drain writes part i's columns straight
 * into outs[i] (bf16 [M, N] each) -- no int32 [M, nparts*N] accumulator in
 * HBM.  Bit-identical to linear_acc + xpuint8_dequant_epilogue_slice per part.
 * xq [M,K], xs [M] are caller scratch.  N % 32 == 0, nparts <= 8.  Replaces
 * the reference's fused qkv pattern, python/xpu_kernels/int8/ops.py:500-525
 * (linear_acc, dequant_slice) as used at int8/selftest.py:67-72. */
int xpuint8_linear_split_stream(const void *stream, const void *x, const int8_t *w8,
                                const float *w_scale, const float *bias, void *const *outs,
                                int32_t nparts, int8_t *xq, float *xs, int64_t M, int64_t N,
                                int64_t K, int32_t activation);

/* RMS norm + rotary embedding of attention heads, B x S rows of H heads of
 * D elements (D 64, 128 or 256): x is bf16 (x_is_int32 = 0) or the INT8 GEMM's
 * int32 accumulator (x_is_int32 = 1: first dequantized as bf16(float(acc) *
 * (w_scale[h*D+d] * x_scale[row])), w_scale [H*D], x_scale [B*S]); per head
 * y = bf16((x * rsqrt(mean(x^2) + eps)) * weight) (weight [D]), then each pair
 * (d, d + D/2) (split_half) or (2i, 2i+1) rotated by freqs [freqs_batch,
 * freqs_seq, D/2, 2, 2] fp32 ([[cos, -sin], [sin, cos]]; 1 broadcasts) into
 * out bf16.  ldx / ldo: elements between rows (an accumulator slice of a fused
 * qkv GEMM has ldx = 3 * H * D).  Replaces python/xpu_kernels/triton/rope.py
 * :360-408 (_rows, _rows_dq) behind rms_rope_split_half(_dequant) (:643-652,
 * :694), the chain of triton/reference.py:63-98. */
int xpuint8_rms_rope_stream(const void *stream, const void *x, int32_t x_is_int32, int64_t ldx,
                            const float *x_scale, const float *w_scale, const float *weight,
                            const float *freqs, int64_t freqs_batch, int64_t freqs_seq, void *out,
                            int64_t ldo, int64_t B, int64_t S, int64_t H, int64_t D, float eps,
                            int32_t split_half);

/* The fused FFN down(act(up(x))) (ops.py:649-719) in one C call; activation 3
 * situ, 4 GEGLU (fused into the up-projection's epilogue), 5 GELU-erf.
 * `workspace` holds xpuint8_ffn_workspace_bytes(M, K, inner, activation)
 * bytes of caller-provided scratch. */
int64_t xpuint8_ffn_workspace_bytes(int64_t M, int64_t K, int64_t inner, int32_t activation);
int xpuint8_ffn_stream(const void *stream, const void *x, const int8_t *up_w8,
                       const float *up_scale, const int8_t *down_w8, const float *down_scale,
                       const float *down_bias, void *out, void *workspace, int64_t M, int64_t K,
                       int64_t inner, int32_t activation);

/* Per-row int8 quantization without rotation (the gradient quantizer):
 * scale = max(amax/127, 1e-30), q = rint(x / scale).  With col_scale non-NULL
 * the input is bf16(x * bf16(col_scale[k])) (linear_dx_int8's column scale).
 * Replaces the Triton kernel triton/quantize.py:63-126 and the chain
 * quantize_row_torch (ops.py:320-330).  K % 8 == 0. */
int xpuint8_quantize_row_stream(const void *stream, const void *x, const float *col_scale,
                                int8_t *q, float *scale, int64_t M, int64_t K);

/* dL/dx of the INT8 linear with the weight kept in int8, in one C call:
 * dy bf16 [M,N], w8 int8 [N,K] and w_scale fp32 [N] (the forward's prepared
 * weight) -> dx bf16 [M,K].  The column-scaled row quantizer, the int8 GEMM
 * reading w8 as stored with the row-scale epilogue, and the rotation undone
 * along K, launched back to back (the GEMM with programmatic serialization).
 * `workspace` holds xpuint8_linear_dx_int8_workspace_bytes(M, N, K) bytes.
 * K % 256 == 0, N % 16 == 0.  Replaces the chain of
 * python/xpu_kernels/int8/ops.py:353-377 (linear_dx_int8). */
int64_t xpuint8_linear_dx_int8_workspace_bytes(int64_t M, int64_t N, int64_t K);
int xpuint8_linear_dx_int8_stream(const void *stream, const void *dy, const int8_t *w8,
                                  const float *w_scale, void *dx, void *workspace, int64_t M,
                                  int64_t N, int64_t K);

/* dL/dW with both GEMM operands int8, in one C call: dy bf16 [M,N], the
 * forward's rotated int8 activation xq [M,K] and its row scales x_scale [M]
 * -> dW bf16 [N,K] = rotate_K(bf16(colquant(dy*xs)^T @ xq * tg)).  The column
 * quantizer, the int8 GEMM with both operands MN-major, and the rotation.
 * `workspace` holds xpuint8_linear_dw_int8_workspace_bytes(M, N, K) bytes.
 * K % 256 == 0, N % 16 == 0.  No counterpart in the reference, whose weight
 * gradient is the bf16 matmul of python/xpu_kernels/int8/ops.py:207-238. */
int64_t xpuint8_linear_dw_int8_workspace_bytes(int64_t M, int64_t N, int64_t K);
int xpuint8_linear_dw_int8_stream(const void *stream, const void *dy, const int8_t *xq,
                                  const float *x_scale, void *dw, void *workspace, int64_t M,
                                  int64_t N, int64_t K);

/* Column quantization of g = dy[m,n] * x_scale[m] over m, for the int8 weight
 * gradient: gq int8 [M,N], tg fp32 [N].  N % 16 == 0. */
int xpuint8_colquant_stream(const void *stream, const void *dy, const float *x_scale, int8_t *gq,
                            float *tg, int64_t M, int64_t N);

/* The device fault words of the bounded waits (0 = none: the GEMM's, then the
 * wait probe's), read with a device synchronisation; reset != 0 clears them.
 * A GEMM wait that gave up records its site here and the kernel returns. */
int xpuint8_fault_status(int32_t reset);

/* Self-test of the bounded device waits (blocking, legacy default stream):
 * one CTA waits on a shared-memory mbarrier that nothing arrives on, through
 * the GEMM's own bounded wait, with a limit of limit_ns (clamped to
 * [1 us, 2 s]).  The wait gives up, records `site` (non-zero) in the fault
 * word xpuint8_fault_status reports, and the kernel returns; *elapsed_ns
 * (if not NULL) receives how long it waited.  The probe's word is separate
 * from the GEMM's, so it never stops a later GEMM.  No counterpart in the
 * reference, whose failure model is the return code and last-error text
 * (src/xpuint8.cpp:47-50). */
int xpuint8_wait_probe(int64_t limit_ns, int32_t site, int64_t *elapsed_ns);

/* The N-sharded INT8 linear with its output all-gather fused into the GEMM
 * (BASELINE config C5's large-weight variant; the reference has no
 * distributed code).  Rank `rank` of `nranks` holds weight rows
 * [rank*N, (rank+1)*N) (w8 [N,K] int8, w_scale [N] fp32, bias [N] or NULL)
 * and the whole activation x [M,K] bf16; outs[r] is rank r's output
 * [M, nranks*N] bf16 as mapped in this process (its own buffer and the
 * peers' through xpuint8_ipc_open).  Every output tile of this rank's
 * block is written by the TMA unit into all nranks buffers at columns
 * [rank*N, (rank+1)*N), over NVLink as the tiles finish.  xq [M,K] int8 and
 * xs [M] fp32 are caller scratch.  The caller orders the ranks around the
 * call: every rank's previous readers of its output before, every rank's
 * call before readers after (a device-side barrier such as a one-element
 * all-reduce on the same stream).  nranks <= 8, N % 16 == 0, K % 256 == 0. */
int xpuint8_linear_allgather_stream(const void *stream, const void *x, const int8_t *w8,
                                    const float *w_scale, const float *bias, void *const *outs,
                                    int32_t nranks, int32_t rank, int8_t *xq, float *xs, int64_t M,
                                    int64_t N, int64_t K, int32_t activation);

/* The same with the column block given explicitly, for blocks of unequal
 * width (N output columns not divisible into equal multiple-of-16 blocks):
 * this rank's tiles land at columns [col_offset, col_offset + N) of every
 * rank's [M, n_total] output.  col_offset and n_total are multiples of 16.
 * xpuint8_linear_allgather_stream is this call with col_offset = rank * N and
 * n_total = nranks * N. */
int xpuint8_linear_allgather_cols_stream(const void *stream, const void *x, const int8_t *w8,
                                         const float *w_scale, const float *bias,
                                         void *const *outs, int32_t nranks, int64_t col_offset,
                                         int64_t n_total, int8_t *xq, float *xs, int64_t M,
                                         int64_t N, int64_t K, int32_t activation);

/* Peer-visible device buffers for the fused all-gather (set-up time, not per
 * call): xpuint8_ipc_alloc allocates `bytes` on the current device and
 * writes its 64-byte CUDA IPC handle; another process opens it with
 * xpuint8_ipc_open (a mapping valid on its current device, peer access
 * enabled lazily), releases the mapping with xpuint8_ipc_close; the owner
 * frees with xpuint8_ipc_free.  No counterpart in the reference. */
int xpuint8_ipc_alloc(int64_t bytes, void **ptr, void *handle);
int xpuint8_ipc_open(const void *handle, void **ptr);
int xpuint8_ipc_close(void *ptr);
int xpuint8_ipc_free(void *ptr);

/* Self-check of the quantizers' scale arithmetic (blocking, default stream):
 * the fast row scale s = max(amax/127, 1e-30) and 1/s against the IEEE
 * divide / reciprocal on every non-negative float, and the packed
 * product-then-add of the code computation against the scalar operations.
 * Writes the mismatch counts (both 0 on a correct build).  No counterpart in
 * the reference, whose quantizers call the divide per row. */
int xpuint8_check_scale_math(int64_t *bad_scale, int64_t *bad_quant);

/* xpuint8_linear_stream for callers that cannot allocate device memory (a
 * plugin inside an application that owns the GPU's memory pool, a C caller
 * without a device allocator, a path where cudaMalloc would synchronise).
 * No counterpart in the reference.  Same arguments minus the scratch: the
 * int8 activation and its row scales live in a fixed array inside the
 * library (8 MiB + 64 KiB, held on every GPU that loads the library until
 * exit), so M <= 16384 and M * K <= 8 MiB; larger calls return 2.  All calls
 * on a device share that array: calls whose work overlaps on the GPU race.
 * The first call on a device (in each CUDA context there: a device reset or
 * another current context looks it up anew) resolves the array's address and
 * may load the library's device code; make it before any stream capture. */
int xpuint8_linear_noalloc_stream(const void *stream, const void *x, const int8_t *w8,
                                  const float *w_scale, const float *bias, void *out, int64_t M,
                                  int64_t N, int64_t K, int32_t activation);

#ifdef __cplusplus
}
#endif
#endif /* XPU_INT8_H */
