// The fused input activations of the quantizers (the reference's
// load_activated_reg / situ_reg, src/xpuint8.cpp:142-160,190-220), with every
// bf16 rounding of the reference's chain.
//
// Every activation input is a bf16 value: the bf16 activation itself (mode 0)
// or the dequantized accumulator rounded to bf16 (mode 1, src/xpuint8.cpp:
// 236-248).  Each activation is therefore built from one-input pieces, each a
// function on the 65 536 bf16 values whose result is a bf16 value, joined by at
// most one product and rounding:
//
//   act 1  GELU-tanh   piece_gelu_tanh(a)
//   act 2  SwiGLU      bf16(piece_silu(a) * b)
//   act 3  situ        bf16(piece_situ_gate(g) * piece_situ_hidden(h))
//   act 4  GEGLU       bf16(h * piece_gelu_erf(g))
//   act 5  GELU-erf    piece_gelu_erf(a)
//
// Both rotation kernel files evaluate the activations through these.
#pragma once

#include "common.cuh"

namespace xpuint8 {

__device__ __forceinline__ float gelu_erf_f(float x) {
    const float t = __fmul_rn(x, 0.7071067811865476f);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(t)));
}
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float x2 = __fmul_rn(x, x);
    const float inner = __fmul_rn(__fmul_rn(0.7978845608028654f, x),
                                  __fadd_rn(1.0f, __fmul_rn(0.044715f, x2)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// the one-input pieces (bf16 values held in fp32)
__device__ __forceinline__ float piece_gelu_tanh(float x) { return round_bf16(gelu_tanh_f(x)); }
__device__ __forceinline__ float piece_silu(float a) {
    return round_bf16(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))));
}
// MossImage's situ (src/xpuint8.cpp:142-160): the gate's factor
// bf16(bf16(tanh(bf16(g/4))) * bf16(sigmoid(g))) and the hidden one
// bf16(tanh(bf16(h/25)))
__device__ __forceinline__ float piece_situ_gate(float g) {
    const float tg = round_bf16(tanhf(round_bf16(__fdiv_rn(g, 4.0f))));
    const float sg = round_bf16(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
    return round_bf16(__fmul_rn(tg, sg));
}
__device__ __forceinline__ float piece_situ_hidden(float h) {
    return round_bf16(tanhf(round_bf16(__fdiv_rn(h, 25.0f))));
}
__device__ __forceinline__ float piece_gelu_erf(float x) { return round_bf16(gelu_erf_f(x)); }

__host__ __device__ constexpr bool act_paired(int act) { return act == 2 || act == 3 || act == 4; }

// the activation evaluated directly; a, b are exact bf16 values (b: the second
// input of a paired activation -- SwiGLU's up, situ's and GEGLU's gate)
template <int ACT>
__device__ __forceinline__ float activate(float a, float b) {
    if constexpr (ACT == 0) {
        return a;
    } else if constexpr (ACT == 1) {
        return piece_gelu_tanh(a);
    } else if constexpr (ACT == 2) {
        return round_bf16(__fmul_rn(piece_silu(a), b));
    } else if constexpr (ACT == 3) {
        return round_bf16(__fmul_rn(piece_situ_gate(b), piece_situ_hidden(a)));
    } else if constexpr (ACT == 4) {
        return round_bf16(__fmul_rn(a, piece_gelu_erf(b)));
    } else {
        return piece_gelu_erf(a);
    }
}

}  // namespace xpuint8
