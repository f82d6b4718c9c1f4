// rope.cuh -- rotary position embedding as ggml_rope_ext applies it in the
// reference (src/cosyvoice-llm.cpp:56-57,180: NEOX per head, n_dims = head_dim,
// freq_base = rope_theta; src/cosyvoice-graph.cpp:354-355: NORMAL on the first
// head_dim elements of the whole 1024-wide row, freq_base 10000), with
// ext_factor 0 and no frequency factors, the only form the reference uses.
//
// The angles follow ggml's CPU backend: the host forms theta_scale =
// powf(freq_base, -2 / n_dims) with the C library, and pair k at position p
// has angle p * theta_scale^k built by k sequential f32 products, times
// freq_scale.  cos / sin (CUDA's sincosf) are scaled by attn_factor.  A
// rotated pair (a, b) becomes (a cos - b sin, a sin + b cos), each as two
// rounded products and one rounded sum.
#pragma once

#include "common.cuh"
#include "internal.h"

namespace cvattn {

// Angle of pair k0 at position p (k0 sequential products), advanced by
// rope_next for k0 + 1, k0 + 2, ...: the same rounding as forming each one
// from scratch.
__device__ __forceinline__ float rope_theta(const RopeDev& r, int p, int k0) {
    float theta = (float)p;
    for (int i = 0; i < k0; ++i) theta = __fmul_rn(theta, r.theta_scale);
    return theta;
}
__device__ __forceinline__ float rope_next(const RopeDev& r, float theta) { return __fmul_rn(theta, r.theta_scale); }

// (cos, sin) * attn_factor of an angle.
__device__ __forceinline__ float2 rope_cs(const RopeDev& r, float theta) {
    float s, c;
    sincosf(__fmul_rn(r.freq_scale, theta), &s, &c);
    return make_float2(__fmul_rn(c, r.attn_factor), __fmul_rn(s, r.attn_factor));
}

// Rotated value of one element: self is the element, partner the other one of
// its pair, first whether self is the pair's first element.
__device__ __forceinline__ float rope_rotate(float self, float partner, float2 cs, bool first) {
    return first ? __fsub_rn(__fmul_rn(self, cs.x), __fmul_rn(partner, cs.y))
                 : __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(self, cs.x));
}

// Pair of element e of a row (row-local index): returns the partner's index,
// or -1 when e is not rotated; k is the pair index, first as above.
__device__ __forceinline__ int rope_pair(const RopeDev& r, int e, int& k, bool& first) {
    const int u0 = e - e % r.unit_len, d = e - u0;
    if (d >= r.n_dims) return -1;
    if (r.mode & 2) {
        const int half = r.n_dims >> 1;
        first = d < half;
        k = first ? d : d - half;
        return u0 + (first ? d + half : d - half);
    }
    first = (d & 1) == 0;
    k = d >> 1;
    return u0 + (d ^ 1);
}

}  // namespace cvattn
