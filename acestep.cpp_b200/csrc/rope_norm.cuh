// rope_norm.cuh -- the attention prologue of acestep.cpp (RMSNorm times a
// per-dimension weight, then RoPE in NEOX order) applied to rows that the
// kernels already hold in registers: Q rows as the attention kernels load them,
// the new K row of a fused decode append, K rows in fa_kv_prologue.
//
// Arithmetic, per row x of D values (ggml_rms_norm + ggml_mul, then
// ggml_rope_ext mode 2 with n_dims = D, freq_scale 1, no YaRN):
//   sc   = 1 / sqrtf(sum(x^2) / D + eps);       y = (x * sc) * w
//   a_k  = (float) pos * inv_freq[k],  k < D/2   (inv_freq from the host)
//   y'_k = y_k cos a_k - y_{k+D/2} sin a_k;  y'_{k+D/2} = y_k sin a_k + y_{k+D/2} cos a_k
#pragma once

#include "fa_internal.h"

namespace acefa {

__device__ __forceinline__ float rn_scale(const RopeNorm &p, float ss, int D) {
    return 1.0f / sqrtf(ss / (float) D + p.eps);
}

// cos and sin of a RoPE angle.  Kept out of line: sincosf's argument
// reduction for large angles is long, and the prologue calls it from many
// unrolled sites that would otherwise each carry a copy.  (The dense kernel,
// whose warps re-split their registers, calls no functions: it uses the inline
// form from a single site.)
__device__ __forceinline__ float2 rn_cos_sin_inline(float a) {
    float s, c;
    sincosf(a, &s, &c);
    return make_float2(c, s);
}
static __device__ __noinline__ float2 rn_cos_sin(float a) { return rn_cos_sin_inline(a); }

// Rotation of one pair: `first` holds y_k (partner y_{k+D/2}), else the reverse.
__device__ __forceinline__ float rn_rotate(const RopeNorm &p, float own, float partner, bool first, int pos, int k) {
    const float2 cs = rn_cos_sin((float) pos * p.inv_freq[k]);
    return first ? own * cs.x - partner * cs.y : partner * cs.y + own * cs.x;
}

// A row spread over a warp, lane l holding the DPL consecutive dims
// DPL*l .. DPL*l + DPL-1 (D = 32 * DPL): the partner of dim d < D/2 is held by
// lane l ^ 16 at the same slot.
template <int DPL>
__device__ __forceinline__ void rn_warp_row(const RopeNorm &p, float (&x)[DPL], int lane, int pos) {
    constexpr int D = 32 * DPL;
    if (p.w) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            ss = fmaf(x[e], x[e], ss);
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, off);
        }
        const float sc = rn_scale(p, ss, D);
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            x[e] = (x[e] * sc) * __ldg(p.w + DPL * lane + e);
        }
    }
    if (p.rope) {
        const bool first = lane < 16;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
            x[e]                = rn_rotate(p, x[e], partner, first, pos, (DPL * lane + e) & (D / 2 - 1));
        }
    }
}

}  // namespace acefa
