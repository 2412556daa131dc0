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

// cos and sin of a RoPE angle a = pos * inv_freq (a >= 0, up to ~1e5 rad).
// The angle is reduced to [-pi, pi] in double precision (a - 2 pi n with
// n = rint(a / 2 pi): for a < 2^24 the reduction error stays below 1e-9 rad),
// then the hardware __sincosf evaluates it (absolute error ~4e-7 on
// [-pi, pi]).  Short and register-light, unlike the general sincosf whose
// large-argument path would dominate these kernels' prologues.
__device__ __forceinline__ float2 rn_cos_sin(float a) {
    const double ad = (double) a;
    const double n  = rint(ad * 0.15915494309189535);  // 1 / (2 pi)
    const float  r  = (float) fma(-n, 6.283185307179586, ad);
    float        s, c;
    __sincosf(r, &s, &c);
    return make_float2(c, s);
}

// Rotation of one pair: `first` holds y_k (partner y_{k+D/2}), else the reverse.
__device__ __forceinline__ float rn_rotate(const RopeNorm &p, float own, float partner, bool first, int pos, int k) {
    const float2 cs = rn_cos_sin((float) pos * p.inv_freq[k]);
    return first ? own * cs.x - partner * cs.y : partner * cs.y + own * cs.x;
}

// A row spread over a warp, lane l holding the DPL consecutive dims
// DPL*l .. DPL*l + DPL-1 (D = 32 * DPL): the partner of dim d < D/2 is held by
// lane l ^ 16 at the same slot, and both lanes need the same DPL angles, so
// each computes half of them and takes the other half from its partner.
template <int DPL>
__device__ __forceinline__ void rn_warp_row(const RopeNorm &p, float (&x)[DPL], int lane, int pos) {
    constexpr int D = 32 * DPL;
    constexpr int H = DPL / 2;
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
        const int  e0    = first ? 0 : H;  // the half of the angles this lane computes
        float2     cs[DPL];
#pragma unroll
        for (int j = 0; j < H; ++j) {
            const float2 mine  = rn_cos_sin((float) pos * p.inv_freq[(DPL * lane + e0 + j) & (D / 2 - 1)]);
            const float2 other = make_float2(__shfl_xor_sync(0xffffffffu, mine.x, 16),
                                             __shfl_xor_sync(0xffffffffu, mine.y, 16));
            cs[j]     = first ? mine : other;
            cs[j + H] = first ? other : mine;
        }
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
            x[e] = first ? x[e] * cs[e].x - partner * cs[e].y : partner * cs[e].y + x[e] * cs[e].x;
        }
    }
}

}  // namespace acefa
