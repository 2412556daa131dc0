// fa_prologue.cu -- acefa_kv_prologue(): K and V of a dense attention node
// prepared in one pass.  acestep.cpp runs, per layer, rms_norm, mul (norm
// weight), rope, cont (permute) and a cast or set_rows for K and a cont and a
// cast or set_rows for V (src/dit-graph.h:181-213, src/qwen3-lm.h:423-449);
// here one warp takes one row: it loads the f32 row, applies RMSNorm and RoPE
// in registers (rope_norm.cuh) and stores it converted to F16 / BF16 at the
// destination view's strides.  HBM-bound: 4 B read and 2 B written per value.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstring>

#include "fa_internal.h"
#include "ptx.cuh"
#include "rope_norm.cuh"

namespace acefa {

namespace {

constexpr int kProWarps  = 8;  // warps per CTA
constexpr int kProUnroll = 4;  // rows per warp in flight

struct KvSide {
    const char *src;
    char       *dst;
    int64_t     s_nb1, s_nb2, s_nb3;
    int64_t     d_nb1, d_nb2, d_nb3;
    int         vec;  // every lane's chunk aligned on both sides: vector loads / stores
};

struct KvProParams {
    KvSide   side[2];  // K, V (V.src == nullptr: none)
    int      D, rows, H, B;
    int      dst_bf16;
    int64_t  n_rows;   // rows * H * B
    RopeNorm kp;
};

// Row r of the [D, rows, H, B] operands -> (i, h, b) in 32-bit arithmetic
// (the host checks rows * H * B < 2^31).
struct RowCoord {
    int i, h, b;
};
__device__ __forceinline__ RowCoord row_coord(const KvProParams &P, int r) {
    const unsigned q = (unsigned) r / (unsigned) P.rows;
    return RowCoord{(int) ((unsigned) r - q * (unsigned) P.rows), (int) (q % (unsigned) P.H), (int) (q / (unsigned) P.H)};
}

template <int DPL>
__device__ __forceinline__ void load_row(const KvSide &s, const RowCoord &rc, int lane, float (&x)[DPL]) {
    const float *sp = reinterpret_cast<const float *>(s.src + (int64_t) rc.i * s.s_nb1 + (int64_t) rc.h * s.s_nb2 +
                                                      (int64_t) rc.b * s.s_nb3) +
                      DPL * lane;
    if (s.vec) {
        if constexpr (DPL == 4) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(sp));
            x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
        } else {
            const float2 v = __ldg(reinterpret_cast<const float2 *>(sp));
            x[0] = v.x, x[1] = v.y;
        }
    } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            x[e] = __ldg(sp + e);
        }
    }
}

template <int DPL>
__device__ __forceinline__ void store_row(const KvSide &s, const RowCoord &rc, int lane, bool bf16,
                                          const float (&x)[DPL]) {
    uint16_t *dp = reinterpret_cast<uint16_t *>(s.dst + (int64_t) rc.i * s.d_nb1 + (int64_t) rc.h * s.d_nb2 +
                                                (int64_t) rc.b * s.d_nb3) +
                   DPL * lane;
    uint16_t u[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
        u[e] = bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(x[e])) : __half_as_ushort(__float2half_rn(x[e]));
    }
    if (s.vec) {
        if constexpr (DPL == 4) {
            *reinterpret_cast<uint2 *>(dp) =
                make_uint2((uint32_t) u[0] | ((uint32_t) u[1] << 16), (uint32_t) u[2] | ((uint32_t) u[3] << 16));
        } else {
            *reinterpret_cast<uint32_t *>(dp) = (uint32_t) u[0] | ((uint32_t) u[1] << 16);
        }
    } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            dp[e] = u[e];
        }
    }
}

template <int DPL>
__global__ void __launch_bounds__(kProWarps * 32, 3) fa_kv_prologue(const __grid_constant__ KvProParams P) {
    constexpr int D = 32 * DPL, H = DPL / 2;
    const int     lane   = threadIdx.x & 31;
    const int     warp0  = (int) blockIdx.x * kProWarps + (int) (threadIdx.x >> 5);
    const int     stride = (int) gridDim.x * kProWarps;
    const int     n      = (int) P.n_rows;
    const RopeNorm &kp   = P.kp;
    // Per-lane constants: this lane's norm weights and the frequencies of the
    // half of its angles it computes (lane ^ 16 computes the other half).
    const bool first = lane < 16;
    float      wreg[DPL], freq[H];
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
        wreg[e] = kp.w ? __ldg(kp.w + DPL * lane + e) : 1.0f;
    }
#pragma unroll
    for (int j = 0; j < H; ++j) {
        freq[j] = kp.inv_freq[(DPL * lane + (first ? 0 : H) + j) & (D / 2 - 1)];
    }
    for (int r0 = warp0; r0 < n; r0 += stride * kProUnroll) {
        float    k[kProUnroll][DPL], v[kProUnroll][DPL];
        RowCoord rc[kProUnroll];
        int      pos[kProUnroll];
#pragma unroll
        for (int u = 0; u < kProUnroll; ++u) {
            const int r = r0 + u * stride;
            rc[u]       = row_coord(P, r < n ? r : 0);
            pos[u]      = 0;
            if (r < n) {
                load_row<DPL>(P.side[0], rc[u], lane, k[u]);
                if (P.side[1].src) {
                    load_row<DPL>(P.side[1], rc[u], lane, v[u]);
                }
                if (kp.rope) {
                    pos[u] = __ldg(kp.pos + rc[u].i + (int64_t) rc[u].b * P.rows);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kProUnroll; ++u) {
            if (r0 + u * stride >= n) {  // warp-uniform
                break;
            }
            float(&x)[DPL] = k[u];
            if (kp.w) {
                float ss = 0.0f;
#pragma unroll
                for (int e = 0; e < DPL; ++e) {
                    ss = fmaf(x[e], x[e], ss);
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    ss += __shfl_xor_sync(0xffffffffu, ss, off);
                }
                const float sc = rn_scale(kp, ss, D);
#pragma unroll
                for (int e = 0; e < DPL; ++e) {
                    x[e] = (x[e] * sc) * wreg[e];
                }
            }
            if (kp.rope) {
                float2 cs[DPL];
#pragma unroll
                for (int j = 0; j < H; ++j) {
                    const float2 mine  = rn_cos_sin((float) pos[u] * freq[j]);
                    const float2 other = make_float2(__shfl_xor_sync(0xffffffffu, mine.x, 16),
                                                     __shfl_xor_sync(0xffffffffu, mine.y, 16));
                    cs[j]     = first ? mine : other;
                    cs[j + H] = first ? other : mine;
                }
#pragma unroll
                for (int e = 0; e < DPL; ++e) {
                    const float pt = __shfl_xor_sync(0xffffffffu, x[e], 16);
                    x[e]           = first ? x[e] * cs[e].x - pt * cs[e].y : pt * cs[e].y + x[e] * cs[e].x;
                }
            }
            store_row<DPL>(P.side[0], rc[u], lane, P.dst_bf16, x);
            if (P.side[1].src) {
                store_row<DPL>(P.side[1], rc[u], lane, P.dst_bf16, v[u]);
            }
        }
    }
}

}  // namespace

// Launch for operands validated by acefa_kv_prologue (fa_api.cu).
int kv_prologue_launch(const acefa_tensor *k_src, const acefa_tensor *v_src, const acefa_tensor *k_dst,
                       const acefa_tensor *v_dst, const RopeNorm &kp, int sm_count, cudaStream_t stream) {
    KvProParams P;
    std::memset(&P, 0, sizeof(P));
    P.D    = (int) k_src->ne[0];
    P.rows = (int) k_src->ne[1];
    P.H    = (int) k_src->ne[2];
    P.B    = (int) k_src->ne[3];
    P.dst_bf16 = k_dst->type == ACEFA_TYPE_BF16;
    P.n_rows   = (int64_t) P.rows * P.H * P.B;
    P.kp       = kp;
    const acefa_tensor *src[2] = {k_src, v_src}, *dst[2] = {k_dst, v_dst};
    for (int s = 0; s < 2; ++s) {
        if (!src[s]) {
            continue;
        }
        KvSide &d = P.side[s];
        d.src     = static_cast<const char *>(src[s]->data);
        d.dst     = static_cast<char *>(dst[s]->data);
        d.s_nb1 = src[s]->nb[1], d.s_nb2 = src[s]->nb[2], d.s_nb3 = src[s]->nb[3];
        d.d_nb1 = dst[s]->nb[1], d.d_nb2 = dst[s]->nb[2], d.d_nb3 = dst[s]->nb[3];
        const int    dpl  = P.D / 32;
        const size_t sa   = (size_t) 4 * dpl, da = (size_t) 2 * dpl;  // per-lane chunk bytes
        const bool   s_ok = reinterpret_cast<uintptr_t>(d.src) % sa == 0 && d.s_nb1 % sa == 0 && d.s_nb2 % sa == 0 &&
                          d.s_nb3 % sa == 0;
        const bool   d_ok = reinterpret_cast<uintptr_t>(d.dst) % da == 0 && d.d_nb1 % da == 0 && d.d_nb2 % da == 0 &&
                          d.d_nb3 % da == 0;
        d.vec = s_ok && d_ok;
    }
    // one wave of resident CTAs (three per SM), each warp looping over rows:
    // no partial last wave (8% faster than 8 CTAs per SM queued in waves)
    const int64_t warps = (P.n_rows + kProUnroll - 1) / kProUnroll;
    int64_t       grid  = (warps + kProWarps - 1) / kProWarps;
    const int64_t cap   = (int64_t) sm_count * 3;
    grid                = grid < cap ? grid : cap;
    if (grid < 1) {
        grid = 1;
    }
    if (P.D == 128) {
        fa_kv_prologue<4><<<(unsigned) grid, kProWarps * 32, 0, stream>>>(P);
    } else {
        fa_kv_prologue<2><<<(unsigned) grid, kProWarps * 32, 0, stream>>>(P);
    }
    return cudaGetLastError() == cudaSuccess ? ACEFA_OK : ACEFA_ERR_CUDA;
}

}  // namespace acefa
