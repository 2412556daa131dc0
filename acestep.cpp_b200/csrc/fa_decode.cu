// fa_decode.cu -- split-KV flash-decode for sm_100a.
//
// Serves ggml_flash_attn_ext nodes whose query side is small: acestep.cpp's
// batched CFG decode (src/qwen3-lm.h:789-794: Q [128,1,Hq,N], K/V views
// [128,n_kv_pad,8,N] of the F16 cache), single-sequence decode
// (src/qwen3-lm.h:465-469 with n_tokens == 1) and the short FSQ encoders
// (src/fsq-tok.h:183, src/fsq-detok.h:171; S = 5..6).
//
// Design (memory bound; the roofline is HBM bytes of K and V):
//   * Work unit = (batch b, kv head hk, row block rb).  A unit's rows are the
//     G*n_q (query, q-head) pairs that share K/V head hk, 16 per block, so each
//     K/V byte is read once per unit and feeds G*n_q rows of tensor-core math.
//   * The flattened (unit, 64-key tile) list is cut into equal contiguous
//     ranges, one per persistent CTA (2 CTAs per SM).  A CTA that sees a unit
//     only partly writes an unnormalised partial (m, l, O); the combine kernel
//     merges partials.  Grid and splits depend on shapes only, so a captured
//     CUDA graph replays with any mask contents.
//   * Warp-specialised pipeline: one producer warp streams K/V tiles into a
//     3-stage shared-memory ring -- TMA tensor tiles with 128-B swizzle for
//     F16/BF16, 1-D bulk copies of whole 34-B-block rows for Q8_0 -- and skips
//     tiles whose mask is entirely -inf (the padded decode window tail).
//   * Four consumer warps each take 16 keys of every tile: S = Q K^T and O += P V
//     on mma.sync m16n8k16 with F32 accumulation, online softmax in the log2
//     domain with quad shuffles.  Q8_0 K/V are dequantised in registers
//     (int8 -> f16 by exponent splicing, times the block scale).
//   * Every mbarrier wait is bounded; on expiry the CTA records an error word,
//     drains its in-flight copies (bounded) and exits.
#include <cfloat>

#include "fa_internal.h"
#include "ptx.cuh"
#include "rope_norm.cuh"

namespace acefa {

namespace {

constexpr int kMetaData  = 1;
constexpr int kMetaFlush = 2;
constexpr int kMetaTerm  = 3;

constexpr uint16_t kHalfNegInf = 0xFC00u;

template <int KV_TYPE, int D>
struct DecCfg {
    static constexpr bool kQ8        = KV_TYPE == ACEFA_TYPE_Q8_0;
    static constexpr bool kBF16      = KV_TYPE == ACEFA_TYPE_BF16;
    static constexpr int  kRowBytes  = kQ8 ? D / 32 * 34 : D * 2;
    // F16/BF16: exactly the TMA boxes (D/64 swizzled 64-key x 128-B boxes).
    // Q8_0: raw rows plus up to 15 lead bytes, rounded to keep stages 1 KB aligned.
    static constexpr int  kTmaBytes  = kDecBN * kRowBytes;
    static constexpr int  kTileBytes = kQ8 ? ((kDecBN * kRowBytes + 16) + 1023) / 1024 * 1024 : kTmaBytes;
    static constexpr int  kMaskBytes  = kDecRows * kDecBN * 2;  // up to 16 mask rows x 64 keys (f16)
    static constexpr int  kStageBytes = 2 * kTileBytes + kMaskBytes;
    static_assert(kQ8 || kTileBytes % 1024 == 0, "TMA 128-B swizzle needs 1 KB aligned boxes");
    static_assert(kStageBytes % 1024 == 0, "stages must stay 1 KB aligned");
    static constexpr int  kMergeStride = D + 8;  // floats per merge row (bank spread)
    // shared memory carve-up (offsets from the 1024-B aligned base)
    static constexpr int kOffStages = 0;
    static constexpr int kOffMerge  = kOffStages + kDecStages * kStageBytes;
    static constexpr int kOffStats  = kOffMerge + kDecRows * kMergeStride * 4;  // m,l per warp per row
    static constexpr int kOffFin    = kOffStats + 2 * kDecWarps * kDecRows * 4;  // merged m,l per row
    static constexpr int kOffBars   = kOffFin + 2 * kDecRows * 4;
    static constexpr int kOffMeta   = kOffBars + 2 * kDecStages * 8;
    static constexpr int kOffFlags  = kOffMeta + kDecStages * 16;
    static constexpr int kSmemBytes = kOffFlags + 16 + 1024;  // + alignment slack
    static constexpr int kThreads   = (kDecWarps + 1) * 32;
};

// a * b / c, by 32-bit division when the plan says every such product fits
// (a 64-bit division is a long emulated sequence on the critical path).
__device__ __forceinline__ int64_t mul_div(int64_t a, int64_t b, int64_t c, int div32) {
    return div32 ? (int64_t) ((uint32_t) (a * b) / (uint32_t) c) : a * b / c;
}
__device__ __forceinline__ int64_t cta_of_tile(int64_t t, int64_t T, int C, int div32) {
    return div32 ? (int64_t) (((uint32_t) (t + 1) * (uint32_t) C - 1u) / (uint32_t) T) : ((t + 1) * C - 1) / T;
}

struct UnitCoord {
    int b, hk, rb, bk, rows;
};

__device__ __forceinline__ UnitCoord unit_coord(const DecodeParams &P, int u) {
    UnitCoord c;
    c.rb            = u % P.n_rb;
    c.hk            = (u / P.n_rb) % P.op.Hkv;
    c.b             = u / (P.n_rb * P.op.Hkv);
    c.bk            = c.b / P.op.rk3;
    const int total = P.op.G * P.op.n_q;
    c.rows          = min(kDecRows, total - c.rb * kDecRows);
    return c;
}

// Row rr of unit -> (query index iq, q head hq).
__device__ __forceinline__ void row_coord(const DecodeParams &P, const UnitCoord &uc, int rr, int &iq, int &hq) {
    const int gr = uc.rb * kDecRows + rr;
    iq           = gr / P.op.G;
    hq           = uc.hk * P.op.G + gr % P.op.G;
}

__device__ __forceinline__ const uint16_t *mask_row(const OpDesc &o, int iq, int hq, int b) {
    return reinterpret_cast<const uint16_t *>(o.mask + (int64_t) iq * o.m_nb1 + (int64_t) (hq % o.m_ne2) * o.m_nb2 +
                                              (int64_t) (b % o.m_ne3) * o.m_nb3);
}

// True if some mask entry of this tile, for some row of the unit, is not -inf
// (under a mask rule: some key of the tile is in some row's visible range).
__device__ bool tile_live(const DecodeParams &P, const UnitCoord &uc, int tile) {
    const OpDesc &o   = P.op;
    const int     j0  = tile * kDecBN;
    const int     cnt = min(kDecBN, o.n_kv - j0);
    if (o.mg_kind) {
        int lo0, hi0, lo1, hi1;
        mg_range(o, uc.b, (uc.rb * kDecRows) / o.G, lo0, hi0);
        mg_range(o, uc.b, (uc.rb * kDecRows + uc.rows - 1) / o.G, lo1, hi1);
        return max(lo0, j0) < min(hi1, j0 + cnt);
    }
    if (o.mask == nullptr) {
        return true;
    }
    const uint16_t *prev = nullptr;
    for (int rr = 0; rr < uc.rows; ++rr) {
        int iq, hq;
        row_coord(P, uc, rr, iq, hq);
        const uint16_t *m = mask_row(o, iq, hq, uc.b);
        if (m == prev) {
            continue;
        }
        prev = m;
        m += j0;
        bool dead = true;
        for (int j = 0; j < cnt; j += 8) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                if (j + e < cnt) {
                    dead &= (__ldg(m + j + e) == kHalfNegInf);
                }
            }
            if (!dead) {
                return true;
            }
        }
    }
    return false;
}

// -------------------------------------------------------------------------
// int8 -> f16 pair helpers (exact): byte b becomes 1024 + (b ^ 0x80) by exponent
// splicing; subtracting 1152 recovers the signed value exactly.
__device__ __forceinline__ __half2 i8pair_to_h2(uint32_t spliced) {
    const uint32_t t = (spliced & 0x00FF00FFu) ^ 0x64806480u;
    return __hsub2(*reinterpret_cast<const __half2 *>(&t), __half2half2(__ushort_as_half((unsigned short) 0x6480u)));
}

// Residual of a bf16x2 rounding: bf16(x - float(bf16(x))) for both lanes.
__device__ __forceinline__ uint32_t split_lo_bf16(float x0, float x1, uint32_t hi) {
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162 *>(&hi);
    const float2         f = __bfloat1622float2(h);
    return pack2<true>(x0 - f.x, x1 - f.y);
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// N bytes starting at a 2-B aligned shared address, as N/4 words.
template <int NW>
__device__ __forceinline__ void lds_bytes_unaligned(uint32_t addr, uint32_t (&out)[NW]) {
    const uint32_t base = addr & ~3u;
    const uint32_t sh   = (addr & 3u) * 8u;
    uint32_t       w[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) {
        w[i] = lds32(base + 4 * i);
    }
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        out[i] = __funnelshift_r(w[i], w[i + 1], sh);
    }
}

}  // namespace

// Fused KV-cache append, run by the producer warp of the CTA whose tile range
// holds the new row's tile: the f32 row of K and of V for (kv head, set) is
// converted to the cache type -- F16 / BF16 rounded to nearest even, Q8_0 by
// ggml's reference quantiser (d = amax/127, q = roundf(x * (1/d)), d stored
// as f16) -- and stored at cache row append_pos[set].  append_load fetches the
// lane's four values of each row early (their latency overlaps the unit's
// first copies); append_store writes them, and its proxy fence orders the
// generic stores before the warp's later TMA / bulk-copy reads of that row.
// Lane mapping: F16/BF16 dims lane + 32k; Q8_0 block lane/8, values 4*(lane%8)+k.
template <int KV_TYPE, int D>
__device__ __forceinline__ int append_index(int lane, int k) {
    return KV_TYPE == ACEFA_TYPE_Q8_0 ? (lane >> 3) * 32 + (lane & 7) * 4 + k : lane + 32 * k;
}

template <int KV_TYPE, int D, bool PRO>
__device__ __forceinline__ void append_load(const DecodeParams &P, int hk, int bk, int lane, float (&xk)[4],
                                            float (&xv)[4]) {
    const float *ks = reinterpret_cast<const float *>(P.k_new + (int64_t) hk * P.kn_nb2 + (int64_t) bk * P.kn_nb3);
    const float *vs = reinterpret_cast<const float *>(P.v_new + (int64_t) hk * P.vn_nb2 + (int64_t) bk * P.vn_nb3);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int  i  = append_index<KV_TYPE, D>(lane, k);
        const bool in = KV_TYPE == ACEFA_TYPE_Q8_0 ? (lane >> 3) < D / 32 : k < D / 32;
        xk[k]         = in ? ks[i] : 0.0f;
        xv[k]         = in ? vs[i] : 0.0f;
    }
    const RopeNorm &kp = P.kp;
    if (PRO && kp.on) {
        // QK-norm + RoPE of the new K row (values outside the row are 0)
        if (kp.w) {
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                ss = fmaf(xk[k], xk[k], ss);
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                ss += __shfl_xor_sync(0xffffffffu, ss, off);
            }
            const float sc = rn_scale(kp, ss, D);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const bool in = KV_TYPE == ACEFA_TYPE_Q8_0 ? (lane >> 3) < D / 32 : k < D / 32;
                xk[k]         = in ? (xk[k] * sc) * __ldg(kp.w + append_index<KV_TYPE, D>(lane, k)) : 0.0f;
            }
        }
        if (kp.rope) {
            const int pos = __ldg(kp.pos + bk);
            if constexpr (KV_TYPE == ACEFA_TYPE_Q8_0) {
                // dim d + D/2 is D/64 blocks (8 lanes each) further: lane ^ (D/8)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int   d  = append_index<KV_TYPE, D>(lane, k);
                    const float pt = __shfl_xor_sync(0xffffffffu, xk[k], D / 8);
                    xk[k] = (lane >> 3) < D / 32 ? rn_rotate(kp, xk[k], pt, d < D / 2, pos, d & (D / 2 - 1)) : 0.0f;
                }
            } else {
                // dim lane + 32k pairs with lane + 32(k + D/64): same lane
#pragma unroll
                for (int k = 0; k < D / 64; ++k) {
                    const float a = xk[k], b = xk[k + D / 64];
                    const int   d = append_index<KV_TYPE, D>(lane, k);
                    xk[k]          = rn_rotate(kp, a, b, true, pos, d);
                    xk[k + D / 64] = rn_rotate(kp, b, a, false, pos, d);
                }
            }
        }
    }
}

template <int KV_TYPE, int D>
__device__ __forceinline__ void append_store(const DecodeParams &P, int64_t pr, int lane, const char *kbase,
                                             const char *vbase, const float (&xk)[4], const float (&xv)[4]) {
    const OpDesc &o = P.op;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        const float(&x)[4] = which ? xv : xk;
        char *dst          = const_cast<char *>(which ? vbase + pr * o.v_nb1 : kbase + pr * o.k_nb1);
        if constexpr (KV_TYPE == ACEFA_TYPE_Q8_0) {
            // 32-value blocks, eight lanes per block, four values per lane
            constexpr int NB   = D / 32;
            const int     blk  = lane >> 3;
            const int     sub  = lane & 7;
            float         amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                amax = fmaxf(amax, fabsf(x[k]));
            }
#pragma unroll
            for (int off = 4; off > 0; off >>= 1) {
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            }
            const float d  = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            if (blk < NB) {
                // rows and blocks start at even addresses (34-B blocks, rows of
                // D/32 blocks, validated 2-B aligned): 16-bit stores throughout
                uint16_t *bp = reinterpret_cast<uint16_t *>(dst + blk * 34);
                if (sub == 0) {
                    bp[0] = __half_as_ushort(__float2half_rn(d));
                }
#pragma unroll
                for (int k = 0; k < 4; k += 2) {
                    const uint32_t q0 = (uint32_t) (uint8_t) (int8_t) roundf(x[k] * id);
                    const uint32_t q1 = (uint32_t) (uint8_t) (int8_t) roundf(x[k + 1] * id);
                    bp[1 + sub * 2 + k / 2] = (uint16_t) (q0 | (q1 << 8));
                }
            }
        } else {
            uint16_t *dh = reinterpret_cast<uint16_t *>(dst);
#pragma unroll
            for (int k = 0; k < D / 32; ++k) {
                const float v = x[k];
                dh[append_index<KV_TYPE, D>(lane, k)] =
                    KV_TYPE == ACEFA_TYPE_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                               : __half_as_ushort(__float2half_rn(v));
            }
        }
    }
    fence_proxy_async_global();
    __syncwarp();
}

// PRO: the instance that applies the QK-norm + RoPE prologues (Q rows, the
// appended K row); the others carry none of that code.
template <int KV_TYPE, int D, bool PRO>
__global__ void __launch_bounds__(DecCfg<KV_TYPE, D>::kThreads, 2)
    fa_decode_kernel(const __grid_constant__ DecodeParams P, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap) {
    using Cfg                 = DecCfg<KV_TYPE, D>;
    constexpr bool kQ8        = Cfg::kQ8;
    constexpr bool kBF16      = Cfg::kBF16;
    constexpr int  KS         = D / 16;  // k-steps over the head dim
    constexpr int  NT         = D / 8;   // n8 tiles over the head dim

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    uint64_t     *full_bar  = reinterpret_cast<uint64_t *>(smem + Cfg::kOffBars);
    uint64_t     *empty_bar = full_bar + kDecStages;
    int4         *meta      = reinterpret_cast<int4 *>(smem + Cfg::kOffMeta);
    volatile int *abort_f   = reinterpret_cast<volatile int *>(smem + Cfg::kOffFlags);
    float        *merge     = reinterpret_cast<float *>(smem + Cfg::kOffMerge);
    float        *s_m       = reinterpret_cast<float *>(smem + Cfg::kOffStats);
    float        *s_l       = s_m + kDecWarps * kDecRows;
    float        *s_fin     = reinterpret_cast<float *>(smem + Cfg::kOffFin);  // [0,16) max, [16,32) sum

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kDecStages; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], kDecWarps);
        }
        *abort_f = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // Everything below reads tensors that an earlier kernel may have written.
    pdl_wait_primary();
    pdl_launch_dependents();

    const OpDesc &o  = P.op;
    const int64_t T  = P.total_tiles;
    const int     C  = P.n_ctas;
    const int64_t t0 = mul_div(blockIdx.x, T, C, P.div32);
    const int64_t t1 = mul_div(blockIdx.x + 1, T, C, P.div32);
    const int     tpu = P.tiles_per_unit;

    if (warp == kDecWarps) {
        // ============================ producer ============================
        if (!kQ8 && lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
        }
        int      stage = 0;
        uint32_t phase = 0;
        bool     ok    = true;
        int      pend[kDecStages];  // parity of the last phase armed on each full barrier
        for (int i = 0; i < kDecStages; ++i) {
            pend[i] = -1;
        }
        auto advance = [&]() {
            if (++stage == kDecStages) {
                stage = 0;
                phase ^= 1u;
            }
        };
        auto acquire = [&]() -> bool {
            // all lanes poll; the outcome is made warp-uniform because the
            // ballots and shuffles after it need the whole warp
            return __all_sync(0xffffffffu, mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_f, P.dev_err,
                                                             DEVERR_TIMEOUT_EMPTY, P.wait_limit_ns));
        };
        // Stage the mask segment [64*ti, 64*ti + 64) of every slot row.  Returns
        // the bytes the caller must add to the barrier's transaction count (the
        // bulk-copy case, issued by the caller after arming the barrier); rows
        // that are not 16-B aligned, or a segment running past the mask's row
        // length, are copied here with plain loads instead.
        auto stage_mask = [&](int ti, int n_ms, const uint16_t *my_mr, bool bulk, uint8_t *dst) -> uint32_t {
            if (n_ms == 0) {
                return 0;
            }
            const int j0 = ti * kDecBN;
            if (bulk && j0 + kDecBN <= o.m_ne0) {
                return (uint32_t) (n_ms * kDecBN * 2);
            }
            uint16_t *d16 = reinterpret_cast<uint16_t *>(dst);
            for (int sl = 0; sl < n_ms; ++sl) {
                const uint16_t *src = reinterpret_cast<const uint16_t *>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_mr), sl));
                for (int j = lane; j < kDecBN; j += 32) {
                    d16[sl * kDecBN + j] = j0 + j < o.m_ne0 ? __ldg(src + j0 + j) : kHalfNegInf;
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            return 0;
        };
        for (int64_t t = t0; t < t1 && ok;) {
            const int       u   = (int) mul_div(t, 1, tpu, P.div32);
            const int64_t   ue  = min(t1, (int64_t) (u + 1) * tpu);
            const int       tlo = (int) (t - (int64_t) u * tpu);
            const int       thi = (int) (ue - (int64_t) u * tpu);
            const UnitCoord uc  = unit_coord(P, u);
            const char *kbase = o.k + (int64_t) uc.hk * o.k_nb2 + (int64_t) uc.bk * o.k_nb3;
            const char *vbase = o.v + (int64_t) uc.hk * o.v_nb2 + (int64_t) uc.bk * o.v_nb3;
            // Fused append: the row is written by the CTA whose range holds its
            // tile, just before that tile's copy is issued (after the earlier
            // tiles' copies, so its latency overlaps them), or after the unit's
            // tiles when the mask makes that tile dead.
            int64_t app_row  = -1;
            int     app_tile = -1;
            float   app_k[4], app_v[4];
            if (P.append_pos) {
                app_row = P.append_pos[uc.bk];
                if (app_row < 0 || app_row >= o.n_kv) {
                    if (lane == 0) {
                        atomicCAS(P.dev_err, 0, DEVERR_APPEND_POS);
                    }
                } else if (app_row / kDecBN >= tlo && app_row / kDecBN < thi) {
                    app_tile = (int) (app_row / kDecBN);
                    append_load<KV_TYPE, D, PRO>(P, uc.hk, uc.bk, lane, app_k, app_v);
                }
            }
            // Mask slots: the distinct mask rows this unit reads (one per query
            // index when the mask is shared by all heads).  Lane s owns slot s and
            // stages its 64-key segment of every tile into shared memory.
            int             n_ms   = 0;
            const uint16_t *my_mr  = nullptr;
            if (o.mask) {
                if (o.m_ne2 == 1) {
                    const int iq0 = (uc.rb * kDecRows) / o.G;
                    n_ms          = (uc.rb * kDecRows + uc.rows - 1) / o.G - iq0 + 1;
                    if (lane < n_ms) {
                        my_mr = mask_row(o, iq0 + lane, 0, uc.b);
                    }
                } else {
                    n_ms = uc.rows;
                    if (lane < n_ms) {
                        int iq, hq;
                        row_coord(P, uc, lane, iq, hq);
                        my_mr = mask_row(o, iq, hq, uc.b);
                    }
                }
            }
            const bool mask_bulk =
                __all_sync(0xffffffffu, lane >= n_ms || (reinterpret_cast<uintptr_t>(my_mr) & 15u) == 0);
            for (int tb = tlo; tb < thi && ok; tb += 32) {
                const int  tile = tb + lane;
                const bool live = tile < thi && tile_live(P, uc, tile);
                uint32_t   bits = __ballot_sync(0xffffffffu, live);
                while (bits && ok) {
                    const int i = __ffs(bits) - 1;
                    bits &= bits - 1;
                    const int ti = tb + i;
                    if (ti == app_tile) {
                        append_store<KV_TYPE, D>(P, app_row, lane, kbase, vbase, app_k, app_v);
                        app_tile = -1;
                    }
                    ok           = acquire();
                    if (!ok) {
                        break;
                    }
                    uint8_t *sK = smem + Cfg::kOffStages + stage * Cfg::kStageBytes;
                    uint8_t *sV = sK + Cfg::kTileBytes;
                    if constexpr (kQ8) {
                        // Rows are contiguous 34-B blocks; a tile starts at any even
                        // address.  Copy from the 16-B boundary below it (inside the
                        // tensor: its base is 16-B aligned) and let the consumers
                        // index from the lead; the last <16 bytes go by plain copies.
                        const int      j0     = ti * kDecBN;
                        const int      nrows  = min(kDecBN, o.n_kv - j0);
                        const uint32_t bytes  = (uint32_t) nrows * Cfg::kRowBytes;
                        const char    *kg     = kbase + (int64_t) j0 * Cfg::kRowBytes;
                        const char    *vg     = vbase + (int64_t) j0 * Cfg::kRowBytes;
                        const uint32_t lead_k = (uint32_t) (reinterpret_cast<uintptr_t>(kg) & 15u);
                        const uint32_t lead_v = (uint32_t) (reinterpret_cast<uintptr_t>(vg) & 15u);
                        const uint32_t bulk_k = (lead_k + bytes) & ~15u;
                        const uint32_t bulk_v = (lead_v + bytes) & ~15u;
                        if ((uint32_t) lane < lead_k + bytes - bulk_k) {
                            sK[bulk_k + lane] = (uint8_t) kg[(int) (bulk_k + lane) - (int) lead_k];
                        }
                        if ((uint32_t) lane < lead_v + bytes - bulk_v) {
                            sV[bulk_v + lane] = (uint8_t) vg[(int) (bulk_v + lane) - (int) lead_v];
                        }
                        const uint32_t mbytes = stage_mask(ti, n_ms, my_mr, mask_bulk, sK + 2 * Cfg::kTileBytes);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (mbytes && lane < n_ms) {
                            bulk_load(sK + 2 * Cfg::kTileBytes + lane * kDecBN * 2, my_mr + ti * kDecBN, kDecBN * 2,
                                      &full_bar[stage]);
                        }
                        if (lane == 0) {
                            meta[stage] = make_int4(u, ti, kMetaData, (int) (lead_k | (lead_v << 8)));
                            mbar_arrive_expect_tx(&full_bar[stage], bulk_k + bulk_v + mbytes);
                            if (bulk_k) {
                                bulk_load(sK, kg - lead_k, bulk_k, &full_bar[stage]);
                            }
                            if (bulk_v) {
                                bulk_load(sV, vg - lead_v, bulk_v, &full_bar[stage]);
                            }
                        }
                    } else {
                        const uint32_t mbytes = stage_mask(ti, n_ms, my_mr, mask_bulk, sK + 2 * Cfg::kTileBytes);
                        if (lane == 0) {
                            meta[stage] = make_int4(u, ti, kMetaData, 0);
                            mbar_arrive_expect_tx(&full_bar[stage], (uint32_t) (2 * Cfg::kTmaBytes) + mbytes);
#pragma unroll
                            for (int h = 0; h < D / 64; ++h) {
                                tma_load_4d(sK + h * kDecBN * 128, &kmap, 64 * h, ti * kDecBN, uc.hk, uc.bk,
                                            &full_bar[stage]);
                                tma_load_4d(sV + h * kDecBN * 128, &vmap, 64 * h, ti * kDecBN, uc.hk, uc.bk,
                                            &full_bar[stage]);
                            }
                        }
                        __syncwarp();
                        if (mbytes && lane < n_ms) {
                            bulk_load(sK + 2 * Cfg::kTileBytes + lane * kDecBN * 2, my_mr + ti * kDecBN, kDecBN * 2,
                                      &full_bar[stage]);
                        }
                    }
                    pend[stage] = (int) phase;
                    __syncwarp();
                    advance();
                }
            }
            if (app_tile >= 0) {  // the row's tile is dead for this unit: no read to order
                append_store<KV_TYPE, D>(P, app_row, lane, kbase, vbase, app_k, app_v);
            }
            if (!ok) {
                break;
            }
            ok = acquire();
            if (!ok) {
                break;
            }
            if (lane == 0) {
                meta[stage] = make_int4(u, 0, kMetaFlush, 0);
                mbar_arrive(&full_bar[stage]);
            }
            pend[stage] = (int) phase;
            __syncwarp();
            advance();
            t = ue;
        }
        if (ok) {
            ok = acquire();
            if (ok && lane == 0) {
                meta[stage] = make_int4(-1, 0, kMetaTerm, 0);
                mbar_arrive(&full_bar[stage]);
            }
        }
        if (!ok) {
            // Aborting: let the last copy armed on each stage land before the CTA
            // exits (a phase can never run more than one ahead of its last arm).
            for (int i = 0; i < kDecStages; ++i) {
                if (pend[i] < 0) {
                    continue;
                }
                const uint64_t t_start = globaltimer_ns();
                while (!mbar_try_wait(&full_bar[i], (uint32_t) pend[i])) {
                    if (globaltimer_ns() - t_start > P.wait_limit_ns) {
                        atomicCAS(P.dev_err, 0, DEVERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
        return;
    }

    // ============================== consumers ==============================
    const int g = lane >> 2;  // fragment row group
    const int c = lane & 3;   // fragment column pair
    int       stage = 0;
    uint32_t  phase = 0;

    int       cur_unit = -1;
    UnitCoord uc{};
    float     m_run[2], l_run[2];
    float     oacc[NT][4];
    uint32_t  qa[KS][4];
    // BF16 operands keep ~16 mantissa bits of Q and P by a hi + lo split
    // (two MMAs each); the F16 and Q8_0 paths never touch qlo.
    uint32_t  qlo[kBF16 ? KS : 1][4];
    int       mslot[2];  // mask slot (staged row) of fragment rows g and g+8
    int       vlo[2], vhi[2];  // mask rule: visible keys [vlo, vhi) of rows g and g+8
    float     slope[2];

    auto setup_unit = [&](int u) {
        uc = unit_coord(P, u);
        m_run[0] = m_run[1] = -INFINITY;
        l_run[0] = l_run[1] = 0.0f;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                oacc[j][e] = 0.0f;
            }
        }
        const float *qrow[2];
        int          qpos[2] = {0, 0};  // RoPE positions of rows g and g+8 (Q prologue)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int rr = g + 8 * i;
            int       iq, hq;
            row_coord(P, uc, rr < uc.rows ? rr : 0, iq, hq);
            qrow[i]  = rr < uc.rows ? reinterpret_cast<const float *>(o.q + (int64_t) iq * o.q_nb1 +
                                                                     (int64_t) hq * o.q_nb2 + (int64_t) uc.b * o.q_nb3)
                                    : nullptr;
            mslot[i] = o.m_ne2 == 1 ? iq - (uc.rb * kDecRows) / o.G : (rr < uc.rows ? rr : 0);
            slope[i] = alibi_slope(o, hq);
            if (o.mg_kind) {
                mg_range(o, uc.b, iq, vlo[i], vhi[i]);
            }
            if (PRO && o.qp.rope && rr < uc.rows) {
                qpos[i] = __ldg(o.qp.pos + iq + (int64_t) uc.b * o.n_q);
            }
        }
        if constexpr (!PRO) {
            auto qv = [&](int i, int d) -> float { return qrow[i] ? __ldg(qrow[i] + d) : 0.0f; };
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                if constexpr (kQ8) {
                    // dims permuted so each thread's K bytes are one contiguous run
                    const int d0 = c * (D / 4) + 4 * ks;
                    qa[ks][0]    = pack2<false>(qv(0, d0), qv(0, d0 + 1));
                    qa[ks][1]    = pack2<false>(qv(1, d0), qv(1, d0 + 1));
                    qa[ks][2]    = pack2<false>(qv(0, d0 + 2), qv(0, d0 + 3));
                    qa[ks][3]    = pack2<false>(qv(1, d0 + 2), qv(1, d0 + 3));
                } else {
                    const int d0    = 16 * ks + 2 * c;
                    const int ii[4] = {0, 1, 0, 1};
                    const int dd[4] = {d0, d0, d0 + 8, d0 + 8};
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float x0 = qv(ii[r], dd[r]), x1 = qv(ii[r], dd[r] + 1);
                        qa[ks][r]      = pack2<kBF16>(x0, x1);
                        if constexpr (kBF16) {
                            qlo[ks][r] = split_lo_bf16(x0, x1, qa[ks][r]);
                        }
                    }
                }
            }
        } else {
            // This thread's Q values, x[i][ks][e] of row g + 8i: dims
            // c*(D/4) + 4ks + e for Q8_0 (each thread's K bytes are one run), else
            // 16ks + 2c + (e & 1) + 8(e >> 1) (the m16n8k16 A fragment).
            auto qdim = [&](int ks, int e) -> int {
                return kQ8 ? c * (D / 4) + 4 * ks + e : 16 * ks + 2 * c + (e & 1) + 8 * (e >> 1);
            };
            float x[2][KS][4];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        x[i][ks][e] = qrow[i] ? __ldg(qrow[i] + qdim(ks, e)) : 0.0f;
                    }
                }
            }
            if (o.qp.on) {
                // QK-norm + RoPE: a row's D values are spread over its quad (c = 0..3)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    if (o.qp.w) {
                        float ss = 0.0f;
#pragma unroll
                        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                ss = fmaf(x[i][ks][e], x[i][ks][e], ss);
                            }
                        }
                        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                        const float sc = rn_scale(o.qp, ss, D);
#pragma unroll
                        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                x[i][ks][e] = (x[i][ks][e] * sc) * __ldg(o.qp.w + qdim(ks, e));
                            }
                        }
                    }
                    if (o.qp.rope) {
                        if constexpr (kQ8) {
                            // dim d + D/2 sits on thread c ^ 2 at the same (ks, e)
#pragma unroll
                            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float pt = __shfl_xor_sync(0xffffffffu, x[i][ks][e], 2);
                                    x[i][ks][e]    = rn_rotate(o.qp, x[i][ks][e], pt, c < 2, qpos[i], qdim(ks, e) & (D / 2 - 1));
                                }
                            }
                        } else {
                            // dim d + D/2 is this thread's (ks + KS/2, e)
#pragma unroll
                            for (int ks = 0; ks < KS / 2; ++ks) {
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const float a = x[i][ks][e], bb = x[i][ks + KS / 2][e];
                                    x[i][ks][e]          = rn_rotate(o.qp, a, bb, true, qpos[i], qdim(ks, e));
                                    x[i][ks + KS / 2][e] = rn_rotate(o.qp, bb, a, false, qpos[i], qdim(ks, e));
                                }
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    // fragment register r: row r & 1, value pair (r >> 1)
                    const float x0 = x[r & 1][ks][2 * (r >> 1)], x1 = x[r & 1][ks][2 * (r >> 1) + 1];
                    qa[ks][r]      = pack2<kBF16>(x0, x1);
                    if constexpr (kBF16) {
                        qlo[ks][r] = split_lo_bf16(x0, x1, qa[ks][r]);
                    }
                }
            }
        }
    };

    // Head-dim index held by accumulator element (j, e) (column part only).
    auto out_dim = [&](int j, int e) -> int {
        if constexpr (kQ8) {
            return (D / 8) * (2 * c + (e & 1)) + j;
        } else {
            return 8 * j + 2 * c + (e & 1);
        }
    };

    auto process_tile = [&](const uint8_t *sK, const uint8_t *sV, const uint16_t *sM, int tile) {
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s[nt][e] = 0.0f;
            }
        }
        // ---- S = Q K^T over this warp's 16 keys
        if constexpr (kQ8) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int      row   = 16 * warp + 8 * nt + g;
                const int      dim0  = c * (D / 4);
                const uint32_t rbase = smem_u32(sK) + row * Cfg::kRowBytes + (dim0 / 32) * 34;
                uint32_t       qw[D / 16];
                lds_bytes_unaligned<D / 16>(rbase + 2 + (dim0 % 32), qw);
                const __half  dsc = __ushort_as_half(lds16(rbase));
                const __half2 d2  = __half2half2(dsc);
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    const __half2 lo = __hmul2(i8pair_to_h2(__byte_perm(qw[ks], 0, 0x4140)), d2);
                    const __half2 hi = __hmul2(i8pair_to_h2(__byte_perm(qw[ks], 0, 0x4342)), d2);
                    mma_16816<false>(s[nt], qa[ks], *reinterpret_cast<const uint32_t *>(&lo),
                                     *reinterpret_cast<const uint32_t *>(&hi));
                }
            }
        } else {
            const int mi   = lane >> 3;
            const int r8   = lane & 7;
            const int krow = 16 * warp + (mi >> 1) * 8 + r8;
            float s2[2][4];  // second accumulator chain (odd k-steps) for more MMA overlap
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s2[nt][e] = 0.0f;
                }
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int      dim  = 16 * ks + (mi & 1) * 8;
                const uint32_t addr = smem_u32(sK) + (dim >> 6) * (kDecBN * 128) + krow * 128 +
                                      ((((dim & 63) >> 3) ^ r8) << 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(addr, b0, b1, b2, b3);
                float(&acc)[2][4] = (!kBF16 && (ks & 1)) ? s2 : s;  // BF16 already pairs hi+lo MMAs
                mma_16816<kBF16>(acc[0], qa[ks], b0, b1);
                mma_16816<kBF16>(acc[1], qa[ks], b2, b3);
                if constexpr (kBF16) {
                    mma_16816<true>(acc[0], qlo[ks], b0, b1);
                    mma_16816<true>(acc[1], qlo[ks], b2, b3);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s[nt][e] += s2[nt][e];
                }
            }
        }
        // ---- scale, softcap, mask, bounds; to log2 units
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i   = e >> 1;
                const int pos = tile * kDecBN + 16 * warp + 8 * nt + 2 * c + (e & 1);
                float     x   = s[nt][e] * o.scale_eff;
                if (o.softcap != 0.0f) {
                    x = o.softcap * tanhf(x);
                }
                if (pos < o.n_kv) {
                    if (o.mask) {
                        // a -inf entry removes the key outright, whatever K held there
                        const float mv = slope[i] * __half2float(__ushort_as_half(
                                                        sM[mslot[i] * kDecBN + 16 * warp + 8 * nt + 2 * c + (e & 1)]));
                        x              = mv == -INFINITY ? -INFINITY : x + mv;
                    } else if (o.mg_kind) {
                        // a visible key adds the rule's 0 like a 0 mask entry
                        x = pos >= vlo[i] && pos < vhi[i] ? x + 0.0f : -INFINITY;
                    }
                    x *= kLog2e;
                } else {
                    x = -INFINITY;
                }
                s[nt][e] = x;
            }
        }
        // ---- online softmax (rows g and g+8)
        float alpha[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            float mx = fmaxf(fmaxf(s[0][2 * i], s[0][2 * i + 1]), fmaxf(s[1][2 * i], s[1][2 * i + 1]));
            mx       = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx       = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mnew = fmaxf(m_run[i], mx);
            const float muse = mnew == -INFINITY ? 0.0f : mnew;
            alpha[i]         = fast_exp2(m_run[i] - muse);
            m_run[i]         = mnew;
            float rs         = 0.0f;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                s[nt][2 * i]     = fast_exp2(s[nt][2 * i] - muse);
                s[nt][2 * i + 1] = fast_exp2(s[nt][2 * i + 1] - muse);
                rs += s[nt][2 * i] + s[nt][2 * i + 1];
            }
            l_run[i] = l_run[i] * alpha[i] + rs;
        }
        if (__any_sync(0xffffffffu, alpha[0] != 1.0f || alpha[1] != 1.0f)) {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                oacc[j][0] *= alpha[0];
                oacc[j][1] *= alpha[0];
                oacc[j][2] *= alpha[1];
                oacc[j][3] *= alpha[1];
            }
        }
        // ---- O += P V
        constexpr bool kPB = kQ8 ? false : kBF16;
        uint32_t       pa[4];
        pa[0] = pack2<kPB>(s[0][0], s[0][1]);
        pa[1] = pack2<kPB>(s[0][2], s[0][3]);
        pa[2] = pack2<kPB>(s[1][0], s[1][1]);
        pa[3] = pack2<kPB>(s[1][2], s[1][3]);
        uint32_t palo[4];
        if constexpr (kBF16) {
            palo[0] = split_lo_bf16(s[0][0], s[0][1], pa[0]);
            palo[1] = split_lo_bf16(s[0][2], s[0][3], pa[1]);
            palo[2] = split_lo_bf16(s[1][0], s[1][1], pa[2]);
            palo[3] = split_lo_bf16(s[1][2], s[1][3], pa[3]);
        }
        if constexpr (kQ8) {
            // this thread's B fragments: keys 2c,2c+1 (b0) and 2c+8,2c+9 (b1) of the
            // warp's 16, head dims (D/8)*g .. +D/8 (one contiguous byte run per key)
            const int dim0 = (D / 8) * g;
            uint32_t  qv[4][D / 32];
            __half    dv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int      key   = 16 * warp + 2 * c + (r & 1) + 8 * (r >> 1);
                const uint32_t rbase = smem_u32(sV) + key * Cfg::kRowBytes + (dim0 / 32) * 34;
                lds_bytes_unaligned<D / 32>(rbase + 2 + (dim0 % 32), qv[r]);
                // rows past n_kv in the last tile hold stale bytes: a zero scale
                // keeps them finite (their P is 0, but 0 * inf would be NaN)
                dv[r] = tile * kDecBN + key < o.n_kv ? __ushort_as_half(lds16(rbase)) : __float2half(0.0f);
            }
            const __half2 d01 = __halves2half2(dv[0], dv[1]);
            const __half2 d89 = __halves2half2(dv[2], dv[3]);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int      wi  = j >> 2;
                const uint32_t sel = (uint32_t) (j & 3) | ((uint32_t) (4 + (j & 3)) << 8);
                const __half2  b0  = __hmul2(i8pair_to_h2(__byte_perm(qv[0][wi], qv[1][wi], sel)), d01);
                const __half2  b1  = __hmul2(i8pair_to_h2(__byte_perm(qv[2][wi], qv[3][wi], sel)), d89);
                mma_16816<false>(oacc[j], pa, *reinterpret_cast<const uint32_t *>(&b0),
                                 *reinterpret_cast<const uint32_t *>(&b1));
            }
        } else {
            const int mi   = lane >> 3;
            const int r8   = lane & 7;
            const int vrow = 16 * warp + (mi & 1) * 8 + r8;
#pragma unroll
            for (int dn = 0; dn < D / 16; ++dn) {
                const int      dim  = 16 * dn + (mi >> 1) * 8;
                const uint32_t addr = smem_u32(sV) + (dim >> 6) * (kDecBN * 128) + vrow * 128 +
                                      ((((dim & 63) >> 3) ^ r8) << 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(addr, b0, b1, b2, b3);
                mma_16816<kBF16>(oacc[2 * dn], pa, b0, b1);
                mma_16816<kBF16>(oacc[2 * dn + 1], pa, b2, b3);
                if constexpr (kBF16) {
                    mma_16816<true>(oacc[2 * dn], palo, b0, b1);
                    mma_16816<true>(oacc[2 * dn + 1], palo, b2, b3);
                }
            }
        }
    };

    auto flush_unit = [&](int u) {
        // per-warp row statistics
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 1);
            l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 2);
        }
        if (c == 0) {
            s_m[warp * kDecRows + g]     = m_run[0];
            s_m[warp * kDecRows + g + 8] = m_run[1];
            s_l[warp * kDecRows + g]     = l_run[0];
            s_l[warp * kDecRows + g + 8] = l_run[1];
        }
        named_bar_sync(1, kDecWarps * 32);
        float fac[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int row = g + 8 * i;
            float     mx  = -INFINITY;
#pragma unroll
            for (int w = 0; w < kDecWarps; ++w) {
                mx = fmaxf(mx, s_m[w * kDecRows + row]);
            }
            fac[i] = m_run[i] == -INFINITY ? 0.0f : fast_exp2(m_run[i] - mx);
        }
        // The four warps' partial O, rescaled to the common row max, summed in
        // shared memory in four turns; in turn t warp w adds its n8 tiles of
        // column block (w + t) % 4, so every warp works in every turn and each
        // element has one writer per turn (plain stores, no atomics).  Threads
        // 0-15 also merge the row statistics.
        constexpr int NTB = NT / 4;  // n8 tiles per column block
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int bsel = (warp + t) & 3;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                if (bb == bsel) {
#pragma unroll
                    for (int jj = 0; jj < NTB; ++jj) {
                        const int j = bb * NTB + jj;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float      *mp = &merge[(g + 8 * (e >> 1)) * Cfg::kMergeStride + out_dim(j, e)];
                            const float v  = oacc[j][e] * fac[e >> 1];
                            *mp            = t == 0 ? v : *mp + v;
                        }
                    }
                }
            }
            if (t == 0 && threadIdx.x < kDecRows) {
                const int row = threadIdx.x;
                float     mx  = -INFINITY;
#pragma unroll
                for (int ww = 0; ww < kDecWarps; ++ww) {
                    mx = fmaxf(mx, s_m[ww * kDecRows + row]);
                }
                float l = 0.0f;
#pragma unroll
                for (int ww = 0; ww < kDecWarps; ++ww) {
                    const float mw = s_m[ww * kDecRows + row];
                    l += mw == -INFINITY ? 0.0f : s_l[ww * kDecRows + row] * fast_exp2(mw - mx);
                }
                s_fin[row]            = mx;
                s_fin[kDecRows + row] = l;
            }
            named_bar_sync(1, kDecWarps * 32);
        }
        // this CTA holds every tile of the unit: write the output itself
        const bool direct = t0 <= (int64_t) u * tpu && (int64_t) (u + 1) * tpu <= t1;
        float     *slot   = P.partials + (int64_t) (blockIdx.x + u) * dec_slot_floats(D);
        if (!direct && threadIdx.x < kDecRows && threadIdx.x < uc.rows) {
            slot[threadIdx.x]            = s_fin[threadIdx.x];
            slot[kDecRows + threadIdx.x] = s_fin[kDecRows + threadIdx.x];
        }
        // four consecutive head dims per thread and step
        for (int idx = threadIdx.x; idx < kDecRows * (D / 4); idx += kDecWarps * 32) {
            const int row = idx / (D / 4);
            const int d   = (idx % (D / 4)) * 4;
            if (row >= uc.rows) {
                continue;
            }
            float4 acc = *reinterpret_cast<const float4 *>(&merge[row * Cfg::kMergeStride + d]);
            if (direct) {
                const float mx = s_fin[row];
                float       l  = s_fin[kDecRows + row];
                float       fs = 1.0f;
                int         iq, hq;
                row_coord(P, uc, row, iq, hq);
                if (o.sinks) {
                    const float ts = o.sinks[hq] * kLog2e;
                    if (ts > mx) {
                        fs = fast_exp2(mx - ts);
                        l  = l * fs + 1.0f;
                    } else {
                        l += fast_exp2(ts - mx);
                    }
                }
                const float inv = l == 0.0f ? 0.0f : fs / l;
                acc             = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
                char *dp = o.dst + (int64_t) d * o.d_nb0 + (int64_t) hq * o.d_nb1 + (int64_t) iq * o.d_nb2 +
                           (int64_t) uc.b * o.d_nb3;
                if (o.d_nb0 == 4 && (reinterpret_cast<uintptr_t>(dp) & 15u) == 0) {
                    // mirrors are congruent to dst modulo 16 B
                    *reinterpret_cast<float4 *>(dp) = acc;
                    for (int mi = 0; mi < o.n_mirror; ++mi) {
                        *reinterpret_cast<float4 *>(dp + o.mirror_delta[mi]) = acc;
                    }
                } else {
                    const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        char *dk = dp + (int64_t) k * o.d_nb0;
                        *reinterpret_cast<float *>(dk) = a4[k];
                        for (int mi = 0; mi < o.n_mirror; ++mi) {
                            *reinterpret_cast<float *>(dk + o.mirror_delta[mi]) = a4[k];
                        }
                    }
                }
                if (o.n_mirror) {
                    __threadfence_system();
                }
            } else {
                *reinterpret_cast<float4 *>(slot + 2 * kDecRows + row * D + d) = acc;
            }
        }
        named_bar_sync(1, kDecWarps * 32);  // merge and s_fin are free for the next unit
    };

    // The first unit is known from the tile range: fetch its Q while the
    // producer scans the mask and issues the first copies.
    if (t0 < t1) {
        cur_unit = (int) mul_div(t0, 1, tpu, P.div32);
        setup_unit(cur_unit);
    }
    while (true) {
        const bool got =
            mbar_wait_bounded(&full_bar[stage], phase, abort_f, P.dev_err, DEVERR_TIMEOUT_FULL, P.wait_limit_ns);
        // ldmatrix / mma.sync / shuffles below are warp-collective: leave together
        if (!__all_sync(0xffffffffu, got)) {
            break;
        }
        const int4 md = meta[stage];
        if (md.z == kMetaTerm) {
            break;
        }
        if (md.x != cur_unit) {
            setup_unit(md.x);
            cur_unit = md.x;
        }
        if (md.z == kMetaData) {
            const uint8_t *sK = smem + Cfg::kOffStages + stage * Cfg::kStageBytes;
            const uint8_t *sV = sK + Cfg::kTileBytes;
            if constexpr (kQ8) {
                sK += md.w & 0xff;
                sV += (md.w >> 8) & 0xff;
            }
            process_tile(sK, sV,
                         reinterpret_cast<const uint16_t *>(smem + Cfg::kOffStages + stage * Cfg::kStageBytes +
                                                            2 * Cfg::kTileBytes),
                         md.y);
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty_bar[stage]);
        }
        if (md.z == kMetaFlush) {
            flush_unit(cur_unit);
            cur_unit = -1;
        }
        if (++stage == kDecStages) {
            stage = 0;
            phase ^= 1u;
        }
    }
}

// ---------------------------------------------------------------------------
// Combine: merge the partials of every unit split across CTAs.  One CTA per
// unit; 16 threads per row, each owning D/16 contiguous head dims, so all rows
// and parts are read in parallel (the kernel is latency bound).
constexpr int kCombThreads = kDecRows * 16;

template <int D>
__global__ void __launch_bounds__(kCombThreads) fa_decode_combine(const __grid_constant__ DecodeParams P) {
    constexpr int DPT = D / 16;  // dims per thread
    pdl_wait_primary();
    const OpDesc &o   = P.op;
    const int     u   = blockIdx.x;
    const int64_t T   = P.total_tiles;
    const int     C   = P.n_ctas;
    const int     tpu = P.tiles_per_unit;
    const int64_t cf  = cta_of_tile((int64_t) u * tpu, T, C, P.div32);
    const int64_t cl  = cta_of_tile((int64_t) (u + 1) * tpu - 1, T, C, P.div32);
    if (cf == cl) {
        return;
    }
    const UnitCoord uc  = unit_coord(P, u);
    const int       row = threadIdx.x / 16;
    const int       d0  = (threadIdx.x % 16) * DPT;
    // rows past uc.rows still run (the shuffles below need full warps); they
    // read their slot's unused rows and write nothing
    const bool    active = row < uc.rows;
    const int64_t stride = dec_slot_floats(D);
    const float  *base   = P.partials + (cf + u) * stride;
    const int     np     = (int) (cl - cf + 1);  // <= kDecMaxParts + 1
    const int     sub    = threadIdx.x % 16;
    // Thread `sub` of a row reads part sub's max and sum (at most 16 parts), so
    // the row statistics take one round of loads and two shuffle reductions;
    // then every part's slice of O is requested before any is summed.
    float m_p = -INFINITY, l_p = 0.0f;
    if (sub < np) {
        m_p = __ldg(base + sub * stride + row);
        l_p = __ldg(base + sub * stride + kDecRows + row);
    }
    float mx = m_p;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    const float f_p = m_p == -INFINITY ? 0.0f : fast_exp2(m_p - mx);
    float       l   = l_p * f_p;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, off);
    }
    float acc[DPT];
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
        acc[i] = 0.0f;
    }
    const int grp = (threadIdx.x & 31) & ~15;  // first lane of this row's 16 in the warp
    // a unit spans at most kDecMaxParts + 1 CTAs (its ends need not align with
    // theirs): at most 16 parts, one per thread of the row.  The weights are
    // gathered first so that no shuffle sits between the loads below.
    static_assert(kDecMaxParts + 1 <= 16, "one part per thread of a row");
    float fw[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        fw[p] = __shfl_sync(0xffffffffu, f_p, grp + p);
    }
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        if (p < np) {  // uniform over the CTA
            const float   f   = fw[p];
            const float4 *op4 = reinterpret_cast<const float4 *>(base + p * stride + 2 * kDecRows + row * D + d0);
#pragma unroll
            for (int i = 0; i < DPT / 4; ++i) {
                const float4 v = __ldg(op4 + i);
                acc[4 * i + 0] += f * v.x;
                acc[4 * i + 1] += f * v.y;
                acc[4 * i + 2] += f * v.z;
                acc[4 * i + 3] += f * v.w;
            }
        }
    }
    if (!active) {
        return;
    }
    int iq, hq;
    row_coord(P, uc, row, iq, hq);
    float fs = 1.0f;
    if (o.sinks) {
        const float ts = o.sinks[hq] * kLog2e;
        if (ts > mx) {
            fs = fast_exp2(mx - ts);
            l  = l * fs + 1.0f;
        } else {
            l += fast_exp2(ts - mx);
        }
    }
    const float inv = l == 0.0f ? 0.0f : fs / l;
    char       *out = o.dst + (int64_t) hq * o.d_nb1 + (int64_t) iq * o.d_nb2 + (int64_t) uc.b * o.d_nb3;
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
        char *dp = out + (int64_t) (d0 + i) * o.d_nb0;
        *reinterpret_cast<float *>(dp) = acc[i] * inv;
        for (int mi = 0; mi < o.n_mirror; ++mi) {
            *reinterpret_cast<float *>(dp + o.mirror_delta[mi]) = acc[i] * inv;
        }
    }
    if (o.n_mirror) {
        __threadfence_system();
    }
}

// ---------------------------------------------------------------------------
// host side

namespace {

template <int KV_TYPE, int D>
cudaError_t launch_impl(const DecodeLaunch &L, cudaStream_t s, int *launches) {
    using Cfg = DecCfg<KV_TYPE, D>;
    const bool pro  = L.p.op.qp.on || L.p.kp.on;
    auto       kern = pro ? fa_decode_kernel<KV_TYPE, D, true> : fa_decode_kernel<KV_TYPE, D, false>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        for (auto k : {fa_decode_kernel<KV_TYPE, D, false>, fa_decode_kernel<KV_TYPE, D, true>}) {
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
            if (e != cudaSuccess) {
                return e;
            }
        }
        configured_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) L.p.n_ctas);
    cfg.blockDim           = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes   = Cfg::kSmemBytes;
    cfg.stream             = s;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, L.p, L.kmap, L.vmap);
    if (e != cudaSuccess) {
        return e;
    }
    int n = 1;
    // The combine only has work when some unit spans several CTAs.
    if (decode_needs_combine(L.p)) {
        cudaLaunchConfig_t c2 = cfg;
        c2.gridDim            = dim3((unsigned) L.p.units);
        c2.blockDim           = dim3(kCombThreads);
        c2.dynamicSmemBytes   = 0;
        e                     = cudaLaunchKernelEx(&c2, fa_decode_combine<D>, L.p);
        if (e != cudaSuccess) {
            return e;
        }
        n = 2;
    }
    if (launches) {
        *launches = n;
    }
    return cudaSuccess;
}

}  // namespace

bool decode_needs_combine(const DecodeParams &p) {
    // a unit is split iff some CTA range boundary falls strictly inside it
    for (int c = 1; c < p.n_ctas; ++c) {
        const int64_t lo = (int64_t) c * p.total_tiles / p.n_ctas;
        if (lo % p.tiles_per_unit != 0) {
            return true;
        }
    }
    return false;
}

cudaError_t launch_decode(const DecodeLaunch &L, cudaStream_t s, int *launches) {
    const int t = L.p.op.kv_type, D = L.p.op.D;
    if (t == ACEFA_TYPE_F16 && D == 128) return launch_impl<ACEFA_TYPE_F16, 128>(L, s, launches);
    if (t == ACEFA_TYPE_F16 && D == 64) return launch_impl<ACEFA_TYPE_F16, 64>(L, s, launches);
    if (t == ACEFA_TYPE_BF16 && D == 128) return launch_impl<ACEFA_TYPE_BF16, 128>(L, s, launches);
    if (t == ACEFA_TYPE_BF16 && D == 64) return launch_impl<ACEFA_TYPE_BF16, 64>(L, s, launches);
    if (t == ACEFA_TYPE_Q8_0 && D == 128) return launch_impl<ACEFA_TYPE_Q8_0, 128>(L, s, launches);
    if (t == ACEFA_TYPE_Q8_0 && D == 64) return launch_impl<ACEFA_TYPE_Q8_0, 64>(L, s, launches);
    return cudaErrorInvalidValue;
}

size_t decode_smem_bytes(int kv_type, int D) {
    if (kv_type == ACEFA_TYPE_Q8_0) {
        return D == 128 ? DecCfg<ACEFA_TYPE_Q8_0, 128>::kSmemBytes : DecCfg<ACEFA_TYPE_Q8_0, 64>::kSmemBytes;
    }
    return D == 128 ? DecCfg<ACEFA_TYPE_F16, 128>::kSmemBytes : DecCfg<ACEFA_TYPE_F16, 64>::kSmemBytes;
}

int decode_ctas_per_sm(int kv_type, int D) {
    // Two CTAs per SM share the 228 KB of shared memory; the launch bounds ask
    // the register allocator for the same.
    const size_t per = decode_smem_bytes(kv_type, D) + 1024;  // + per-CTA reserve
    return per * 2 <= 228 * 1024 ? 2 : 1;
}

}  // namespace acefa
