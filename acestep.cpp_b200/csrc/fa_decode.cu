// fa_decode.cu -- split-KV flash-decode for sm_100a.
//
// Serves ggml_flash_attn_ext nodes whose query side is small: acestep.cpp's
// batched CFG decode (src/qwen3-lm.h:789-794: Q [128,1,Hq,N], K/V views
// [128,n_kv_pad,8,N] of the KV cache), single-sequence decode
// (src/qwen3-lm.h:465-469 with n_tokens == 1) and the short FSQ encoders
// (src/fsq-tok.h:183, src/fsq-detok.h:171; S = 5..6).
//
// Design (memory bound; the roofline is HBM bytes of K and V):
//   * Work unit = (batch b, kv head hk, row block rb).  A unit's rows are the
//     G*n_q (query, q-head) pairs that share K/V head hk, 16 per block, so each
//     K/V byte is read once per unit and feeds G*n_q rows of tensor-core math.
//   * A unit runs on one thread-block cluster of C CTAs (C chosen on the host
//     so that units * C fills the SMs); CTA r of the cluster streams the r-th
//     contiguous range of the unit's 64-key tiles.  At the end the CTAs merge
//     their partial results (running max, row sum, unnormalised O) through
//     distributed shared memory, each CTA finishing one slice of the head
//     dims.  One launch per op, no workspace, no second kernel; grid and
//     cluster size depend on shapes only, so a captured CUDA graph replays
//     with any mask contents.
//   * One producer warp streams K/V tiles into a 3-stage shared-memory ring --
//     TMA tensor tiles with 128-B swizzle for F16/BF16, 1-D bulk copies of
//     whole 34-B-block rows for Q8_0 -- and skips tiles whose mask is entirely
//     -inf (the padded decode window tail).
//   * Four consumer warps each take 16 keys of every tile, on mma.sync
//     m16n8k16 with F32 accumulation and an online softmax in the log2 domain.
//     F16/BF16: S = Q K^T and O += P V over 16-row units, K and V by ldmatrix
//     from the swizzled tiles.  Q8_0: transposed, S^T = K Q^T and
//     O^T += V^T P^T over 8-row units (the keys fill the MMA's M dimension, so
//     a 4-head GQA group wastes half an n8 tile instead of three quarters of an
//     m16 tile); head dims are assigned so that each thread's K and V bytes
//     are contiguous runs of Q8_0 blocks, dequantised once in registers as
//     f16(d * q).
//   * Every wait is bounded; on expiry the CTA records an error word, drains
//     its in-flight copies (bounded) and exits.
#include <cfloat>
#include <mutex>

#include "fa_internal.h"
#include "ptx.cuh"
#include "q8.cuh"
#include "rope_norm.cuh"

// Largest cluster the host plan may pick (a tuning macro; the device may
// allow less), and the largest it picks when some SMs would hold two CTAs.
#ifndef ACEFA_DEC_MAX_CLUSTER
#define ACEFA_DEC_MAX_CLUSTER 8
#endif
#ifndef ACEFA_DEC_SHARE_CLUSTER
#define ACEFA_DEC_SHARE_CLUSTER 6
#endif
// Q8_0 stages in flight and CTAs per SM (tuning macros).
#ifndef ACEFA_Q8_STAGES
#define ACEFA_Q8_STAGES 4
#endif
#ifndef ACEFA_Q8_CTAS
#define ACEFA_Q8_CTAS 2
#endif
// The same for the wide Q8_0 instance (decode_wide).
#ifndef ACEFA_Q8W_STAGES
#define ACEFA_Q8W_STAGES 3
#endif
#ifndef ACEFA_Q8W_CTAS
#define ACEFA_Q8W_CTAS 3
#endif

namespace acefa {

namespace {

constexpr int kDecShareCluster = ACEFA_DEC_SHARE_CLUSTER;
constexpr int kMetaData = 1;
constexpr int kMetaTerm = 3;

constexpr uint16_t kHalfNegInf = 0xFC00u;
constexpr float    kQ8RescaleLog2 = 8.0f;  // Q8_0 consumer: rescale when the max grows by > 2^8

// WIDE (Q8_0, D = 128): three CTAs per SM with three stages each instead of
// two with four -- more warps to hide the dequantisation's latency; chosen by
// decode_wide for ops with many long units (elsewhere the shallower pipeline
// and the larger cluster merge cost more than the extra warps gain).
template <int KV_TYPE, int D, bool WIDE = false>
struct DecCfg {
    static constexpr bool kQ8         = KV_TYPE == ACEFA_TYPE_Q8_0;
    static constexpr bool kBF16       = KV_TYPE == ACEFA_TYPE_BF16;
    static constexpr int  kRowBytes   = kQ8 ? D / 32 * 34 : D * 2;  // one cache row
    // rows per unit: the m16 tile of the F16/BF16 consumer, the n8 tile of the
    // transposed Q8_0 consumer
    static constexpr int  kRows       = decode_unit_rows(KV_TYPE);
    // staged tile: F16/BF16 = the TMA boxes (D/64 swizzled boxes of 64 keys x
    // 128 B, 1 KB aligned); Q8_0 = whole block rows plus up to 15 lead bytes
    // (bulk copies only need 16-B alignment)
    static constexpr int  kTile       = kQ8 ? (kDecBN * kRowBytes + 16 + 15) / 16 * 16 : kDecBN * D * 2;
    static constexpr int  kMaskBytes  = kRows * kDecBN * 2;  // a mask row per unit row at most x 64 keys (f16)
    static constexpr int  kStageBytes = 2 * kTile + kMaskBytes;
    static constexpr int  kStages     = kQ8 ? (WIDE ? ACEFA_Q8W_STAGES : ACEFA_Q8_STAGES) : kDecStages;
    static_assert(kQ8 || kStageBytes % 1024 == 0, "TMA stages must stay 1 KB aligned");
    static constexpr int  kThreads     = (kDecWarps + 1) * 32;  // 4 consumer warps + the producer
    // Merge rows: F16/BF16 D + 8 floats.  Q8_0 threads write dims 16g + k
    // (g = lane / 4) of rows 2c + e: with a plain layout 16g aliases on two
    // banks (a 16-way conflict), so every 16-dim group is skewed by one float
    // (merge_at) and the row stride is 4 (mod 16) -- the 32 lanes of a store
    // then hit 32 banks.
    static constexpr int  kMergeStride = kQ8 ? ((D + D / 16 - 4 + 15) / 16) * 16 + 4 : D + 8;
    __device__ static int merge_at(int row, int dim) { return row * kMergeStride + (kQ8 ? dim + (dim >> 4) : dim); }
    // shared memory carve-up (offsets from the 1024-B aligned base).  Q8_0:
    // the merge rows live in the stage memory, idle once every warp has left
    // the tile loop (past the cluster merge's [C][rows] statistics table at
    // the stages' start), so that four CTAs with three stages fit an SM.
    static constexpr int kOffStages = 0;
    static constexpr int kMergeBytes = kDecRows * kMergeStride * 4;
    static constexpr int kOffMerge  = kQ8 ? 1024 : kStages * kStageBytes;
    static_assert(!kQ8 || 1024 + kMergeBytes <= kStages * kStageBytes, "merge rows exceed the stage memory");
    static constexpr int kOffStats  = kQ8 ? kStages * kStageBytes : kOffMerge + kMergeBytes;  // m,l per warp per row
    static constexpr int kOffFin    = kOffStats + 2 * kDecWarps * kDecRows * 4;  // merged m,l per row
    static constexpr int kOffBars   = kOffFin + 2 * kDecRows * 4;
    static constexpr int kNumBars   = 2 * kStages;  // full / empty per stage
    static constexpr int kOffMeta   = kOffBars + kNumBars * 8;
    static constexpr int kOffFlags  = kOffMeta + kStages * 16;
    static constexpr int kSmemBytes = kOffFlags + 16 + 1024;  // + alignment slack
    // D = 256: a 66 KB stage, one CTA per SM
    static constexpr int kCtasPerSm = D > 128 ? 1 : (kQ8 ? (WIDE ? ACEFA_Q8W_CTAS : ACEFA_Q8_CTAS) : 2);
    static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 228 * 1024, "CTAs per SM exceed shared memory");
    static_assert(kSmemBytes <= 232448, "stages exceed the 227 KB per CTA");
    static_assert(D <= 128 || !kQ8, "D = 256 serves F16 and BF16 K/V");
};

struct UnitCoord {
    int b, hk, rb, bk, rows;
};

template <int R>
__device__ __forceinline__ UnitCoord unit_coord(const DecodeParams &P, int u) {
    UnitCoord c;
    c.rb            = u % P.n_rb;
    c.hk            = (u / P.n_rb) % P.op.Hkv;
    c.b             = u / (P.n_rb * P.op.Hkv);
    c.bk            = c.b / P.op.rk3;
    const int total = P.op.G * P.op.n_q;
    c.rows          = min(R, total - c.rb * R);
    return c;
}

// Row rr of unit -> (query index iq, q head hq).
template <int R>
__device__ __forceinline__ void row_coord(const DecodeParams &P, const UnitCoord &uc, int rr, int &iq, int &hq) {
    const int gr = uc.rb * R + rr;
    iq           = gr / P.op.G;
    hq           = uc.hk * P.op.G + gr % P.op.G;
}

__device__ __forceinline__ const uint16_t *mask_row(const OpDesc &o, int iq, int hq, int b) {
    return reinterpret_cast<const uint16_t *>(o.mask + (int64_t) iq * o.m_nb1 + (int64_t) (hq % o.m_ne2) * o.m_nb2 +
                                              (int64_t) (b % o.m_ne3) * o.m_nb3);
}

// True if some mask entry of this tile, for some row of the unit, is not -inf
// (under a mask rule: some key of the tile is in some row's visible range).
template <int R>
__device__ bool tile_live(const DecodeParams &P, const UnitCoord &uc, int tile) {
    const OpDesc &o   = P.op;
    const int     j0  = tile * kDecBN;
    const int     cnt = min(kDecBN, o.n_kv - j0);
    if (o.mg_kind) {
        int lo0, hi0, lo1, hi1;
        mg_range(o, uc.b, (uc.rb * R) / o.G, lo0, hi0);
        mg_range(o, uc.b, (uc.rb * R + uc.rows - 1) / o.G, lo1, hi1);
        return max(lo0, j0) < min(hi1, j0 + cnt);
    }
    if (o.mask == nullptr) {
        return true;
    }
    const uint16_t *prev = nullptr;
    for (int rr = 0; rr < uc.rows; ++rr) {
        int iq, hq;
        row_coord<R>(P, uc, rr, iq, hq);
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

// Residual of a bf16x2 rounding: bf16(x - float(bf16(x))) for both lanes.
__device__ __forceinline__ uint32_t split_lo_bf16(float x0, float x1, uint32_t hi) {
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162 *>(&hi);
    const float2         f = __bfloat1622float2(h);
    return pack2<true>(x0 - f.x, x1 - f.y);
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
template <int KV_TYPE, int D, bool PRO, bool WIDE = false>
__global__ void __launch_bounds__(DecCfg<KV_TYPE, D, WIDE>::kThreads, DecCfg<KV_TYPE, D, WIDE>::kCtasPerSm)
    fa_decode_kernel(const __grid_constant__ DecodeParams P, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap) {
    using Cfg            = DecCfg<KV_TYPE, D, WIDE>;
    constexpr bool kQ8   = Cfg::kQ8;
    constexpr bool kBF16 = Cfg::kBF16;
    constexpr int  KS    = D / 16;      // k-steps over the head dim
    constexpr int  NT    = D / 8;       // n8 tiles over the head dim
    constexpr int  R     = Cfg::kRows;  // rows per unit

    extern __shared__ uint8_t smem_raw[];
    // 1 KB aligned base, derived from smem_raw by an offset so that the
    // compiler keeps the shared address space: every access through it is an
    // ld/st.shared (a pointer rebuilt from an integer would be generic).
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

    uint64_t     *full_bar  = reinterpret_cast<uint64_t *>(smem + Cfg::kOffBars);
    uint64_t     *empty_bar = full_bar + Cfg::kStages;
    int4         *meta      = reinterpret_cast<int4 *>(smem + Cfg::kOffMeta);
    volatile int *abort_f   = reinterpret_cast<volatile int *>(smem + Cfg::kOffFlags);
    float        *merge     = reinterpret_cast<float *>(smem + Cfg::kOffMerge);
    float        *s_m       = reinterpret_cast<float *>(smem + Cfg::kOffStats);
    float        *s_l       = s_m + kDecWarps * kDecRows;
    float        *s_fin     = reinterpret_cast<float *>(smem + Cfg::kOffFin);  // [0,16) max, [16,32) sum

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int C    = P.cluster;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(&full_bar[i], 1);
            mbar_init(&empty_bar[i], kDecWarps);
        }
        *abort_f = 0;
        fence_barrier_init();
    }
    if (C > 1) {
        cluster_sync_all();  // every CTA's barriers exist before any remote arrival
    } else {
        __syncthreads();
    }

    // The next kernel of the stream may start its own set-up now.  Each role
    // waits for the previous kernel (pdl_wait_primary) just before its first
    // read of a tensor that kernel may have written: the address arithmetic
    // before that reads kernel parameters only and overlaps the previous
    // kernel's tail.
    pdl_launch_dependents();

    const OpDesc   &o   = P.op;
    const int       u   = (int) (blockIdx.x / (unsigned) C);
    const int       r   = (int) (blockIdx.x % (unsigned) C);  // == %cluster_ctarank
    const int       tpu = P.tiles_per_unit;
    const int       tlo = (int) ((int64_t) tpu * r / C);
    const int       thi = (int) ((int64_t) tpu * (r + 1) / C);
    const UnitCoord uc  = unit_coord<R>(P, u);

    // Mask slots: the distinct mask rows this unit reads (one per query index
    // when the mask is shared by all heads).
    int n_ms = 0;
    if (o.mask) {
        n_ms = o.m_ne2 == 1 ? (uc.rb * R + uc.rows - 1) / o.G - (uc.rb * R) / o.G + 1 : uc.rows;
    }

    if (warp == kDecWarps) {
        // ============================ producer ============================
        if (!kQ8 && lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
        }
        int      stage = 0;
        uint32_t phase = 0;
        bool     ok    = true;
        int      pend[Cfg::kStages];  // parity of the last phase armed on each full barrier
        for (int i = 0; i < Cfg::kStages; ++i) {
            pend[i] = -1;
        }
        auto advance = [&]() {
            if (++stage == Cfg::kStages) {
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
        // Lane s owns mask slot s and stages its 64-key segment of every tile.
        const uint16_t *my_mr = nullptr;
        if (o.mask && lane < n_ms) {
            if (o.m_ne2 == 1) {
                my_mr = mask_row(o, (uc.rb * R) / o.G + lane, 0, uc.b);
            } else {
                int iq, hq;
                row_coord<R>(P, uc, lane, iq, hq);
                my_mr = mask_row(o, iq, hq, uc.b);
            }
        }
        const bool mask_bulk =
            __all_sync(0xffffffffu, lane >= n_ms || (reinterpret_cast<uintptr_t>(my_mr) & 15u) == 0);
        // Stage the mask segment [64*ti, 64*ti + 64) of every slot row.  Returns
        // the bytes the caller must add to the barrier's transaction count (the
        // bulk-copy case, issued by the caller after arming the barrier); rows
        // that are not 16-B aligned, or a segment running past the mask's row
        // length, are copied here with plain loads instead.
        auto stage_mask = [&](int ti, uint8_t *dst) -> uint32_t {
            if (n_ms == 0) {
                return 0;
            }
            const int j0 = ti * kDecBN;
            if (mask_bulk && j0 + kDecBN <= o.m_ne0) {
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
        const char *kbase = o.k + (int64_t) uc.hk * o.k_nb2 + (int64_t) uc.bk * o.k_nb3;
        const char *vbase = o.v + (int64_t) uc.hk * o.v_nb2 + (int64_t) uc.bk * o.v_nb3;
        pdl_wait_primary();  // K/V, the mask and the append rows below
        // Fused append: the row is written by the CTA whose range holds its
        // tile, just before that tile's copy is issued (after the earlier
        // tiles' copies, so its latency overlaps them), or after the range's
        // tiles when the mask makes that tile dead.
        int64_t app_row  = -1;
        int     app_tile = -1;
        float   app_k[4], app_v[4];
        if (P.append_pos) {
            app_row = P.append_pos[uc.bk];
            if (app_row < 0 || app_row >= o.n_kv) {
                if (lane == 0 && r == 0) {
                    atomicCAS(P.dev_err, 0, DEVERR_APPEND_POS);
                }
            } else if (app_row / kDecBN >= tlo && app_row / kDecBN < thi) {
                app_tile = (int) (app_row / kDecBN);
                append_load<KV_TYPE, D, PRO>(P, uc.hk, uc.bk, lane, app_k, app_v);
            }
        }
        // Copies tile ti into the next stage (K, V, and the mask segments).
        auto issue = [&](int ti) {
            ok = acquire();
            if (!ok) {
                return;
            }
            uint8_t *sK = smem + Cfg::kOffStages + stage * Cfg::kStageBytes;
            uint8_t *sV = sK + Cfg::kTile;
            uint8_t *sM = sK + 2 * Cfg::kTile;
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
                const uint32_t mbytes = stage_mask(ti, sM);
                fence_proxy_async_smem();
                __syncwarp();
                if (mbytes && lane < n_ms) {
                    bulk_load(sM + lane * kDecBN * 2, my_mr + ti * kDecBN, kDecBN * 2, &full_bar[stage]);
                }
                if (lane == 0) {
                    meta[stage] = make_int4(nrows, ti, kMetaData, (int) (lead_k | (lead_v << 8)));
                    mbar_arrive_expect_tx(&full_bar[stage], bulk_k + bulk_v + mbytes);
                    if (bulk_k) {
                        bulk_load(sK, kg - lead_k, bulk_k, &full_bar[stage]);
                    }
                    if (bulk_v) {
                        bulk_load(sV, vg - lead_v, bulk_v, &full_bar[stage]);
                    }
                }
            } else {
                const uint32_t mbytes = stage_mask(ti, sM);
                if (lane == 0) {
                    meta[stage] = make_int4(0, ti, kMetaData, 0);
                    mbar_arrive_expect_tx(&full_bar[stage], (uint32_t) (2 * Cfg::kTile) + mbytes);
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
                    bulk_load(sM + lane * kDecBN * 2, my_mr + ti * kDecBN, kDecBN * 2, &full_bar[stage]);
                }
            }
            pend[stage] = (int) phase;
            __syncwarp();
            advance();
        };
        // The first stages go out before the liveness scan of the mask (a
        // global-memory round trip) returns: a dead tile among them only adds
        // keys of zero weight.  Not with a fused append, whose row must be
        // written before its tile is read.
        int spec_end = tlo;
        if (!P.append_pos) {
            spec_end = min(thi, tlo + Cfg::kStages);
            for (int ti = tlo; ti < spec_end && ok; ++ti) {
                issue(ti);
            }
        }
        for (int tb = tlo; tb < thi && ok; tb += 32) {
            const int  tile = tb + lane;
            const bool live = tile >= spec_end && tile < thi && tile_live<R>(P, uc, tile);
            uint32_t   bits = __ballot_sync(0xffffffffu, live);
            while (bits && ok) {
                const int i = __ffs(bits) - 1;
                bits &= bits - 1;
                const int ti = tb + i;
                if (ti == app_tile) {
                    append_store<KV_TYPE, D>(P, app_row, lane, kbase, vbase, app_k, app_v);
                    app_tile = -1;
                }
                issue(ti);
            }
        }
        if (app_tile >= 0) {  // the row's tile is dead for this unit: no read to order
            append_store<KV_TYPE, D>(P, app_row, lane, kbase, vbase, app_k, app_v);
        }
        if (ok) {
            ok = acquire();
            if (ok && lane == 0) {
                meta[stage] = make_int4(0, 0, kMetaTerm, 0);
                mbar_arrive(&full_bar[stage]);
            }
        }
        if (!ok) {
            // Aborting: let the last copy armed on each stage land before the CTA
            // exits (a phase can never run more than one ahead of its last arm).
            for (int i = 0; i < Cfg::kStages; ++i) {
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

    pdl_wait_primary();  // consumers: Q (and, at the end, the output)
    if constexpr (kQ8) {
        // ======================= consumers, Q8_0 (transposed) ========================
        // S^T = K Q^T and O^T += V^T P^T on mma.sync m16n8k16: the warp's 16 keys
        // of a tile are the M dimension, the unit's 8 rows the N dimension.
        // Head dims are assigned so that every K or V byte a thread needs is one
        // contiguous run of a Q8_0 block: for S, thread (g, c) holds K dims
        // [c*D/4, (c+1)*D/4) of keys g and g+8 (k-step ks: dims c*D/4 + 4ks +
        // {0,1} and {2,3}, the same for Q^T); for PV it holds dims
        // [g*D/8, (g+1)*D/8) of keys 2c, 2c+1, 2c+8, 2c+9 (m-tile mt: dims
        // g*D/8 + mt and g*D/8 + D/16 + mt).  Every K and V value is
        // dequantised once, in registers, as f16(d * q).
        constexpr int KSQ = D / 16;  // k-steps of S^T = quant words of K per key and thread
        constexpr int MT  = D / 16;  // m-tiles of O^T
        constexpr int VW  = D / 32;  // quant words of V per key and thread (D/8 bytes)
        constexpr int RB  = Cfg::kRowBytes;
        const int     g   = lane >> 2;
        const int     c   = lane & 3;
        float         m_run[2] = {-INFINITY, -INFINITY};  // rows 2c, 2c+1 (log2 units)
        float         l_run[2] = {0.0f, 0.0f};             // this thread's keys only until the flush
        float         oacc[MT][4];
        uint32_t      qb[KSQ][2];  // Q^T fragments of row g
        int           mslot[2], vlo[2] = {0, 0}, vhi[2] = {0, 0};
        float         slope[2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                oacc[mt][e] = 0.0f;
            }
        }
        {
            int iq, hq;
            row_coord<R>(P, uc, g < uc.rows ? g : 0, iq, hq);
            const float *qrow = g < uc.rows ? reinterpret_cast<const float *>(o.q + (int64_t) iq * o.q_nb1 +
                                                                              (int64_t) hq * o.q_nb2 +
                                                                              (int64_t) uc.b * o.q_nb3)
                                            : nullptr;
            const int d0 = c * (D / 4);
            float     x[KSQ][4];
#pragma unroll
            for (int ks = 0; ks < KSQ; ++ks) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    x[ks][e] = qrow ? __ldg(qrow + d0 + 4 * ks + e) : 0.0f;
                }
            }
            if (PRO && o.qp.on) {
                // QK-norm + RoPE: row g's D values are spread over its quad (c = 0..3)
                if (o.qp.w) {
                    float ss = 0.0f;
#pragma unroll
                    for (int ks = 0; ks < KSQ; ++ks) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            ss = fmaf(x[ks][e], x[ks][e], ss);
                        }
                    }
                    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                    const float sc = rn_scale(o.qp, ss, D);
#pragma unroll
                    for (int ks = 0; ks < KSQ; ++ks) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            x[ks][e] = (x[ks][e] * sc) * __ldg(o.qp.w + d0 + 4 * ks + e);
                        }
                    }
                }
                if (o.qp.rope) {
                    // dim d + D/2 sits on thread c ^ 2 at the same (ks, e)
                    const int qpos = g < uc.rows ? __ldg(o.qp.pos + iq + (int64_t) uc.b * o.n_q) : 0;
#pragma unroll
                    for (int ks = 0; ks < KSQ; ++ks) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float pt = __shfl_xor_sync(0xffffffffu, x[ks][e], 2);
                            x[ks][e] = rn_rotate(o.qp, x[ks][e], pt, c < 2, qpos, (d0 + 4 * ks + e) & (D / 2 - 1));
                        }
                    }
                }
            }
#pragma unroll
            for (int ks = 0; ks < KSQ; ++ks) {
                qb[ks][0] = pack2<false>(x[ks][0], x[ks][1]);
                qb[ks][1] = pack2<false>(x[ks][2], x[ks][3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int rr = 2 * c + i;
            int       iq, hq;
            row_coord<R>(P, uc, rr < uc.rows ? rr : 0, iq, hq);
            mslot[i] = o.m_ne2 == 1 ? iq - (uc.rb * R) / o.G : (rr < uc.rows ? rr : 0);
            slope[i] = alibi_slope(o, hq);
            if (o.mg_kind) {
                mg_range(o, uc.b, iq, vlo[i], vhi[i]);
            }
        }
        const int      kd0      = c * (D / 4);  // this thread's K dims (scores)
        const int      vd0      = g * (D / 8);  // this thread's V dims (PV)
        const uint32_t sel_half = (g & 1) ? 0x7632u : 0x5410u;
        const int      src1     = 8 * c + (g >> 1);  // lanes holding P[row g][keys 2c, 2c+8] and [2c+1, 2c+9]
        const int      src2     = src1 + 4;

        int      stage = 0;
        uint32_t phase = 0;
        while (true) {
            const bool got =
                mbar_wait_bounded(&full_bar[stage], phase, abort_f, P.dev_err, DEVERR_TIMEOUT_FULL, P.wait_limit_ns);
            if (!__all_sync(0xffffffffu, got)) {  // the shuffles and MMAs below need the whole warp
                break;
            }
            const int4 md = meta[stage];
            if (md.z != kMetaData) {
                break;
            }
            const uint8_t  *stg  = smem + Cfg::kOffStages + stage * Cfg::kStageBytes;
            const uint32_t  sK   = smem_u32(stg) + (uint32_t) (md.w & 0xff);
            const uint32_t  sV   = smem_u32(stg + Cfg::kTile) + (uint32_t) ((md.w >> 8) & 0xff);
            const uint16_t *sM   = reinterpret_cast<const uint16_t *>(stg + 2 * Cfg::kTile);
            const int       tile = md.y;
            const int       key0 = 16 * warp + g;  // keys key0 and key0 + 8 of the tile
            // ---- S^T = K Q^T
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            {
                uint32_t       k0[KSQ], k1[KSQ];
                const uint16_t e0 = q8_load_run<KSQ>(sK + key0 * RB + 34 * (kd0 / 32), kd0 % 32, k0);
                const uint16_t e1 = q8_load_run<KSQ>(sK + (key0 + 8) * RB + 34 * (kd0 / 32), kd0 % 32, k1);
                const __half2  d0 = __half2half2(__ushort_as_half(e0));
                const __half2  d1 = __half2half2(__ushort_as_half(e1));
#pragma unroll
                for (int ks = 0; ks < KSQ; ++ks) {
                    const uint32_t a[4] = {i8x2_scaled(k0[ks], 0x4140u, d0), i8x2_scaled(k1[ks], 0x4140u, d1),
                                           i8x2_scaled(k0[ks], 0x4342u, d0), i8x2_scaled(k1[ks], 0x4342u, d1)};
                    mma_16816<false>((ks & 1) ? s2 : s, a, qb[ks][0], qb[ks][1]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s[e] += s2[e];
                }
            }
            // ---- scale, softcap, mask, bounds; online softmax over keys (rows 2c, 2c+1)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i   = e & 1;
                const int kk  = key0 + 8 * (e >> 1);
                const int pos = tile * kDecBN + kk;
                float     x   = s[e] * o.scale_eff;
                if (o.softcap != 0.0f) {
                    x = o.softcap * tanhf(x);
                }
                if (pos < o.n_kv) {
                    if (o.mask) {
                        // a -inf entry removes the key outright, whatever K held there
                        const float mv = slope[i] * __half2float(__ushort_as_half(sM[mslot[i] * kDecBN + kk]));
                        x              = mv == -INFINITY ? -INFINITY : x + mv;
                    } else if (o.mg_kind) {
                        // a visible key adds the rule's 0 like a 0 mask entry
                        x = pos >= vlo[i] && pos < vhi[i] ? x + 0.0f : -INFINITY;
                    }
                    x *= kLog2e;
                } else {
                    x = -INFINITY;
                }
                s[e] = x;
            }
            // A row's keys are spread over the 8 lanes of its column c, so its
            // maximum takes three shuffles.  They run only when some score
            // exceeds the running max by more than 2^8 (one vote); otherwise
            // P = 2^(s - m) <= 2^8 against the running max, exact enough in f16
            // (the dense kernel's rule).
            const bool grow = s[0] > m_run[0] + kQ8RescaleLog2 || s[2] > m_run[0] + kQ8RescaleLog2 ||
                              s[1] > m_run[1] + kQ8RescaleLog2 || s[3] > m_run[1] + kQ8RescaleLog2;
            if (__any_sync(0xffffffffu, grow)) {
                float alpha[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    float mx = fmaxf(s[i], s[2 + i]);
                    mx       = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx       = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx       = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float mnew = fmaxf(m_run[i], mx);
                    alpha[i]         = mnew == -INFINITY ? 1.0f : fast_exp2(m_run[i] - mnew);
                    m_run[i]         = mnew;
                    l_run[i] *= alpha[i];
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    oacc[mt][0] *= alpha[0];
                    oacc[mt][1] *= alpha[1];
                    oacc[mt][2] *= alpha[0];
                    oacc[mt][3] *= alpha[1];
                }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float muse = m_run[i] == -INFINITY ? 0.0f : m_run[i];
                s[i]             = fast_exp2(s[i] - muse);
                s[2 + i]         = fast_exp2(s[2 + i] - muse);
                l_run[i] += s[i] + s[2 + i];
            }
            // ---- P^T fragments: P[row g][keys 2c, 2c+1] and [2c+8, 2c+9], from
            // the lanes whose S^T rows are those keys
            const uint32_t hlo = pack2<false>(s[0], s[1]);  // key key0: rows 2c, 2c+1
            const uint32_t hhi = pack2<false>(s[2], s[3]);  // key key0 + 8
            const uint32_t x1  = __shfl_sync(0xffffffffu, hlo, src1);
            const uint32_t x2  = __shfl_sync(0xffffffffu, hlo, src2);
            const uint32_t y1  = __shfl_sync(0xffffffffu, hhi, src1);
            const uint32_t y2  = __shfl_sync(0xffffffffu, hhi, src2);
            const uint32_t pb0 = __byte_perm(x1, x2, sel_half);
            const uint32_t pb1 = __byte_perm(y1, y2, sel_half);
            // ---- O^T += V^T P^T
            {
                uint32_t vw[4][VW];
                uint16_t dvb[4];
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int key = 16 * warp + 2 * c + (jj & 1) + 8 * (jj >> 1);
                    dvb[jj]       = q8_load_run<VW>(sV + key * RB + 34 * (vd0 / 32), vd0 % 32, vw[jj]);
                    // rows past n_kv in the last tile hold stale bytes: a zero scale
                    // keeps them finite (their P is 0, but 0 * inf would be NaN)
                    dvb[jj] = tile * kDecBN + key < o.n_kv ? dvb[jj] : (uint16_t) 0;
                }
                const __half2 dA = __halves2half2(__ushort_as_half(dvb[0]), __ushort_as_half(dvb[1]));
                const __half2 dB = __halves2half2(__ushort_as_half(dvb[2]), __ushort_as_half(dvb[3]));
                // the two keys of each pair interleaved byte by byte: word k holds
                // run bytes 2k, 2k+1 of both keys ([A B A B])
                uint32_t ia[2 * VW], ib[2 * VW];
#pragma unroll
                for (int q = 0; q < VW; ++q) {
                    ia[2 * q]     = __byte_perm(vw[0][q], vw[1][q], 0x5140u);
                    ia[2 * q + 1] = __byte_perm(vw[0][q], vw[1][q], 0x7362u);
                    ib[2 * q]     = __byte_perm(vw[2][q], vw[3][q], 0x5140u);
                    ib[2 * q + 1] = __byte_perm(vw[2][q], vw[3][q], 0x7362u);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    constexpr int  kHalfRun = D / 16;
                    const int      b0 = mt, b1 = kHalfRun + mt;  // run bytes of dims vd0 + mt, vd0 + D/16 + mt
                    const uint32_t s0 = (b0 & 1) ? 0x4342u : 0x4140u;
                    const uint32_t s1 = (b1 & 1) ? 0x4342u : 0x4140u;
                    const uint32_t a[4] = {i8x2_scaled(ia[b0 >> 1], s0, dA), i8x2_scaled(ia[b1 >> 1], s1, dA),
                                           i8x2_scaled(ib[b0 >> 1], s0, dB), i8x2_scaled(ib[b1 >> 1], s1, dB)};
                    mma_16816<false>(oacc[mt], a, pb0, pb1);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty_bar[stage]);
            }
            if (++stage == Cfg::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }

        // ---- merge of the four warps' partial results
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 4);
            l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 8);
            l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 16);
        }
        if (g == 0) {
            s_m[warp * kDecRows + 2 * c]     = m_run[0];
            s_m[warp * kDecRows + 2 * c + 1] = m_run[1];
            s_l[warp * kDecRows + 2 * c]     = l_run[0];
            s_l[warp * kDecRows + 2 * c + 1] = l_run[1];
        }
        named_bar_sync(1, kDecWarps * 32);
        float fac[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            float mx = -INFINITY;
#pragma unroll
            for (int w = 0; w < kDecWarps; ++w) {
                mx = fmaxf(mx, s_m[w * kDecRows + 2 * c + i]);
            }
            fac[i] = m_run[i] == -INFINITY ? 0.0f : fast_exp2(m_run[i] - mx);
        }
        // four turns; in turn t warp w adds its m-tiles of block (w + t) % 4, so
        // each element has one writer per turn (plain stores, no atomics)
        constexpr int MTB = MT / 4;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int bsel = (warp + t) & 3;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                if (bb == bsel) {
#pragma unroll
                    for (int jj = 0; jj < MTB; ++jj) {
                        const int mt = bb * MTB + jj;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int   row = 2 * c + (e & 1);
                            const int   dim = vd0 + (e >> 1) * (D / 16) + mt;
                            float      *mp  = &merge[Cfg::merge_at(row, dim)];
                            const float v   = oacc[mt][e] * fac[e & 1];
                            *mp             = t == 0 ? v : *mp + v;
                        }
                    }
                }
            }
            if (t == 0 && threadIdx.x < R) {
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
    } else {
        // ======================= consumers, F16 / BF16 ========================
        const int g = lane >> 2;  // fragment row group
        const int c = lane & 3;   // fragment column pair

        float    m_run[2], l_run[2];
        float    oacc[NT][4];
        uint32_t qa[KS][4];
        // BF16 operands keep ~16 mantissa bits of Q and P by a hi + lo split
        // (two MMAs each); the F16 and Q8_0 paths never touch qlo.
        uint32_t qlo[kBF16 ? KS : 1][4];
        int      mslot[2];        // mask slot (staged row) of fragment rows g and g+8
        int      vlo[2], vhi[2];  // mask rule: visible keys [vlo, vhi) of rows g and g+8
        float    slope[2];

        // ---- Q fragments of rows g and g+8 (QK-norm + RoPE applied in the PRO instance)
        {
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
                row_coord<R>(P, uc, rr < uc.rows ? rr : 0, iq, hq);
                qrow[i]  = rr < uc.rows ? reinterpret_cast<const float *>(o.q + (int64_t) iq * o.q_nb1 +
                                                                         (int64_t) hq * o.q_nb2 + (int64_t) uc.b * o.q_nb3)
                                        : nullptr;
                mslot[i] = o.m_ne2 == 1 ? iq - (uc.rb * R) / o.G : (rr < uc.rows ? rr : 0);
                slope[i] = alibi_slope(o, hq);
                if (o.mg_kind) {
                    mg_range(o, uc.b, iq, vlo[i], vhi[i]);
                }
                if (PRO && o.qp.rope && rr < uc.rows) {
                    qpos[i] = __ldg(o.qp.pos + iq + (int64_t) uc.b * o.n_q);
                }
            }
            // This thread's Q values, x[i][ks][e] of row g + 8i: dims
            // 16ks + 2c + (e & 1) + 8(e >> 1) (the m16n8k16 A fragment).
            auto qdim = [&](int ks, int e) -> int { return 16 * ks + 2 * c + (e & 1) + 8 * (e >> 1); };
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
            if (PRO && o.qp.on) {
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
    #pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
    #pragma unroll
                for (int rg = 0; rg < 4; ++rg) {
                    // fragment register rg: row rg & 1, value pair (rg >> 1)
                    const float x0 = x[rg & 1][ks][2 * (rg >> 1)], x1 = x[rg & 1][ks][2 * (rg >> 1) + 1];
                    qa[ks][rg]     = pack2<kBF16>(x0, x1);
                    if constexpr (kBF16) {
                        qlo[ks][rg] = split_lo_bf16(x0, x1, qa[ks][rg]);
                    }
                }
            }
        }

        // ---- S = Q K^T over this warp's 16 keys of a swizzled 16-bit tile
        auto tile_scores = [&](const uint8_t *sK, float (&s)[2][4]) {
            const int mi   = lane >> 3;
            const int r8   = lane & 7;
            const int krow = 16 * warp + (mi >> 1) * 8 + r8;
            float     s2[2][4];  // second accumulator chain (odd k-steps) for more MMA overlap
    #pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s[nt][e]  = 0.0f;
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
        };

        // ---- scale, softcap, mask, bounds; online softmax; P as A fragments
        auto tile_softmax = [&](float (&s)[2][4], const uint16_t *sM, int tile, uint32_t (&pa)[4], uint32_t (&palo)[4]) {
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
            pa[0] = pack2<kBF16>(s[0][0], s[0][1]);
            pa[1] = pack2<kBF16>(s[0][2], s[0][3]);
            pa[2] = pack2<kBF16>(s[1][0], s[1][1]);
            pa[3] = pack2<kBF16>(s[1][2], s[1][3]);
            if constexpr (kBF16) {
                palo[0] = split_lo_bf16(s[0][0], s[0][1], pa[0]);
                palo[1] = split_lo_bf16(s[0][2], s[0][3], pa[1]);
                palo[2] = split_lo_bf16(s[1][0], s[1][1], pa[2]);
                palo[3] = split_lo_bf16(s[1][2], s[1][3], pa[3]);
            }
        };

        // ---- O += P V over this warp's 16 keys
        auto tile_pv = [&](const uint8_t *sV, const uint32_t (&pa)[4], const uint32_t (&palo)[4]) {
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
        };

        int      stage = 0;
        uint32_t phase = 0;
        while (true) {
            const bool got =
                mbar_wait_bounded(&full_bar[stage], phase, abort_f, P.dev_err, DEVERR_TIMEOUT_FULL, P.wait_limit_ns);
            // ldmatrix / mma.sync / shuffles below are warp-collective: leave together
            if (!__all_sync(0xffffffffu, got)) {
                break;
            }
            const int4 md = meta[stage];
            if (md.z != kMetaData) {
                break;
            }
            const uint8_t *sK = smem + Cfg::kOffStages + stage * Cfg::kStageBytes;
            float          s[2][4];
            uint32_t       pa[4], palo[4];
            tile_scores(sK, s);
            tile_softmax(s, reinterpret_cast<const uint16_t *>(sK + 2 * Cfg::kTile), md.y, pa, palo);
            tile_pv(sK + Cfg::kTile, pa, palo);
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty_bar[stage]);
            }
            if (++stage == Cfg::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }

        // ---- merge of the four warps' partial results (rows of this CTA's range)
        // Head-dim index held by accumulator element (j, e) (column part only).
        auto out_dim = [&](int j, int e) -> int { return 8 * j + 2 * c + (e & 1); };
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
                            float      *mp = &merge[Cfg::merge_at(g + 8 * (e >> 1), out_dim(j, e))];
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
    }

    // ---- merge across the cluster and write the output
    // CTA r finishes its share of the head dims (the r-th of C nearly equal
    // ranges of float4 chunks) of every row from all C partials, read from the
    // peers' shared memory; C == 1 writes them all.  Two phases of the
    // hardware cluster barrier order it: every partial is published before any
    // CTA reads, and every read is done before any CTA exits (this CTA arrives
    // once its reads have returned, then stores, then waits).  Every CTA
    // reaches both phases: each wait of the pipeline before them is bounded,
    // and the producer warps have exited.
    if (C > 1) {
        cluster_arrive();
        cluster_wait();
    }
    // this CTA's float4 chunks of every row: [ch0, ch1) of the row's D / 4
    const int      ch0    = r * (D / 4) / C;
    const int      chunks = (r + 1) * (D / 4) / C - ch0;
    const uint32_t fin_a  = smem_u32(s_fin);
    const uint32_t mrg_a  = smem_u32(merge);
    constexpr int  kItems = (kDecRows * (D / 4) + kDecWarps * 32 - 1) / (kDecWarps * 32);  // per thread at C == 1
    static_assert((kDecRows * ((D / 4 + 1) / 2) + kDecWarps * 32 - 1) / (kDecWarps * 32) <= kItems, "item count");
    constexpr int  kMaxC  = ACEFA_DEC_MAX_CLUSTER < kDecMaxCluster ? ACEFA_DEC_MAX_CLUSTER : kDecMaxCluster;
    float4         res[kItems];
    char          *res_dp[kItems];
    // Row r's result from the C parts' statistics (m, l) and values v.
    auto finish = [&](int it, int row, int d, const float (&mk0)[kMaxC], const float (&lk)[kMaxC],
                      const float4 (&vk)[kMaxC]) {
        float mk[kMaxC];
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < kMaxC; ++k) {
            mx = fmaxf(mx, mk0[k]);
        }
        float l = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxC; ++k) {
            mk[k] = mk0[k] == -INFINITY ? 0.0f : fast_exp2(mk0[k] - mx);  // the part's weight
            l += lk[k] * mk[k];
        }
        int iq, hq;
        row_coord<R>(P, uc, row, iq, hq);
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
        float4      acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kMaxC; ++k) {
            if (k < C) {
                acc.x += mk[k] * vk[k].x;
                acc.y += mk[k] * vk[k].y;
                acc.z += mk[k] * vk[k].z;
                acc.w += mk[k] * vk[k].w;
            }
        }
        res[it]    = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        res_dp[it] = o.dst + (int64_t) d * o.d_nb0 + (int64_t) hq * o.d_nb1 + (int64_t) iq * o.d_nb2 +
                     (int64_t) uc.b * o.d_nb3;
    };
#pragma unroll
    for (int it = 0; it < kItems; ++it) {
        res_dp[it] = nullptr;
    }
    if (C == 1) {
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            const int idx = (int) threadIdx.x + it * kDecWarps * 32;
            const int row = idx / chunks;
            const int d   = (ch0 + idx % chunks) * 4;
            if (idx >= kDecRows * chunks || row >= uc.rows) {
                continue;
            }
            float  mk[kMaxC], lk[kMaxC];
            float4 vk[kMaxC];
#pragma unroll
            for (int k = 0; k < kMaxC; ++k) {
                mk[k] = k == 0 ? s_fin[row] : -INFINITY;
                lk[k] = k == 0 ? s_fin[kDecRows + row] : 0.0f;
                vk[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if constexpr (kQ8) {  // four dims of one skewed group: contiguous, 4-B aligned
                const float *mp = &merge[Cfg::merge_at(row, d)];
                vk[0]           = make_float4(mp[0], mp[1], mp[2], mp[3]);
            } else {
                vk[0] = *reinterpret_cast<const float4 *>(&merge[Cfg::merge_at(row, d)]);
            }
            finish(it, row, d, mk, lk, vk);
        }
    } else {
        // The parts' values for this thread's items are requested first, then
        // each part's row statistics once per (part, row) into a table in the
        // (now idle) first pipeline stage, so both kinds of distributed
        // shared-memory loads are in flight together and no statistic is
        // fetched more than once.
        constexpr int kItemsC = (kDecRows * ((D / 4 + 1) / 2) + kDecWarps * 32 - 1) / (kDecWarps * 32);
        float4        vk[kItemsC][kMaxC];
#pragma unroll
        for (int it = 0; it < kItemsC; ++it) {
            const int idx = (int) threadIdx.x + it * kDecWarps * 32;
            const int row = idx / chunks;
            const int d   = (ch0 + idx % chunks) * 4;
            const bool live = idx < kDecRows * chunks && row < uc.rows;
#pragma unroll
            for (int k = 0; k < kMaxC; ++k) {
                vk[it][k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (live && k < C) {
                    const uint32_t a = mapa_shared(mrg_a + 4 * Cfg::merge_at(row, d), (uint32_t) k);
                    if constexpr (kQ8) {
                        vk[it][k] = make_float4(ld_cluster_f32(a), ld_cluster_f32(a + 4), ld_cluster_f32(a + 8),
                                                ld_cluster_f32(a + 12));
                    } else {
                        vk[it][k] = ld_cluster_f32x4(a);
                    }
                }
            }
        }
        float2 *stab = reinterpret_cast<float2 *>(smem + Cfg::kOffStages);  // [C][kDecRows] (m, l)
        for (int t = threadIdx.x; t < C * kDecRows; t += kDecWarps * 32) {
            const int k = t / kDecRows, row = t % kDecRows;
            stab[t]     = make_float2(ld_cluster_f32(mapa_shared(fin_a + 4 * row, (uint32_t) k)),
                                      ld_cluster_f32(mapa_shared(fin_a + 4 * (kDecRows + row), (uint32_t) k)));
        }
        named_bar_sync(1, kDecWarps * 32);
#pragma unroll
        for (int it = 0; it < kItemsC; ++it) {
            const int idx = (int) threadIdx.x + it * kDecWarps * 32;
            const int row = idx / chunks;
            const int d   = (ch0 + idx % chunks) * 4;
            if (idx >= kDecRows * chunks || row >= uc.rows) {
                continue;
            }
            float mk[kMaxC], lk[kMaxC];
#pragma unroll
            for (int k = 0; k < kMaxC; ++k) {
                const float2 st = k < C ? stab[k * kDecRows + row] : make_float2(-INFINITY, 0.0f);
                mk[k]           = st.x;
                lk[k]           = st.y;
            }
            finish(it, row, d, mk, lk, vk[it]);
        }
    }
    if (C > 1) {
        // this CTA's reads of the peers' partials have returned (their values
        // are in res): the arrive needs no memory ordering
        cluster_arrive_relaxed();
    }
#pragma unroll
    for (int it = 0; it < kItems; ++it) {
        char *dp = res_dp[it];
        if (!dp) {
            continue;
        }
        const float4 acc = res[it];
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
                char *dk                       = dp + (int64_t) k * o.d_nb0;
                *reinterpret_cast<float *>(dk) = a4[k];
                for (int mi = 0; mi < o.n_mirror; ++mi) {
                    *reinterpret_cast<float *>(dk + o.mirror_delta[mi]) = a4[k];
                }
            }
        }
    }
    if (o.n_mirror) {
        __threadfence_system();
    }
    if (C > 1) {
        cluster_wait();  // this CTA's partial stays readable until every peer is done
    }
}

// ---------------------------------------------------------------------------
// host side

namespace {

// Per-device, per-instance launch set-up (shared-memory size, the
// non-portable cluster size) and the cluster sizes the device schedules for it.
struct InstInfo {
    bool ok = false;
    // clusters of c CTAs the device keeps resident at once (0 = not launchable)
    int active[kDecMaxCluster + 1] = {};
    int sms = 0;  // the device's SM count
};
constexpr int kMaxDev = 64;
std::mutex    g_inst_mutex;

template <int KV_TYPE, int D, bool PRO, bool WIDE>
const InstInfo &inst_info(int dev) {
    static InstInfo info[kMaxDev];
    static bool     done[kMaxDev];
    using Cfg = DecCfg<KV_TYPE, D, WIDE>;
    std::lock_guard<std::mutex> lock(g_inst_mutex);
    InstInfo &in = info[dev];
    if (done[dev]) {
        return in;
    }
    done[dev] = true;
    auto k    = fa_decode_kernel<KV_TYPE, D, PRO, WIDE>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess) {
        return in;
    }
    in.ok = true;
    cudaDeviceGetAttribute(&in.sms, cudaDevAttrMultiProcessorCount, dev);
    const bool big =
        ACEFA_DEC_MAX_CLUSTER > 8 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                                         cudaSuccess;
    for (int c = 1; c <= ACEFA_DEC_MAX_CLUSTER && c <= kDecMaxCluster; ++c) {
        if (c > 8 && !big) {
            break;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim            = dim3((unsigned) c);
        cfg.blockDim           = dim3(Cfg::kThreads);
        cfg.dynamicSmemBytes   = Cfg::kSmemBytes;
        cudaLaunchAttribute at[1];
        at[0].id               = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned) c;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs              = at;
        cfg.numAttrs           = 1;
        int n                  = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess) {
            in.active[c] = n;
        }
    }
    cudaGetLastError();  // a refused query leaves no sticky error
    return in;
}

// The instance with the prologue exists for D <= 128 (the host refuses
// prologues and appends at D = 256).
template <int KV_TYPE, int D>
constexpr bool kHasPro = D <= 128;

template <int KV_TYPE, int D, bool WIDE>
const InstInfo &pro_info(bool pro, int dev) {
    if constexpr (kHasPro<KV_TYPE, D>) {
        if (pro) {
            return inst_info<KV_TYPE, D, true, WIDE>(dev);
        }
    }
    return inst_info<KV_TYPE, D, false, WIDE>(dev);
}

template <int KV_TYPE, int D, bool WIDE = false>
cudaError_t launch_impl(const DecodeLaunch &L, cudaStream_t s, int *launches) {
    using Cfg      = DecCfg<KV_TYPE, D, WIDE>;
    const bool pro = L.p.op.qp.on || L.p.kp.on;
    if (pro && !kHasPro<KV_TYPE, D>) {
        return cudaErrorInvalidValue;
    }
    auto kern = fa_decode_kernel<KV_TYPE, D, false, WIDE>;
    if constexpr (kHasPro<KV_TYPE, D>) {
        if (pro) {
            kern = fa_decode_kernel<KV_TYPE, D, true, WIDE>;
        }
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        return cudaErrorInvalidDevice;
    }
    const InstInfo &in = pro_info<KV_TYPE, D, WIDE>(pro, dev);
    if (!in.ok) {
        return cudaErrorInvalidConfiguration;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) (L.p.units * L.p.cluster));
    cfg.blockDim           = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes   = Cfg::kSmemBytes;
    cfg.stream             = s;
    cudaLaunchAttribute attr[2];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id                                         = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x                           = (unsigned) L.p.cluster;
    attr[1].val.clusterDim.y                           = 1;
    attr[1].val.clusterDim.z                           = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = L.p.cluster > 1 ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, L.p, L.kmap, L.vmap);
    if (e != cudaSuccess) {
        return e;
    }
    if (launches) {
        *launches = 1;
    }
    return cudaSuccess;
}

// The largest cluster size whose clusters for all `units` are resident at
// once (so the op runs in one wave), or 1.
template <int KV_TYPE, int D, bool WIDE = false>
int cluster_for(bool pro, int units, int tiles_per_unit) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        return 1;
    }
    const InstInfo &in   = pro_info<KV_TYPE, D, WIDE>(pro, dev);
    int             best = 1;
    for (int c = 2; c <= kDecMaxCluster && in.ok; ++c) {
        // Clusters of more than kDecShareCluster CTAs only while every CTA
        // still has an SM to itself: shared SMs slow the short per-CTA key
        // ranges more than the wider merge saves (32 units: 6 CTAs per unit
        // 20-29 % faster than 8).
        const bool own_sm = in.sms <= 0 || (int64_t) units * c <= in.sms;
        if (c <= tiles_per_unit && units <= in.active[c] && (c <= kDecShareCluster || own_sm)) {
            best = c;
        }
    }
    return best;
}

}  // namespace

cudaError_t launch_decode(const DecodeLaunch &L, cudaStream_t s, int *launches) {
    const int t = L.p.op.kv_type, D = L.p.op.D;
    if (t == ACEFA_TYPE_F16 && D == 128) return launch_impl<ACEFA_TYPE_F16, 128>(L, s, launches);
    if (t == ACEFA_TYPE_F16 && D == 64) return launch_impl<ACEFA_TYPE_F16, 64>(L, s, launches);
    if (t == ACEFA_TYPE_BF16 && D == 128) return launch_impl<ACEFA_TYPE_BF16, 128>(L, s, launches);
    if (t == ACEFA_TYPE_BF16 && D == 64) return launch_impl<ACEFA_TYPE_BF16, 64>(L, s, launches);
    if (t == ACEFA_TYPE_Q8_0 && D == 128 && L.p.wide) return launch_impl<ACEFA_TYPE_Q8_0, 128, true>(L, s, launches);
    if (t == ACEFA_TYPE_Q8_0 && D == 128) return launch_impl<ACEFA_TYPE_Q8_0, 128>(L, s, launches);
    if (t == ACEFA_TYPE_Q8_0 && D == 64) return launch_impl<ACEFA_TYPE_Q8_0, 64>(L, s, launches);
    if (t == ACEFA_TYPE_F16 && D == 256) return launch_impl<ACEFA_TYPE_F16, 256>(L, s, launches);
    if (t == ACEFA_TYPE_BF16 && D == 256) return launch_impl<ACEFA_TYPE_BF16, 256>(L, s, launches);
    return cudaErrorInvalidValue;
}

int decode_cluster(int kv_type, int D, bool pro, int units, int tiles_per_unit, bool wide) {
    const int u = units, t = tiles_per_unit;
    if (wide && kv_type == ACEFA_TYPE_Q8_0 && D == 128) {
        return cluster_for<ACEFA_TYPE_Q8_0, 128, true>(pro, u, t);
    }
    if (kv_type == ACEFA_TYPE_F16) {
        return D == 128 ? cluster_for<ACEFA_TYPE_F16, 128>(pro, u, t)
                        : (D == 64 ? cluster_for<ACEFA_TYPE_F16, 64>(pro, u, t) : cluster_for<ACEFA_TYPE_F16, 256>(pro, u, t));
    }
    if (kv_type == ACEFA_TYPE_BF16) {
        return D == 128 ? cluster_for<ACEFA_TYPE_BF16, 128>(pro, u, t)
                        : (D == 64 ? cluster_for<ACEFA_TYPE_BF16, 64>(pro, u, t)
                                   : cluster_for<ACEFA_TYPE_BF16, 256>(pro, u, t));
    }
    return D == 128 ? cluster_for<ACEFA_TYPE_Q8_0, 128>(pro, u, t) : cluster_for<ACEFA_TYPE_Q8_0, 64>(pro, u, t);
}

}  // namespace acefa
