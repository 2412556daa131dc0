// fa_dense.cu -- tcgen05/TMEM flash attention for query-heavy ggml_flash_attn_ext
// nodes: LM causal prefill (src/qwen3-lm.h:465-469, n_tokens > 1), the Qwen3
// encoders (src/qwen3-enc.h:195-199) and DiT self/cross attention
// (src/dit-graph.h:227-231, :348-352).
//
// One CTA owns two 128-row tiles of a (batch, kv head) unit -- the rows are
// the unit's (query, q head) pairs, so GQA heads that share K/V share the
// stream -- and walks the unit's 128-key tiles:
//   warp 0      TMA producer: K_j and V_j into a 4 x 32 KB shared ring (128-B
//               swizzle, two 64-dim boxes per tile), skipping key tiles that
//               no row of either tile can see.
//   warp 1      owns 512 TMEM columns (O0 | O1 | S0 | S1) and issues the MMAs
//               from one thread: S_i = Q_i K_j^T (SS form, K-major operands)
//               and O_i += P_i V_j (TS form: P read from TMEM, V MN-major).
//   warps 4-7   softmax for row tile 0, warps 8-11 for row tile 1: one thread
//               per row reads S with tcgen05.ld, applies scale / softcap /
//               mask / ALiBi in log2 units, keeps a running max that only
//               moves (and rescales O in TMEM) when it grows by more than 2^8,
//               and writes P as f16 over the S columns it just read.
// Q arrives as f32 rows by TMA into the K/V ring (idle until then) and every
// thread converts it to swizzled f16 once per CTA; the output leaves by TMA
// stores of 32-dim chunks staged in the idle Q buffers (per-thread loads and
// per-lane stores where a tensor map cannot describe the tensor).
// The two row tiles ping-pong: while one warpgroup exponentiates, the tensor
// core runs the other tile's PV and next S.  When the work units leave the
// last wave mostly idle, the leftover units are cut into key ranges whose
// partial results fa_dense_combine merges.  A pre-pass classifies each
// (row tile, key tile) of the mask as dead / all-zero / mixed so that causal
// and window masks never load or multiply their dead tiles.
// Every wait is bounded (error word + drain on expiry).
#include "fa_internal.h"
#include "ptx.cuh"
#include "q8.cuh"
#include "rope_norm.cuh"

namespace acefa {
namespace {

constexpr int      kThreads    = 384;  // warp 0 TMA, warp 1 MMA, 2-3 spare, 4-7 / 8-11 softmax
constexpr int      kRing       = 4;
constexpr int      kTileBytes  = kDenseBN * 128 * 2;  // 32 KB: 128 keys x 128 dims f16
constexpr int      kQBytes     = kDenseBM * 128 * 2;  // 32 KB
constexpr int      kOffQ       = 0;
constexpr int      kOffRing    = kOffQ + 2 * kQBytes;
constexpr int      kOffBars    = kOffRing + kRing * kTileBytes;
constexpr int      kNumBars    = 2 * kRing + 2 * 3 + 2;  // ... + fin + the Q staging barrier
constexpr int      kOffCls     = kOffBars + kNumBars * 8;
constexpr int      kOffMisc    = kOffCls + 2 * kDenseMaxKT;
constexpr int      kSmemBytes  = kOffMisc + 16 + 1024;
constexpr uint32_t kTmemCols   = 512;
constexpr float    kRescaleLog2 = 8.0f;  // O is rescaled only when the max grows by > 2^8
// Register split between the warpgroups (setmaxnreg): warps 0-3 (TMA, MMA)
// give registers to the two softmax warpgroups.  The sum must stay within
// what the block was launched with (384 threads x 168 registers = 64512), or
// setmaxnreg.inc would wait forever: 128 x 112 + 256 x 192 = 63488.
constexpr uint32_t kRegsControl = 112;
constexpr uint32_t kRegsSoftmax = 192;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= 384 * 168, "register split exceeds the launch pool");


constexpr uint16_t kHalfNegInf = 0xFC00u;

// K/V element type of an instance.  F16 tiles go from TMA straight to the
// tensor core.  BF16 tiles land by TMA and warps 2-3 convert them in place to
// F16 (exact for values inside F16's range, as ggml's CUDA backend converts
// BF16 K/V to F16 for its tensor-core attention).  Q8_0 rows are staged raw, in
// half tiles of 64 keys, by bulk copies, and warps 2-3 dequantise them into the
// F16 tiles the MMAs read (f16(d * q), one rounding).
constexpr int kKvF16 = 0, kKvBF16 = 1, kKvQ8 = 2;
constexpr int kConvWarps = 2;                                       // warps 2 and 3
constexpr int kRawRows   = kDenseBN / 2;                            // Q8_0 keys per staged half tile
constexpr int kRawRowBytes = 136;                                   // largest row (D = 128): 4 blocks of 34 B
constexpr int kRawBytes  = (kRawRows * kRawRowBytes + 16 + 15) / 16 * 16;  // + up to 15 lead bytes
constexpr int kRawStages = 3;
constexpr int kOffExt     = (kOffMisc + 16 + 15) / 16 * 16;
// ready[kRing] (BF16: converted), raw_full / raw_empty [kRawStages] (Q8_0)
constexpr int kNumExtBars = kRing + 2 * kRawStages;
constexpr int kOffRawMeta = kOffExt + kNumExtBars * 8;             // int4 [kRawStages]
constexpr int kOffRaw     = kOffRawMeta + kRawStages * 16;
static_assert(kOffRaw % 16 == 0, "bulk copies need 16-B aligned staging");
template <int KVT>
constexpr int dense_smem_bytes() {
    // (+ 16: the converters' last 4-B loads of a staged row may reach 3 bytes
    // past the staging ring; + 1024: alignment of the dynamic base)
    return KVT == kKvF16 ? kSmemBytes
                         : (KVT == kKvBF16 ? kOffRawMeta + 1024 : kOffRaw + kRawStages * kRawBytes + 16 + 1024);
}
static_assert(dense_smem_bytes<kKvQ8>() <= 232448, "Q8_0 staging exceeds the 227 KB per CTA");


__device__ __forceinline__ void row_to_query(int gr, int G, int hk, int &iq, int &hq) {
    iq = gr / G;
    hq = hk * G + gr % G;
}

}  // namespace

// ---------------------------------------------------------------------------
// Mask classification: one CTA per (key tile, row tile, mask batch).  The
// tile's mask rows (at most 128 query rows x 128 keys) are cut into 8-key
// chunks; each thread takes up to 8 chunks and issues all their 16-B loads
// before looking at any (the pass is a stream over the mask: it must run at
// HBM speed, not at load latency).  Chunks that are not 16-B aligned or run
// past n_kv are read element by element.
__device__ __forceinline__ void classify_halves(const uint32_t (&w)[4], int kk, int &live, int &nonzero,
                                                int &nonbinary) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t h = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
        if (e < kk) {
            live |= h != kHalfNegInf;
            nonzero |= (h & 0x7FFFu) != 0;
            nonbinary |= (h & 0x7FFFu) != 0 && h != kHalfNegInf;
        }
    }
}

__global__ void __launch_bounds__(256) fa_mask_classify(const __grid_constant__ DenseParams P) {
    constexpr int kChunks = kDenseBN / 8;                  // 8-key chunks per row of a tile
    constexpr int kItems  = kDenseBM * kChunks / 256;      // chunks per thread (rows <= 128)
    const OpDesc &o   = P.op;
    const int     kt  = blockIdx.x;
    const int     t   = blockIdx.y;
    const int     bm  = blockIdx.z;
    const int     G   = o.G;
    const int     gr0 = t * kDenseBM;
    const int     gr1 = min(P.rows_total, gr0 + kDenseBM) - 1;
    const int     iq0 = gr0 / G, iq1 = gr1 / G;
    const int     nrow = iq1 - iq0 + 1;  // <= 128: G = 1 gives 128 rows, G >= 2 at most 65
    const int     j0 = kt * kDenseBN, j1 = min(o.n_kv, j0 + kDenseBN);
    const int     nj = j1 - j0;
    int           live = 0, nonzero = 0, nonbinary = 0;
    pdl_wait_primary();
    const char *mbase = o.mask + (int64_t) bm * o.m_nb3 + (int64_t) iq0 * o.m_nb1 + (int64_t) j0 * 2;
    const bool  vec   = ((reinterpret_cast<uintptr_t>(mbase) | (uintptr_t) o.m_nb1) & 15u) == 0;
    uint4       v[kItems];
#pragma unroll
    for (int it = 0; it < kItems; ++it) {
        const int idx = (int) threadIdx.x + 256 * it;
        const int r = idx / kChunks, ch = idx % kChunks;
        v[it]       = make_uint4(0u, 0u, 0u, 0u);
        if (vec && r < nrow && nj - 8 * ch >= 8) {
            v[it] = __ldg(reinterpret_cast<const uint4 *>(mbase + (int64_t) r * o.m_nb1) + ch);
        }
    }
#pragma unroll
    for (int it = 0; it < kItems; ++it) {
        const int idx = (int) threadIdx.x + 256 * it;
        const int r = idx / kChunks, ch = idx % kChunks;
        const int kk = nj - 8 * ch;  // keys of this chunk inside the tile
        if (r >= nrow || kk <= 0) {
            continue;
        }
        uint32_t w[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
        if (!vec || kk < 8) {
            const uint16_t *p = reinterpret_cast<const uint16_t *>(mbase + (int64_t) r * o.m_nb1) + 8 * ch;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t h = e < kk ? __ldg(p + e) : 0u;
                w[e >> 1]        = (e & 1) ? (w[e >> 1] & 0xFFFFu) | (h << 16) : h;
            }
        }
        classify_halves(w, kk, live, nonzero, nonbinary);
    }
    live      = __syncthreads_or(live);
    nonzero   = __syncthreads_or(nonzero);
    nonbinary = __syncthreads_or(nonbinary);
    if (threadIdx.x == 0) {
        P.cls_out[((int64_t) bm * P.n_rt + t) * P.n_kt + kt] =
            (uint8_t) ((live ? kClsLive : 0) | (live && nonzero ? kClsMask : 0) |
                       (live && nonzero && !nonbinary ? kClsBinary : 0));
    }
    pdl_launch_dependents();
}

// Class of (row tile t, key tile kt) under a mask rule: the classes the
// classify pass gives the equivalent 0 / -inf mask (dead, all visible, or
// binary), from the rows' visible key ranges alone.
__device__ __forceinline__ uint8_t rule_class(const OpDesc &o, int b, int t, int kt, int rows_total) {
    const int gr0 = t * kDenseBM;
    const int gr1 = min(rows_total, gr0 + kDenseBM) - 1;
    const int j0 = kt * kDenseBN, j1 = min(o.n_kv, j0 + kDenseBN);
    int       lo0, hi0, lo1, hi1;
    mg_range(o, b, gr0 / o.G, lo0, hi0);
    mg_range(o, b, gr1 / o.G, lo1, hi1);
    if (max(lo0, j0) >= min(hi1, j1)) {
        return 0;
    }
    return lo1 <= j0 && hi0 >= j1 ? kClsLive : (uint8_t) (kClsLive | kClsMask | kClsBinary);
}

// Bits [a, b) of a 32-bit word (a, b clipped to 0..32).
__device__ __forceinline__ uint32_t range_bits(int a, int b) {
    a = max(a, 0);
    b = min(b, 32);
    if (a >= b) {
        return 0u;
    }
    return (b >= 32 ? ~0u : ((1u << b) - 1u)) & ~((1u << a) - 1u);
}

// ---------------------------------------------------------------------------
// K/V conversion into the F16 tiles the MMAs read (warps 2-3).

// bf16x2 -> f16x2 (exact for values inside F16's range)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
    return cvt_f16x2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// kRawRows staged Q8_0 rows (HD/32 blocks of 34 B each, any 2-B alignment) ->
// rows [row0, row0 + kRawRows) of a 128-key F16 tile in the 128-B swizzled
// layout of the TMA boxes {64 dims, 128 keys}.  A warp iteration converts
// 32 / (HD/32) rows, lane = (row, 32-value block).  Rows at or past `nvalid`
// become zeros.
template <int HD>
__device__ __forceinline__ void q8_rows_to_f16(uint32_t src, uint32_t tile, int row0, int nvalid, int cw, int lane) {
    constexpr int kBlk  = HD / 32;      // blocks per row
    constexpr int kRows = 32 / kBlk;    // rows per warp iteration
    const int     blk   = lane % kBlk;
    const int     rr    = lane / kBlk;
#pragma unroll 1
    for (int it = cw; it < kRawRows / kRows; it += kConvWarps) {
        const int j  = it * kRows + rr;
        uint32_t  q[8];
        const uint16_t dbits = q8_load_run<8>(src + (uint32_t) (j * kBlk * 34 + 34 * blk), 0, q);
        const __half2  d2    = __half2half2(__ushort_as_half(j < nvalid ? dbits : (uint16_t) 0));
        uint32_t       o[16];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            o[2 * k]     = i8x2_scaled(q[k], 0x4140u, d2);
            o[2 * k + 1] = i8x2_scaled(q[k], 0x4342u, d2);
        }
        const int row = row0 + j;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int cc = 4 * blk + m;  // 16-B chunk (8 dims) of the row
            const uint32_t a =
                tile + (uint32_t) ((cc >> 3) * (kDenseBN * 128) + row * 128 + (((cc & 7) ^ (row & 7)) << 4));
            sts128(a, o[4 * m], o[4 * m + 1], o[4 * m + 2], o[4 * m + 3]);
        }
    }
}

// ---------------------------------------------------------------------------
// Softmax helpers of one row (thread) over one 128-key tile held in TMEM.

// Bit k of vis[k/32] = key j0+k visible: inside n_kv and (for binary-mask
// tiles) a mask entry that is not -inf, or under a mask rule (rule set) inside
// the row's visible range [vlo, vhi).
__device__ __forceinline__ void build_visibility(uint32_t (&vis)[4], uint8_t c, const uint16_t *mrow, int j0,
                                                 int n_kv, int m_ne0, bool rule, int vlo, int vhi) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t bits = ~0u;
        if (c & kClsBounds) {
            const int room = n_kv - (j0 + 32 * w);
            bits           = room >= 32 ? ~0u : (room <= 0 ? 0u : ((1u << room) - 1u));
        }
        if ((c & kClsMask) && rule) {
            bits &= range_bits(vlo - (j0 + 32 * w), vhi - (j0 + 32 * w));
        } else if (c & kClsMask) {
            const uint16_t *mp = mrow + j0 + 32 * w;
            uint32_t        mb = 0;
            if ((reinterpret_cast<uintptr_t>(mp) & 15u) == 0 && j0 + 32 * w + 32 <= m_ne0) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const uint4    v     = __ldg(reinterpret_cast<const uint4 *>(mp) + q4);
                    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        mb |= (uint32_t) ((ws[e] & 0xFFFFu) != kHalfNegInf) << (8 * q4 + 2 * e);
                        mb |= (uint32_t) ((ws[e] >> 16) != kHalfNegInf) << (8 * q4 + 2 * e + 1);
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const bool in = j0 + 32 * w + e < m_ne0 && __ldg(mp + e) != kHalfNegInf;
                    mb |= (uint32_t) in << e;
                }
            }
            bits &= mb;
        }
        vis[w] = bits;
    }
}

template <bool VIS>
__device__ __forceinline__ float pass1_max(uint32_t tS, const uint32_t (&vis)[4]) {
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
    for (int ch = 0; ch < 4; ch += 2) {
        uint32_t x[32], y[32];
        tmem_ld32(tS + 32 * ch, x);
        tmem_ld32(tS + 32 * ch + 32, y);
        tmem_ld_wait32(x);
        tmem_ld_wait32(y);
        const uint32_t va = ch == 0 ? vis[0] : vis[2];  // keep vis in registers
        const uint32_t vb = ch == 0 ? vis[1] : vis[3];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            float a = __uint_as_float(x[e]), b = __uint_as_float(y[e]);
            if constexpr (VIS) {
                a = (va >> e) & 1u ? a : -INFINITY;
                b = (vb >> e) & 1u ? b : -INFINITY;
            }
            mx[e & 3] = fmax3(mx[e & 3], a, b);
        }
    }
    return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// Fast-tile P: t = s * c - m by packed FMA (two scores per instruction),
// rounded to f16x2 and exponentiated by ex2.approx.f16x2 (two results per MUFU
// op), which is already P's storage format.  Masked keys get t = -inf, so
// P = 0 exactly.  Row sums add the f16 pairs in groups of four and fold them into
// f32 once per 32 keys.
template <bool VIS>
__device__ __forceinline__ void pass2_exp_packed(uint32_t tS, const uint32_t (&vis)[4], float mul, float m_use,
                                                 float (&ls)[4]) {
    const uint64_t c2 = f32x2(mul, mul);
    const uint64_t m2 = f32x2(-m_use, -m_use);
#pragma unroll 1
    for (int ch = 0; ch < 4; ch += 2) {
        uint32_t x[32], y[32];
        tmem_ld32(tS + 32 * ch, x);
        tmem_ld32(tS + 32 * ch + 32, y);
        tmem_ld_wait32(x);
        tmem_ld_wait32(y);
        const uint32_t va = ch == 0 ? vis[0] : vis[2];
        const uint32_t vb = ch == 0 ? vis[1] : vis[3];
        uint32_t       pk[16], pk2[16];
        uint32_t       ha[4], hb[4];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            float a0, a1, b0, b1;
            f32x2_split(ffma2(f32x2(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1])), c2, m2), a0, a1);
            f32x2_split(ffma2(f32x2(__uint_as_float(y[2 * e]), __uint_as_float(y[2 * e + 1])), c2, m2), b0, b1);
            if constexpr (VIS) {
                a0 = (va >> (2 * e)) & 1u ? a0 : -INFINITY;
                a1 = (va >> (2 * e + 1)) & 1u ? a1 : -INFINITY;
                b0 = (vb >> (2 * e)) & 1u ? b0 : -INFINITY;
                b1 = (vb >> (2 * e + 1)) & 1u ? b1 : -INFINITY;
            }
            pk[e]  = ex2_f16x2(cvt_f16x2(a0, a1));
            pk2[e] = ex2_f16x2(cvt_f16x2(b0, b1));
            if (e < 4) {
                ha[e] = pk[e];
                hb[e] = pk2[e];
            } else {
                ha[e & 3] = hadd2_u(ha[e & 3], pk[e]);
                hb[e & 3] = hadd2_u(hb[e & 3], pk2[e]);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half2 s2 = __hadd2(*reinterpret_cast<const __half2 *>(&ha[k]),
                                       *reinterpret_cast<const __half2 *>(&hb[k]));
            const float2  f  = __half22float2(s2);
            ls[k] += f.x + f.y;
        }
        tmem_st16(tS + 16 * ch, pk);
        tmem_st16(tS + 16 * ch + 16, pk2);
    }
}

// Steady-state fast tile: P = exp2(s * c - m) for all 128 keys into pk (f16
// pairs, not yet stored), row sums into ls, and the raw (unscaled) max of the
// visible scores returned, all from one read of S.
// 64 scores (two 32-column chunks) against the running max m: P into
// pk[0..31] (f16 pairs, chunk x then chunk y), raw maxima into mx, sums into ls.
template <bool VIS>
__device__ __forceinline__ void exp_pair(const uint32_t (&x)[32], const uint32_t (&y)[32], uint32_t vx,
                                         uint32_t vy, float c, float m, float (&mx)[2], float (&ls)[4],
                                         uint32_t *pk) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        float a0 = __uint_as_float(x[2 * e]), a1 = __uint_as_float(x[2 * e + 1]);
        float b0 = __uint_as_float(y[2 * e]), b1 = __uint_as_float(y[2 * e + 1]);
        if constexpr (VIS) {
            a0 = (vx >> (2 * e)) & 1u ? a0 : -INFINITY;
            a1 = (vx >> (2 * e + 1)) & 1u ? a1 : -INFINITY;
            b0 = (vy >> (2 * e)) & 1u ? b0 : -INFINITY;
            b1 = (vy >> (2 * e + 1)) & 1u ? b1 : -INFINITY;
        }
        mx[0] = fmax3(mx[0], a0, a1);
        mx[1] = fmax3(mx[1], b0, b1);
        const float p0 = fast_exp2(fmaf(a0, c, -m)), p1 = fast_exp2(fmaf(a1, c, -m));
        const float q0 = fast_exp2(fmaf(b0, c, -m)), q1 = fast_exp2(fmaf(b1, c, -m));
        ls[e & 3] += (p0 + p1) + (q0 + q1);
        pk[e]      = pack2<false>(p0, p1);
        pk[16 + e] = pack2<false>(q0, q1);
    }
}

// One tile row against the running max: the second half's TMEM loads are
// issued before the first half is exponentiated, so their latency hides
// behind it.  P stays in registers (pk) and the raw tile max is returned.
template <bool VIS>
__device__ __forceinline__ float exp_tile_regs(uint32_t tS, const uint32_t (&vis)[4], float c, float m,
                                               float (&ls)[4], uint32_t (&pk)[64]) {
    float    mx[2] = {-INFINITY, -INFINITY};
    uint32_t x0[32], x1[32], y0[32], y1[32];
    tmem_ld32(tS, x0);
    tmem_ld32(tS + 32, x1);
    tmem_ld_wait32(x0);
    tmem_ld_wait32(x1);
    tmem_ld32(tS + 64, y0);
    tmem_ld32(tS + 96, y1);
    exp_pair<VIS>(x0, x1, vis[0], vis[1], c, m, mx, ls, pk);
    tmem_ld_wait32(y0);
    tmem_ld_wait32(y1);
    exp_pair<VIS>(y0, y1, vis[2], vis[3], c, m, mx, ls, pk + 32);
    return fmaxf(mx[0], mx[1]);
}

// P = exp2(x * mul - m) as f16 pairs written over the first 64 S columns;
// row sums accumulate into ls[4].
template <bool VIS>
__device__ __forceinline__ void pass2_exp(uint32_t tS, const uint32_t (&vis)[4], float mul, float m_use,
                                          float (&ls)[4]) {
#pragma unroll 1
    for (int ch = 0; ch < 4; ch += 2) {
        uint32_t x[32], y[32];
        tmem_ld32(tS + 32 * ch, x);
        tmem_ld32(tS + 32 * ch + 32, y);
        tmem_ld_wait32(x);
        tmem_ld_wait32(y);
        uint32_t       pk[16], pk2[16];
        const uint32_t va = ch == 0 ? vis[0] : vis[2];
        const uint32_t vb = ch == 0 ? vis[1] : vis[3];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            float p0 = fast_exp2(fmaf(__uint_as_float(x[2 * e]), mul, -m_use));
            float p1 = fast_exp2(fmaf(__uint_as_float(x[2 * e + 1]), mul, -m_use));
            float q0 = fast_exp2(fmaf(__uint_as_float(y[2 * e]), mul, -m_use));
            float q1 = fast_exp2(fmaf(__uint_as_float(y[2 * e + 1]), mul, -m_use));
            if constexpr (VIS) {
                p0 = (va >> (2 * e)) & 1u ? p0 : 0.0f;
                p1 = (va >> (2 * e + 1)) & 1u ? p1 : 0.0f;
                q0 = (vb >> (2 * e)) & 1u ? q0 : 0.0f;
                q1 = (vb >> (2 * e + 1)) & 1u ? q1 : 0.0f;
            }
            ls[e & 3] += (p0 + p1) + (q0 + q1);
            pk[e]  = pack2<false>(p0, p1);
            pk2[e] = pack2<false>(q0, q1);
        }
        tmem_st16(tS + 16 * ch, pk);
        tmem_st16(tS + 16 * ch + 16, pk2);
    }
}

// ---------------------------------------------------------------------------
// PRO: the instance that applies the QK-norm + RoPE prologue to Q rows; KVT:
// the K/V element type (kKvF16 / kKvBF16 / kKvQ8).
// HD = head dim, 64 or 128: D = 64 reads one 64-dim box per K/V tile, runs
// half the S k-steps and an N = 64 PV MMA, and leaves O in 64 TMEM columns.
template <bool PRO, int KVT, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    fa_dense_kernel(const __grid_constant__ DenseParams P, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap qmap,
                    const __grid_constant__ CUtensorMap omap) {
    extern __shared__ uint8_t smem_raw[];
    // 1 KB aligned base, derived from smem_raw by an offset so that the
    // compiler keeps the shared address space: every access through it is an
    // ld/st.shared (a pointer rebuilt from an integer would be generic).
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

    uint64_t     *bars    = reinterpret_cast<uint64_t *>(smem + kOffBars);
    uint64_t     *full    = bars;
    uint64_t     *empty   = bars + kRing;
    uint64_t     *s_ready = bars + 2 * kRing;
    uint64_t     *p_ready = s_ready + 2;
    uint64_t     *o_done  = p_ready + 2;
    uint64_t     *fin     = o_done + 2;
    uint64_t     *q_full  = fin + 1;  // the unit's f32 Q rows staged in the K/V ring
    uint64_t     *ready     = reinterpret_cast<uint64_t *>(smem + kOffExt);  // [kRing] BF16 tile converted
    uint64_t     *raw_full  = ready + kRing;                                  // [kRawStages] Q8_0 half tile staged
    uint64_t     *raw_empty = raw_full + kRawStages;                         // [kRawStages] staging free again
    int4         *raw_meta  = reinterpret_cast<int4 *>(smem + kOffRawMeta);  // (rows, lead bytes) per staging
    uint8_t      *s_cls   = smem + kOffCls;  // [2][kDenseMaxKT]
    uint32_t     *s_tmem  = reinterpret_cast<uint32_t *>(smem + kOffMisc);
    volatile int *abort_f = reinterpret_cast<volatile int *>(smem + kOffMisc + 4);

    const OpDesc &o    = P.op;
    const int     warp = threadIdx.x >> 5;
    const int     lane = threadIdx.x & 31;
    // 1-D grid of work units.  Masked nodes: pair index slowest and descending,
    // so every (batch, head)'s late (for causal masks, heaviest) row tiles are
    // scheduled first.  Unmasked nodes (every unit the same work): (batch, kv
    // head) slowest, so the CTAs in flight share few heads' K/V and re-read them
    // from L2.  CTAs past n_full each take one key range of a split unit.
    const int     units   = o.B * o.Hkv;
    const bool    is_part = (int) blockIdx.x >= P.n_full;
    const int     xs      = (int) blockIdx.x - P.n_full;
    const int     unit_id = is_part ? P.n_full + xs / P.n_split : (int) blockIdx.x;
    const int     sp      = is_part ? xs % P.n_split : 0;
    const int     kt_lo   = is_part ? (int) ((int64_t) P.n_kt * sp / P.n_split) : 0;
    const int     kt_hi   = is_part ? (int) ((int64_t) P.n_kt * (sp + 1) / P.n_split) : P.n_kt;
    const int     pair    = P.head_major ? unit_id % P.n_pairs : P.n_pairs - 1 - unit_id / units;
    const int     bh      = P.head_major ? unit_id / P.n_pairs : unit_id % units;
    const int     hk      = bh % o.Hkv;
    const int     b       = bh / o.Hkv;
    const int     bk   = b / o.rk3;
    const int     t0   = 2 * pair;
    const bool    has_tile[2] = {t0 < P.n_rt, t0 + 1 < P.n_rt};

    if (warp == 1) {
        tmem_alloc(s_tmem, kTmemCols);
        tmem_relinquish();
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRing; ++i) {
            mbar_init(&full[i], KVT == kKvQ8 ? kConvWarps : 1);
            mbar_init(&empty[i], 1);
            if constexpr (KVT == kKvBF16) {
                mbar_init(&ready[i], kConvWarps);
            }
        }
        if constexpr (KVT == kKvQ8) {
            for (int i = 0; i < kRawStages; ++i) {
                mbar_init(&raw_full[i], 1);
                mbar_init(&raw_empty[i], kConvWarps);
            }
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_ready[i], 1);
            mbar_init(&p_ready[i], 128);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(fin, 1);
        mbar_init(q_full, 1);
        *abort_f = 0;
        fence_barrier_init();
    }
    if (KVT != kKvQ8 && warp == 0 && lane == 0) {
        prefetch_tensormap(&kmap);
        prefetch_tensormap(&vmap);
    }
    if (P.q_tma && warp == 0 && lane == 0) {
        prefetch_tensormap(&qmap);
    }
    pdl_wait_primary();

    // The unit's Q rows (f32) by TMA into the K/V ring, idle until Q has been
    // converted: far more bytes in flight than per-thread loads give.  Issued
    // by the thread that initialised the barriers, before the class table.
    if (P.q_tma && threadIdx.x == 0) {
        const uint32_t tile_bytes = kDenseBM * HD * 4;
        mbar_arrive_expect_tx(q_full, tile_bytes * ((has_tile[0] ? 1u : 0u) + (has_tile[1] ? 1u : 0u)));
        for (int i = 0; i < 2; ++i) {
            if (has_tile[i]) {
                tma_load_4d(smem + kOffRing + i * tile_bytes, &qmap, 0, hk * o.G, (t0 + i) * (kDenseBM / o.G), b,
                            q_full);
            }
        }
    }

    // ---- key-tile classes of both row tiles
    for (int j = threadIdx.x; j < P.n_kt; j += kThreads) {
        for (int i = 0; i < 2; ++i) {
            uint8_t c = 0;
            if (has_tile[i] && j >= kt_lo && j < kt_hi) {
                if (P.cls) {
                    c = P.cls[((int64_t) (b % o.m_ne3) * P.n_rt + t0 + i) * P.n_kt + j];
                } else if (o.mg_kind) {
                    c = rule_class(o, b, t0 + i, j, P.rows_total);
                } else {
                    c = kClsLive | (o.mask ? kClsMask : 0);
                }
                if ((c & kClsLive) && j == P.n_kt - 1 && (o.n_kv % kDenseBN) != 0) {
                    c |= kClsBounds;
                }
            }
            s_cls[i * kDenseMaxKT + j] = c;
        }
    }

    __syncthreads();  // barriers initialised, class table complete

    auto live_of  = [&](int i, int j) -> bool { return (s_cls[i * kDenseMaxKT + j] & kClsLive) != 0; };
    auto any_live = [&](int j) -> bool { return live_of(0, j) || live_of(1, j); };

    // TMA producer state (warp 0, lane 0).  (Issuing its first key steps
    // before the Q conversion below measured slower: the K/V burst competes
    // with the Q loads at every wave start.)
    int  pend[kRing];
    int  p_j = 0, p_use = 0;
    bool p_ok = true;
    auto produce = [&](int max_steps) {
        for (int n = 0; p_j < P.n_kt && p_ok && n < max_steps; ++p_j) {
            if (!any_live(p_j)) {
                continue;
            }
            for (int h = 0; h < 2 && p_ok; ++h) {
                const int seq = 2 * p_use + h;
                const int buf = seq % kRing;
                const int u   = seq / kRing;
                p_ok = mbar_wait_bounded(&empty[buf], (uint32_t) ((u & 1) ^ 1), abort_f, P.dev_err,
                                         DEVERR_TIMEOUT_EMPTY, P.wait_limit_ns);
                if (!p_ok) {
                    break;
                }
                uint8_t           *dst = smem + kOffRing + buf * kTileBytes;
                const CUtensorMap *map = h == 0 ? &kmap : &vmap;
                mbar_arrive_expect_tx(&full[buf], kTileBytes * HD / 128);
                tma_load_4d(dst, map, 0, p_j * kDenseBN, hk, bk, &full[buf]);
                if constexpr (HD == 128) {
                    tma_load_4d(dst + kDenseBN * 128, map, 64, p_j * kDenseBN, hk, bk, &full[buf]);
                }
                pend[buf] = u & 1;
            }
            ++p_use;
            ++n;
        }
    };
    if (warp == 0 && lane == 0) {
        for (int k = 0; k < kRing; ++k) {
            pend[k] = -1;
        }
    }

    // ---- Q: f32 rows -> f16, 128-B swizzled K-major tiles [HD/64 x 64 dims][128 rows].
    // 16-B chunks, eight loads in flight per thread before any is converted.
    // A warp's chunks of one load step are 32 / kCpr rows (chunk c of a row:
    // dims 4c..4c+3).
    {
        constexpr int kCpr    = HD / 4;  // chunks per row
        constexpr int kChunks = 2 * kDenseBM * kCpr;
        constexpr int kUnroll = 8;
        auto store_q = [&](int ch, float4 x) {
            const int      rr = ch / kCpr;
            const int      i  = rr / kDenseBM;
            const int      r  = rr % kDenseBM;
            const int      d  = 4 * (ch % kCpr);
            const uint32_t lo = pack2<false>(x.x, x.y), hi = pack2<false>(x.z, x.w);
            uint8_t *dst = smem + kOffQ + i * kQBytes + (d >> 6) * (kDenseBM * 128) + r * 128 +
                           ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2;
            *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
        };
        const float *q_st = reinterpret_cast<const float *>(smem + kOffRing);  // [2][128][HD] when q_tma
        if (P.q_tma &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(q_full, 0u, abort_f, P.dev_err, DEVERR_TIMEOUT_FULL,
                                                       P.wait_limit_ns))) {
            *abort_f = 1;  // the waits below give up at once; the Q copy is drained before exit
        }
        for (int base = threadIdx.x; base < kChunks; base += kThreads * kUnroll) {
            float4 v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int ch = base + u * kThreads;
                v[u]         = make_float4(0.f, 0.f, 0.f, 0.f);
                const int rr = ch / kCpr;
                const int i  = rr / kDenseBM;
                const int gr = (t0 + i) * kDenseBM + rr % kDenseBM;
                if (P.q_tma) {
                    if (ch < kChunks && has_tile[i] && gr < P.rows_total) {
                        v[u] = *reinterpret_cast<const float4 *>(q_st + (size_t) rr * HD + 4 * (ch % kCpr));
                    }
                } else if (ch < kChunks && has_tile[i] && gr < P.rows_total) {
                    int iq, hq;
                    row_to_query(gr, o.G, hk, iq, hq);
                    const char  *qrow = o.q + (int64_t) iq * o.q_nb1 + (int64_t) hq * o.q_nb2 + (int64_t) b * o.q_nb3;
                    const float *qf   = reinterpret_cast<const float *>(qrow) + 4 * (ch % kCpr);
                    if ((reinterpret_cast<uintptr_t>(qf) & 15u) == 0) {
                        v[u] = __ldg(reinterpret_cast<const float4 *>(qf));
                    } else {
                        v[u] = make_float4(__ldg(qf), __ldg(qf + 1), __ldg(qf + 2), __ldg(qf + 3));
                    }
                }
            }
            if (!PRO || !o.qp.on) {
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    if (base + u * kThreads < kChunks) {
                        store_q(base + u * kThreads, v[u]);
                    }
                }
                continue;
            }
            // QK-norm + RoPE of each row (one row per warp and step), one step
            // at a time: the loads above are already in flight
            float4 vl[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                vl[u] = v[u];
            }
#pragma unroll 1
            for (int u = 0; u < kUnroll; ++u) {
                const int ch = base + u * kThreads;
                if (ch >= kChunks) {
                    break;
                }
                const int rr  = ch / kCpr;
                const int i   = rr / kDenseBM;
                const int gr  = (t0 + i) * kDenseBM + rr % kDenseBM;
                const int cr  = lane % kCpr;  // this lane's chunk of its row
                int       pos = 0;
                if (o.qp.rope && has_tile[i] && gr < P.rows_total) {
                    int iq, hq;
                    row_to_query(gr, o.G, hk, iq, hq);
                    pos = __ldg(o.qp.pos + iq + (int64_t) b * o.n_q);
                }
                float x[4] = {vl[u].x, vl[u].y, vl[u].z, vl[u].w};
                if (o.qp.w) {
                    float ss = 0.0f;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        ss = fmaf(x[e], x[e], ss);
                    }
#pragma unroll
                    for (int off = kCpr / 2; off; off >>= 1) {
                        ss += __shfl_xor_sync(0xffffffffu, ss, off);
                    }
                    const float sc = rn_scale(o.qp, ss, HD);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        x[e] = (x[e] * sc) * __ldg(o.qp.w + 4 * cr + e);
                    }
                }
                if (o.qp.rope) {
                    float2 cs[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        cs[e] = rn_cos_sin((float) pos * o.qp.inv_freq[(4 * cr + e) & (HD / 2 - 1)]);
                    }
                    const bool first = cr < kCpr / 2;  // dim d < HD/2 pairs with d + HD/2
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float pt = __shfl_xor_sync(0xffffffffu, x[e], kCpr / 2);
                        x[e] = first ? x[e] * cs[e].x - pt * cs[e].y : pt * cs[e].y + x[e] * cs[e].x;
                    }
                }
                store_q(ch, make_float4(x[0], x[1], x[2], x[3]));
            }
        }
    }
    fence_proxy_async_smem();  // Q is read by the tensor core (async proxy)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp < 4) {
      setmaxnreg_dec<kRegsControl>();
      if (KVT == kKvQ8 && warp == 0) {
        // ======================= Q8_0 staging producer ========================
        // Each live key tile's K then V rows, in halves of 64 keys, by bulk
        // copies into the staging ring (from the 16-B boundary below each half,
        // inside the tensor; the ragged last bytes by plain copies).
        const char *kb    = o.k + (int64_t) hk * o.k_nb2 + (int64_t) bk * o.k_nb3;
        const char *vb    = o.v + (int64_t) hk * o.v_nb2 + (int64_t) bk * o.v_nb3;
        int         rs    = 0;
        uint32_t    rph   = 0;
        int         rpend[kRawStages];
        bool        ok    = true;
        for (int i = 0; i < kRawStages; ++i) {
            rpend[i] = -1;
        }
        for (int j = 0; j < P.n_kt && ok; ++j) {
            if (!any_live(j)) {
                continue;
            }
            for (int h = 0; h < 2 && ok; ++h) {
                for (int q = 0; q < 2 && ok; ++q) {
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&raw_empty[rs], rph ^ 1u, abort_f, P.dev_err,
                                                                   DEVERR_TIMEOUT_EMPTY, P.wait_limit_ns));
                    if (!ok) {
                        break;
                    }
                    const int      row0  = j * kDenseBN + q * kRawRows;
                    const int      nrows = max(0, min(kRawRows, o.n_kv - row0));
                    const char    *src   = (h ? vb : kb) + (int64_t) row0 * (HD / 32 * 34);
                    const uint32_t lead  = (uint32_t) (reinterpret_cast<uintptr_t>(src) & 15u);
                    const uint32_t bytes = (uint32_t) nrows * (HD / 32 * 34);
                    const uint32_t bulk  = (lead + bytes) & ~15u;
                    uint8_t       *dst   = smem + kOffRaw + rs * kRawBytes;
                    if (nrows > 0 && (uint32_t) lane < lead + bytes - bulk && bulk + (uint32_t) lane >= lead) {
                        dst[bulk + lane] = (uint8_t) src[(int) (bulk + lane) - (int) lead];
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        raw_meta[rs] = make_int4(nrows, (int) lead, 0, 0);
                        mbar_arrive_expect_tx(&raw_full[rs], bulk);
                        if (bulk) {
                            bulk_load(dst, src - lead, bulk, &raw_full[rs]);
                        }
                    }
                    rpend[rs] = (int) rph;
                    __syncwarp();
                    if (++rs == kRawStages) {
                        rs = 0;
                        rph ^= 1u;
                    }
                }
            }
        }
        if (!ok && lane == 0) {
            // let the copies in flight land before the CTA exits
            for (int i = 0; i < kRawStages; ++i) {
                if (rpend[i] < 0) {
                    continue;
                }
                const uint64_t ts = globaltimer_ns();
                while (!mbar_try_wait(&raw_full[i], (uint32_t) rpend[i])) {
                    if (globaltimer_ns() - ts > P.wait_limit_ns) {
                        atomicCAS(P.dev_err, 0, DEVERR_TIMEOUT_DRAIN);
                        break;
                    }
                }
            }
        }
      } else if (warp == 0) {
        // ============================ TMA producer ============================
        if (lane == 0) {
            produce(P.n_kt);
            if (!p_ok) {
                for (int i = 0; i < kRing; ++i) {
                    if (pend[i] < 0) {
                        continue;
                    }
                    const uint64_t ts = globaltimer_ns();
                    while (!mbar_try_wait(&full[i], (uint32_t) pend[i])) {
                        if (globaltimer_ns() - ts > P.wait_limit_ns) {
                            atomicCAS(P.dev_err, 0, DEVERR_TIMEOUT_DRAIN);
                            break;
                        }
                    }
                }
            }
        }
      } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        if (lane == 0) {
            constexpr uint32_t idS = umma_idesc_f16(128, 128, false, false, false);
            constexpr uint32_t idO = umma_idesc_f16(128, HD, false, true, false);
            // Base descriptors, built once.  Advancing a descriptor is a 64-bit add
            // to its start-address field (16-B units): k-step ks of a K-major
            // operand sits at (ks/4)*16 KB + (ks%4)*32 B; of the MN-major V at
            // ks*16 keys*128 B; ring slot s at s*32 KB.
            const uint64_t qd0   = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
            const uint64_t qd1   = umma_desc_sw128(smem_u32(smem + kOffQ + kQBytes), 16, 1024);
            const uint64_t kd0   = umma_desc_sw128(smem_u32(smem + kOffRing), 16, 1024);
            const uint64_t vd0   = umma_desc_sw128(smem_u32(smem + kOffRing), kDenseBN * 128, 1024);
            const uint32_t tO0   = tmem + 0, tO1 = tmem + 128, tS0 = tmem + 256, tS1 = tmem + 384;
            uint32_t       p_ph0 = 0, p_ph1 = 0, has_o0 = 0, has_o1 = 0;
            bool           ok    = true;

            // a ring slot is ready once its tile landed (F16) or was converted
            // to F16 (BF16: `ready`; Q8_0: the converters arrive on `full`)
            auto wait_full = [&](int seq) -> bool {
                uint64_t *bar = KVT == kKvBF16 ? &ready[seq % kRing] : &full[seq % kRing];
                return mbar_wait_bounded(bar, (uint32_t) ((seq / kRing) & 1), abort_f, P.dev_err, DEVERR_TIMEOUT_FULL,
                                         P.wait_limit_ns);
            };
            auto issue_s = [&](uint32_t tS, uint64_t qd, int slot) {
                const uint64_t kd = kd0 + (uint64_t) (slot * (kTileBytes >> 4));
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks) {
                    const uint64_t off = (uint64_t) ((ks >> 2) * (kDenseBM * 128 >> 4) + (ks & 3) * 2);
                    umma_ss(tS, qd + off, kd + off, idS, ks > 0 ? 1u : 0u);
                }
            };
            auto issue_pv = [&](uint32_t tO, uint32_t tS, int slot, uint32_t acc) {
                const uint64_t vd = vd0 + (uint64_t) (slot * (kTileBytes >> 4));
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    umma_ts(tO, tS + ks * 8, vd + (uint64_t) (ks * (16 * 128 >> 4)), idO, (ks > 0 || acc) ? 1u : 0u);
                }
            };
            auto next_live = [&](int j) {
                while (j < P.n_kt && !any_live(j)) {
                    ++j;
                }
                return j;
            };

            int use = 0;
            int j   = next_live(0);
            if (j < P.n_kt) {
                ok = wait_full(2 * use);
                if (ok) {
                    tc_fence_after();
                    const int ks0 = (2 * use) % kRing;
                    if (live_of(0, j)) {
                        issue_s(tS0, qd0, ks0);
                        tc_commit(&s_ready[0]);
                    }
                    if (live_of(1, j)) {
                        issue_s(tS1, qd1, ks0);
                        tc_commit(&s_ready[1]);
                    }
                    tc_commit(&empty[ks0]);
                }
            }
            while (ok && j < P.n_kt) {
                const int  jn    = next_live(j + 1);
                const bool nxt   = jn < P.n_kt;
                const int  vslot = (2 * use + 1) % kRing;
                const int  kslot = (2 * (use + 1)) % kRing;
                const bool l0 = live_of(0, j), l1 = live_of(1, j);
                const bool n0 = nxt && live_of(0, jn), n1 = nxt && live_of(1, jn);
                ok = wait_full(2 * use + 1);
                if (!ok) {
                    break;
                }
                tc_fence_after();
                bool kready = false;
                // row tile 0: O0 += P0 V_j, then S0 = Q0 K_jn
                if (l0) {
                    ok = mbar_wait_bounded(&p_ready[0], p_ph0, abort_f, P.dev_err, DEVERR_TIMEOUT_MMA, P.wait_limit_ns);
                    if (!ok) {
                        break;
                    }
                    p_ph0 ^= 1u;
                    tc_fence_after();
                    issue_pv(tO0, tS0, vslot, has_o0);
                    has_o0 = 1;
                    tc_commit(&o_done[0]);
                }
                if (n0) {
                    ok = wait_full(2 * (use + 1));
                    if (!ok) {
                        break;
                    }
                    tc_fence_after();
                    kready = true;
                    issue_s(tS0, qd0, kslot);
                    tc_commit(&s_ready[0]);
                }
                // row tile 1
                if (l1) {
                    ok = mbar_wait_bounded(&p_ready[1], p_ph1, abort_f, P.dev_err, DEVERR_TIMEOUT_MMA, P.wait_limit_ns);
                    if (!ok) {
                        break;
                    }
                    p_ph1 ^= 1u;
                    tc_fence_after();
                    issue_pv(tO1, tS1, vslot, has_o1);
                    has_o1 = 1;
                    tc_commit(&o_done[1]);
                }
                tc_commit(&empty[vslot]);
                if (nxt) {
                    if (!kready) {
                        ok = wait_full(2 * (use + 1));
                        if (!ok) {
                            break;
                        }
                        tc_fence_after();
                    }
                    if (n1) {
                        issue_s(tS1, qd1, kslot);
                        tc_commit(&s_ready[1]);
                    }
                    tc_commit(&empty[kslot]);
                }
                ++use;
                j = jn;
            }
            // every MMA issued by this thread completes before TMEM is released
            tc_commit(fin);
            const uint64_t ts = globaltimer_ns();
            while (!mbar_try_wait(fin, 0)) {
                if (globaltimer_ns() - ts > P.wait_limit_ns) {
                    atomicCAS(P.dev_err, 0, DEVERR_TIMEOUT_MMA);
                    break;
                }
            }
        }
      } else if (KVT != kKvF16) {
        // ============================ converters (warps 2-3) ===================
        // Ring slots in the producer's order: each live key tile's K, then V.
        const int cw  = warp - 2;
        const int ct  = cw * 32 + lane;
        bool      ok  = true;
        int       use = 0;
        int       rs  = 0;  // Q8_0 staging position
        uint32_t  rph = 0;
        for (int j = 0; j < P.n_kt && ok; ++j) {
            if (!any_live(j)) {
                continue;
            }
            for (int h = 0; h < 2 && ok; ++h) {
                const int seq  = 2 * use + h;
                const int buf  = seq % kRing;
                const int u    = seq / kRing;
                uint8_t  *tile = smem + kOffRing + buf * kTileBytes;
                if constexpr (KVT == kKvBF16) {
                    // the TMA-landed bf16 tile, converted in place, 16 B at a time
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[buf], (uint32_t) (u & 1), abort_f, P.dev_err,
                                                                   DEVERR_TIMEOUT_FULL, P.wait_limit_ns));
                    if (!ok) {
                        break;
                    }
#pragma unroll 4
                    for (int x = ct; x < kTileBytes * HD / 128 / 16; x += 32 * kConvWarps) {
                        uint4 w = *reinterpret_cast<const uint4 *>(tile + 16 * x);
                        w.x     = bf16x2_to_f16x2(w.x);
                        w.y     = bf16x2_to_f16x2(w.y);
                        w.z     = bf16x2_to_f16x2(w.z);
                        w.w     = bf16x2_to_f16x2(w.w);
                        *reinterpret_cast<uint4 *>(tile + 16 * x) = w;
                    }
                    fence_proxy_async_smem();  // read next by the tensor core (async proxy)
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&ready[buf]);
                    }
                } else {
                    // the slot's previous tile is no longer read by the MMAs;
                    // fill it from two staged halves
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&empty[buf], (uint32_t) ((u & 1) ^ 1), abort_f,
                                                                   P.dev_err, DEVERR_TIMEOUT_EMPTY, P.wait_limit_ns));
                    for (int q = 0; q < 2 && ok; ++q) {
                        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&raw_full[rs], rph, abort_f, P.dev_err,
                                                                       DEVERR_TIMEOUT_FULL, P.wait_limit_ns));
                        if (!ok) {
                            break;
                        }
                        const int4 md = raw_meta[rs];
                        q8_rows_to_f16<HD>(smem_u32(smem + kOffRaw + rs * kRawBytes) + (uint32_t) md.y, smem_u32(tile),
                                       q * kRawRows, md.x, cw, lane);
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&raw_empty[rs]);
                        }
                        if (++rs == kRawStages) {
                            rs = 0;
                            rph ^= 1u;
                        }
                    }
                    if (!ok) {
                        break;
                    }
                    fence_proxy_async_smem();  // read next by the tensor core (async proxy)
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&full[buf]);
                    }
                }
            }
            ++use;
        }
      }
    } else {
        // ============================ softmax =================================
        setmaxnreg_inc<kRegsSoftmax>();
        // warps 4-7 own row tile 0 and warps 8-11 row tile 1; a warp may only
        // touch TMEM lanes 32*(warp%4) .. +31
        const int      i     = (warp - 4) >> 2;  // row tile
        const int      wq    = warp & 3;         // TMEM lane quarter
        const int      r     = wq * 32 + lane;
        const int      gr    = (t0 + i) * kDenseBM + r;
        const bool     vrow  = has_tile[i] && gr < P.rows_total;
        const uint32_t lanes = (uint32_t) (wq * 32) << 16;
        const uint32_t tS    = tmem + lanes + 256 + 128 * i;
        const uint32_t tO    = tmem + lanes + 128 * i;
        int            iq = 0, hq = 0;
        if (vrow) {
            row_to_query(gr, o.G, hk, iq, hq);
        }
        const uint16_t *mrow = nullptr;
        if (o.mask) {
            mrow = reinterpret_cast<const uint16_t *>(o.mask + (int64_t) iq * o.m_nb1 +
                                                      (int64_t) (hq % o.m_ne2) * o.m_nb2 +
                                                      (int64_t) (b % o.m_ne3) * o.m_nb3);
        }
        // mask rule: this row's visible keys [vlo, vhi)
        const bool rule = o.mg_kind != 0;
        int        vlo = 0, vhi = 0;
        if (rule) {
            mg_range(o, b, iq, vlo, vhi);
        }
        const float slope = alibi_slope(o, hq);
        // softcap or a non-positive scale take the general path on every tile
        const bool  general    = o.softcap != 0.0f || !(o.scale_eff > 0.0f);
        const float scale_log2 = o.scale_eff * kLog2e;
        float       m_run = -INFINITY;  // log2 units
        float       l_run = 0.0f;
        int         cnt   = 0;
        bool        ok    = true;

        // Folds the tile max into the running max and rescales O and l when it
        // grew by more than 2^8.  tcgen05.ld/st are warp-collective, so the whole warp
        // walks O when any of its rows needs it (the others multiply by 1).
        // (No wait for the previous PV here: S of this tile was issued after it,
        // and the s_ready commit only fires once every earlier MMA is done.)
        auto update_max = [&](float tmax) -> bool {
            const float m_new = fmaxf(m_run, tmax);
            const bool  need  = m_run != -INFINITY && m_new > m_run + kRescaleLog2;
            float       f     = 1.0f;
            if (need) {
                f = fast_exp2(m_run - m_new);
                l_run *= f;
                m_run = m_new;
            }
            if (m_run == -INFINITY) {
                m_run = m_new;  // nothing accumulated yet for this row
            }
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
                for (int ch = 0; ch < HD / 16; ++ch) {
                    uint32_t x[16];
                    tmem_ld16(tO + 16 * ch, x);
                    tmem_ld_wait16(x);
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        x[e] = __float_as_uint(__uint_as_float(x[e]) * f);
                    }
                    tmem_st16(tO + 16 * ch, x);
                }
            }
            return true;
        };

        for (int j = 0; j < P.n_kt && ok; ++j) {
            const uint8_t c = s_cls[i * kDenseMaxKT + j];
            if (!(c & kClsLive)) {
                continue;
            }
            const int j0 = j * kDenseBN;
            // Fast tiles (no mask values other than 0 / -inf, no softcap,
            // positive scale): max of the raw scores, then exp2(s * c - m) in
            // one FMA + ex2 per score.  Binary-mask and ragged tiles use a
            // 128-bit visibility mask per row, built (from the mask in global
            // memory) before the wait for S, so its loads overlap the MMA.
            // Other tiles rewrite S as finished log2-unit logits in TMEM first.
            const bool fast    = (!(c & kClsMask) || (c & kClsBinary)) && !general;
            const bool use_vis = fast && (c & (kClsMask | kClsBounds)) != 0;
            uint32_t   vis[4]  = {~0u, ~0u, ~0u, ~0u};
            if (use_vis) {
                build_visibility(vis, c, mrow, j0, o.n_kv, o.m_ne0, rule, vlo, vhi);
            }
            ok = mbar_wait_bounded(&s_ready[i], (uint32_t) (cnt & 1), abort_f, P.dev_err, DEVERR_TIMEOUT_MMA,
                                   P.wait_limit_ns);
            ok = __all_sync(0xffffffffu, ok);  // the collectives below need the whole warp
            if (!ok) {
                break;
            }
            tc_fence_after();
            if (fast) {
                float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (__any_sync(0xffffffffu, m_run == -INFINITY)) {
                    // some row has no max yet: classic max pass first
                    const float tmax =
                        (use_vis ? pass1_max<true>(tS, vis) : pass1_max<false>(tS, vis)) * scale_log2;
                    update_max(tmax);
                    const float m_use = m_run == -INFINITY ? 0.0f : m_run;
                    if (use_vis) {
                        pass2_exp_packed<true>(tS, vis, scale_log2, m_use, ls);
                    } else {
                        pass2_exp_packed<false>(tS, vis, scale_log2, m_use, ls);
                    }
                } else {
                    // Steady state: exponentiate against the running max while
                    // finding the tile max; P stays in registers until the max is
                    // known to have grown by at most 2^8 (else redo with the new max).
                    uint32_t    pk[64];
                    const float tmax =
                        (use_vis ? exp_tile_regs<true>(tS, vis, scale_log2, m_run, ls, pk)
                                 : exp_tile_regs<false>(tS, vis, scale_log2, m_run, ls, pk)) *
                        scale_log2;
                    if (__any_sync(0xffffffffu, tmax > m_run + kRescaleLog2)) {
                        update_max(tmax);
                        ls[0] = ls[1] = ls[2] = ls[3] = 0.0f;
                        if (use_vis) {
                            exp_tile_regs<true>(tS, vis, scale_log2, m_run, ls, pk);
                        } else {
                            exp_tile_regs<false>(tS, vis, scale_log2, m_run, ls, pk);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t part[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            part[e] = pk[16 * q + e];
                        }
                        tmem_st16(tS + 16 * q, part);
                    }
                }
                l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
            } else {
                // ---- pass 1 (general): logits in log2 units, written back
                float tmax = -INFINITY;
#pragma unroll 1
                for (int ch = 0; ch < 4; ++ch) {
                    uint32_t x[32];
                    tmem_ld32(tS + 32 * ch, x);
                    tmem_ld_wait32(x);
                    uint16_t mk[32];
                    if ((c & kClsMask) && !rule) {
                        const uint16_t *mp = mrow + j0 + 32 * ch;
                        if ((reinterpret_cast<uintptr_t>(mp) & 15u) == 0 && j0 + 32 * ch + 32 <= o.m_ne0) {
#pragma unroll
                            for (int q4 = 0; q4 < 4; ++q4) {
                                const uint4    w     = __ldg(reinterpret_cast<const uint4 *>(mp) + q4);
                                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    mk[8 * q4 + 2 * e]     = (uint16_t) (ws[e] & 0xFFFFu);
                                    mk[8 * q4 + 2 * e + 1] = (uint16_t) (ws[e] >> 16);
                                }
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                mk[e] = j0 + 32 * ch + e < o.m_ne0 ? __ldg(mp + e) : kHalfNegInf;
                            }
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        float v = __uint_as_float(x[e]) * o.scale_eff;
                        if (o.softcap != 0.0f) {
                            v = o.softcap * tanhf(v);
                        }
                        if ((c & kClsMask) && rule) {
                            // a visible key adds the rule's 0 like a 0 mask entry
                            const int jj = j0 + 32 * ch + e;
                            v            = jj >= vlo && jj < vhi ? v + 0.0f : -INFINITY;
                        } else if (c & kClsMask) {
                            const float mv = slope * __half2float(__ushort_as_half(mk[e]));
                            v              = mv == -INFINITY ? -INFINITY : v + mv;
                        }
                        if ((c & kClsBounds) && j0 + 32 * ch + e >= o.n_kv) {
                            v = -INFINITY;
                        }
                        v *= kLog2e;
                        tmax = fmaxf(tmax, v);
                        x[e] = __float_as_uint(v);
                    }
                    tmem_st32(tS + 32 * ch, x);
                }
                tmem_st_wait();
                if (!update_max(tmax)) {
                    break;
                }
                // ---- pass 2 (general): P = exp2(x - m) over the S columns
                const float m_use = m_run == -INFINITY ? 0.0f : m_run;
                float       ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t all[4] = {~0u, ~0u, ~0u, ~0u};
                pass2_exp<false>(tS, all, 1.0f, m_use, ls);
                l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_ready[i]);
            ++cnt;
        }
        // ---- epilogue: O / l
        if (ok && cnt > 0) {
            ok = mbar_wait_bounded(&o_done[i], (uint32_t) ((cnt - 1) & 1), abort_f, P.dev_err, DEVERR_TIMEOUT_MMA,
                                   P.wait_limit_ns);
            tc_fence_after();
        }
        ok = __all_sync(0xffffffffu, ok);
        if (is_part) {
            // key range of a split unit: unnormalised O, running max and row
            // sum to this range's slot; fa_dense_combine finishes the rows
            float *slot = P.part + ((int64_t) ((unit_id - P.n_full) * P.n_split + sp) * 2 + i) * dense_part_floats();
#pragma unroll 1
            for (int ch = 0; ch < HD / 32; ++ch) {
                uint32_t xo[32];
                if (ok && cnt > 0) {
                    tmem_ld32(tO + 32 * ch, xo);
                    tmem_ld_wait32(xo);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        xo[e] = 0u;
                    }
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    slot[(32 * ch + e) * kDenseBM + r] = __uint_as_float(xo[e]);
                }
            }
            const bool has = ok && cnt > 0;
            slot[128 * kDenseBM + r]            = has ? m_run : -INFINITY;
            slot[128 * kDenseBM + kDenseBM + r] = has ? l_run : 0.0f;
        } else {
        float fs = 1.0f;
        if (o.sinks && vrow) {
            const float ts = o.sinks[hq] * kLog2e;
            if (ts > m_run) {
                fs    = m_run == -INFINITY ? 0.0f : fast_exp2(m_run - ts);
                l_run = l_run * fs + 1.0f;
            } else {
                l_run += fast_exp2(ts - m_run);
            }
        }
        const float inv = l_run > 0.0f ? fs / l_run : 0.0f;
        float      *orow = vrow ? reinterpret_cast<float *>(o.dst + (int64_t) hq * o.d_nb1 + (int64_t) iq * o.d_nb2 +
                                                            (int64_t) b * o.d_nb3)
                                : nullptr;
        // Rows leave through a per-warp staging slab in this row tile's Q
        // buffer (idle once its last MMA has completed): each lane parks its
        // row's 32-float chunk, then every store instruction of the warp writes
        // four rows x 128 B, i.e. whole lines -- for the NVLink stores to the
        // mirrors as much as for HBM.  16-B chunk j of row r sits at slot
        // j ^ (r & 7), so both the parking and the read-back are conflict-free.
        const bool al16 = __all_sync(0xffffffffu, (reinterpret_cast<uintptr_t>(orow) & 15u) == 0);
        uint8_t   *stage = smem + kOffQ + i * kQBytes + wq * 8192;
        if (P.o_tma) {
            // The warp's 32 rows leave by TMA stores of 32-dim chunks, two 4 KB
            // slabs alternating (the 128-B swizzle is the slab's XOR layout);
            // rows past the node are clipped by the tensor map.
            const int row0 = (t0 + i) * kDenseBM + 32 * wq;  // first unit row of this warp
#pragma unroll 1
            for (int ch = 0; ch < HD / 32; ++ch) {
                uint32_t x[32];
                if (ok && cnt > 0) {
                    tmem_ld32(tO + 32 * ch, x);
                    tmem_ld_wait32(x);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        x[e] = 0u;
                    }
                }
                uint8_t *slab = stage + (ch & 1) * 4096;
                if (ch >= 2 && lane == 0) {
                    bulk_wait_read<1>();  // the store of chunk ch - 2 has read this slab
                }
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    *reinterpret_cast<float4 *>(slab + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(__uint_as_float(x[4 * j]) * inv, __uint_as_float(x[4 * j + 1]) * inv,
                                    __uint_as_float(x[4 * j + 2]) * inv, __uint_as_float(x[4 * j + 3]) * inv);
                }
                fence_proxy_async_smem();  // the slab is read by the async proxy
                __syncwarp();
                if (lane == 0) {
                    tma_store_4d(&omap, slab, 32 * ch, hk * o.G, row0 / o.G, b);
                    bulk_commit();
                }
            }
            if (lane == 0) {
                bulk_wait_read<0>();  // shared memory read out; the global writes complete with the grid
            }
            __syncwarp();
        } else {
        char      *rowp[8];
#pragma unroll
        for (int st = 0; st < 8; ++st) {
            rowp[st] = reinterpret_cast<char *>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(orow),
                                                            4 * st + (lane >> 3)));
        }
#pragma unroll 1
        for (int ch = 0; ch < HD / 32; ++ch) {
            uint32_t x[32];
            if (ok && cnt > 0) {
                tmem_ld32(tO + 32 * ch, x);
                tmem_ld_wait32(x);
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    x[e] = 0u;
                }
            }
            if (al16) {
                __syncwarp();  // the previous chunk's read-back is done
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    *reinterpret_cast<float4 *>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(__uint_as_float(x[4 * j]) * inv, __uint_as_float(x[4 * j + 1]) * inv,
                                    __uint_as_float(x[4 * j + 2]) * inv, __uint_as_float(x[4 * j + 3]) * inv);
                }
                __syncwarp();
                const int c = lane & 7;
#pragma unroll
                for (int st = 0; st < 8; ++st) {
                    const int    rr = 4 * st + (lane >> 3);
                    const float4 w4 = *reinterpret_cast<const float4 *>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
                    if (rowp[st]) {
                        char *dp = rowp[st] + 128 * ch + 16 * c;
                        *reinterpret_cast<float4 *>(dp) = w4;
                        for (int mi = 0; mi < o.n_mirror; ++mi) {  // peers' outputs (NVLink stores)
                            *reinterpret_cast<float4 *>(dp + o.mirror_delta[mi]) = w4;
                        }
                    }
                }
            } else if (vrow) {
                float *op = orow + 32 * ch;
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float w1 = __uint_as_float(x[e]) * inv;
                    op[e]          = w1;
                    for (int mi = 0; mi < o.n_mirror; ++mi) {
                        *reinterpret_cast<float *>(reinterpret_cast<char *>(op + e) + o.mirror_delta[mi]) = w1;
                    }
                }
            }
        }
        }
        if (o.n_mirror) {
            __threadfence_system();  // peer stores performed before the kernel retires
        }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (P.q_tma && warp == 0 && lane == 0 && !mbar_try_wait(q_full, 0u)) {
        // only after an abort: let the Q copy land before the CTA exits
        const uint64_t t_start = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0u)) {
            if (globaltimer_ns() - t_start > P.wait_limit_ns) {
                atomicCAS(P.dev_err, 0, DEVERR_TIMEOUT_DRAIN);
                break;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Merge of the key ranges of split units: one CTA per (split unit, row tile,
// 8-dim chunk), one thread per row, every load of the chunk independent.
// O = sum_k 2^(m_k - M) O_k / (sum_k 2^(m_k - M) l_k [+ sink]).
constexpr int kCombineDims = 8;

__global__ void __launch_bounds__(kDenseBM) fa_dense_combine(const __grid_constant__ DenseParams P) {
    const OpDesc &o     = P.op;
    const int     t     = blockIdx.x;  // split unit
    const int     i     = blockIdx.y;  // row tile of its pair
    const int     d0    = blockIdx.z * kCombineDims;
    const int     r     = threadIdx.x;
    const int     units = o.B * o.Hkv;
    const int     unit  = P.n_full + t;
    const int     pair  = P.head_major ? unit % P.n_pairs : P.n_pairs - 1 - unit / units;
    const int     bh    = P.head_major ? unit / P.n_pairs : unit % units;
    const int     hk    = bh % o.Hkv;
    const int     b     = bh / o.Hkv;
    const int     gr    = (2 * pair + i) * kDenseBM + r;
    pdl_wait_primary();
    if (2 * pair + i >= P.n_rt || gr >= P.rows_total) {
        return;
    }
    int iq, hq;
    row_to_query(gr, o.G, hk, iq, hq);
    const float *base = P.part + (int64_t) t * P.n_split * 2 * dense_part_floats() + (int64_t) i * dense_part_floats();
    const int64_t step = 2 * (int64_t) dense_part_floats();  // next key range of the same row tile
    float         mk[kDenseMaxSplit], lk[kDenseMaxSplit];
    float         M = -INFINITY;
#pragma unroll
    for (int k = 0; k < kDenseMaxSplit; ++k) {
        mk[k] = k < P.n_split ? __ldg(base + k * step + 128 * kDenseBM + r) : -INFINITY;
        lk[k] = k < P.n_split ? __ldg(base + k * step + 128 * kDenseBM + kDenseBM + r) : 0.0f;
        M     = fmaxf(M, mk[k]);
    }
    float L = 0.0f;
#pragma unroll
    for (int k = 0; k < kDenseMaxSplit; ++k) {
        L += mk[k] == -INFINITY ? 0.0f : lk[k] * fast_exp2(mk[k] - M);
    }
    float fs = 1.0f;
    if (o.sinks) {
        const float ts = o.sinks[hq] * kLog2e;
        if (ts > M) {
            fs = M == -INFINITY ? 0.0f : fast_exp2(M - ts);
            L  = L * fs + 1.0f;
        } else {
            L += fast_exp2(ts - M);
        }
    }
    const float inv = L > 0.0f ? fs / L : 0.0f;
    float       acc[kCombineDims];
#pragma unroll
    for (int e = 0; e < kCombineDims; ++e) {
        acc[e] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kDenseMaxSplit; ++k) {
        if (k < P.n_split && mk[k] != -INFINITY) {
            const float w = fast_exp2(mk[k] - M) * inv;
#pragma unroll
            for (int e = 0; e < kCombineDims; ++e) {
                acc[e] += __ldg(base + k * step + (int64_t) (d0 + e) * kDenseBM + r) * w;
            }
        }
    }
    char *orow = o.dst + (int64_t) hq * o.d_nb1 + (int64_t) iq * o.d_nb2 + (int64_t) b * o.d_nb3;
#pragma unroll
    for (int e = 0; e < kCombineDims; ++e) {
        char *dp                        = orow + (int64_t) (d0 + e) * o.d_nb0;
        *reinterpret_cast<float *>(dp) = acc[e];
        for (int mi = 0; mi < o.n_mirror; ++mi) {
            *reinterpret_cast<float *>(dp + o.mirror_delta[mi]) = acc[e];
        }
    }
    if (o.n_mirror) {
        __threadfence_system();
    }
}

// ---------------------------------------------------------------------------
// BF16 K/V -> contiguous F16 copies [Bk][Hkv][n_kv][D] in the caller's
// workspace, when it holds them: the dense kernel then runs its F16 instance
// instead of converting every staged tile with two warps.  The same rounding
// as those warps (bf16 -> f32 exactly, then f16 to nearest even), so either
// route gives bit-identical results.  Grid (16-B chunks of one head's rows /
// 256, Hkv * Bk, K / V); HBM-bound: 2 B read and 2 B written per value.
namespace {

struct CvtSide {
    const char *src;
    int64_t     nb1, nb2, nb3;
    uint4      *dst;
};

__global__ void __launch_bounds__(256) fa_bf16_to_f16(const CvtSide ks, const CvtSide vs, int cpr_log2, int n_kv,
                                                      int Hkv) {
    const CvtSide &sd    = blockIdx.z ? vs : ks;
    const int      hb    = (int) blockIdx.y;
    const int      h     = hb % Hkv, b = hb / Hkv;
    const int      per_h = n_kv << cpr_log2;  // chunks of one head
    const int      x     = (int) blockIdx.x * 256 + (int) threadIdx.x;
    if (x >= per_h) {
        return;
    }
    const int   j  = x >> cpr_log2, ch = x & ((1 << cpr_log2) - 1);
    const uint4 w  = __ldcs(reinterpret_cast<const uint4 *>(sd.src + (int64_t) j * sd.nb1 + (int64_t) h * sd.nb2 +
                                                           (int64_t) b * sd.nb3) + ch);
    const uint4 o4 = make_uint4(bf16x2_to_f16x2(w.x), bf16x2_to_f16x2(w.y), bf16x2_to_f16x2(w.z),
                                bf16x2_to_f16x2(w.w));
    sd.dst[(int64_t) hb * per_h + x] = o4;
}

}  // namespace

cudaError_t dense_bf16_to_f16(const OpDesc &o, uint16_t *k_dst, uint16_t *v_dst, cudaStream_t s) {
    CvtSide ks = {o.k, o.k_nb1, o.k_nb2, o.k_nb3, reinterpret_cast<uint4 *>(k_dst)};
    CvtSide vs = {o.v, o.v_nb1, o.v_nb2, o.v_nb3, reinterpret_cast<uint4 *>(v_dst)};
    const int cpr_log2 = o.D == 128 ? 4 : 3;  // 16-B chunks per row: D / 8
    const int per_h    = o.n_kv << cpr_log2;
    dim3      grid((unsigned) ((per_h + 255) / 256), (unsigned) (o.Hkv * o.Bk), 2);
    fa_bf16_to_f16<<<grid, 256, 0, s>>>(ks, vs, cpr_log2, o.n_kv, o.Hkv);
    return cudaGetLastError();
}

namespace {

template <int KVT>
cudaError_t configure_dense() {
    for (auto k : {fa_dense_kernel<false, KVT, 128>, fa_dense_kernel<true, KVT, 128>, fa_dense_kernel<false, KVT, 64>,
                   fa_dense_kernel<true, KVT, 64>}) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dense_smem_bytes<KVT>());
        if (e != cudaSuccess) {
            return e;
        }
    }
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_dense(const DenseLaunch &L, cudaStream_t s, int *launches) {
    static thread_local int configured_dev = -1;
    int                     dev            = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = configure_dense<kKvF16>();
        if (e == cudaSuccess) {
            e = configure_dense<kKvBF16>();
        }
        if (e == cudaSuccess) {
            e = configure_dense<kKvQ8>();
        }
        if (e != cudaSuccess) {
            return e;
        }
        configured_dev = dev;
    }
    int                 n = 0;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    if (L.classify) {
        cudaLaunchConfig_t c = {};
        c.gridDim            = dim3((unsigned) L.p.n_kt, (unsigned) L.p.n_rt, (unsigned) L.p.op.m_ne3);
        c.blockDim           = dim3(256);
        c.stream             = s;
        c.attrs              = attr;
        c.numAttrs           = 1;
        cudaError_t e        = cudaLaunchKernelEx(&c, fa_mask_classify, L.p);
        if (e != cudaSuccess) {
            return e;
        }
        ++n;
    }
    const int   kvt = L.p.op.kv_type == ACEFA_TYPE_Q8_0 ? kKvQ8 : (L.p.op.kv_type == ACEFA_TYPE_BF16 ? kKvBF16 : kKvF16);
    const bool  pro = L.p.op.qp.on;
    const bool  d64  = L.p.op.D == 64;
    auto        kern = d64 ? (kvt == kKvQ8    ? (pro ? fa_dense_kernel<true, kKvQ8, 64> : fa_dense_kernel<false, kKvQ8, 64>)
                              : kvt == kKvBF16 ? (pro ? fa_dense_kernel<true, kKvBF16, 64>
                                                      : fa_dense_kernel<false, kKvBF16, 64>)
                                               : (pro ? fa_dense_kernel<true, kKvF16, 64> : fa_dense_kernel<false, kKvF16, 64>))
                           : (kvt == kKvQ8    ? (pro ? fa_dense_kernel<true, kKvQ8, 128> : fa_dense_kernel<false, kKvQ8, 128>)
                              : kvt == kKvBF16 ? (pro ? fa_dense_kernel<true, kKvBF16, 128>
                                                      : fa_dense_kernel<false, kKvBF16, 128>)
                                               : (pro ? fa_dense_kernel<true, kKvF16, 128>
                                                      : fa_dense_kernel<false, kKvF16, 128>));
    const int   smem = kvt == kKvQ8 ? dense_smem_bytes<kKvQ8>()
                                    : (kvt == kKvBF16 ? dense_smem_bytes<kKvBF16>() : dense_smem_bytes<kKvF16>());
    cudaLaunchConfig_t c = {};
    c.gridDim            = dim3((unsigned) (L.p.n_full + (int64_t) L.p.n_tail * L.p.n_split));
    c.blockDim           = dim3(kThreads);
    c.dynamicSmemBytes   = (size_t) smem;
    c.stream             = s;
    c.attrs              = attr;
    c.numAttrs           = 1;
    cudaError_t e        = cudaLaunchKernelEx(&c, kern, L.p, L.kmap, L.vmap, L.qmap, L.omap);
    if (e != cudaSuccess) {
        return e;
    }
    ++n;
    if (L.p.n_tail > 0) {
        cudaLaunchConfig_t cc = {};
        cc.gridDim            = dim3((unsigned) L.p.n_tail, 2, (unsigned) (L.p.op.D / kCombineDims));
        cc.blockDim           = dim3(kDenseBM);
        cc.stream             = s;
        cc.attrs              = attr;
        cc.numAttrs           = 1;
        e                     = cudaLaunchKernelEx(&cc, fa_dense_combine, L.p);
        if (e != cudaSuccess) {
            return e;
        }
        ++n;
    }
    if (launches) {
        *launches = n;
    }
    return cudaSuccess;
}

}  // namespace acefa
