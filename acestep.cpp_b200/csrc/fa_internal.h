// fa_internal.h -- host/device shared parameter blocks of the attention kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "acefa.h"  // include/ is on the compiler include path

namespace acefa {

constexpr float kLog2e = 1.4426950408889634f;

// RMSNorm + RoPE (NEOX) of rows of D values, device form of acefa_rope_norm.
// inv_freq[k] = theta_base^(-2k/D) is computed once on the host (powf), so
// every kernel -- and the CPU oracle -- rotates by the same f32 angles
// positions[..] * inv_freq[k].
constexpr int kRopeMaxPairs = 64;  // D <= 128
struct RopeNorm {
    int            on;        // apply (a prologue was given)
    int            rope;      // rotate (theta_base != 0)
    const float   *w;         // RMSNorm weight [D], or nullptr: no RMSNorm
    const int32_t *pos;       // positions
    float          eps;
    float          inv_freq[kRopeMaxPairs];
};

// Operands after host-side validation, in ggml terms.  Strides in bytes.
struct OpDesc {
    // Q [D, n_q, Hq, B] f32
    const char *q;
    int64_t     q_nb1, q_nb2, q_nb3;
    // K/V [D, n_kv, Hkv, Bk]
    const char *k, *v;
    int64_t     k_nb1, k_nb2, k_nb3;
    int64_t     v_nb1, v_nb2, v_nb3;
    int         kv_type;  // ACEFA_TYPE_F16 / BF16 / Q8_0
    // mask [>=n_kv, >=n_q, m_ne2, m_ne3] f16 (nullptr = none)
    const char *mask;
    int64_t     m_nb1, m_nb2, m_nb3;
    int         m_ne0, m_ne2, m_ne3;
    // mask given by rule (acefa_flash_attn_ext_gen): mg_kind != 0 replaces
    // `mask` (which is then null); see acefa_mask_gen
    int     mg_kind, mg_window;
    int64_t mg_pos0[ACEFA_MASK_GEN_MAX_BATCH];
    int64_t mg_len[ACEFA_MASK_GEN_MAX_BATCH];
    // Q prologue (acefa_op_ext::q_prologue): Q rows are raw projections,
    // normalised and rotated as they are loaded; row (iq, b) has position
    // qp.pos[iq + b * n_q]
    RopeNorm qp;
    // sinks [Hq] f32 (nullptr = none)
    const float *sinks;
    // dst [D, Hq, n_q, B] f32
    char   *dst;
    int64_t d_nb0, d_nb1, d_nb2, d_nb3;
    // Mirrors: the same output also stored at dst + mirror_delta[i] (peer GPUs'
    // buffers mapped into this address space; plain stores over NVLink).
    int     n_mirror;
    int64_t mirror_delta[ACEFA_MAX_MIRRORS];
    // shapes
    int D, n_q, Hq, B, n_kv, Hkv, Bk;
    int G;    // Hq / Hkv
    int rk3;  // B / Bk
    // scalars
    float scale_eff;  // scale, divided by softcap when softcap != 0
    float softcap;
    float max_bias, alibi_m0, alibi_m1;
    int   n_head_log2;
};

// Keys visible to query iq of batch b under the mask rule (mg_kind != 0):
// [lo, hi), clipped to [0, n_kv].  lo and hi never decrease with iq, so the
// keys visible to some query of a run iq0..iq1 are [lo(iq0), hi(iq1)) and the
// keys visible to all of them [lo(iq1), hi(iq0)).  The host clamps pos0 and
// len into [-(n_q + 1), n_kv], which keeps every sum below in range.
__host__ __device__ inline void mg_range(const OpDesc &o, int b, int iq, int &lo, int &hi) {
    int64_t l = 0, h = o.n_kv;
    if (o.mg_kind == ACEFA_MASK_CAUSAL) {
        h = o.mg_pos0[b] + iq + 1;
    } else if (o.mg_kind == ACEFA_MASK_WINDOW) {
        l = (int64_t) iq - o.mg_window;
        h = (int64_t) iq + o.mg_window + 1;
    } else {
        h = o.mg_len[b];
    }
    l  = l < 0 ? 0 : (l > o.n_kv ? o.n_kv : l);
    h  = h < 0 ? 0 : (h > o.n_kv ? o.n_kv : h);
    lo = (int) l;
    hi = (int) h;
}

__host__ __device__ inline float alibi_slope(const OpDesc &o, int h) {
    if (o.max_bias <= 0.0f) {
        return 1.0f;
    }
#ifdef __CUDA_ARCH__
    return h < o.n_head_log2 ? powf(o.alibi_m0, (float) (h + 1)) : powf(o.alibi_m1, (float) (2 * (h - o.n_head_log2) + 1));
#else
    return h < o.n_head_log2 ? powf(o.alibi_m0, (float) (h + 1)) : powf(o.alibi_m1, (float) (2 * (h - o.n_head_log2) + 1));
#endif
}

// ------------------------------------------------------------------ decode
// The split-KV decode kernel works on "units" (batch b, kv head hk, row block
// rb); a unit's rows are the G*n_q (query, head) pairs that share one K/V head,
// 16 at a time.  Its keys are cut into tiles of kDecBN positions.  A unit runs
// on one thread-block cluster of `cluster` CTAs, each streaming a contiguous
// range of the unit's tiles; the CTAs merge their partial results through
// distributed shared memory, so the op is one launch and needs no workspace.
constexpr int kDecBN         = 64;  // keys per pipeline stage
constexpr int kDecWarps      = 4;   // consumer warps (16 keys each per stage)
constexpr int kDecStages     = 3;   // pipeline depth
constexpr int kDecRows       = 16;  // rows per unit (one m16 MMA tile)
constexpr int kDecMaxCluster = 16;  // CTAs per unit (16 needs the non-portable cluster size)

// Rows per unit: one m16 MMA tile for F16/BF16; one n8 tile of the transposed
// Q8_0 consumer.
__host__ __device__ constexpr int decode_unit_rows(int kv_type) { return kv_type == ACEFA_TYPE_Q8_0 ? 8 : kDecRows; }

struct DecodeParams {
    OpDesc  op;
    int     n_rb;            // row blocks per (b, hk)
    int     units;           // B * Hkv * n_rb
    int     tiles_per_unit;  // ceil(n_kv / kDecBN)
    int     cluster;         // CTAs per unit (grid = units * cluster)
    int     wide;            // Q8_0: the three-CTAs-per-SM instance (decode_wide)
    // Fused KV-cache append (acefa_flash_attn_ext_append), or all null: the
    // new K/V row of (kv head h, set s) is f32 at k_new + h*kn_nb2 + s*kn_nb3
    // and goes into cache row append_pos[s] before that row is read.
    const char    *k_new, *v_new;
    int64_t        kn_nb2, kn_nb3, vn_nb2, vn_nb3;
    const int64_t *append_pos;
    RopeNorm       kp;  // prologue of the new K row (position kp.pos[set])
    int    *dev_err;
    uint64_t wait_limit_ns;
};

struct DecodeLaunch {
    DecodeParams p;
    CUtensorMap  kmap, vmap;  // F16/BF16 tiles via TMA (unused for Q8_0)
};

cudaError_t launch_decode(const DecodeLaunch &L, cudaStream_t s, int *launches);
// CTAs per unit for the decode kernel of these operands on the current
// device: the largest size (<= kDecMaxCluster, <= the unit's key tiles)
// whose clusters for all `units` are resident at once; 1 otherwise.
int         decode_cluster(int kv_type, int D, bool prologue, int units, int tiles_per_unit, bool wide);
// Q8_0 ops of at least kDecWideUnits units of at least kDecWideTiles key tiles
// run three CTAs per SM (measured crossovers: 16 sets x 8 heads gain from 1280
// keys on; 8 sets, 2 sets and shorter windows lose to the shallower pipeline)
constexpr int kDecWideTiles = 20;
constexpr int kDecWideUnits = 128;
inline bool   decode_wide(int kv_type, int D, int tiles_per_unit, int units) {
    return kv_type == ACEFA_TYPE_Q8_0 && D == 128 && tiles_per_unit >= kDecWideTiles && units >= kDecWideUnits;
}

// ------------------------------------------------------------------ dense
// tcgen05 kernel for query-heavy nodes (LM prefill, DiT self/cross, encoders):
// a CTA owns two 128-row tiles of one (batch, kv head) unit and streams the
// unit's 128-key tiles through tensor memory.
constexpr int kDenseBM    = 128;  // rows per row tile (MMA M)
constexpr int kDenseBN    = 128;  // keys per key tile (MMA N of S)
constexpr int kDenseMaxKT = 512;  // key tiles the class table holds (n_kv <= 65536)

// mask tile classes
constexpr uint8_t kClsLive   = 1;  // some key of the tile is visible to some row
constexpr uint8_t kClsMask   = 2;  // entries other than 0 present: read the mask
constexpr uint8_t kClsBounds = 4;  // tile runs past n_kv
constexpr uint8_t kClsBinary = 8;  // every mask entry of the tile is 0 or -inf

// Work units are (row-tile pair, batch, kv head), numbered pair-major from
// the heaviest pair (head-major for unmasked nodes).  The first n_full units
// run whole, one CTA each; when the last wave would leave most SMs idle, each
// of the n_tail remaining units is cut into n_split key ranges run by
// separate CTAs, which write unnormalised partial results (O, running max,
// row sum) that fa_dense_combine merges.
struct DenseParams {
    OpDesc         op;
    int            rows_total;  // G * n_q rows per (b, hk) unit
    int            n_rt;        // 128-row tiles per unit
    int            n_pairs;     // row-tile pairs per unit
    int            n_kt;        // key tiles
    int            n_full;      // units run whole
    int            n_tail;      // units split over key ranges
    int            n_split;     // key ranges per split unit (1 = none)
    int            head_major;  // units numbered (batch, kv head) slowest: a head's pairs run together
    const uint8_t *cls;         // [m_ne3][n_rt][n_kt] classes, or nullptr (no per-tile info)
    uint8_t       *cls_out;     // same buffer, written by the classify pre-pass
    float         *part;        // [n_tail][n_split][2 tiles] partial slots (dense_part_floats each)
    int           *dev_err;
    uint64_t       wait_limit_ns;
    int            q_tma;       // Q rows staged by TMA (qmap) instead of per-thread loads
    int            o_tma;       // output rows leave by TMA stores (omap) instead of per-lane stores
};

constexpr int kDenseMaxSplit = 8;  // key ranges per split unit

// One partial slot: O [128 dims][128 rows] (row fastest), then m[128], l[128].
constexpr int dense_part_floats() { return 128 * kDenseBM + 2 * kDenseBM; }

struct DenseLaunch {
    DenseParams p;
    CUtensorMap kmap, vmap;  // box {64, 128, 1, 1}, 128-B swizzle
    CUtensorMap qmap;        // f32 Q rows of one row tile (when p.q_tma)
    CUtensorMap omap;        // f32 output: 32 dims x 32 unit rows, 128-B swizzle (when p.o_tma)
    bool        classify;    // run the mask-classification pre-pass
};

cudaError_t launch_dense(const DenseLaunch &L, cudaStream_t s, int *launches);

// BF16 K/V of `o` -> contiguous F16 copies [Bk][Hkv][n_kv][D] (one launch).
cudaError_t dense_bf16_to_f16(const OpDesc &o, uint16_t *k_dst, uint16_t *v_dst, cudaStream_t s);

// ------------------------------------------------------------------ workspace
// Bytes of workspace the operator needs when it is offered at most `limit`
// (acefa_workspace_bytes is limit = SIZE_MAX); 0 for unsupported operands.
size_t workspace_bytes_within(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                              const acefa_tensor *mask, const acefa_tensor *dst, size_t limit);

// ------------------------------------------------------------------ K/V prologue
int kv_prologue_launch(const acefa_tensor *k_src, const acefa_tensor *v_src, const acefa_tensor *k_dst,
                       const acefa_tensor *v_dst, const RopeNorm &kp, int sm_count, cudaStream_t stream);

// ------------------------------------------------------------------ CFG logit combine
// Launch for arguments validated by acefa_cfg_logit_combine (fa_api.cu).
int cfg_combine_launch(const float *cond, const float *uncond, int64_t row_stride, int n, int eos_idx,
                       int code_offset, int cols, float cfg_scale, float *compact, cudaStream_t stream);

}  // namespace acefa
