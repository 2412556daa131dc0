// fa_api.cu -- the C ABI (include/acefa.h): operand validation in ggml terms,
// workspace sizing, TMA descriptor encoding and kernel dispatch.
//
// Mirrors what ggml's CUDA backend does for GGML_OP_FLASH_ATTN_EXT
// (supports_op check, then ggml_cuda_flash_attn_ext(ctx, dst) reading
// dst->src[0..4] and dst->op_params {scale, max_bias, logit_softcap}) without any
// ggml type in the signature.  Status codes replace ggml's GGML_ABORT.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "fa_internal.h"
#include "ptx.cuh"

namespace acefa {

__device__ int g_dev_err;  // device-side failure word (see DEVERR_*)

namespace {

thread_local int t_last_launches = 0;
thread_local int t_last_path     = 0;

constexpr int kMaxDevices = 64;

struct DevInfo {
    int               sm_count = 0;
    int               cc_major = 0, cc_minor = 0;
    int              *err_ptr  = nullptr;
    std::atomic<bool> ready{false};  // set once the fields above are filled
};
DevInfo    g_dev[kMaxDevices];  // per-device properties, immutable once ready
std::mutex g_dev_mutex;         // serialises the one-time fill

int dev_info(DevInfo **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        return ACEFA_ERR_CUDA;
    }
    DevInfo &d = g_dev[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_dev_mutex);
        if (!d.ready.load(std::memory_order_relaxed)) {  // retried on a later call if it fails
            int   sm = 0, major = 0, minor = 0;
            void *p  = nullptr;
            if (cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
                cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) {
                return ACEFA_ERR_CUDA;
            }
            d.sm_count = sm;
            d.cc_major = major;
            d.cc_minor = minor;
            d.err_ptr  = static_cast<int *>(p);
            d.ready.store(true, std::memory_order_release);
        }
    }
    if (d.cc_major != 10 || d.cc_minor != 0) {
        return ACEFA_ERR_DEVICE;
    }
    *out = &d;
    return ACEFA_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = [] {  // thread-safe one-time lookup
        void                           *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            return reinterpret_cast<EncodeTiledFn>(p);
        }
        return static_cast<EncodeTiledFn>(nullptr);
    }();
    return fn;
}

uint64_t wait_limit_ns() {
    static const uint64_t lim = [] {
        const char *e  = std::getenv("ACEFA_WAIT_LIMIT_MS");
        long        ms = e ? std::atol(e) : 0;
        return (ms > 0 ? (uint64_t) ms : 1000ull) * 1000000ull;
    }();
    return lim;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------------ validation
struct Checked {
    OpDesc op;
    int    status;
};

Checked check_operands(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                       const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst) {
    Checked r;
    std::memset(&r.op, 0, sizeof(r.op));
    r.status = ACEFA_OK;
    auto fail = [&](int s) {
        r.status = s;
        return r;
    };
    if (!q || !k || !v || !dst || !q->data || !k->data || !v->data || !dst->data) {
        return fail(ACEFA_ERR_NULL);
    }
    if (q->type != ACEFA_TYPE_F32 || dst->type != ACEFA_TYPE_F32) {
        return fail(ACEFA_ERR_TYPE);
    }
    if (k->type != ACEFA_TYPE_F16 && k->type != ACEFA_TYPE_BF16 && k->type != ACEFA_TYPE_Q8_0) {
        return fail(ACEFA_ERR_TYPE);
    }
    if (v->type != k->type) {
        return fail(ACEFA_ERR_TYPE);
    }
    for (int i = 0; i < 4; ++i) {
        if (q->ne[i] <= 0 || k->ne[i] <= 0 || v->ne[i] <= 0 || dst->ne[i] <= 0) {
            return fail(ACEFA_ERR_SHAPE);
        }
    }
    const int64_t D = q->ne[0], n_q = q->ne[1], Hq = q->ne[2], B = q->ne[3];
    const int64_t n_kv = k->ne[1], Hkv = k->ne[2], Bk = k->ne[3];
    if (k->ne[0] != D || v->ne[0] != D || v->ne[1] != n_kv || v->ne[2] != Hkv || v->ne[3] != Bk) {
        return fail(ACEFA_ERR_SHAPE);
    }
    if (Hq % Hkv != 0 || B % Bk != 0) {
        return fail(ACEFA_ERR_SHAPE);
    }
    if (dst->ne[0] != D || dst->ne[1] != Hq || dst->ne[2] != n_q || dst->ne[3] != B) {
        return fail(ACEFA_ERR_SHAPE);
    }
    if (D != 64 && D != 128 && D != 256) {
        return fail(ACEFA_ERR_SHAPE);
    }
    if (D == 256 && k->type == ACEFA_TYPE_Q8_0) {
        return fail(ACEFA_ERR_TYPE);  // D = 256 serves F16 and BF16 K/V
    }
    if (n_kv > (1ll << 30) || n_q > (1ll << 30) || Hq > 4096 || B > (1ll << 20) ||
        (Hq / Hkv) * n_q > (1ll << 30)) {
        return fail(ACEFA_ERR_SHAPE);
    }
    if (mask) {
        if (!mask->data) {
            return fail(ACEFA_ERR_NULL);
        }
        if (mask->type != ACEFA_TYPE_F16) {
            return fail(ACEFA_ERR_TYPE);
        }
        if (mask->ne[0] < n_kv || mask->ne[1] < n_q || mask->ne[2] <= 0 || mask->ne[3] <= 0 ||
            Hq % mask->ne[2] != 0 || B % mask->ne[3] != 0) {
            return fail(ACEFA_ERR_SHAPE);
        }
        if (mask->nb[0] != 2 || mask->nb[1] % 2 || mask->nb[2] % 2 || mask->nb[3] % 2 || !aligned(mask->data, 2)) {
            return fail(ACEFA_ERR_LAYOUT);
        }
    }
    if (sinks) {
        if (!sinks->data) {
            return fail(ACEFA_ERR_NULL);
        }
        if (sinks->type != ACEFA_TYPE_F32) {
            return fail(ACEFA_ERR_TYPE);
        }
        if (sinks->ne[0] < Hq || sinks->nb[0] != 4 || !aligned(sinks->data, 4)) {
            return fail(ACEFA_ERR_SHAPE);
        }
    }
    // Q: f32 elements contiguous along D
    if (q->nb[0] != 4 || q->nb[1] % 4 || q->nb[2] % 4 || q->nb[3] % 4 || !aligned(q->data, 4)) {
        return fail(ACEFA_ERR_LAYOUT);
    }
    if (dst->nb[0] != 4 || dst->nb[1] % 4 || dst->nb[2] % 4 || dst->nb[3] % 4 || !aligned(dst->data, 4)) {
        return fail(ACEFA_ERR_LAYOUT);
    }
    // K/V: the streaming kernels need 16-B aligned rows and head/batch strides
    for (const acefa_tensor *t : {k, v}) {
        if (!aligned(t->data, 16)) {
            return fail(ACEFA_ERR_LAYOUT);
        }
        if (t->type == ACEFA_TYPE_Q8_0) {
            if (D % 32 || t->nb[0] != 34 || t->nb[1] != (size_t) (D / 32 * 34)) {
                return fail(ACEFA_ERR_LAYOUT);
            }
        } else {
            if (t->nb[0] != 2 || t->nb[1] % 16 || t->nb[1] < (size_t) (2 * D)) {
                return fail(ACEFA_ERR_LAYOUT);
            }
        }
        // F16/BF16 go through TMA tensor maps (16-B strides); Q8_0 tiles are
        // copied from the 16-B boundary below them, so even strides suffice.
        const size_t sa = t->type == ACEFA_TYPE_Q8_0 ? 2 : 16;
        if ((t->ne[2] > 1 && t->nb[2] % sa) || (t->ne[3] > 1 && t->nb[3] % sa)) {
            return fail(ACEFA_ERR_LAYOUT);
        }
    }

    OpDesc &o = r.op;
    o.q       = static_cast<const char *>(q->data);
    o.q_nb1 = q->nb[1], o.q_nb2 = q->nb[2], o.q_nb3 = q->nb[3];
    o.k = static_cast<const char *>(k->data), o.v = static_cast<const char *>(v->data);
    o.k_nb1 = k->nb[1], o.k_nb2 = k->nb[2], o.k_nb3 = k->nb[3];
    o.v_nb1 = v->nb[1], o.v_nb2 = v->nb[2], o.v_nb3 = v->nb[3];
    o.kv_type = k->type;
    if (mask) {
        o.mask  = static_cast<const char *>(mask->data);
        o.m_nb1 = mask->nb[1], o.m_nb2 = mask->nb[2], o.m_nb3 = mask->nb[3];
        o.m_ne0 = (int) mask->ne[0], o.m_ne2 = (int) mask->ne[2], o.m_ne3 = (int) mask->ne[3];
    } else {
        o.m_ne2 = o.m_ne3 = 1;
    }
    o.sinks = sinks ? static_cast<const float *>(sinks->data) : nullptr;
    o.dst   = static_cast<char *>(dst->data);
    o.d_nb0 = dst->nb[0], o.d_nb1 = dst->nb[1], o.d_nb2 = dst->nb[2], o.d_nb3 = dst->nb[3];
    o.D = (int) D, o.n_q = (int) n_q, o.Hq = (int) Hq, o.B = (int) B;
    o.n_kv = (int) n_kv, o.Hkv = (int) Hkv, o.Bk = (int) Bk;
    o.G   = (int) (Hq / Hkv);
    o.rk3 = (int) (B / Bk);
    return r;
}

void set_scalars(OpDesc &o, float scale, float max_bias, float softcap) {
    o.softcap   = softcap;
    o.scale_eff = softcap != 0.0f ? scale / softcap : scale;
    o.max_bias  = max_bias;
    const int n_head_log2 = 1 << (int) std::floor(std::log2((float) o.Hq));
    o.n_head_log2         = n_head_log2;
    o.alibi_m0            = std::pow(2.0f, -(max_bias) / (float) n_head_log2);
    o.alibi_m1            = std::pow(2.0f, -(max_bias / 2.0f) / (float) n_head_log2);
}

// ------------------------------------------------------------------ decode plan
// A unit (batch, kv head, 16-row block) runs on a cluster of C CTAs that split
// its keys and merge through distributed shared memory.  C is the largest
// size (<= 16, <= the unit's key tiles) for which the device keeps every
// unit's cluster resident at once, so the op runs in one wave -- and above 6
// only while every CTA has an SM to itself; units beyond that run one CTA
// each.  A function of shapes and the device only.
struct DecodePlan {
    int  n_rb, units, tpu, cluster;
    bool wide;
};

DecodePlan plan_decode(const OpDesc &o, bool prologue) {
    DecodePlan p;
    const int rows = o.G * o.n_q;
    const int R    = decode_unit_rows(o.kv_type);
    p.n_rb         = (rows + R - 1) / R;
    p.units        = o.B * o.Hkv * p.n_rb;
    p.tpu          = (o.n_kv + kDecBN - 1) / kDecBN;
    p.wide         = decode_wide(o.kv_type, o.D, p.tpu, p.units);
    p.cluster      = decode_cluster(o.kv_type, o.D, prologue, p.units, p.tpu, p.wide);
    return p;
}

// ------------------------------------------------------------------ dense plan
// The dense tcgen05 kernel serves D = 64 and 128 (F16, BF16 or Q8_0 K/V) when a K/V
// head has more than 64 rows of queries (G * n_q) -- prefill, encoders, DiT.  A
// function of shapes only, so the choice (and the workspace) is fixed before
// capture.
bool use_dense(const OpDesc &o) {
    const int64_t rows = (int64_t) o.G * o.n_q;
    const int64_t n_kt = ((int64_t) o.n_kv + kDenseBN - 1) / kDenseBN;
    const int64_t n_pairs = ((rows + kDenseBM - 1) / kDenseBM + 1) / 2;
    return (o.D == 128 || o.D == 64) && rows > 64 && n_kt <= kDenseMaxKT && n_pairs * o.Hkv * o.B < (1ll << 31);
}

struct DensePlan {
    int    rows_total, n_rt, n_pairs, n_kt;
    int    n_full, n_tail, n_split;
    bool   classify;
    size_t cls_bytes;   // class table at the start of the workspace (256-B aligned)
    size_t conv_bytes;  // F16 copies of BF16 K/V at the end of the workspace, or 0
    size_t ws_bytes;
};

// One CTA per SM at a time.  The units that do not fill a whole last wave
// ("tail") may be cut into key ranges run by separate CTAs and merged by
// fa_dense_combine, so that the last wave ends sooner.  The split is chosen by
// the estimated duration of that wave, in key-tile steps of one CTA: a CTA's
// fixed cost (launch, Q conversion, output stores) measured ~5.6 steps and the
// merge ~1.3 (per-CTA %globaltimer stamps on B200).  Only for unmasked nodes
// (every unit the same work; a causal mask's heavy-first order already packs
// the last wave), at most 8 ranges of at least 8 key tiles (shorter ranges
// measured slower than no split: DiT S = 1500, 3 ranges of 4 tiles, -7 %),
// the ranges of the tail within one wave, and the partial results within the
// caller's workspace.  A function of shapes, the SM count and the workspace
// size.
DensePlan plan_dense(const OpDesc &o, int sm_count, size_t ws_limit) {
    constexpr double kFixedSteps = 5.6, kMergeSteps = 1.3;
    DensePlan p;
    p.rows_total = o.G * o.n_q;
    p.n_rt       = (p.rows_total + kDenseBM - 1) / kDenseBM;
    p.n_pairs    = (p.n_rt + 1) / 2;
    p.n_kt       = (o.n_kv + kDenseBN - 1) / kDenseBN;
    // per-tile classes need one mask row per query: a mask shared by all heads
    p.classify          = o.mask != nullptr && o.m_ne2 == 1;
    size_t b            = p.classify ? (size_t) o.m_ne3 * p.n_rt * p.n_kt : 0;
    p.cls_bytes         = (b + 255) / 256 * 256;
    const int64_t units = (int64_t) p.n_pairs * o.B * o.Hkv;
    const int64_t sms   = sm_count > 0 ? sm_count : 1;
    const int64_t tail  = units % sms;
    auto part_bytes     = [&](int64_t split) {
        return (size_t) tail * (size_t) split * 2 * dense_part_floats() * sizeof(float);
    };
    int64_t split = 1;
    if (o.mask == nullptr && o.mg_kind == 0 && tail > 0) {
        double best = kFixedSteps + (double) p.n_kt;
        for (int64_t sp = 2; sp <= kDenseMaxSplit && tail * sp <= sms && p.n_kt / sp >= 8; ++sp) {
            if (p.cls_bytes + part_bytes(sp) > ws_limit) {
                break;
            }
            const double t = kMergeSteps + kFixedSteps + (double) ((p.n_kt + sp - 1) / sp);
            if (t < best) {
                best  = t;
                split = sp;
            }
        }
    }
    p.n_split  = (int) split;
    p.n_tail   = split > 1 ? (int) tail : 0;
    p.n_full   = (int) (units - p.n_tail);
    p.ws_bytes = p.cls_bytes + (split > 1 ? (part_bytes(split) + 255) / 256 * 256 : 0);
    // BF16 K/V: F16 copies made by one conversion pass when they fit the
    // offer (the kernel's converter warps otherwise)
    p.conv_bytes = 0;
    if (o.kv_type == ACEFA_TYPE_BF16) {
        const size_t conv = ((size_t) 2 * o.Bk * o.Hkv * o.n_kv * o.D * 2 + 255) / 256 * 256;
        if (p.ws_bytes + conv <= ws_limit && (int64_t) o.n_kv * (o.D / 8) < (1ll << 31)) {
            p.conv_bytes = conv;
            p.ws_bytes += conv;
        }
    }
    if (p.ws_bytes == 0) {
        p.ws_bytes = 256;
    }
    return p;
}

int encode_kv_map(CUtensorMap *map, const acefa_tensor *t, int D, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        return ACEFA_ERR_CUDA;
    }
    cuuint64_t dims[4]    = {(cuuint64_t) D, (cuuint64_t) t->ne[1], (cuuint64_t) t->ne[2], (cuuint64_t) t->ne[3]};
    cuuint64_t s1         = t->nb[1];
    cuuint64_t s2         = t->ne[2] > 1 ? t->nb[2] : s1 * (cuuint64_t) t->ne[1];
    cuuint64_t s3         = t->ne[3] > 1 ? t->nb[3] : s2 * (cuuint64_t) t->ne[2];
    cuuint64_t strides[3] = {s1, s2, s3};
    cuuint32_t box[4]     = {64, (cuuint32_t) box_rows, 1, 1};
    cuuint32_t estr[4]    = {1, 1, 1, 1};
    CUresult   rc = enc(map, t->type == ACEFA_TYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        4, t->data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return rc == CUDA_SUCCESS ? ACEFA_OK : ACEFA_ERR_LAYOUT;
}

// f32 Q rows of one 128-row tile of a unit, for the dense kernel's TMA:
// unit row r of kv head hk is query r / G of head hk * G + r % G, so the box
// is {D dims, G heads, 128 / G queries, 1 batch} over dims ordered (dim,
// head, query, batch) -- it lands in shared memory as 128 rows of D floats in
// unit-row order.  Returns false (per-thread loads instead) when the layout
// does not fit a tensor map: 16-B aligned base and strides, 128 % G == 0.
bool encode_q_map(CUtensorMap *map, const acefa_tensor *q, int D, int G) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || q->type != ACEFA_TYPE_F32 || q->nb[0] != 4 || G <= 0 || kDenseBM % G != 0 ||
        (reinterpret_cast<uintptr_t>(q->data) & 15u) != 0) {
        return false;
    }
    const cuuint64_t nq = (cuuint64_t) q->ne[1], nh = (cuuint64_t) q->ne[2], nb = (cuuint64_t) q->ne[3];
    // strides of extent-1 dimensions do not matter; keep them 16-B multiples
    const cuuint64_t sq = nq > 1 ? (cuuint64_t) q->nb[1] : 16u * ((4u * (cuuint64_t) D + 15u) / 16u);
    const cuuint64_t sh = nh > 1 ? (cuuint64_t) q->nb[2] : sq * nq;
    const cuuint64_t sb = nb > 1 ? (cuuint64_t) q->nb[3] : sh * nh + sq * nq;
    if ((sq | sh | sb) & 15u) {
        return false;
    }
    cuuint64_t dims[4]    = {(cuuint64_t) D, nh, nq, nb};
    cuuint64_t strides[3] = {sh, sq, sb};
    cuuint32_t box[4]     = {(cuuint32_t) D, (cuuint32_t) G, (cuuint32_t) (kDenseBM / G), 1};
    cuuint32_t estr[4]    = {1, 1, 1, 1};
    CUresult   rc = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, q->data, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return rc == CUDA_SUCCESS;
}

// The f32 output rows of 32 unit rows x 32 dims, for the dense kernel's TMA
// stores: dst [D, Hq, n_q, B] ordered (dim, head, query, batch), box {32, G,
// 32 / G, 1} with the 128-B swizzle of the kernel's per-warp staging slab.
// Returns false (per-lane stores instead) when the layout does not fit a
// tensor map: 16-B aligned base and strides, 32 % G == 0, or mirrors (peer
// buffers) to store into as well.
bool encode_o_map(CUtensorMap *map, const acefa_tensor *d, int D, int G, int n_mirror) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || n_mirror != 0 || d->type != ACEFA_TYPE_F32 || d->nb[0] != 4 || G <= 0 || 32 % G != 0 ||
        (reinterpret_cast<uintptr_t>(d->data) & 15u) != 0) {
        return false;
    }
    const cuuint64_t nh = (cuuint64_t) d->ne[1], nq = (cuuint64_t) d->ne[2], nb = (cuuint64_t) d->ne[3];
    const cuuint64_t sh = nh > 1 ? (cuuint64_t) d->nb[1] : 16u * ((4u * (cuuint64_t) D + 15u) / 16u);
    const cuuint64_t sq = nq > 1 ? (cuuint64_t) d->nb[2] : sh * nh;
    const cuuint64_t sb = nb > 1 ? (cuuint64_t) d->nb[3] : sq * nq + sh * nh;
    if ((sh | sq | sb) & 15u) {
        return false;
    }
    cuuint64_t dims[4]    = {(cuuint64_t) D, nh, nq, nb};
    cuuint64_t strides[3] = {sh, sq, sb};
    cuuint32_t box[4]     = {32, (cuuint32_t) G, (cuuint32_t) (32 / G), 1};
    cuuint32_t estr[4]    = {1, 1, 1, 1};
    CUresult   rc = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d->data, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return rc == CUDA_SUCCESS;
}

}  // namespace
}  // namespace acefa

using namespace acefa;

// Copies a mask rule into the operand block.  pos0 and len are clamped into
// [-(n_q + 1), n_kv]: for keys 0 .. n_kv-1 and queries 0 .. n_q-1 that keeps
// every visibility decision and bounds the device-side sums.
static int rc_of_rule(OpDesc &o, const acefa_mask_gen *mg) {
    const bool per_batch = mg->kind == ACEFA_MASK_CAUSAL || mg->kind == ACEFA_MASK_PADDING;
    if ((!per_batch && mg->kind != ACEFA_MASK_WINDOW) || (per_batch && o.B > ACEFA_MASK_GEN_MAX_BATCH) ||
        (mg->kind == ACEFA_MASK_WINDOW && mg->window < 0)) {
        return ACEFA_ERR_SHAPE;
    }
    o.mg_kind   = mg->kind;
    o.mg_window = mg->window;
    const int64_t lo = -((int64_t) o.n_q + 1), hi = o.n_kv;
    for (int b = 0; b < ACEFA_MASK_GEN_MAX_BATCH; ++b) {
        const bool in = per_batch && b < o.B;
        o.mg_pos0[b]  = in ? std::min(std::max(mg->pos0[b], lo), hi) : 0;
        o.mg_len[b]   = in ? std::min(std::max(mg->len[b], lo), hi) : 0;
    }
    return ACEFA_OK;
}

// New K/V rows of a fused KV-cache append.
struct AppendArgs {
    const char    *k_new, *v_new;
    int64_t        kn_nb2, kn_nb3, vn_nb2, vn_nb3;
    const int64_t *pos;
};

// RMSNorm + RoPE parameters for the kernels.  inv_freq[k] = theta_base^(-2k/D)
// is computed here, once, with the C library's powf.
static int fill_rope_norm(RopeNorm &r, const acefa_rope_norm *p, int D) {
    std::memset(&r, 0, sizeof(r));
    if (!p) {
        return ACEFA_OK;
    }
    if (!std::isfinite(p->eps) || p->eps < 0.0f || !std::isfinite(p->theta_base) || p->theta_base < 0.0f ||
        D / 2 > kRopeMaxPairs || D % 64) {
        return ACEFA_ERR_SHAPE;
    }
    if (p->theta_base > 0.0f && !p->positions) {
        return ACEFA_ERR_NULL;
    }
    if (!aligned(p->norm_weight, 4) || !aligned(p->positions, 4)) {
        return ACEFA_ERR_LAYOUT;
    }
    r.on   = 1;
    r.rope = p->theta_base > 0.0f;
    r.w    = p->norm_weight;
    r.pos  = p->positions;
    r.eps  = p->eps;
    for (int k = 0; k < D / 2; ++k) {
        r.inv_freq[k] = r.rope ? std::pow(p->theta_base, -(float) (2 * k) / (float) D) : 0.0f;
    }
    return ACEFA_OK;
}

// The operator with any of the fusions of acefa_op_ext.
static int run_op(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v, const acefa_tensor *mask,
                  const acefa_tensor *sinks, const acefa_tensor *dst, float scale, float max_bias,
                  float logit_softcap, int prec, const acefa_op_ext *ext, void *stream, void *workspace,
                  size_t workspace_bytes) {
    (void) prec;  // accumulation is F32 for both GGML_PREC_DEFAULT and GGML_PREC_F32
    static const acefa_op_ext kNone = {};
    const acefa_op_ext       &x     = ext ? *ext : kNone;
    Checked c = check_operands(q, k, v, mask, sinks, dst);
    if (c.status != ACEFA_OK) {
        return c.status;
    }
    if (x.mask_gen && (mask || rc_of_rule(c.op, x.mask_gen) != ACEFA_OK)) {
        return ACEFA_ERR_SHAPE;
    }
    if (!std::isfinite(scale) || !std::isfinite(max_bias) || !std::isfinite(logit_softcap) || max_bias < 0.0f) {
        return ACEFA_ERR_SHAPE;
    }
    int rc = fill_rope_norm(c.op.qp, x.q_prologue, c.op.D);
    if (rc != ACEFA_OK) {
        return rc;
    }
    // fused KV append: new rows [D, 1, Hkv, Bk] f32, one cache row per set
    AppendArgs        app_args{};
    const AppendArgs *app = nullptr;
    RopeNorm          kp;
    if (x.k_new || x.v_new || x.append_pos) {
        const acefa_tensor *kn = x.k_new, *vn = x.v_new;
        if (!kn || !vn || !x.append_pos || !kn->data || !vn->data) {
            return ACEFA_ERR_NULL;
        }
        if (kn->type != ACEFA_TYPE_F32 || vn->type != ACEFA_TYPE_F32) {
            return ACEFA_ERR_TYPE;
        }
        if (c.op.D > 128) {
            return ACEFA_ERR_SHAPE;  // one warp lane holds four values of the new row
        }
        for (const acefa_tensor *t : {kn, vn}) {
            if (t->ne[0] != k->ne[0] || t->ne[1] != 1 || t->ne[2] != k->ne[2] || t->ne[3] != k->ne[3]) {
                return ACEFA_ERR_SHAPE;
            }
            if (t->nb[0] != 4 || t->nb[2] % 4 || t->nb[3] % 4 || !aligned(t->data, 4)) {
                return ACEFA_ERR_LAYOUT;
            }
        }
        app_args = AppendArgs{static_cast<const char *>(kn->data), static_cast<const char *>(vn->data),
                              (int64_t) kn->nb[2], (int64_t) kn->nb[3], (int64_t) vn->nb[2], (int64_t) vn->nb[3],
                              x.append_pos};
        app      = &app_args;
    } else if (x.k_prologue) {
        return ACEFA_ERR_SHAPE;  // the K prologue applies to the appended row
    }
    if ((rc = fill_rope_norm(kp, x.k_prologue, c.op.D)) != ACEFA_OK) {
        return rc;
    }
    void *const *mirrors   = x.mirrors;
    const int    n_mirrors = x.n_mirrors;
    if (n_mirrors < 0 || n_mirrors > ACEFA_MAX_MIRRORS || (n_mirrors > 0 && !mirrors)) {
        return n_mirrors > 0 && !mirrors ? ACEFA_ERR_NULL : ACEFA_ERR_SHAPE;
    }
    for (int i = 0; i < n_mirrors; ++i) {
        if (!mirrors[i]) {
            return ACEFA_ERR_NULL;
        }
        const int64_t delta = static_cast<int64_t>(reinterpret_cast<uintptr_t>(mirrors[i]) -
                                                   reinterpret_cast<uintptr_t>(dst->data));
        if (delta % 16 != 0 || delta == 0) {
            return ACEFA_ERR_LAYOUT;
        }
        c.op.mirror_delta[i] = delta;
    }
    c.op.n_mirror = n_mirrors;
    DevInfo *di = nullptr;
    if ((rc = dev_info(&di)) != ACEFA_OK) {
        return rc;
    }
    set_scalars(c.op, scale, max_bias, logit_softcap);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    if (use_dense(c.op)) {
        if (app) {
            return ACEFA_ERR_SHAPE;  // the fused append serves the decode path (one new row per set)
        }
        const DensePlan dp = plan_dense(c.op, di->sm_count, workspace_bytes);
        if (workspace_bytes < dp.ws_bytes || !workspace || !aligned(workspace, 256)) {
            return ACEFA_ERR_WORKSPACE;
        }
        acefa_tensor kc, vc;  // the F16 copies of BF16 K/V, when the plan makes them
        int          pre = 0;
        if (dp.conv_bytes) {
            const size_t per = dp.conv_bytes / 2 / 256 * 256;
            uint16_t *kd = reinterpret_cast<uint16_t *>(static_cast<char *>(workspace) + dp.ws_bytes - dp.conv_bytes);
            uint16_t *vd = reinterpret_cast<uint16_t *>(reinterpret_cast<char *>(kd) + per);
            if (dense_bf16_to_f16(c.op, kd, vd, s) != cudaSuccess) {
                return ACEFA_ERR_CUDA;
            }
            pre = 1;
            for (int side = 0; side < 2; ++side) {
                acefa_tensor &t = side ? vc : kc;
                t               = side ? *v : *k;
                t.type          = ACEFA_TYPE_F16;
                t.data          = side ? static_cast<void *>(vd) : static_cast<void *>(kd);
                t.nb[0]         = 2;
                t.nb[1]         = (size_t) 2 * c.op.D;
                t.nb[2]         = t.nb[1] * (size_t) c.op.n_kv;
                t.nb[3]         = t.nb[2] * (size_t) c.op.Hkv;
            }
            c.op.k = static_cast<const char *>(kc.data), c.op.v = static_cast<const char *>(vc.data);
            c.op.k_nb1 = c.op.v_nb1 = (int64_t) kc.nb[1];
            c.op.k_nb2 = c.op.v_nb2 = (int64_t) kc.nb[2];
            c.op.k_nb3 = c.op.v_nb3 = (int64_t) kc.nb[3];
            c.op.kv_type = ACEFA_TYPE_F16;
            k = &kc, v = &vc;
        }
        DenseLaunch L;
        std::memset(&L, 0, sizeof(L));
        L.p.op            = c.op;
        L.p.rows_total    = dp.rows_total;
        L.p.n_rt          = dp.n_rt;
        L.p.n_pairs       = dp.n_pairs;
        L.p.n_kt          = dp.n_kt;
        L.p.n_full        = dp.n_full;
        L.p.n_tail        = dp.n_tail;
        L.p.n_split       = dp.n_split;
        // (batch, head)-major unit order (a head's pairs in flight together,
        // sharing its K/V tiles in L2) wherever the pairs' work is uniform:
        // no mask, or a window / padding rule.  Causal rules and f16 masks
        // (whose pattern the host does not see) keep the heavy-first order.
        L.p.head_major    = c.op.mask == nullptr &&
                         (c.op.mg_kind == 0 || c.op.mg_kind == ACEFA_MASK_WINDOW || c.op.mg_kind == ACEFA_MASK_PADDING);
        L.p.cls           = dp.classify ? static_cast<const uint8_t *>(workspace) : nullptr;
        L.p.cls_out       = dp.classify ? static_cast<uint8_t *>(workspace) : nullptr;
        L.p.part          = dp.n_tail ? reinterpret_cast<float *>(static_cast<char *>(workspace) + dp.cls_bytes)
                                      : nullptr;
        L.p.dev_err       = di->err_ptr;
        L.p.wait_limit_ns = wait_limit_ns();
        L.classify        = dp.classify;
        L.p.q_tma         = encode_q_map(&L.qmap, q, c.op.D, c.op.G) ? 1 : 0;
        L.p.o_tma         = encode_o_map(&L.omap, dst, c.op.D, c.op.G, c.op.n_mirror) ? 1 : 0;
        if (c.op.kv_type != ACEFA_TYPE_Q8_0 &&  // Q8_0 rows are staged by bulk copies
            ((rc = encode_kv_map(&L.kmap, k, c.op.D, kDenseBN)) != ACEFA_OK ||
             (rc = encode_kv_map(&L.vmap, v, c.op.D, kDenseBN)) != ACEFA_OK)) {
            return rc;
        }
        int launches = 0;
        if (launch_dense(L, s, &launches) != cudaSuccess) {
            return ACEFA_ERR_CUDA;
        }
        t_last_launches = launches + pre;
        t_last_path     = 2;
        return ACEFA_OK;
    }

    // the decode path needs no workspace: split keys merge inside the cluster
    const bool pro  = c.op.qp.on || kp.on;
    DecodePlan plan = plan_decode(c.op, pro);
    if ((int64_t) plan.units * plan.cluster >= (1ll << 31)) {
        return ACEFA_ERR_SHAPE;
    }
    DecodeLaunch L;
    std::memset(&L, 0, sizeof(L));
    L.p.op             = c.op;
    L.p.n_rb           = plan.n_rb;
    L.p.units          = plan.units;
    L.p.tiles_per_unit = plan.tpu;
    L.p.cluster        = plan.cluster;
    L.p.wide           = plan.wide;
    if (app) {
        L.p.k_new      = app->k_new;
        L.p.v_new      = app->v_new;
        L.p.kn_nb2     = app->kn_nb2;
        L.p.kn_nb3     = app->kn_nb3;
        L.p.vn_nb2     = app->vn_nb2;
        L.p.vn_nb3     = app->vn_nb3;
        L.p.append_pos = app->pos;
        L.p.kp         = kp;
    }
    L.p.dev_err        = di->err_ptr;
    L.p.wait_limit_ns  = wait_limit_ns();
    if (c.op.kv_type != ACEFA_TYPE_Q8_0) {
        if ((rc = encode_kv_map(&L.kmap, k, c.op.D, kDecBN)) != ACEFA_OK ||
            (rc = encode_kv_map(&L.vmap, v, c.op.D, kDecBN)) != ACEFA_OK) {
            return rc;
        }
    }
    int         launches = 0;
    cudaError_t e        = launch_decode(L, s, &launches);
    if (e != cudaSuccess) {
        return ACEFA_ERR_CUDA;
    }
    t_last_launches = launches;
    t_last_path     = 1;
    return ACEFA_OK;
}

// Workspace the operator needs when the caller offers at most `limit` bytes:
// the dense plan shrinks its last-wave split to fit (down to no split), so a
// smaller offer can need less.  0 = unsupported operands or no device.
size_t acefa::workspace_bytes_within(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                     const acefa_tensor *mask, const acefa_tensor *dst, size_t limit) {
    Checked c = check_operands(q, k, v, mask, nullptr, dst);
    if (c.status != ACEFA_OK) {
        return 0;
    }
    DevInfo *di = nullptr;
    if (dev_info(&di) != ACEFA_OK) {
        return 0;
    }
    if (use_dense(c.op)) {
        return plan_dense(c.op, di->sm_count, limit).ws_bytes;
    }
    return 256;  // the decode path uses none; a nonzero size marks the operands supported
}

extern "C" {

ACEFA_API int acefa_check(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                          const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst) {
    return check_operands(q, k, v, mask, sinks, dst).status;
}

ACEFA_API int acefa_supports(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                             const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst) {
    return check_operands(q, k, v, mask, sinks, dst).status == ACEFA_OK ? 1 : 0;
}

ACEFA_API size_t acefa_workspace_bytes(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                       const acefa_tensor *mask, const acefa_tensor *dst) {
    return acefa::workspace_bytes_within(q, k, v, mask, dst, SIZE_MAX);
}

ACEFA_API int acefa_flash_attn_ext(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                   const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst,
                                   float scale, float max_bias, float logit_softcap, int prec, void *stream,
                                   void *workspace, size_t workspace_bytes) {
    return run_op(q, k, v, mask, sinks, dst, scale, max_bias, logit_softcap, prec, nullptr, stream, workspace,
                  workspace_bytes);
}

ACEFA_API int acefa_flash_attn_ext_mirrored(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                            const acefa_tensor *mask, const acefa_tensor *sinks,
                                            const acefa_tensor *dst, float scale, float max_bias,
                                            float logit_softcap, int prec, void *const *mirrors, int n_mirrors,
                                            void *stream, void *workspace, size_t workspace_bytes) {
    acefa_op_ext x = {};
    x.mirrors      = mirrors;
    x.n_mirrors    = n_mirrors;
    return run_op(q, k, v, mask, sinks, dst, scale, max_bias, logit_softcap, prec, &x, stream, workspace,
                  workspace_bytes);
}

ACEFA_API int acefa_flash_attn_ext_append(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                          const acefa_tensor *mask, const acefa_tensor *sinks,
                                          const acefa_tensor *dst, float scale, float max_bias, float logit_softcap,
                                          int prec, const acefa_tensor *k_new, const acefa_tensor *v_new,
                                          const int64_t *pos, void *stream, void *workspace,
                                          size_t workspace_bytes) {
    if (!k_new || !v_new || !pos) {
        return ACEFA_ERR_NULL;
    }
    acefa_op_ext x = {};
    x.k_new        = k_new;
    x.v_new        = v_new;
    x.append_pos   = pos;
    return run_op(q, k, v, mask, sinks, dst, scale, max_bias, logit_softcap, prec, &x, stream, workspace,
                  workspace_bytes);
}

ACEFA_API int acefa_flash_attn_ext_gen(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                       const acefa_mask_gen *mask_gen, const acefa_tensor *sinks,
                                       const acefa_tensor *dst, float scale, float max_bias, float logit_softcap,
                                       int prec, void *stream, void *workspace, size_t workspace_bytes) {
    if (!mask_gen) {
        return ACEFA_ERR_NULL;
    }
    acefa_op_ext x = {};
    x.mask_gen     = mask_gen;
    return run_op(q, k, v, nullptr, sinks, dst, scale, max_bias, logit_softcap, prec, &x, stream, workspace,
                  workspace_bytes);
}

ACEFA_API int acefa_flash_attn_ext_fused(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                         const acefa_tensor *mask, const acefa_tensor *sinks,
                                         const acefa_tensor *dst, float scale, float max_bias,
                                         float logit_softcap, int prec, const acefa_op_ext *ext, void *stream,
                                         void *workspace, size_t workspace_bytes) {
    return run_op(q, k, v, mask, sinks, dst, scale, max_bias, logit_softcap, prec, ext, stream, workspace,
                  workspace_bytes);
}

ACEFA_API int acefa_kv_prologue(const acefa_tensor *k_src, const acefa_tensor *v_src, const acefa_tensor *k_dst,
                                const acefa_tensor *v_dst, const acefa_rope_norm *k_prologue, void *stream) {
    if (!k_src || !k_dst || !k_src->data || !k_dst->data || (!v_src != !v_dst) ||
        (v_src && (!v_src->data || !v_dst->data))) {
        return ACEFA_ERR_NULL;
    }
    const acefa_tensor *src[2] = {k_src, v_src}, *dstt[2] = {k_dst, v_dst};
    for (int i = 0; i < 2; ++i) {
        if (!src[i]) {
            continue;
        }
        if (src[i]->type != ACEFA_TYPE_F32 || dstt[i]->type != k_dst->type ||
            (k_dst->type != ACEFA_TYPE_F16 && k_dst->type != ACEFA_TYPE_BF16)) {
            return ACEFA_ERR_TYPE;
        }
        for (int d = 0; d < 4; ++d) {
            if (src[i]->ne[d] <= 0 || src[i]->ne[d] != k_src->ne[d] || dstt[i]->ne[d] != k_src->ne[d]) {
                return ACEFA_ERR_SHAPE;
            }
        }
        if (src[i]->nb[0] != 4 || dstt[i]->nb[0] != 2 || !aligned(src[i]->data, 4) || !aligned(dstt[i]->data, 2)) {
            return ACEFA_ERR_LAYOUT;
        }
        for (int d = 1; d < 4; ++d) {
            if (src[i]->nb[d] % 4 || dstt[i]->nb[d] % 2) {
                return ACEFA_ERR_LAYOUT;
            }
        }
    }
    const int64_t D = k_src->ne[0];
    if ((D != 64 && D != 128) || k_src->ne[1] * k_src->ne[2] * k_src->ne[3] > INT32_MAX) {
        return ACEFA_ERR_SHAPE;  // rows are numbered in 32 bits
    }
    RopeNorm kp;
    int      rc = fill_rope_norm(kp, k_prologue, (int) D);
    if (rc != ACEFA_OK) {
        return rc;
    }
    DevInfo *di = nullptr;
    if ((rc = dev_info(&di)) != ACEFA_OK) {
        return rc;
    }
    rc = kv_prologue_launch(k_src, v_src, k_dst, v_dst, kp, di->sm_count, static_cast<cudaStream_t>(stream));
    if (rc == ACEFA_OK) {
        t_last_launches = 1;
    }
    return rc;
}

ACEFA_API int acefa_cfg_logit_combine(const float *cond, const float *uncond, int64_t row_stride, int n,
                                      int eos_idx, int code_offset, int code_count, float cfg_scale,
                                      float *compact, void *stream) {
    if (n != 0 && (!cond || !compact)) {  // n == 0 reads and writes nothing
        return ACEFA_ERR_NULL;
    }
    if (n < 0 || n > 65535 || row_stride <= 0 || code_count < 0 || code_offset < 0 ||
        (int64_t) code_offset + code_count > row_stride || eos_idx >= row_stride ||
        (int64_t) code_count + 1 > INT32_MAX) {
        return ACEFA_ERR_SHAPE;
    }
    if (!aligned(cond, 4) || !aligned(compact, 4) || (uncond && !aligned(uncond, 4))) {
        return ACEFA_ERR_LAYOUT;
    }
    const int cols = code_count + (eos_idx >= 0 ? 1 : 0);
    const auto lo = reinterpret_cast<uintptr_t>(compact), hi = lo + (uintptr_t) n * cols * sizeof(float);
    const bool in_place = compact == cond && eos_idx < 0 && code_offset == 0 && code_count == row_stride;
    auto overlaps = [&](const float *rows) {  // the byte range n rows of row_stride floats span
        if (!rows || n == 0) {
            return false;
        }
        const auto b = reinterpret_cast<uintptr_t>(rows);
        const auto e = b + ((uintptr_t) (n - 1) * row_stride + row_stride) * sizeof(float);
        return b < hi && lo < e;
    };
    if ((!in_place && overlaps(cond)) || overlaps(uncond)) {
        return ACEFA_ERR_LAYOUT;
    }
    DevInfo *di = nullptr;
    int      rc = dev_info(&di);
    if (rc != ACEFA_OK) {
        return rc;
    }
    if (n == 0 || cols == 0) {
        t_last_launches = 0;
        return ACEFA_OK;
    }
    rc = cfg_combine_launch(cond, uncond, row_stride, n, eos_idx, code_offset, cols, cfg_scale, compact,
                            static_cast<cudaStream_t>(stream));
    if (rc == ACEFA_OK) {
        t_last_launches = 1;
    }
    return rc;
}

ACEFA_API int acefa_device_error(void *stream) {
    DevInfo *di = nullptr;
    int      rc = dev_info(&di);
    if (rc != ACEFA_OK) {
        return rc;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        return ACEFA_ERR_CUDA;
    }
    int v = 0;
    if (cudaMemcpy(&v, di->err_ptr, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        return ACEFA_ERR_CUDA;
    }
    const int zero = 0;
    if (cudaMemcpy(di->err_ptr, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
        return ACEFA_ERR_CUDA;
    }
    return v;
}

ACEFA_API const char *acefa_status_string(int status) {
    switch (status) {
        case ACEFA_OK: return "ok";
        case ACEFA_ERR_NULL: return "null tensor or pointer";
        case ACEFA_ERR_TYPE: return "unsupported element type";
        case ACEFA_ERR_SHAPE: return "shapes violate the flash_attn_ext contract";
        case ACEFA_ERR_LAYOUT: return "unsupported stride or alignment";
        case ACEFA_ERR_WORKSPACE: return "workspace too small or misaligned";
        case ACEFA_ERR_CUDA: return "CUDA call failed";
        case ACEFA_ERR_DEVICE: return "device is not sm_100";
        case ACEFA_ERR_DEVICE_TIMEOUT: return "device-side wait expired";
        case ACEFA_ERR_NOALLOC_LIMIT: return "operands need more scratch than the fixed no-alloc buffer (8 MiB) holds";
        default: return "unknown status";
    }
}

ACEFA_API int acefa_last_launch_count(void) { return t_last_launches; }
ACEFA_API int acefa_last_path(void) { return t_last_path; }
ACEFA_API int acefa_version(void) { return 100; }

}  // extern "C"
