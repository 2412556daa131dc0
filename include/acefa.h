/*
 * acefa.h -- C ABI of the B200 (sm_100a) attention engine behind acestep.cpp's
 * ggml_flash_attn_ext operator.
 *
 * The engine replaces the CUDA-side execution of one GGML_OP_FLASH_ATTN_EXT
 * graph node.  acestep.cpp creates those nodes at
 *   src/qwen3-lm.h:465-469    (LM prefill / single decode, PREC_F32)
 *   src/qwen3-lm.h:789-794    (LM batched CFG decode, PREC_F32)
 *   src/qwen3-enc.h:195-199   (text / lyric / timbre / FSQ encoders)
 *   src/dit-graph.h:227-231   (DiT self-attention)
 *   src/dit-graph.h:348-352   (DiT cross-attention)
 * and ggml's CUDA backend executes them in its per-node switch
 * (case GGML_OP_FLASH_ATTN_EXT -> ggml_cuda_flash_attn_ext(ctx, dst) in the
 * ggml fork that acestep.cpp pins as a submodule, .gitmodules:1-3).  That call
 * is what acefa_flash_attn_ext() replaces; acefa_supports() replaces the
 * GGML_OP_FLASH_ATTN_EXT branch of ggml_backend_cuda_device_supports_op, which
 * acestep.cpp's static_graph_alloc consults (src/static-graph.h:12-19).
 *
 * Tensors use ggml's conventions: ne[0] innermost, nb[] byte strides, type ids
 * equal to enum ggml_type.  All data pointers are device pointers owned by the
 * caller (ggml's allocator).  No entry point allocates device memory or aborts;
 * acefa_flash_attn_ext() also never synchronises, so it is safe inside
 * CUDA-graph stream capture.
 */
#ifndef ACEFA_H
#define ACEFA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define ACEFA_API __attribute__((visibility("default")))
#else
#define ACEFA_API
#endif

/* Same numeric values as enum ggml_type. */
typedef enum acefa_type {
    ACEFA_TYPE_F32  = 0,
    ACEFA_TYPE_F16  = 1,
    ACEFA_TYPE_Q8_0 = 8,
    ACEFA_TYPE_BF16 = 30,
} acefa_type;

/* Same numeric values as enum ggml_prec (ggml_flash_attn_ext_set_prec). */
typedef enum acefa_prec {
    ACEFA_PREC_DEFAULT = 0,
    ACEFA_PREC_F32     = 10,
} acefa_prec;

typedef enum acefa_status {
    ACEFA_OK             = 0,
    ACEFA_ERR_NULL       = -1, /* a required tensor or pointer is NULL */
    ACEFA_ERR_TYPE       = -2, /* unsupported element type */
    ACEFA_ERR_SHAPE      = -3, /* shapes violate the ggml_flash_attn_ext contract */
    ACEFA_ERR_LAYOUT     = -4, /* stride/alignment this engine does not support */
    ACEFA_ERR_WORKSPACE  = -5, /* workspace too small or not 256-B aligned */
    ACEFA_ERR_CUDA       = -6, /* a CUDA runtime/driver call failed */
    ACEFA_ERR_DEVICE     = -7, /* current device is not sm_100 */
    ACEFA_ERR_DEVICE_TIMEOUT = -8, /* a bounded device-side wait expired */
    ACEFA_ERR_NOALLOC_LIMIT  = -9, /* operands need more scratch than acefa_flash_attn_ext_noalloc's fixed buffer */
} acefa_status;

/* ggml_tensor reduced to what the operator reads. */
typedef struct acefa_tensor {
    int32_t type;  /* acefa_type */
    int64_t ne[4]; /* elements per dimension, ne[0] innermost */
    size_t  nb[4]; /* byte strides; for Q8_0 nb[0] = 34 (block bytes) */
    void   *data;  /* device pointer */
} acefa_tensor;

/*
 * dst = softmax(scale * Q K^T [softcap] + slope * mask [+ sinks]) V, permuted.
 *
 *   q     [D,  n_q,  Hq,  B ]  F32, any strides with nb[0] == 4
 *   k     [D,  n_kv, Hkv, Bk]  F16, BF16 or Q8_0; Hq % Hkv == 0, B % Bk == 0
 *   v     [Dv, n_kv, Hkv, Bk]  same type as k, Dv == D
 *   mask  [>=n_kv, >=n_q, Hm, Bm] F16 or NULL; Hq % Hm == 0, B % Bm == 0
 *   sinks [Hq] F32 or NULL (extra softmax logit per head, no value row)
 *   dst   [Dv, Hq, n_q, B] F32
 *
 * scale, max_bias (ALiBi) and logit_softcap have ggml's meaning.  prec is
 * accepted for either value; accumulation is always F32.  stream is a
 * cudaStream_t (NULL = legacy default stream).  workspace must hold
 * acefa_workspace_bytes() bytes, 256-B aligned, caller-owned; its contents need
 * no initialisation and are dead after the call's kernels finish.
 * Returns ACEFA_OK or a negative acefa_status; launches nothing on error.
 */
ACEFA_API int acefa_flash_attn_ext(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                   const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst,
                                   float scale, float max_bias, float logit_softcap, int prec, void *stream,
                                   void *workspace, size_t workspace_bytes);

/*
 * The same operator for callers that cannot hand the engine any device memory:
 * hosts whose device memory is entirely owned by another allocator (a ggml
 * backend whose graph allocator has planned every buffer, a plugin inside a
 * framework that forbids foreign allocations), threads that must never block
 * (cudaMalloc can synchronise the whole device), and builds that forbid runtime
 * allocation after start-up.  No counterpart in the reference: ggml's CUDA
 * backend always draws flash-attention scratch from its own memory pool.
 *
 * Arguments and results are those of acefa_flash_attn_ext() without the
 * workspace pair.  The scratch is a fixed 8 MiB array inside the library, one
 * per GPU, held from library load until process exit; only the dense
 * (query-heavy) path uses it -- its mask-class table, the partial results of
 * its last-wave key-range split, F16 copies of BF16 K/V when they fit -- while
 * decode nodes need none.  The call plans its work for that 8 MiB (the dense
 * path shrinks or drops its split and skips the BF16 copies to fit, exactly as
 * acefa_flash_attn_ext would with an 8 MiB workspace); operands that need more
 * even then -- a mask-class table over 8 MiB -- are refused with
 * ACEFA_ERR_NOALLOC_LIMIT and nothing is launched.  The first call on each
 * device looks up that array's device address (with the device current), so
 * make that first call before any stream capture.  The address is kept for the
 * life of the process: after cudaDeviceReset() on a device this entry (like the
 * engine's device error word) must not be used on it again.  Every call on a device
 * shares the array: calls whose kernels may overlap on the GPU (other streams or
 * other threads without ordering) race and must be serialised by the caller.
 * Nothing is allocated, freed or zeroed by the call.
 */
ACEFA_API int acefa_flash_attn_ext_noalloc(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                           const acefa_tensor *mask, const acefa_tensor *sinks,
                                           const acefa_tensor *dst, float scale, float max_bias, float logit_softcap,
                                           int prec, void *stream);

/*
 * Multi-GPU extension; no counterpart in the reference, which runs every module
 * on one device.  The operator with its result also written to up to
 * ACEFA_MAX_MIRRORS further buffers ("mirrors"), each laid out exactly like dst
 * (same ne and nb) at another address: typically this rank's head slice of a
 * peer GPU's full output, mapped with acefa_peer_import().  The kernels' output
 * stage stores every row to dst and to each mirror (plain stores, over NVLink
 * for peer memory), so a head-sharded attention layer assembles its full
 * output on every GPU with no separate all-gather.  Each mirror must be
 * congruent to dst modulo 16 bytes.  n_mirrors == 0 is acefa_flash_attn_ext().
 * The call signals nothing to the peers: before a peer reads its output the
 * caller orders it after this stream's work (a collective on this stream after
 * the call, or an IPC event).  Returns ACEFA_ERR_NULL / ACEFA_ERR_LAYOUT for a
 * NULL or misaligned mirror, ACEFA_ERR_SHAPE for n_mirrors out of range.
 */
#define ACEFA_MAX_MIRRORS 7
ACEFA_API int acefa_flash_attn_ext_mirrored(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                            const acefa_tensor *mask, const acefa_tensor *sinks,
                                            const acefa_tensor *dst, float scale, float max_bias,
                                            float logit_softcap, int prec, void *const *mirrors, int n_mirrors,
                                            void *stream, void *workspace, size_t workspace_bytes);

/*
 * The operator fused with the KV-cache append that precedes it in a decode
 * step.  The reference writes the new row with two ggml_set_rows nodes (K and V
 * at src/qwen3-lm.h:776-777, inside qw3lm_forward_batch) and then runs the
 * attention node over the cache views; this entry does both in one launch.
 *
 *   k_new, v_new  [D, 1, Hkv, Bk] F32, nb[0] == 4: the new row of every
 *                 (kv head, set), already projected, normed and rotated
 *   pos           device array of Bk int64: the cache row (0 <= pos < n_kv of
 *                 the k/v views) that receives set s's new row
 *
 * Row pos[s] of every head of set s in k and v is overwritten with k_new /
 * v_new converted to the cache type (F16 / BF16 rounded to nearest even; Q8_0
 * by ggml's reference quantiser: d = amax/127, q = roundf(x * (1/d)), d as f16), and
 * the attention then reads the updated cache exactly as acefa_flash_attn_ext
 * would have after the two set_rows.  The k and v views must be writable and
 * each (head, set) row written once: sets whose views alias each other, or a
 * mask that hides row pos[s], are the caller's concern.  Served by the decode
 * path only (query rows per kv head <= 64, i.e. decode steps); other shapes
 * return ACEFA_ERR_SHAPE.  A pos outside [0, n_kv) leaves that set's row
 * unwritten and raises device error 5 (acefa_device_error()).  Other
 * arguments and results are those of acefa_flash_attn_ext().
 */
ACEFA_API int acefa_flash_attn_ext_append(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                          const acefa_tensor *mask, const acefa_tensor *sinks,
                                          const acefa_tensor *dst, float scale, float max_bias, float logit_softcap,
                                          int prec, const acefa_tensor *k_new, const acefa_tensor *v_new,
                                          const int64_t *pos, void *stream, void *workspace, size_t workspace_bytes);

/*
 * A mask given by its rule instead of an f16 tensor.  acestep.cpp fills these
 * masks on the host and the attention node reads them back from HBM: the LM
 * prefill causal mask (src/qwen3-lm.h:597-609), the batched decode validity
 * mask (src/qwen3-lm.h:872-881), the DiT sliding window sa_mask_sw and the
 * cross-attention padding ca_mask (src/dit-sampler.h:262-311).
 * Key j is visible to query i (0-based within n_q) of batch b when
 *   ACEFA_MASK_CAUSAL   j <= pos0[b] + i   (LM prefill with the cache holding
 *                       pos0 earlier tokens; a decode step is i = 0, keys
 *                       0 .. kv_pos)
 *   ACEFA_MASK_WINDOW   |i - j| <= window  (DiT self-attention, sliding-window
 *                       layers; where the reference's window is off -- win <= 0
 *                       or S <= win -- the node is unmasked: pass no mask)
 *   ACEFA_MASK_PADDING  j < len[b]         (DiT cross-attention padding)
 * Visible keys add 0 and hidden keys -inf, exactly as the equivalent f16
 * mask would; results are bit-identical to acefa_flash_attn_ext with that mask.
 * pos0 / len are read for b < B (at most ACEFA_MASK_GEN_MAX_BATCH batches).
 */
#define ACEFA_MASK_GEN_MAX_BATCH 32
typedef enum acefa_mask_kind {
    ACEFA_MASK_CAUSAL  = 1,
    ACEFA_MASK_WINDOW  = 2,
    ACEFA_MASK_PADDING = 3,
} acefa_mask_kind;

typedef struct acefa_mask_gen {
    int32_t kind;    /* acefa_mask_kind */
    int32_t window;  /* ACEFA_MASK_WINDOW */
    int64_t pos0[ACEFA_MASK_GEN_MAX_BATCH];  /* ACEFA_MASK_CAUSAL */
    int64_t len[ACEFA_MASK_GEN_MAX_BATCH];   /* ACEFA_MASK_PADDING */
} acefa_mask_gen;

/* acefa_flash_attn_ext() with the mask given by rule (mask_gen, host memory,
 * read during the call) instead of a tensor: no mask is read on the device and
 * the dense path needs no mask-classification pass.  The rule is copied into
 * the launch, so mask_gen may be reused or freed once the call returns.
 * acefa_workspace_bytes(q, k, v, NULL, dst) is enough workspace.  Returns
 * ACEFA_ERR_SHAPE for an unknown kind, B > ACEFA_MASK_GEN_MAX_BATCH with a
 * per-batch kind (CAUSAL, PADDING), or a negative window. */
ACEFA_API int acefa_flash_attn_ext_gen(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                       const acefa_mask_gen *mask_gen, const acefa_tensor *sinks,
                                       const acefa_tensor *dst, float scale, float max_bias, float logit_softcap,
                                       int prec, void *stream, void *workspace, size_t workspace_bytes);

/*
 * The attention prologue acestep.cpp runs as separate graph nodes before the
 * attention node (src/qwen3-lm.h:423-431, src/dit-graph.h:181-197):
 *   y = ggml_rms_norm(x, eps) * norm_weight        (per row of D values)
 *   y = ggml_rope_ext(y, positions, mode 2 = NEOX, n_dims = D, freq_base =
 *       theta_base, freq_scale 1, no YaRN)
 * i.e. pair k < D/2 rotates (y[k], y[k + D/2]) by positions[..] *
 * theta_base^(-2k/D).  Row i of batch b has position positions[i + b * n],
 * n being the rows per batch of the tensor it applies to (n_q for Q; for a
 * decode step's new K row, n = 1: positions[set]).
 */
typedef struct acefa_rope_norm {
    const float   *norm_weight;  /* [D] f32, device; NULL = no RMSNorm */
    float          eps;          /* rms_norm_eps */
    float          theta_base;   /* rope_theta; 0 = no RoPE */
    const int32_t *positions;    /* int32, device (ggml's positions tensor); unused without RoPE */
} acefa_rope_norm;

/*
 * Options of acefa_flash_attn_ext_fused().  Zero-initialise and set what is
 * used; every member may be NULL / 0.
 */
typedef struct acefa_op_ext {
    const acefa_mask_gen  *mask_gen;    /* mask by rule; `mask` must then be NULL */
    const acefa_rope_norm *q_prologue;  /* applied to each Q row as the kernels load it */
    /* Fused KV-cache append (decode path), as acefa_flash_attn_ext_append: */
    const acefa_tensor    *k_new, *v_new;
    const int64_t         *append_pos;
    const acefa_rope_norm *k_prologue;  /* applied to k_new before it is converted and stored */
    /* Mirrors, as acefa_flash_attn_ext_mirrored: */
    void *const           *mirrors;
    int                    n_mirrors;
} acefa_op_ext;

/* The operator with any combination of the fusions above (NULL ext = plain
 * acefa_flash_attn_ext).  Q given with a q_prologue is the raw projection
 * output (before RMSNorm and RoPE), in the same [D, n_q, Hq, B] view. */
ACEFA_API int acefa_flash_attn_ext_fused(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                         const acefa_tensor *mask, const acefa_tensor *sinks,
                                         const acefa_tensor *dst, float scale, float max_bias,
                                         float logit_softcap, int prec, const acefa_op_ext *ext, void *stream,
                                         void *workspace, size_t workspace_bytes);

/*
 * K / V preparation for the dense path in one pass: k_dst = RoPE(RMSNorm(k_src))
 * and v_dst = v_src, converted to the destination type (F16 or BF16), at any
 * strides on either side (so the permute of the reference's graph and a
 * write into a KV-cache window are both just destination views).  Replaces
 * the rms_norm, mul, rope, cont and cast / set_rows nodes of
 * src/dit-graph.h:181-213 and src/qwen3-lm.h:423-449.  k_src / v_src: F32
 * [D, rows, H, B] with rows * H * B < 2^31; k_dst / v_dst: the same ne.
 * v_src / v_dst may be NULL.  Positions index as positions[row + b * rows].
 */
ACEFA_API int acefa_kv_prologue(const acefa_tensor *k_src, const acefa_tensor *v_src, const acefa_tensor *k_dst,
                                const acefa_tensor *v_dst, const acefa_rope_norm *k_prologue, void *stream);

/*
 * CUDA IPC through the ABI, so a host without CUDA bindings can map peer
 * buffers.  acefa_peer_export: an opaque handle (ACEFA_PEER_HANDLE_BYTES bytes)
 * for the allocation holding ptr, plus ptr's byte offset inside it.
 * acefa_peer_import (another process of the same node, its own device current):
 * maps that allocation with peer access enabled and returns the address that
 * corresponds to the exported ptr.  acefa_peer_release: unmaps an address
 * acefa_peer_import returned.  All three return ACEFA_OK or ACEFA_ERR_CUDA /
 * ACEFA_ERR_NULL.
 */
#define ACEFA_PEER_HANDLE_BYTES 64
ACEFA_API int acefa_peer_export(const void *ptr, void *handle, uint64_t *offset);
ACEFA_API int acefa_peer_import(const void *handle, uint64_t offset, void **ptr);
ACEFA_API int acefa_peer_release(void *ptr);

/*
 * CFG combine + logit compaction of a batched LM decode step on the device:
 * the host loop of src/pipeline-lm.cpp:471-492 (and, with eos_idx < 0 and the
 * range [0, V), the full-vocabulary combines of :104-108, :193-199, :364-370),
 * so that only the compact rows cross to the host.  cond / uncond: F32 logits,
 * sequence a's rows at cond + a * row_stride and uncond + a * row_stride (in
 * the reference's batch layout uncond = cond + n * row_stride); uncond NULL:
 * no CFG (the reference's use_cfg false), a plain gather.  compact: n rows of
 * cols = code_count + (eos_idx >= 0) floats, contiguous:
 *   column 0            <- logit eos_idx            (only when eos_idx >= 0)
 *   following columns   <- logits code_offset .. code_offset + code_count - 1
 * each u + cfg_scale * (c - u) with every operation rounded to F32 on its own
 * (no FMA), bit-identical to the reference's x86-64 host arithmetic.
 * compact must not overlap cond or uncond, except compact == cond with
 * eos_idx < 0, code_offset 0 and code_count == row_stride (the in-place
 * full-row combine).  n <= 65535.  Stream-ordered, one launch (none for
 * n == 0, which accepts NULL buffers).  Returns ACEFA_ERR_NULL, ACEFA_ERR_SHAPE (a column outside the row,
 * n out of range), ACEFA_ERR_LAYOUT (misaligned or overlapping buffers).
 */
ACEFA_API int acefa_cfg_logit_combine(const float *cond, const float *uncond, int64_t row_stride, int n,
                                      int eos_idx, int code_offset, int code_count, float cfg_scale,
                                      float *compact, void *stream);

/* Workspace acefa_flash_attn_ext() needs for these operands on the current device
 * (dense path only: mask tile classes, the partial results of the last-wave
 * key-range split, and for BF16 K/V F16 copies of K and V, 4 bytes per K/V
 * value; decode nodes need a token 256 bytes).  A function of shapes,
 * types and the device only -- never of tensor contents -- so it can be sized
 * once before CUDA-graph capture.  A smaller workspace also works where the
 * operator can do without: it then skips the BF16 copies (converting inside
 * the attention kernel, same results) and splits fewer key ranges.  Returns 0
 * for unsupported operands. */
ACEFA_API size_t acefa_workspace_bytes(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                                       const acefa_tensor *mask, const acefa_tensor *dst);

/* 1 if acefa_flash_attn_ext accepts these operands, else 0 (mirrors
 * ggml_backend_cuda_device_supports_op for GGML_OP_FLASH_ATTN_EXT; when it
 * returns 0 the ggml scheduler keeps the node on the CPU backend). */
ACEFA_API int acefa_supports(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                             const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst);

/* Validation only: the status acefa_flash_attn_ext would return before
 * launching (ACEFA_OK when the operands are accepted).  Touches no device. */
ACEFA_API int acefa_check(const acefa_tensor *q, const acefa_tensor *k, const acefa_tensor *v,
                          const acefa_tensor *mask, const acefa_tensor *sinks, const acefa_tensor *dst);

/* Reads and clears the device-side error word set by bounded waits inside the
 * kernels (0 = none).  Synchronises `stream`; for diagnostics, not hot paths.
 * There is ONE word per device, shared by every stream and thread using the
 * engine on it: the first code recorded since the last read is kept, whichever
 * call's kernel recorded it, and a read from one stream also clears what a
 * kernel on another stream recorded.  Callers that run the engine on several
 * streams of one device and need to know which call failed read it with those
 * streams idle.  Returns a negative acefa_status if the read itself fails. */
ACEFA_API int acefa_device_error(void *stream);

/* Human-readable name of an acefa_status. */
ACEFA_API const char *acefa_status_string(int status);

/* Kernel-launch count of the last successful acefa_flash_attn_ext call on this
 * host thread (1 to 3: mask classification, attention, split-KV combine). */
ACEFA_API int acefa_last_launch_count(void);

/* Which kernel family served the last successful call on this thread:
 * 1 = split-KV decode (mma.sync), 2 = dense tcgen05/TMEM. */
ACEFA_API int acefa_last_path(void);

/* ABI version: major*10000 + minor*100 + patch. */
ACEFA_API int acefa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* ACEFA_H */
