// cfg_combine.cu -- the CFG combine and logit compaction of a batched LM
// decode step on the device (acefa_cfg_logit_combine).  acestep.cpp copies the
// logits of all 2n batch entries to the host and there, per sequence, mixes
// the conditional row lc with the unconditional row lu,
// lc[i] = lu[i] + cfg_scale * (lc[i] - lu[i]), on the EOS column and the
// audio-code range, then copies those columns into a compact array for the
// sampler (src/pipeline-lm.cpp:471-492).  Here one launch reads the two rows of
// every sequence and writes only the compact rows, so the host receives
// n * (1 + codes) floats instead of 2n full rows.  HBM-bound: 8 B read and
// 4 B written per compact value.
#include <cuda_runtime.h>

#include <cstdint>

#include "fa_internal.h"

namespace acefa {

namespace {

constexpr int kCfgThreads = 256;
constexpr int kCfgPerThread = 4;  // independent loads in flight per thread

struct CfgParams {
    const float *cond;
    const float *uncond;  // nullptr: no CFG, plain compaction
    float       *out;
    int64_t      row_stride;  // floats between consecutive sequences' rows
    int          cols;        // compact row length
    int          eos;         // EOS column, < 0: none
    int          code_offset;
    float        scale;
};

// blockIdx.y = sequence, blockIdx.x = a chunk of kCfgThreads * kCfgPerThread
// compact columns.  Each operation is rounded on its own (__fsub_rn, __fmul_rn,
// __fadd_rn: no FMA contraction), as the reference computes it on the host.
// Plain (coherent) loads: the in-place form (out == cond) reads and writes the
// same element from the same thread.
__global__ void __launch_bounds__(kCfgThreads) cfg_logit_combine_kernel(const CfgParams P) {
    const int     a    = blockIdx.y;
    const float  *lc   = P.cond + (int64_t) a * P.row_stride;
    const float  *lu   = P.uncond ? P.uncond + (int64_t) a * P.row_stride : nullptr;
    float        *o    = P.out + (int64_t) a * P.cols;
    const int     j0   = blockIdx.x * (kCfgThreads * kCfgPerThread) + threadIdx.x;
    float         c[kCfgPerThread], u[kCfgPerThread];
    int64_t       col[kCfgPerThread];
#pragma unroll
    for (int t = 0; t < kCfgPerThread; ++t) {
        const int j = j0 + t * kCfgThreads;
        col[t]      = P.eos >= 0 ? (j == 0 ? (int64_t) P.eos : (int64_t) P.code_offset + j - 1)
                                 : (int64_t) P.code_offset + j;
        if (j < P.cols) {
            c[t] = __ldcs(lc + col[t]);
            u[t] = lu ? __ldcs(lu + col[t]) : 0.0f;
        }
    }
#pragma unroll
    for (int t = 0; t < kCfgPerThread; ++t) {
        const int j = j0 + t * kCfgThreads;
        if (j < P.cols) {
            const float r = lu ? __fadd_rn(u[t], __fmul_rn(P.scale, __fsub_rn(c[t], u[t]))) : c[t];
            __stcs(o + j, r);
        }
    }
}

}  // namespace

int cfg_combine_launch(const float *cond, const float *uncond, int64_t row_stride, int n, int eos_idx,
                       int code_offset, int cols, float cfg_scale, float *compact, cudaStream_t stream) {
    CfgParams P;
    P.cond        = cond;
    P.uncond      = uncond;
    P.out         = compact;
    P.row_stride  = row_stride;
    P.cols        = cols;
    P.eos         = eos_idx;
    P.code_offset = code_offset;
    P.scale       = cfg_scale;
    const int per = kCfgThreads * kCfgPerThread;
    dim3      grid((unsigned) ((cols + per - 1) / per), (unsigned) n);
    cfg_logit_combine_kernel<<<grid, kCfgThreads, 0, stream>>>(P);
    return cudaGetLastError() == cudaSuccess ? ACEFA_OK : ACEFA_ERR_CUDA;
}

}  // namespace acefa
