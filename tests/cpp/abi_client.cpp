// abi_client.cpp -- a C++ client of libacefa.so that uses only include/acefa.h
// and the CUDA runtime, the way a ggml CUDA-backend bridge would: ggml-style
// descriptors (ne / nb / type), views into a KV cache, a caller-owned
// workspace, a stream.  No Python, no torch.
//
// The node is acestep.cpp's batched CFG decode (src/qwen3-lm.h:776-794):
//   Q    [128, 1, Hq, N]        f32
//   K, V [128, n_kv, Hkv, N]    f16 views of caches [128, max_seq, Hkv, sets]
//   mask [n_kv, 1, 1, N]        f16, 0 for j <= kv_pos[set], -inf after
//   dst  [128, Hq, 1, N]        f32
// and the result is checked against a naive double-precision loop.
//
// Usage: abi_client validate   (descriptor checks only; needs no GPU)
//        abi_client run        (one call on the current GPU + the check)
// Exit status 0 on success.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "acefa.h"

namespace {

constexpr int D = 128, HQ = 16, HKV = 8, N = 2, NKV = 320, MAX_SEQ = 512;
const int     kv_pos[N] = {57, 301};

acefa_tensor desc(int type, const int64_t ne[4], const size_t nb[4], void *data) {
    acefa_tensor t;
    t.type = type;
    for (int i = 0; i < 4; ++i) {
        t.ne[i] = ne[i];
        t.nb[i] = nb[i];
    }
    t.data = data;
    return t;
}

struct Node {
    acefa_tensor q, k, v, mask, dst;
};

// Descriptors of the decode node over the given base pointers.
Node make_node(void *q, void *kc, void *vc, void *mask, void *dst) {
    Node          n;
    const int64_t qne[4] = {D, 1, HQ, N};
    const size_t  qnb[4] = {4, 4 * D, 4 * D, 4 * (size_t) D * HQ};
    const int64_t kne[4] = {D, NKV, HKV, N};  // a view of the first NKV rows of each cache set
    const size_t  knb[4] = {2, 2 * D, 2 * (size_t) D * MAX_SEQ, 2 * (size_t) D * MAX_SEQ * HKV};
    const int64_t mne[4] = {NKV, 1, 1, N};
    const size_t  mnb[4] = {2, 2 * NKV, 2 * NKV, 2 * NKV};
    const int64_t dne[4] = {D, HQ, 1, N};
    const size_t  dnb[4] = {4, 4 * D, 4 * (size_t) D * HQ, 4 * (size_t) D * HQ};
    n.q    = desc(ACEFA_TYPE_F32, qne, qnb, q);
    n.k    = desc(ACEFA_TYPE_F16, kne, knb, kc);
    n.v    = desc(ACEFA_TYPE_F16, kne, knb, vc);
    n.mask = desc(ACEFA_TYPE_F16, mne, mnb, mask);
    n.dst  = desc(ACEFA_TYPE_F32, dne, dnb, dst);
    return n;
}

int fail(const char *what, int got, int want) {
    std::fprintf(stderr, "%s: got %d, want %d\n", what, got, want);
    return 1;
}

// Descriptor validation without a device: fake device addresses, nothing is
// dereferenced before the operands are accepted.
int validate() {
    char *base = reinterpret_cast<char *>(uintptr_t(1) << 20);
    Node  n    = make_node(base, base + (1 << 22), base + (1 << 24), base + (1 << 26), base + (1 << 27));
    int   rc   = acefa_check(&n.q, &n.k, &n.v, &n.mask, nullptr, &n.dst);
    if (rc != ACEFA_OK) {
        return fail("acefa_check(decode node)", rc, ACEFA_OK);
    }
    Node bad = n;
    bad.mask.ne[0] = NKV - 1;  // a mask narrower than n_kv breaks the contract
    if ((rc = acefa_check(&bad.q, &bad.k, &bad.v, &bad.mask, nullptr, &bad.dst)) != ACEFA_ERR_SHAPE) {
        return fail("narrow mask", rc, ACEFA_ERR_SHAPE);
    }
    bad = n;
    bad.v.type = ACEFA_TYPE_Q8_0;  // K and V share one type
    if ((rc = acefa_check(&bad.q, &bad.k, &bad.v, &bad.mask, nullptr, &bad.dst)) != ACEFA_ERR_TYPE) {
        return fail("mixed K/V types", rc, ACEFA_ERR_TYPE);
    }
    if (acefa_supports(&n.q, &n.k, &n.v, &n.mask, nullptr, &n.dst) != 1) {
        return fail("acefa_supports", 0, 1);
    }
    if (std::strlen(acefa_status_string(ACEFA_ERR_SHAPE)) == 0) {
        return fail("status string", 0, 1);
    }
    std::printf("validate ok (ABI version %d)\n", acefa_version());
    return 0;
}

int run() {
    std::mt19937                 rng(4242);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    std::vector<float>           q((size_t) D * HQ * N);
    std::vector<__half>          kc((size_t) D * MAX_SEQ * HKV * N), vc(kc.size());
    std::vector<__half>          mask((size_t) NKV * N);
    for (auto &x : q) x = nd(rng);
    for (auto &x : kc) x = __float2half(nd(rng));
    for (auto &x : vc) x = __float2half(nd(rng));
    for (int s = 0; s < N; ++s) {
        for (int j = 0; j < NKV; ++j) {
            mask[(size_t) s * NKV + j] = __float2half(j <= kv_pos[s] ? 0.0f : -INFINITY);
        }
    }
    void *dq, *dk, *dv, *dm, *dd;
    if (cudaMalloc(&dq, q.size() * 4) || cudaMalloc(&dk, kc.size() * 2) || cudaMalloc(&dv, vc.size() * 2) ||
        cudaMalloc(&dm, mask.size() * 2) || cudaMalloc(&dd, (size_t) D * HQ * N * 4)) {
        return fail("cudaMalloc", 1, 0);
    }
    cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dk, kc.data(), kc.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, vc.data(), vc.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dm, mask.data(), mask.size() * 2, cudaMemcpyHostToDevice);
    Node         n  = make_node(dq, dk, dv, dm, dd);
    const size_t ws = acefa_workspace_bytes(&n.q, &n.k, &n.v, &n.mask, &n.dst);
    void        *dw = nullptr;
    if (ws && cudaMalloc(&dw, ws)) {
        return fail("cudaMalloc workspace", 1, 0);
    }
    cudaStream_t stream;
    cudaStreamCreate(&stream);
    const float scale = 1.0f / std::sqrt((float) D);
    int rc = acefa_flash_attn_ext(&n.q, &n.k, &n.v, &n.mask, nullptr, &n.dst, scale, 0.0f, 0.0f, ACEFA_PREC_F32,
                                  stream, dw, ws);
    if (rc != ACEFA_OK) {
        return fail("acefa_flash_attn_ext", rc, ACEFA_OK);
    }
    if ((rc = acefa_device_error(stream)) != 0) {
        return fail("device error word", rc, 0);
    }
    std::vector<float> out((size_t) D * HQ * N);
    cudaMemcpy(out.data(), dd, out.size() * 4, cudaMemcpyDeviceToHost);
    // naive reference in double precision
    double max_err = 0.0;
    for (int s = 0; s < N; ++s) {
        for (int h = 0; h < HQ; ++h) {
            const int          hk = h / (HQ / HKV);
            std::vector<double> sc(NKV);
            double             mx = -INFINITY;
            for (int j = 0; j <= kv_pos[s]; ++j) {
                double acc = 0.0;
                for (int d = 0; d < D; ++d) {
                    acc += (double) q[((size_t) s * HQ + h) * D + d] *
                           (double) __half2float(kc[(((size_t) s * HKV + hk) * MAX_SEQ + j) * D + d]);
                }
                sc[j] = acc * scale;
                mx    = std::fmax(mx, sc[j]);
            }
            double l = 0.0;
            for (int j = 0; j <= kv_pos[s]; ++j) {
                sc[j] = std::exp(sc[j] - mx);
                l += sc[j];
            }
            for (int d = 0; d < D; ++d) {
                double o = 0.0;
                for (int j = 0; j <= kv_pos[s]; ++j) {
                    o += sc[j] * (double) __half2float(vc[(((size_t) s * HKV + hk) * MAX_SEQ + j) * D + d]);
                }
                const double got = out[((size_t) s * HQ + h) * D + d];  // dst [D, Hq, 1, N]
                max_err          = std::fmax(max_err, std::fabs(got - o / l));
            }
        }
    }
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dm);
    cudaFree(dd);
    cudaFree(dw);
    cudaStreamDestroy(stream);
    if (!(max_err <= 2e-3)) {
        std::fprintf(stderr, "max abs error %.3e above 2e-3\n", max_err);
        return 1;
    }
    std::printf("run ok: max_abs=%.3e launches=%d path=%d workspace=%zu B\n", max_err, acefa_last_launch_count(),
                acefa_last_path(), ws);
    return 0;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc > 1 && std::strcmp(argv[1], "run") == 0) {
        return run();
    }
    return validate();
}
