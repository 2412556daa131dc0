// q8.cuh -- Q8_0 (ggml block: f16 scale d, 32 int8 quants q; value d * q)
// dequantisation helpers shared by the decode and dense kernels.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace acefa {

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
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// NW words of int8 quants of one Q8_0 block starting `sub` bytes into its 32
// values (blk = the block's shared address: f16 scale, then the quants; any
// 2-B alignment), each byte biased to unsigned (b ^ 0x80).  Returns the scale.
template <int NW>
__device__ __forceinline__ uint16_t q8_load_run(uint32_t blk, int sub, uint32_t (&q)[NW]) {
    const uint32_t a  = blk + 2u + (uint32_t) sub;
    const uint32_t aw = a & ~3u;
    const uint32_t sh = (a & 3u) * 8u;  // 0 or 16
    uint32_t       w[NW + 1];
#pragma unroll
    for (int k = 0; k <= NW; ++k) {
        w[k] = lds32(aw + 4u * k);
    }
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        q[k] = __funnelshift_r(w[k], w[k + 1], sh) ^ 0x80808080u;
    }
    return lds16(blk);
}

// Two biased int8 values placed in the low bytes of an f16 pair with exponent
// 0x64 are the f16 values 1152 + b: subtracting 1152 recovers b exactly, and
// the multiply by the block scale rounds once (f16(d * q), as ggml's
// dequantisation to F16).  sel picks the two bytes (0x4140: bytes 0,1;
// 0x4342: bytes 2,3).
__device__ __forceinline__ uint32_t i8x2_scaled(uint32_t biased_word, uint32_t sel, __half2 d2) {
    const uint32_t t = __byte_perm(biased_word, 0x64646464u, sel);
    const __half2  v = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&t), __half2half2(__ushort_as_half(0x6480u))),
                               d2);
    return *reinterpret_cast<const uint32_t *>(&v);
}

}  // namespace acefa
