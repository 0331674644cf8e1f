// mxfp4.cuh — E2M1 x E8M0 decode shared by the MXFP4 matvec and the MXFP4
// MoE expert kernels (FIXED_MXFP4_EXPERT_LAYER_V1; reference
// mxfp4_fma_matvec_e8m0, shaders.metal:200-298, and
// mxfp4_fma_matvec_with_group_size, experts/slots.rs:1239-1287).
//
// Two nibbles at a time are placed into the exponent/mantissa fields of an
// fp16 pair (bits (n & 7) << 9, sign (n & 8) << 12): the fp16 value is
// e2m1(n) * 2^-14 exactly (e = 0 lands in the fp16 subnormals) and converts
// to f32 exactly. A 32-column group's products are summed, then scaled by
// 2^14 and the E8M0 scale (both powers of two), so each term rounds as the
// reference's weight * scale * x does and only the summation order differs.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace pbmoe {

// nibbles n0 (bits 0-3) and n1 (bits 16-19) of `v` -> two floats e2m1 * 2^-14
__device__ __forceinline__ float2 e2m1_pair(uint32_t v) {
    const uint32_t h = ((v & 0x00070007u) << 9) | ((v & 0x00080008u) << 12);
    __half2 hh;
    memcpy(&hh, &h, 4);
    return __half22float2(hh);
}

__device__ __forceinline__ float e8m0_scale(uint32_t e) {
    return __uint_as_float(e == 0 ? 0x00400000u : (e << 23));
}

// Activations of one token for MXFP4 rows in shared memory: 32 columns then 4
// floats of padding (lane l reads group l; unpadded rows would put every
// lane's 16-byte reads in the same banks).
__host__ __device__ inline uint32_t mx_padded_cols(uint32_t cols) { return cols / 32 * 36; }

// sum over one 32-column group of e2m1(w) * 2^-14 * x, for NT tokens whose
// padded rows start `pstride` floats apart at xs (this group's first column)
template <int NT>
__device__ __forceinline__ void mx_group_dot(const uint4 w, const float* xs, uint32_t pstride, float (&part)[NT]) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        // bytes b0..b3 of the word = columns 8q + 2j (low nibble), 8q + 2j + 1 (high)
        const uint32_t v = words[q];
        const float2 lo02 = e2m1_pair(__byte_perm(v, 0, 0x4140));       // cols 0, 2
        const float2 hi02 = e2m1_pair(__byte_perm(v, 0, 0x4140) >> 4);  // cols 1, 3
        const float2 lo46 = e2m1_pair(__byte_perm(v, 0, 0x4342));       // cols 4, 6
        const float2 hi46 = e2m1_pair(__byte_perm(v, 0, 0x4342) >> 4);  // cols 5, 7
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float* xr = xs + t * pstride + q * 8;
            const float4 xa = *reinterpret_cast<const float4*>(xr);
            const float4 xb = *reinterpret_cast<const float4*>(xr + 4);
            float s = part[t];
            s = fmaf(lo02.x, xa.x, s);
            s = fmaf(hi02.x, xa.y, s);
            s = fmaf(lo02.y, xa.z, s);
            s = fmaf(hi02.y, xa.w, s);
            s = fmaf(lo46.x, xb.x, s);
            s = fmaf(hi46.x, xb.y, s);
            s = fmaf(lo46.y, xb.z, s);
            s = fmaf(hi46.y, xb.w, s);
            part[t] = s;
        }
    }
}

}  // namespace pbmoe
