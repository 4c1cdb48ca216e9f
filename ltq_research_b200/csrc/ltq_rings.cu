// int8 ring format of the row tables (lumen-inference/ltq-research src/ple_quant.py:68-77, `int8_rows`): per ring of
// 256 values, d = max(fp16(max|x| / 127), 1e-10) and y = clamp(round_even(x / d), -127, 127) * d, stored in the
// table's dtype.  Every step is an elementwise IEEE operation or an exact maximum, so the result does not depend on
// the order of evaluation; NaN propagates as in the reference's torch operations (a NaN anywhere in a ring makes the
// ring's scale and values NaN; an infinite value makes d infinite).
//
// One warp per ring: lane L holds values 8L .. 8L + 7 (one 16-byte bf16 load or two 16-byte fp32 loads), the ring's
// maximum by a butterfly of shuffles.  HBM-bound: 2 x 2 bytes (bf16) or 2 x 4 bytes (fp32) per value.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "ltq_b200.h"

namespace {

template <bool BF16>
__global__ void __launch_bounds__(256) int8_rings_kernel(const void* __restrict__ in, void* __restrict__ out,
                                                         long long n_rings)
{
    const long long ring = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (ring >= n_rings) return;
    const int lane = threadIdx.x & 31;
    const long long base = ring * 256 + 8 * lane;
    float v[8];
    if constexpr (BF16) {
        const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(in) + base);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __bfloat162float(h[k]);
    } else {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(in) + base);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(in) + base + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    float m = 0.f;
    bool nan = false;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        nan |= v[k] != v[k];
        m = fmaxf(m, fabsf(v[k]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    nan = __any_sync(0xffffffffu, nan);
    float d = __half2float(__float2half_rn(__fdiv_rn(m, 127.f)));
    d = nan ? __int_as_float(0x7fc00000) : fmaxf(d, 1e-10f);
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float q = rintf(__fdiv_rn(v[k], d));
        q = q < -127.f ? -127.f : (q > 127.f ? 127.f : q);  // comparisons keep a NaN
        y[k] = __fmul_rn(q, d);
    }
    if constexpr (BF16) {
        uint4 raw;
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; k++) h[k] = __float2bfloat16_rn(y[k]);
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + base) = raw;
    } else {
        float* o = static_cast<float*>(out) + base;
        *reinterpret_cast<float4*>(o) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(y[4], y[5], y[6], y[7]);
    }
}

}  // namespace

extern "C" int ltq_int8_rings(const void* in, void* out, long long n_rings, int bf16, void* stream)
{
    if (n_rings < 0 || (bf16 != 0 && bf16 != 1)) return -1;
    if (n_rings == 0) return 0;
    if (!in || !out || ((uintptr_t)in & 15) || ((uintptr_t)out & 15)) return -1;
    const long long threads = 32 * n_rings;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (bf16) int8_rings_kernel<true><<<blocks, 256, 0, (cudaStream_t)stream>>>(in, out, n_rings);
    else int8_rings_kernel<false><<<blocks, 256, 0, (cudaStream_t)stream>>>(in, out, n_rings);
    return (int)cudaGetLastError();
}
