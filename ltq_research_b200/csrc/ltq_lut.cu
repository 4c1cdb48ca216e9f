// DP-profile sub-block quantization through a 1-D lookup table (lumen-inference/ltq-research
// src/cuda/tcq_viterbi.cu:768-811 `lut_subs_kernel`, caller src/liqk_v2.py:469-506 `quantize_liqk_v2_diag_rot`).
//
// For every sub-block i of 16 weights x[16 i + j] with weights d[16 i + j]: the bucket of each weight
// b_j = clamp(rint(x * inv_step + half_b), 0, nb - 1) (one fused multiply-add, round to nearest even), the weighted
// error of each of the 64 candidate columns c of the table, err[c] = sum_j d_j (x_j - lut[b_j][c])^2 accumulated over
// j = 0..15 in order as fma(d * e, e, err) with e = x - lut (the reference kernel's contracted arithmetic), the best
// column (smallest err, the lowest c on ties), and out[16 i + j] = lut[b_j][best].
//
// B200 layout: one warp per sub-block, lane L owning candidates 2L and 2L + 1, so a table row (64 floats, 256 bytes)
// is read once per weight by the whole warp as one coalesced 8-byte-per-lane access instead of by one thread
// (16 rows x 256 bytes per thread); the argmin is a shuffle reduction ordered by (err, c).  The table (nb x 64 fp32,
// 2 MB at the reference's 8192 buckets) stays in L2.
#include <cuda_runtime.h>
#include <stdint.h>
#include "ltq_b200.h"

namespace {

__global__ void __launch_bounds__(256) lut_subs_warp_kernel(const float* __restrict__ xs, const float* __restrict__ dh,
                                                            const float* __restrict__ lut, float* __restrict__ out,
                                                            int S, float inv_step, float half_b, int nb)
{
    const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // sub-block of this warp
    if (i >= S) return;
    const int lane = threadIdx.x & 31;
    // lanes 0..15 hold the sub-block's 16 weights; everyone learns them by shuffles
    const float xl = lane < 16 ? xs[i * 16 + lane] : 0.f;
    const float dl = lane < 16 ? dh[i * 16 + lane] : 0.f;
    int bl = 0;
    if (lane < 16) {
        bl = (int)rintf(__fmaf_rn(xl, inv_step, half_b));
        bl = bl < 0 ? 0 : (bl > nb - 1 ? nb - 1 : bl);
    }
    float e0 = 0.f, e1 = 0.f;  // err of candidates 2 lane, 2 lane + 1
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const float x = __shfl_sync(0xffffffffu, xl, j);
        const float d = __shfl_sync(0xffffffffu, dl, j);
        const int b = __shfl_sync(0xffffffffu, bl, j);
        const float2 v = *reinterpret_cast<const float2*>(lut + (long long)b * 64 + 2 * lane);
        const float a0 = __fsub_rn(x, v.x), a1 = __fsub_rn(x, v.y);
        e0 = __fmaf_rn(__fmul_rn(d, a0), a0, e0);
        e1 = __fmaf_rn(__fmul_rn(d, a1), a1, e1);
    }
    // The reference scans c = 1..63 from err[0] and takes err[c] only when strictly smaller: the lowest c of the
    // smallest value, a NaN never taken, and c = 0 whenever err[0] itself is NaN.  Here: the lane's pair first, then a
    // shuffle reduction ordered by (err, c) in which a NaN loses to any number.
    const bool nan0 = __shfl_sync(0xffffffffu, e0 != e0 ? 1 : 0, 0) != 0;
    float be = e0;
    int bc = 2 * lane;
    if (e1 < be || (be != be && e1 == e1)) { be = e1; bc = 2 * lane + 1; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oe = __shfl_down_sync(0xffffffffu, be, off);
        const int oc = __shfl_down_sync(0xffffffffu, bc, off);
        if (oe < be || (oe == be && oc < bc) || (be != be && oe == oe)) { be = oe; bc = oc; }
    }
    bc = nan0 ? 0 : __shfl_sync(0xffffffffu, bc, 0);
    if (lane < 16) out[i * 16 + lane] = lut[(long long)bl * 64 + bc];
}

}  // namespace

extern "C" int lut_subs_quant(const float* xs, const float* dh, const float* lut, float* out, int S, float inv_step,
                              float half_b, int nb, void* stream)
{
    if (S < 0 || nb < 1 || !xs || !dh || !lut || !out || ((uintptr_t)lut & 7)) return -1;
    if (S == 0) return 0;
    const long long threads = 32LL * S;
    lut_subs_warp_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(xs, dh, lut, out, S,
                                                                                             inv_step, half_b, nb);
    return (int)cudaGetLastError();
}
