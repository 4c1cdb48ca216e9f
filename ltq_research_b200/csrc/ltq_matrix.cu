// Matrix-level kernels of the LTQ quantizer path around the Viterbi (lumen-inference/ltq-research src/liqk_v2.py):
//   * ltq_fwht256       — normalized block FWHT-256 along rows with an optional column scale (src/iqk_format.py:153-170,
//                         used by compute_optimal_suh src/liqk_v2.py:409-441 and _fwht_rows :1024-1026);
//   * ltq_scale_fit     — per-(row, 256-block) scale: fp16 d_row and 5-bit exponent (src/liqk_v2.py:938-946);
//   * ltq_ldlq_gather   — the Viterbi input tiles of one 16-column sub-block (src/liqk_v2.py:913-916, :960-963);
//   * ltq_ldlq_feedback — the intra-block LDLQ error feedback after a sub-block (src/liqk_v2.py:964-971);
//   * ltq_ldlq_bcat / ltq_ldlq_inter — the operands of the inter-block update after a 256-column block
//                         (src/liqk_v2.py:972-979) in the six-product bf16 form of an fp32 GEMM on the tensor cores.
// All are memory-bound SIMT kernels: one warp per row or per (row, block), coalesced 16-byte accesses.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>
#include "ltq_b200.h"

namespace {

// ------------------------------------------------------------------------------------------------
// FWHT-256: one warp per (row, 256-block); lane L holds elements 8L .. 8L + 7.  Stages h = 1, 2, 4 pair elements of one
// lane; stages h = 8 .. 128 pair lane L with lane L ^ (h / 8).  At every stage the lower element of a pair becomes
// a + b and the upper a - b (a = lower, b = upper), exactly the order of the reference's butterfly, then one multiply
// by 256^-1/2 = 1/16.
// ------------------------------------------------------------------------------------------------
template <bool BF16>
__global__ void __launch_bounds__(256) fwht256_kernel(const void* __restrict__ in, long long ld_in, float* __restrict__ out,
                                                      long long ld_out, const float* __restrict__ s, int mode, int rows,
                                                      int nblk)
{
    const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= (long long)rows * nblk) return;
    const int lane = threadIdx.x & 31;
    const long long r = wid / nblk;
    const int b = (int)(wid % nblk);
    const int c0 = b * 256 + 8 * lane;
    float v[8];
    if (BF16) {
        const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(in) + r * ld_in + c0);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __bfloat162float(h[k]);
    } else {
        const float* src = reinterpret_cast<const float*>(in) + r * ld_in + c0;
        const float4 a = *reinterpret_cast<const float4*>(src), c = *reinterpret_cast<const float4*>(src + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    }
    if (mode == 1) {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __fdiv_rn(v[k], s[c0 + k]);
    } else if (mode == 2) {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = __fmul_rn(v[k], s[c0 + k]);
    }
#pragma unroll
    for (int h = 1; h < 8; h <<= 1)
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (!(k & h)) {
                const float a = v[k], bb = v[k + h];
                v[k] = __fadd_rn(a, bb);
                v[k + h] = __fsub_rn(a, bb);
            }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = lane & m;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[k], m);
            v[k] = upper ? __fsub_rn(o, v[k]) : __fadd_rn(v[k], o);
        }
    }
    float* dst = out + r * ld_out + c0;
    *reinterpret_cast<float4*>(dst) = make_float4(v[0] * 0.0625f, v[1] * 0.0625f, v[2] * 0.0625f, v[3] * 0.0625f);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4] * 0.0625f, v[5] * 0.0625f, v[6] * 0.0625f, v[7] * 0.0625f);
}

// ------------------------------------------------------------------------------------------------
// scale fit, one warp per row: rms_rb = sqrt(mean_256(x^2)) clamped to 1e-10, times the format scale;
// d_row = fp16(exp(mean_b log rms_rb)) clamped to 1e-8; e = clamp(round(log2(rms_rb / d_row) / e_step), -e_max, e_max-1);
// d_rb = d_row * 2^(e_step * e).  Block sums: each lane adds 8 squares, then a fixed xor-tree over the warp.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) scale_fit_kernel(const float* __restrict__ W, long long ld, int M, int nblk,
                                                        float scale, float e_step, int e_max, __half* d_row_h,
                                                        float* d_row, int8_t* e_out, float* d_rb)
{
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = threadIdx.x & 31;
    extern __shared__ float sm_rms[];
    float* rms = sm_rms + (threadIdx.x >> 5) * nblk;
    float logsum = 0.f;
    for (int b = 0; b < nblk; b++) {
        const float* src = W + (long long)row * ld + b * 256 + 8 * lane;
        const float4 a = *reinterpret_cast<const float4*>(src), c = *reinterpret_cast<const float4*>(src + 4);
        float acc = __fmul_rn(a.x, a.x);
        acc = __fadd_rn(acc, __fmul_rn(a.y, a.y));
        acc = __fadd_rn(acc, __fmul_rn(a.z, a.z));
        acc = __fadd_rn(acc, __fmul_rn(a.w, a.w));
        acc = __fadd_rn(acc, __fmul_rn(c.x, c.x));
        acc = __fadd_rn(acc, __fmul_rn(c.y, c.y));
        acc = __fadd_rn(acc, __fmul_rn(c.z, c.z));
        acc = __fadd_rn(acc, __fmul_rn(c.w, c.w));
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
        const float r = __fmul_rn(fmaxf(sqrtf(__fdiv_rn(acc, 256.f)), 1e-10f), scale);
        if (lane == 0) rms[b] = r;
        logsum = __fadd_rn(logsum, logf(r));
    }
    // the mean over blocks multiplies by the reciprocal of the count, as torch's mean does
    const float dr = fmaxf(__half2float(__float2half_rn(expf(__fmul_rn(logsum, 1.0f / (float)nblk)))), 1e-8f);
    __syncwarp();
    if (lane == 0) {
        if (d_row_h) d_row_h[row] = __float2half_rn(dr);
        if (d_row) d_row[row] = dr;
    }
    for (int b = lane; b < nblk; b += 32) {
        float e = rintf(__fdiv_rn(log2f(__fdiv_rn(rms[b], dr)), e_step));
        e = fminf(fmaxf(e, (float)-e_max), (float)(e_max - 1));
        if (e_out) e_out[(long long)row * nblk + b] = (int8_t)e;
        if (d_rb) d_rb[(long long)row * nblk + b] = __fmul_rn(dr, exp2f(__fmul_rn(e_step, e)));
    }
}

// ------------------------------------------------------------------------------------------------
// LDLQ sub-block tiles: x[n][16 r + c] = w[16 n + r][c] * inv_d[16 n + r]   (w is a [M, 16] column slice, stride ld)
// ------------------------------------------------------------------------------------------------
__global__ void ldlq_gather_kernel(const float* __restrict__ w, long long ld, const float* __restrict__ inv_d, int M,
                                   float* __restrict__ x)
{
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 4 elements
    if (i >= (long long)M * 4) return;
    const int row = (int)(i >> 2), c = (int)(i & 3) * 4;
    const float4 v = *reinterpret_cast<const float4*>(w + row * ld + c);
    const float s = inv_d[row];
    *reinterpret_cast<float4*>(x + (long long)row * 16 + c) =
        make_float4(__fmul_rn(v.x, s), __fmul_rn(v.y, s), __fmul_rn(v.z, s), __fmul_rn(v.w, s));
}

// ------------------------------------------------------------------------------------------------
// LDLQ feedback after the sub-block at columns [s0, s0 + 16) of a 256-column block, one warp per row:
//   G[:, s0:s1] = g (the Viterbi reconstruction; with code: idx = label * U + u, gi = gain index);
//   err = (w[:, s0:s1] - d * g) @ Uinv[s0:s1, s0:s1];   w[:, s1:256] -= err @ U[s0:s1, s1:256]
// The 16 x (256 - s1) slice of U is staged in shared memory once per CTA.  Each dot product is a sequential fma chain.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ldlq_feedback_kernel(float* __restrict__ w, long long ld, int M, int s0,
                                                            const float* __restrict__ d_rb,
                                                            const float* __restrict__ rec, const int* __restrict__ code,
                                                            const float* __restrict__ U, long long ldU,
                                                            const float* __restrict__ Uinv, long long ldUi,
                                                            float* __restrict__ G, long long ldG, int16_t* __restrict__ idx,
                                                            uint8_t* __restrict__ gi, long long ldP)
{
    __shared__ float sU[16 * 256];
    __shared__ float sUi[16 * 16];
    const int s1 = s0 + 16, ncol = 256 - s1;
    for (int i = threadIdx.x; i < 16 * ncol; i += blockDim.x) sU[i] = U[(long long)(s0 + i / ncol) * ldU + s1 + i % ncol];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sUi[i] = Uinv[(long long)(s0 + i / 16) * ldUi + s0 + i % 16];
    __syncthreads();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = threadIdx.x & 31;
    float* wr = w + (long long)row * ld;
    // lanes 0..15: column s0 + lane of this row
    float e = 0.f;
    if (lane < 16) {
        const float g = rec[(long long)row * 16 + lane];
        G[(long long)row * ldG + s0 + lane] = g;
        if (code) {
            const int cd = code[(long long)row * 16 + lane];
            idx[(long long)row * ldP + s0 + lane] = (int16_t)(cd & 0xffff);
            gi[(long long)row * ldP + s0 + lane] = (uint8_t)(cd >> 16);
        }
        e = __fsub_rn(wr[s0 + lane], __fmul_rn(d_rb[row], g));
    }
    if (ncol == 0) return;
    // err[k] = sum_i e[i] * Uinv[i][k], i ascending
    float err = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float ei = __shfl_sync(0xffffffffu, e, i);
        if (lane < 16) err = __fmaf_rn(ei, sUi[i * 16 + lane], err);
    }
    // w[s1 + j] -= sum_k err[k] * U[k][j], k ascending
    float ek[16];
#pragma unroll
    for (int k = 0; k < 16; k++) ek[k] = __shfl_sync(0xffffffffu, err, k);
    for (int j = lane; j < ncol; j += 32) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) acc = __fmaf_rn(ek[k], sU[k * ncol + j], acc);
        wr[s1 + j] = __fsub_rn(wr[s1 + j], acc);
    }
}

// ------------------------------------------------------------------------------------------------
// Six-product bf16 form of an fp32 product: x = x0 + x1 + x2 with x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1)
// (each difference exact in fp32), and a @ b ~ a0 b0 + a0 b1 + a1 b0 + a0 b2 + a1 b1 + a2 b0, i.e. the product of the
// K-concatenations [a0 a0 a1 a0 a1 a2] and [b0; b1; b0; b2; b1; b0] with fp32 accumulation.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void split3_bf16(float x, uint16_t& p0, uint16_t& p1, uint16_t& p2)
{
    const __nv_bfloat16 h0 = __float2bfloat16_rn(x);
    const float r = __fsub_rn(x, __bfloat162float(h0));
    const __nv_bfloat16 h1 = __float2bfloat16_rn(r);
    const __nv_bfloat16 h2 = __float2bfloat16_rn(__fsub_rn(r, __bfloat162float(h1)));
    p0 = __bfloat16_as_ushort(h0);
    p1 = __bfloat16_as_ushort(h1);
    p2 = __bfloat16_as_ushort(h2);
}

// right operands of every block's update: block b's [1536, N_b] (N_b = K - 256 (b + 1)) matrix
// [u0; u1; u0; u2; u1; u0] of U[256 b : 256 b + 256, 256 (b + 1) : K]; one thread per 4 columns of one source row
__global__ void __launch_bounds__(256) ldlq_bcat_kernel(const float* __restrict__ U, long long ldU, int K,
                                                        uint16_t* __restrict__ out)
{
    const int b = blockIdx.y >> 8, i = blockIdx.y & 255;
    const int c0 = 256 * b, c1 = c0 + 256, nb = K - c1;
    const int j = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (j >= nb) return;
    const long long off = 1536LL * ((long long)b * K - 128LL * b * (b + 1));
    const float4 v = *reinterpret_cast<const float4*>(U + (long long)(c0 + i) * ldU + c1 + j);
    const float x[4] = {v.x, v.y, v.z, v.w};
    uint16_t p[3][4];
#pragma unroll
    for (int k = 0; k < 4; k++) split3_bf16(x[k], p[0][k], p[1][k], p[2][k]);
    constexpr int part_of_slot[6] = {0, 1, 0, 2, 1, 0};
#pragma unroll
    for (int sl = 0; sl < 6; sl++) {
        const int q = part_of_slot[sl];
        const uint2 w = make_uint2((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16));
        *reinterpret_cast<uint2*>(out + off + (long long)(256 * sl + i) * nb + j) = w;
    }
}

// The right operands of every block's update in the compact three-part form of the tensor-core GEMM
// (ltq_gemm_bf16x6_tn, both operands K-major): block b's [N_b, 768] matrix with row n = [u0 u1 u2], the three-way split
// of column c1 + n of U[256 b : 256 b + 256, :], i.e. out_b[n][256 p + i] = part_p(U[c0 + i][c1 + n]), at element offset
// 768 * sum_{b' < b} N_b'.  A 32 x 32 tile of U per CTA (32 x 8 threads): read along n (coalesced), split, transposed
// through shared memory, written along i (64 bytes per part and row).  blockIdx = (n tile, i tile, block b).
__global__ void __launch_bounds__(256) ldlq_bcat3_t_kernel(const float* __restrict__ U, long long ldU, int K,
                                                           uint16_t* __restrict__ out)
{
    __shared__ uint16_t sp[3][32][34];  // [part][n][i]
    const int b = blockIdx.z, c0 = 256 * b, c1 = c0 + 256, nb = K - c1;
    const int n0 = 32 * blockIdx.x, i0 = 32 * blockIdx.y;
    if (n0 >= nb) return;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const long long off = 768LL * ((long long)b * K - 128LL * b * (b + 1));
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int i = ty + 8 * q;
        uint16_t p0, p1, p2;
        split3_bf16(U[(long long)(c0 + i0 + i) * ldU + c1 + n0 + tx], p0, p1, p2);
        sp[0][tx][i] = p0;
        sp[1][tx][i] = p1;
        sp[2][tx][i] = p2;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int n = ty + 8 * q;
        uint16_t* row = out + off + (long long)(n0 + n) * 768 + i0 + tx;
#pragma unroll
        for (int pt = 0; pt < 3; pt++) row[256 * pt] = sp[pt][n][tx];
    }
}

// after block [c0, c0 + 256): W_hat = d * G, d_h = fp16(d), e = w - W_hat (the reference's operations, same bits), and
// for the update err = e @ Uinv (Uinv upper triangular: err[k] = sum_{i <= k} e[i] Uinv[i][k], i ascending, fma) split
// into acat [M, 1536] = [e0 e0 e1 e0 e1 e2].  One CTA per 16 rows, thread k = column k.
template <bool COMPACT>
__global__ void __launch_bounds__(256) ldlq_inter_kernel(const float* __restrict__ w, long long ld_w,
                                                         const float* __restrict__ d_rb, long long ld_d,
                                                         const float* __restrict__ G, long long ldG,
                                                         const float* __restrict__ Uinv, long long ldUi,
                                                         float* __restrict__ what, long long ld_what,
                                                         uint16_t* __restrict__ d_h, long long ld_dh,
                                                         uint16_t* __restrict__ acat)
{
    __shared__ __align__(16) float se[256 * 20];  // e[r][i] at se[20 i + r] (rows of one column contiguous)
    __shared__ __align__(16) float su[16 * 256];  // 16 rows of Uinv at a time
    const int k = threadIdx.x;
    const long long r0 = 16LL * blockIdx.x;
#pragma unroll 4
    for (int r = 0; r < 16; r++) {
        const long long row = r0 + r;
        const float d = fmaxf(d_rb[row * ld_d], 1e-8f);
        const float wh = __fmul_rn(d, G[row * ldG + k]);
        what[row * ld_what + k] = wh;
        se[20 * k + r] = __fsub_rn(w[row * ld_w + k], wh);
        if (k == 0 && d_h) d_h[row * ld_dh] = __half_as_ushort(__float2half_rn(d));
    }
    if (!acat) return;
    __syncthreads();
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; r++) acc[r] = 0.f;
    // rows i0 .. i0 + 15 of Uinv staged in shared memory by the whole CTA (coalesced), then consumed by every column
    for (int i0 = 0; i0 < 256; i0 += 16) {
        __syncthreads();
        for (int t = k; t < 16 * 64; t += 256) {
            const int r = t >> 6, c = 4 * (t & 63);
            *reinterpret_cast<float4*>(su + 256 * r + c) =
                *reinterpret_cast<const float4*>(Uinv + (long long)(i0 + r) * ldUi + c);
        }
        __syncthreads();
        const int iend = k + 1 < i0 + 16 ? k + 1 : i0 + 16;
        for (int i = i0; i < iend; i++) {
            const float u = su[256 * (i - i0) + k];
            const float4* e4 = reinterpret_cast<const float4*>(se + 20 * i);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 e = e4[q];
                acc[4 * q] = __fmaf_rn(e.x, u, acc[4 * q]);
                acc[4 * q + 1] = __fmaf_rn(e.y, u, acc[4 * q + 1]);
                acc[4 * q + 2] = __fmaf_rn(e.z, u, acc[4 * q + 2]);
                acc[4 * q + 3] = __fmaf_rn(e.w, u, acc[4 * q + 3]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 16; r++) {
        uint16_t p0, p1, p2;
        split3_bf16(acc[r], p0, p1, p2);
        if constexpr (COMPACT) {  // [e0 e1 e2], row stride 768
            uint16_t* a = acat + (r0 + r) * 768 + k;
            a[0] = p0; a[256] = p1; a[512] = p2;
        } else {  // the six slots [e0 e0 e1 e0 e1 e2], row stride 1536
            uint16_t* a = acat + (r0 + r) * 1536 + k;
            a[0] = p0; a[256] = p0; a[512] = p1; a[768] = p0; a[1024] = p1; a[1280] = p2;
        }
    }
}

// one operand of the six-product form of x (rows x cols, row stride ld; batch element z at x + z * xbs): order 0 puts
// the parts [x0 x0 x1 x0 x1 x2] in the six slots (left operand), order 1 [x0 x1 x0 x2 x1 x0] (right operand); side 0
// concatenates the slots along the columns (out[r][s cols + c]), side 1 along the rows (out[s rows + r][c]); neg splits
// -x (exact).  One thread per 4 columns of one row; blockIdx.y = batch element.
__global__ void __launch_bounds__(256) bf16x6_split_kernel(const float* __restrict__ x, long long ld, long long xbs,
                                                           int rows, int cols, int order, int side, int neg,
                                                           uint16_t* __restrict__ out, long long ld_out, long long obs)
{
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int c4 = cols >> 2;
    if (t >= (long long)rows * c4) return;
    x += (long long)blockIdx.y * xbs;
    out += (long long)blockIdx.y * obs;
    const int r = (int)(t / c4), c = 4 * (int)(t - (long long)r * c4);
    const float4 v = *reinterpret_cast<const float4*>(x + (long long)r * ld + c);
    const float sg = neg ? -1.f : 1.f;
    const float xv[4] = {sg * v.x, sg * v.y, sg * v.z, sg * v.w};
    uint16_t p[3][4];
#pragma unroll
    for (int k = 0; k < 4; k++) split3_bf16(xv[k], p[0][k], p[1][k], p[2][k]);
    constexpr int left[6] = {0, 0, 1, 0, 1, 2}, right[6] = {0, 1, 0, 2, 1, 0};
#pragma unroll
    for (int sl = 0; sl < 6; sl++) {
        const int q = order ? right[sl] : left[sl];
        const uint2 w = make_uint2((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16));
        const long long o = side ? ((long long)sl * rows + r) * ld_out + c : (long long)r * ld_out + (long long)sl * cols + c;
        *reinterpret_cast<uint2*>(out + o) = w;
    }
}

// Compact three-part operand of the tensor-core GEMM (ltq_gemm_bf16x3p_tn) for `batch` fp32 matrices x_z = x + z xbs
// (rows x cols, row stride ld), parts along the columns at stride Kp, zero-padded to Kp:
//   trans 0: out_z[r][p Kp + c] = part_p(s x_z[r][c])   (r < rows; c < Kp, 0 for c >= cols)
//   trans 1: out_z[c][p Kp + r] = part_p(s x_z[r][c])   (c < cols; r < Kp, 0 for r >= rows)
// with s = -1 when neg (exact) else 1, part_p the three-way bf16 split.  trans 0: one thread per 4 columns of a row;
// trans 1: 32 x 32 tiles through shared memory (reads along c, writes along r).
__global__ void __launch_bounds__(256) bf16x3_split_kernel(const float* __restrict__ x, long long ld, long long xbs,
                                                           int rows, int cols, int neg, int Kp,
                                                           uint16_t* __restrict__ out, long long ld_out, long long obs)
{
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int c4 = Kp >> 2;
    if (t >= (long long)rows * c4) return;
    x += (long long)blockIdx.y * xbs;
    out += (long long)blockIdx.y * obs;
    const int r = (int)(t / c4), c = 4 * (int)(t - (long long)r * c4);
    const float sg = neg ? -1.f : 1.f;
    uint16_t p[3][4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float v = c + k < cols ? sg * x[(long long)r * ld + c + k] : 0.f;
        split3_bf16(v, p[0][k], p[1][k], p[2][k]);
    }
#pragma unroll
    for (int q = 0; q < 3; q++)
        *reinterpret_cast<uint2*>(out + (long long)r * ld_out + (long long)q * Kp + c) =
            make_uint2((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16));
}

__global__ void __launch_bounds__(256) bf16x3_split_t_kernel(const float* __restrict__ x, long long ld, long long xbs,
                                                             int rows, int cols, int neg, int Kp,
                                                             uint16_t* __restrict__ out, long long ld_out,
                                                             long long obs)
{
    __shared__ uint16_t sp[3][32][34];  // [part][c][r]
    const int c0 = 32 * blockIdx.x, r0 = 32 * blockIdx.y;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    x += (long long)blockIdx.z * xbs;
    out += (long long)blockIdx.z * obs;
    const float sg = neg ? -1.f : 1.f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int r = r0 + ty + 8 * q, c = c0 + tx;
        const float v = (r < rows && c < cols) ? sg * x[(long long)r * ld + c] : 0.f;
        uint16_t p0, p1, p2;
        split3_bf16(v, p0, p1, p2);
        sp[0][tx][ty + 8 * q] = p0;
        sp[1][tx][ty + 8 * q] = p1;
        sp[2][tx][ty + 8 * q] = p2;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int c = c0 + ty + 8 * q;
        if (c >= cols) continue;
        uint16_t* row = out + (long long)c * ld_out + r0 + tx;
#pragma unroll
        for (int pt = 0; pt < 3; pt++) row[(long long)pt * Kp] = sp[pt][ty + 8 * q][tx];
    }
}

// inverse of the 256 x 256 lower-triangular diagonal block b of L (row-major, row stride ldL) into the diagonal block of
// X (row stride ldX; the block's upper part written as 0), by forward substitution: thread t owns column j = 128 h + t
// (h = blockIdx.y), x_i = (delta_ij - sum_{k < i} L_ik x_k) / L_ii for i >= j, the sum in ascending k; the column lives
// in shared memory (x_k = 0 for k < j, so every thread runs the same k range).
__global__ void __launch_bounds__(128) trtri256_lower_kernel(const float* __restrict__ L, long long ldL,
                                                             float* __restrict__ X, long long ldX)
{
    extern __shared__ float xs[];  // [256][128]
    const int t = threadIdx.x, h = blockIdx.y, j = 128 * h + t, i0 = 128 * h;
    const long long b = blockIdx.x;
    const float* Lb = L + 256 * b * (ldL + 1);
    float* Xb = X + 256 * b * (ldX + 1);
    for (int i = i0; i < 256; i++) {
        const float* Li = Lb + (long long)i * ldL;
        float acc = 0.f;
        int k = i0;
#pragma unroll 4
        for (; k < i; k++) acc = __fmaf_rn(__ldg(Li + k), xs[(k - i0) * 128 + t], acc);
        const float x = i < j ? 0.f : __fdiv_rn(__fsub_rn(i == j ? 1.f : 0.f, acc), __ldg(Li + i));
        xs[(i - i0) * 128 + t] = x;
    }
    for (int i = 0; i < 256; i++) Xb[(long long)i * ldX + j] = i < i0 ? 0.f : xs[(i - i0) * 128 + t];
}

// Cholesky of the 256 x 256 diagonal block at (c0, c0) of A (row-major, row stride ld; lower triangle read; the
// trailing updates of the earlier panels already applied) and the inverse of its factor, the diagonal step of
// hessian.cholesky_lower.  One CTA holds the block in registers: 528 threads each own one 8 x 8 tile (bi >= bk) of the
// lower triangle, ordered by tile column, so that the tiles still active near the end of the sweep fill whole warps.
//   phase 1, the factorization in LDL^T form: at pivot j the owners of tile column j/8 broadcast column j through
//     shared memory (double-buffered, one barrier per pivot) and every tile right of it accumulates
//     s_ik += (a_ij / a_jj) a_kj — 64 fma a thread, the mask on the tile column holding j keeps columns <= j; a value
//     is its loaded one minus its sum, formed once when its column is the pivot column and once at the end (a
//     separate sum keeps the rounding of the left-looking, dot-product form: measured on a damped Gram block, backward
//     error 2.9e-8 against 5.6e-7 when each update was subtracted from the running value); the loaded block waits in
//     the L~ region meanwhile; at the end L_ik = a_ik / sqrt(d_k) goes to A and L~_ik = a_ik / d_k (unit lower) to
//     shared memory, column-major with every column starting at its tile row (32-byte aligned: 132 KB);
//   phase 2, Y = L~^-1 by Gauss-Jordan on the identity: at pivot j the owners of tile row j/8 broadcast row j of Y and
//     every tile below it and left of it takes y_ik -= L~_ij y_jk (rows i > j); then X = L^-1 = D^-1/2 Y;
//   outputs: L in A's block (zeros above the diagonal); xt3 [256][768] (bf16) = the compact right operand of the panel
//     product A_21 X^T for ltq_gemm_bf16x3p_tn, row n = [x0 x1 x2] of row n of X (every element written); X itself at Xo
//     (the block's first element, row stride ldx; tiles on and below the diagonal) when Xo is given; *info = c0 + j + 1
//     for the first pivot that is not
//     positive (or NaN) when *info was 0 (LAPACK's convention).
constexpr int LT_FLOATS = 33792;  // sum over columns of 256 - 8 * (j / 8)
__device__ __forceinline__ int lt_col(int j)
{
    const int jb = j >> 3, c = j & 7;
    return 8 * (256 * jb - 4 * jb * (jb - 1)) + c * (256 - 8 * jb);
}

__global__ void __launch_bounds__(544, 1) chol256_tiled_kernel(float* __restrict__ A, long long ld, int c0,
                                                               uint16_t* __restrict__ xt3, float* __restrict__ Xo,
                                                               long long ldx, int* __restrict__ info)
{
    extern __shared__ __align__(16) float smem[];
    float* lt = smem;                 // L~, column-major from each column's tile row
    float* cb = smem + LT_FLOATS;     // 2 x 256 broadcast buffers
    float* sd = cb + 512;             // the pivots d_j
    const int tid = threadIdx.x;
    int bk = 0, rem = tid;
    while (bk < 32 && rem >= 32 - bk) { rem -= 32 - bk; bk++; }
    const bool own = bk < 32;
    const int bi = bk + rem;
    float* Ab = A + (long long)c0 * (ld + 1);
    float a[8][8];
#pragma unroll
    for (int r = 0; r < 8; r++) {
        float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
        if (own) {
            const float* src = Ab + (long long)(8 * bi + r) * ld + 8 * bk;
            v0 = *reinterpret_cast<const float4*>(src);
            v1 = *reinterpret_cast<const float4*>(src + 4);
        }
        a[r][0] = v0.x; a[r][1] = v0.y; a[r][2] = v0.z; a[r][3] = v0.w;
        a[r][4] = v1.x; a[r][5] = v1.y; a[r][6] = v1.z; a[r][7] = v1.w;
    }
    // the block as loaded goes to shared memory (in the layout of L~ below, each element read back only by its owner);
    // the registers then accumulate the updates sum_j (a_ij / a_jj) a_kj, subtracted from the loaded value once, when
    // the column becomes the pivot column and at the end (one rounding of the running value instead of one per pivot)
    if (own) {
#pragma unroll
        for (int cc = 0; cc < 8; cc++) {
            float* col = lt + lt_col(8 * bk + cc) + 8 * (bi - bk);
            *reinterpret_cast<float4*>(col) = make_float4(a[0][cc], a[1][cc], a[2][cc], a[3][cc]);
            *reinterpret_cast<float4*>(col + 4) = make_float4(a[4][cc], a[5][cc], a[6][cc], a[7][cc]);
        }
    }
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int cc = 0; cc < 8; cc++) a[r][cc] = 0.f;
    for (int jb = 0; jb < 32; jb++) {
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int j = 8 * jb + c;
            float* buf = cb + (c & 1) * 256;
            if (own && bk == jb) {
                const float* col = lt + lt_col(j) + 8 * (bi - jb);
                const float4 o0 = *reinterpret_cast<const float4*>(col);
                const float4 o1 = *reinterpret_cast<const float4*>(col + 4);
                const float v[8] = {__fsub_rn(o0.x, a[0][c]), __fsub_rn(o0.y, a[1][c]), __fsub_rn(o0.z, a[2][c]),
                                    __fsub_rn(o0.w, a[3][c]), __fsub_rn(o1.x, a[4][c]), __fsub_rn(o1.y, a[5][c]),
                                    __fsub_rn(o1.z, a[6][c]), __fsub_rn(o1.w, a[7][c])};
                *reinterpret_cast<float4*>(buf + 8 * bi) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4*>(buf + 8 * bi + 4) = make_float4(v[4], v[5], v[6], v[7]);
                if (bi == jb) {
                    sd[j] = v[c];
                    if (!(v[c] > 0.f)) atomicCAS(info, 0, c0 + j + 1);
                }
            }
            __syncthreads();
            if (own && bk >= jb) {
                const float inv = __frcp_rn(buf[j]);
                const float4 k0 = *reinterpret_cast<const float4*>(buf + 8 * bk);
                const float4 k1 = *reinterpret_cast<const float4*>(buf + 8 * bk + 4);
                float ck[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
                if (bk == jb) {
#pragma unroll
                    for (int cc = 0; cc <= c; cc++) ck[cc] = 0.f;
                }
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const float t = buf[8 * bi + r] * inv;
#pragma unroll
                    for (int cc = 0; cc < 8; cc++) a[r][cc] = __fmaf_rn(t, ck[cc], a[r][cc]);
                }
            }
        }
    }
    __syncthreads();
    if (own) {
        // the final values: loaded minus accumulated (a column's sum stops growing once it has been the pivot column)
#pragma unroll
        for (int cc = 0; cc < 8; cc++) {
            const float* col = lt + lt_col(8 * bk + cc) + 8 * (bi - bk);
            const float4 o0 = *reinterpret_cast<const float4*>(col);
            const float4 o1 = *reinterpret_cast<const float4*>(col + 4);
            a[0][cc] = __fsub_rn(o0.x, a[0][cc]); a[1][cc] = __fsub_rn(o0.y, a[1][cc]);
            a[2][cc] = __fsub_rn(o0.z, a[2][cc]); a[3][cc] = __fsub_rn(o0.w, a[3][cc]);
            a[4][cc] = __fsub_rn(o1.x, a[4][cc]); a[5][cc] = __fsub_rn(o1.y, a[5][cc]);
            a[6][cc] = __fsub_rn(o1.z, a[6][cc]); a[7][cc] = __fsub_rn(o1.w, a[7][cc]);
        }
#pragma unroll
        for (int cc = 0; cc < 8; cc++) {
            const float rd = __frcp_rn(sd[8 * bk + cc]);
            float* col = lt + lt_col(8 * bk + cc) + 8 * (bi - bk);
            *reinterpret_cast<float4*>(col) = make_float4(a[0][cc] * rd, a[1][cc] * rd, a[2][cc] * rd, a[3][cc] * rd);
            *reinterpret_cast<float4*>(col + 4) = make_float4(a[4][cc] * rd, a[5][cc] * rd, a[6][cc] * rd, a[7][cc] * rd);
        }
#pragma unroll
        for (int cc = 0; cc < 8; cc++) {
            const float dk = sd[8 * bk + cc];
            const float rs = __frsqrt_rn(dk);
#pragma unroll
            for (int r = 0; r < 8; r++)
                a[r][cc] = (bi != bk || r > cc) ? a[r][cc] * rs : (r == cc ? __fsqrt_rn(dk) : 0.f);
        }
#pragma unroll
        for (int r = 0; r < 8; r++) {
            float* dst = Ab + (long long)(8 * bi + r) * ld + 8 * bk;
            *reinterpret_cast<float4*>(dst) = make_float4(a[r][0], a[r][1], a[r][2], a[r][3]);
            *reinterpret_cast<float4*>(dst + 4) = make_float4(a[r][4], a[r][5], a[r][6], a[r][7]);
            if (bi != bk) {  // the mirror tile above the diagonal: zeros, so that the block holds exactly L
                float* up = Ab + (long long)(8 * bk + r) * ld + 8 * bi;
                *reinterpret_cast<float4*>(up) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(up + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    // phase 2: Y = L~^-1, in the registers of the factor's tile
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int cc = 0; cc < 8; cc++) a[r][cc] = (bi == bk && r == cc) ? 1.f : 0.f;
    __syncthreads();
    for (int jb = 0; jb < 32; jb++) {
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int j = 8 * jb + c;
            float* buf = cb + (c & 1) * 256;
            if (own && bi == jb) {
                *reinterpret_cast<float4*>(buf + 8 * bk) = make_float4(a[c][0], a[c][1], a[c][2], a[c][3]);
                *reinterpret_cast<float4*>(buf + 8 * bk + 4) = make_float4(a[c][4], a[c][5], a[c][6], a[c][7]);
            }
            __syncthreads();
            if (own && bk <= jb && bi >= jb) {
                const float* col = lt + lt_col(j) + 8 * (bi - jb);
                const float4 y0 = *reinterpret_cast<const float4*>(buf + 8 * bk);
                const float4 y1 = *reinterpret_cast<const float4*>(buf + 8 * bk + 4);
                const float yk[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const float l = (bi == jb && r <= c) ? 0.f : col[r];
#pragma unroll
                    for (int cc = 0; cc < 8; cc++) a[r][cc] = __fmaf_rn(-l, yk[cc], a[r][cc]);
                }
            }
        }
    }
    if (!own) return;
    // X = D^-1/2 Y; X^T's six-slot operand: row k = 8 bk + cc, columns 8 bi .. 8 bi + 7 (and zeros at the mirror)
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const float rs = __frsqrt_rn(sd[8 * bi + r]);
#pragma unroll
        for (int cc = 0; cc < 8; cc++) a[r][cc] *= rs;
    }
    if (Xo) {
        float* Xb = Xo;  // the block's first element (the caller placed it)
#pragma unroll
        for (int r = 0; r < 8; r++) {
            float* dst = Xb + (long long)(8 * bi + r) * ldx + 8 * bk;
            *reinterpret_cast<float4*>(dst) = make_float4(a[r][0], a[r][1], a[r][2], a[r][3]);
            *reinterpret_cast<float4*>(dst + 4) = make_float4(a[r][4], a[r][5], a[r][6], a[r][7]);
        }
    }
    // the compact right operand of the panel product A21 X^T: row n of xt3 = [x0 x1 x2] of row n of X, i.e. this
    // thread's 8 x 8 tile in rows 8 bi + r, columns 8 bk .. 8 bk + 7 of each part (and the zero tile above the diagonal)
#pragma unroll
    for (int r = 0; r < 8; r++) {
        uint32_t w[3][4];  // the three bf16 parts of row r's 8 values, two to a word
#pragma unroll
        for (int cc = 0; cc < 8; cc += 2) {
            uint16_t p0, p1, p2, q0, q1, q2;
            split3_bf16(a[r][cc], p0, p1, p2);
            split3_bf16(a[r][cc + 1], q0, q1, q2);
            w[0][cc / 2] = p0 | (uint32_t)q0 << 16;
            w[1][cc / 2] = p1 | (uint32_t)q1 << 16;
            w[2][cc / 2] = p2 | (uint32_t)q2 << 16;
        }
#pragma unroll
        for (int q = 0; q < 3; q++) {
            *reinterpret_cast<uint4*>(xt3 + (long long)(8 * bi + r) * 768 + 256 * q + 8 * bk) =
                make_uint4(w[q][0], w[q][1], w[q][2], w[q][3]);
            if (bi != bk)
                *reinterpret_cast<uint4*>(xt3 + (long long)(8 * bk + r) * 768 + 256 * q + 8 * bi) = make_uint4(0, 0, 0, 0);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// Solve L L^T x = b for a blocked lower Cholesky factor L [K, K] (row-major, K a multiple of 256) given the inverses
// Dinv[p] of its 256 x 256 diagonal blocks (as the factorization's leaves write them; upper parts zero).  Block forward
// substitution, one launch per 256-row block and direction, no waits between CTAs:
//   forward  step p: y_p = Dinv_p r_p, then r_q -= L[q, p] y_p for the blocks q > p;
//   backward step p: x_p = Dinv_p^T r_p, then r_q -= L[p, q]^T x_p for the blocks q < p.
// Every CTA of a step computes y_p (x_p) itself from the block's residual (a 256 x 256 product, from L2), then updates
// its own 256 entries of r; CTA 0 writes y_p (x_p).  Each entry is one thread's fma chain in a fixed order: the result
// is deterministic.  Multiplying by the inverted diagonal blocks instead of substituting is the form the factorization
// itself uses for its panels (backward stable, slightly larger forward error than substitution).
// ------------------------------------------------------------------------------------------------
// 256 row sums out[i] = sum_k M[i][k] v[k] (k < 256) by a CTA of 1024 threads: warp w takes rows 8 w .. 8 w + 7, each
// lane two float4 of a row (coalesced 512-byte rows), then a fixed shuffle tree per row
__device__ __forceinline__ void rowdot256(const float* __restrict__ M, long long ldm, const float* v, float* out)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    float4 m[8][2];
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int h = 0; h < 2; h++)
            m[r][h] = __ldg(reinterpret_cast<const float4*>(M + (long long)(8 * w + r) * ldm + 128 * h + 4 * lane));
#pragma unroll
    for (int r = 0; r < 8; r++) {
        float a = 0.f;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int k = 128 * h + 4 * lane;
            a = __fmaf_rn(m[r][h].x, v[k], a);
            a = __fmaf_rn(m[r][h].y, v[k + 1], a);
            a = __fmaf_rn(m[r][h].z, v[k + 2], a);
            a = __fmaf_rn(m[r][h].w, v[k + 3], a);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) out[8 * w + r] = a;
    }
}

// 256 column sums out[j] = sum_i M[i][j] v[i] (i < 256) by 1024 threads: thread (j, quarter) sums rows 64 quarter ..
// + 63 of column j (reads coalesced along j), then the four quarters are added in order through `part`
__device__ __forceinline__ void coldot256(const float* __restrict__ M, long long ldm, const float* v, float* part,
                                          float* out)
{
    const int j = threadIdx.x & 255, qtr = threadIdx.x >> 8;
    float a = 0.f;
#pragma unroll 16
    for (int i = 64 * qtr; i < 64 * qtr + 64; i++) a = __fmaf_rn(__ldg(M + (long long)i * ldm + j), v[i], a);
    part[threadIdx.x] = a;
    __syncthreads();
    if (qtr == 0)
        out[j] = __fadd_rn(__fadd_rn(__fadd_rn(part[j], part[256 + j]), part[512 + j]), part[768 + j]);
}

__global__ void __launch_bounds__(1024) chol_solve_fwd_step(const float* __restrict__ L, long long ld,
                                                            const float* __restrict__ Dinv, float* __restrict__ r,
                                                            float* __restrict__ y, int p, int K)
{
    __shared__ float rp[256], yp[256], u[256];
    const int t = threadIdx.x, c0 = 256 * p;
    if (t < 256) rp[t] = r[c0 + t];
    __syncthreads();
    // y_p = Dinv_p r_p (Dinv_p is lower with exact zeros above the diagonal)
    rowdot256(Dinv + (size_t)p * 65536, 256, rp, yp);
    __syncthreads();
    if (blockIdx.x == 0 && t < 256) y[c0 + t] = yp[t];
    const long long q0 = c0 + 256 + 256LL * blockIdx.x;  // this CTA's 256 rows of the blocks below p
    if (q0 < K) {
        rowdot256(L + q0 * ld + c0, ld, yp, u);
        __syncthreads();
        if (t < 256) r[q0 + t] = __fsub_rn(r[q0 + t], u[t]);
    }
}

__global__ void __launch_bounds__(1024) chol_solve_bwd_step(const float* __restrict__ L, long long ld,
                                                            const float* __restrict__ Dinv, float* __restrict__ r,
                                                            float* __restrict__ x, int p)
{
    __shared__ float rp[256], xp[256], u[256], part[1024];
    const int t = threadIdx.x, c0 = 256 * p;
    if (t < 256) rp[t] = r[c0 + t];
    __syncthreads();
    // x_p = Dinv_p^T r_p: column sums of Dinv_p
    coldot256(Dinv + (size_t)p * 65536, 256, rp, part, xp);
    __syncthreads();
    if (blockIdx.x == 0 && t < 256) x[c0 + t] = xp[t];
    const int q0 = 256 * blockIdx.x;  // this CTA's 256 entries of the blocks before p
    if (q0 < c0) {
        coldot256(L + (long long)c0 * ld + q0, ld, xp, part, u);
        __syncthreads();
        if (t < 256) r[q0 + t] = __fsub_rn(r[q0 + t], u[t]);
    }
}

}  // namespace

extern "C" int ltq_fwht256(const void* in, int in_bf16, long long ld_in, float* out, long long ld_out, const float* scale,
                           int mode, int rows, int cols, void* stream)
{
    if (rows < 0 || cols < 0 || cols % 256 || mode < 0 || mode > 2 || (mode && !scale) || ld_in < cols || ld_out < cols ||
        (ld_in % 8) || (ld_out % 4))
        return -1;
    if (rows == 0 || cols == 0) return 0;
    const long long warps = (long long)rows * (cols / 256);
    const int blocks = (int)((warps + 7) / 8);
    if (in_bf16)
        fwht256_kernel<true><<<blocks, 256, 0, (cudaStream_t)stream>>>(in, ld_in, out, ld_out, scale, mode, rows, cols / 256);
    else
        fwht256_kernel<false><<<blocks, 256, 0, (cudaStream_t)stream>>>(in, ld_in, out, ld_out, scale, mode, rows, cols / 256);
    return (int)cudaGetLastError();
}

extern "C" int ltq_scale_fit(const float* W, long long ld, int M, int K, float scale, float e_step, int e_bits,
                             uint16_t* d_row_h, float* d_row, int8_t* e, float* d_rb, void* stream)
{
    if (M < 0 || K <= 0 || K % 256 || ld < K || (ld % 4) || e_bits < 1 || e_bits > 8 || !(e_step > 0.f)) return -1;
    if (M == 0) return 0;
    const int nblk = K / 256;
    const int smem = 8 * nblk * 4;
    if (smem > 48 * 1024) return -1;
    scale_fit_kernel<<<(M + 7) / 8, 256, smem, (cudaStream_t)stream>>>(W, ld, M, nblk, scale, e_step, 1 << (e_bits - 1),
                                                                       reinterpret_cast<__half*>(d_row_h), d_row, e, d_rb);
    return (int)cudaGetLastError();
}

extern "C" int ltq_ldlq_gather(const float* w, long long ld, const float* inv_d, int M, float* x, void* stream)
{
    if (M < 0 || M % 16 || (ld % 4) || ((uintptr_t)w & 15)) return -1;
    if (M == 0) return 0;
    const long long n = (long long)M * 4;
    ldlq_gather_kernel<<<(int)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(w, ld, inv_d, M, x);
    return (int)cudaGetLastError();
}

extern "C" int ltq_ldlq_feedback(float* w, long long ld, int M, int s0, const float* d_rb, const float* rec,
                                 const int* code, const float* U, long long ldU, const float* Uinv, long long ldUi,
                                 float* G, long long ldG, int16_t* idx, uint8_t* gi, long long ldP, void* stream)
{
    if (M < 0 || s0 < 0 || s0 > 240 || s0 % 16 || (code && (!idx || !gi))) return -1;
    if (M == 0) return 0;
    ldlq_feedback_kernel<<<(M + 7) / 8, 256, 0, (cudaStream_t)stream>>>(w, ld, M, s0, d_rb, rec, code, U, ldU, Uinv, ldUi,
                                                                       G, ldG, idx, gi, ldP);
    return (int)cudaGetLastError();
}

extern "C" size_t ltq_ldlq_bcat_elems(int K)
{
    if (K < 256 || K % 256) return 0;
    const long long nb = K / 256 - 1;  // blocks with an update
    return (size_t)(1536LL * (nb * K - 128LL * nb * (nb + 1)));
}

extern "C" int ltq_ldlq_bcat_t(const float* U, long long ldU, int K, uint16_t* bcat, void* stream)
{
    if (K < 512 || K % 256 || ldU < K || !U || !bcat || ((uintptr_t)bcat & 15)) return -1;
    const dim3 grid((K - 256) / 32, 8, K / 256 - 1);
    ldlq_bcat3_t_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(U, ldU, K, bcat);
    return (int)cudaGetLastError();
}

extern "C" int ltq_ldlq_bcat(const float* U, long long ldU, int K, uint16_t* bcat, void* stream)
{
    if (K < 256 || K % 256 || ldU < K || ((uintptr_t)U & 15) || (ldU & 3) || ((uintptr_t)bcat & 7)) return -1;
    const int nb = K / 256 - 1;
    if (nb == 0) return 0;
    const dim3 grid((unsigned)((K - 256) / 4 + 255) / 256, (unsigned)(nb * 256));
    ldlq_bcat_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(U, ldU, K, bcat);
    return (int)cudaGetLastError();
}

extern "C" int ltq_ldlq_inter(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* G,
                              long long ldG, const float* Uinv, long long ldUi, int M, float* what, long long ld_what,
                              uint16_t* d_h, long long ld_dh, uint16_t* acat, void* stream)
{
    if (M < 0 || M % 16 || !w_blk || !d_rb || !G || !what || (acat && (!Uinv || ((uintptr_t)Uinv & 15) || ldUi % 4)))
        return -1;
    if (M == 0) return 0;
    ldlq_inter_kernel<false><<<M / 16, 256, 0, (cudaStream_t)stream>>>(w_blk, ld_w, d_rb, ld_d, G, ldG, Uinv, ldUi,
                                                                      what, ld_what, d_h, ld_dh, acat);
    return (int)cudaGetLastError();
}

extern "C" int ltq_ldlq_inter3(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* G,
                               long long ldG, const float* Uinv, long long ldUi, int M, float* what, long long ld_what,
                               uint16_t* d_h, long long ld_dh, uint16_t* acat3, void* stream)
{
    if (M < 0 || M % 16 || !w_blk || !d_rb || !G || !what || (acat3 && (!Uinv || ((uintptr_t)Uinv & 15) || ldUi % 4)))
        return -1;
    if (M == 0) return 0;
    ldlq_inter_kernel<true><<<M / 16, 256, 0, (cudaStream_t)stream>>>(w_blk, ld_w, d_rb, ld_d, G, ldG, Uinv, ldUi,
                                                                     what, ld_what, d_h, ld_dh, acat3);
    return (int)cudaGetLastError();
}

extern "C" int ltq_bf16x3_split(const float* x, long long ld, long long xbs, int rows, int cols, int batch, int trans,
                                int neg, int Kp, uint16_t* out, long long ld_out, long long obs, void* stream)
{
    if (rows < 0 || cols < 0 || batch < 1 || batch > 65535 || (trans != 0 && trans != 1) || Kp < 0 || Kp % 32 ||
        !x || !out || ld < cols || ld_out < 3LL * Kp || ld_out % 4 || ((uintptr_t)out & 7) ||
        (trans ? Kp < rows : Kp < cols))
        return -1;
    const int orows = trans ? cols : rows;
    if (orows == 0 || Kp == 0) return 0;
    cudaStream_t st = (cudaStream_t)stream;
    if (!trans) {
        const long long threads = (long long)rows * (Kp / 4);
        bf16x3_split_kernel<<<dim3((unsigned)((threads + 255) / 256), batch), 256, 0, st>>>(x, ld, xbs, rows, cols,
                                                                                         neg, Kp, out, ld_out, obs);
    } else {
        bf16x3_split_t_kernel<<<dim3((cols + 31) / 32, Kp / 32, batch), 256, 0, st>>>(x, ld, xbs, rows, cols, neg,
                                                                                       Kp, out, ld_out, obs);
    }
    return (int)cudaGetLastError();
}

extern "C" int ltq_bf16x6_split_batched(const float* x, long long ld, long long xbs, int rows, int cols, int batch,
                                        int order, int side, int neg, uint16_t* out, long long ld_out, long long obs,
                                        void* stream)
{
    if (rows < 0 || cols < 0 || batch < 0 || batch > 65535 || cols % 4 || ld % 4 || ld < cols || xbs % 4 ||
        ld_out % 4 || obs % 4 || ((uintptr_t)x & 15) || ((uintptr_t)out & 7) || (order != 0 && order != 1) ||
        (side != 0 && side != 1) || ld_out < (side ? cols : 6LL * cols))
        return -1;
    const long long n = (long long)rows * (cols / 4);
    if (n == 0 || batch == 0) return 0;
    const dim3 grid((unsigned)((n + 255) / 256), (unsigned)batch);
    bf16x6_split_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, ld, xbs, rows, cols, order, side, neg ? 1 : 0, out,
                                                                ld_out, obs);
    return (int)cudaGetLastError();
}

extern "C" int ltq_bf16x6_split(const float* x, long long ld, int rows, int cols, int order, int side, uint16_t* out,
                                long long ld_out, void* stream)
{
    return ltq_bf16x6_split_batched(x, ld, 0, rows, cols, 1, order, side, 0, out, ld_out, 0, stream);
}

extern "C" int ltq_trtri256_lower(const float* L, long long ldL, int nb, float* X, long long ldX, void* stream)
{
    if (nb < 0 || ldL < 256LL * nb || ldX < 256LL * nb || !L || !X) return -1;
    if (nb == 0) return 0;
    static std::atomic<int> attr_done[64];  // the shared-memory opt-in, once per device
    constexpr int smem = 256 * 128 * 4;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        const cudaError_t e = cudaFuncSetAttribute(trtri256_lower_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int)e;
        attr_done[dev].store(1, std::memory_order_release);
    }
    trtri256_lower_kernel<<<dim3((unsigned)nb, 2), 128, smem, (cudaStream_t)stream>>>(L, ldL, X, ldX);
    return (int)cudaGetLastError();
}

extern "C" int ltq_chol256_diag(float* A, long long ld, int c0, uint16_t* xt3, float* X, long long ldx, int* info,
                                void* stream)
{
    // X: the inverse at (c0, c0) of X (ldx >= c0 + 256), or the 256 x 256 inverse alone at X (ldx == 256)
    if (!A || !xt3 || !info || c0 < 0 || ld < c0 + 256LL || (X && ldx != 256 && ldx < c0 + 256LL)) return -1;
    if (c0 % 4 || ld % 4 || (X && ldx % 4) || ((uintptr_t)A & 15) || ((uintptr_t)xt3 & 15) || ((uintptr_t)X & 15)) return -1;
    static std::atomic<int> attr_done[64];
    constexpr int smem = (LT_FLOATS + 768) * 4;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!attr_done[dev].load(std::memory_order_acquire)) {
        const cudaError_t e = cudaFuncSetAttribute(chol256_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int)e;
        attr_done[dev].store(1, std::memory_order_release);
    }
    float* Xb = X ? (ldx == 256 ? X : X + (long long)c0 * (ldx + 1)) : nullptr;
    chol256_tiled_kernel<<<1, 544, smem, (cudaStream_t)stream>>>(A, ld, c0, xt3, Xb, ldx, info);
    return (int)cudaGetLastError();
}

extern "C" int ltq_chol_solve(const float* L, long long ld, int K, const float* Dinv, const float* b, float* x,
                              float* work, void* stream)
{
    if (!L || !Dinv || !b || !x || !work || K <= 0 || K % 256 || ld < K || (ld % 4) || ((uintptr_t)L & 15)) return -1;
    const cudaStream_t st = (cudaStream_t)stream;
    const int nb = K / 256;
    // work [2 K]: the residual r, then y
    float* r = work;
    float* y = work + K;
    cudaError_t e = cudaMemcpyAsync(r, b, sizeof(float) * K, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return (int)e;
    for (int p = 0; p < nb; p++) {
        const int grid = nb - p - 1 > 0 ? nb - p - 1 : 1;
        chol_solve_fwd_step<<<grid, 1024, 0, st>>>(L, ld, Dinv, r, y, p, K);
    }
    for (int p = nb - 1; p >= 0; p--)
        chol_solve_bwd_step<<<p > 0 ? p : 1, 1024, 0, st>>>(L, ld, Dinv, y, x, p);
    return (int)cudaGetLastError();
}
