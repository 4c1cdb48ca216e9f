// Fused LDLQ block: one 256-column block of the row-scale TCQ quantizer (lumen-inference/ltq-research
// src/liqk_v2.py:956-971, quant_sub :913-936) in one launch.
//
// Rows are independent inside a block (the error feedback only moves error to later columns of the same row), so one
// CTA owns one tile group — 16 consecutive rows — and runs the block's 16 sub-blocks back to back, with no other CTA
// involved.  Per sub-block (columns s0 .. s0 + 15 of the block):
//   1. gather   x[16 r + c] = w[r][s0 + c] * (1 / d_rb[r])      (the Viterbi tile, t = 16 r + c, :914, :963)
//   2. pass 1   forward over the window [128 - W, 128 + W) from a free start + traceback to the state before t = 128
//   3. pass 2   forward over the tile rotated by 128 with start = end = that state + traceback, reconstruction, codes
//               (the tail-biting schedule of src/tcq_proto.py:584-609)
//   4. feedback G[:, s0 + c] = rec, idx / gi from the codes;  e = w[:, s0:s1] - d_rb * rec;
//               err = e @ Uinv[s0:s1, s0:s1];  w[:, s1:256] -= err @ U[s0:s1, s1:256]   (:964-971)
// The forward passes are vit_fwd_tile (G warps, one per gain slot), the tracebacks vit_tb_tile (warp 0); the feedback
// uses the same sequential fma chains as the stand-alone ltq_ldlq_feedback kernel, so both paths give identical bits.
// The block's running copy of w (16 rows x 256 per CTA) lives in the workspace; W_work itself is only read, because
// the inter-block update after the block (:972-979) needs the block's starting values.
#pragma once
#include "tcq_viterbi_kernel.cuh"

namespace ltqb {

struct LdlqParams {
    VitParams p1, p2;         // Viterbi passes 1 and 2 (per-tile buffers indexed by the tile group n)
    const float* wblk;        // W_work[:, c0] (row stride ldw): the block at its start
    long long ldw;
    float* wsub;              // [N * 16][256] running copy of the block
    const float* d_rb;        // d_rb(row, block) at d_rb[row * ldd]
    long long ldd;
    const float* dwrows;      // [16][256]: weights of sub-block ib at t = diag_w[c0 + 16 ib + t % 16]
    const float* U;           // U[c0, c0] (row stride ldU)
    long long ldU;
    const float* Ui;          // U_blk_inv (row stride ldUi)
    long long ldUi;
    float* G;                 // G[:, c0] (row stride ldG)
    long long ldG;
    int16_t* idx;             // idx[:, c0], gi[:, c0] (row stride ldP)
    uint8_t* gi;
    long long ldP;
    float* xbuf;              // [N][256] Viterbi input tile
    float* recbuf;            // [N][256] reconstruction (gain * table value)
    int* codebuf;             // [N][256] codes (gain index << 16 | label * U + u)
    int fb_off;               // shared-memory offset of the feedback scratch and of the traceback warp region
};

// shared memory of the fused kernel: the larger forward layout; the traceback region and the feedback scratch reuse
// the forward pass's metric region (dead once a forward pass has ended)
__host__ __device__ inline int ldlq_smem(const VitParams& a, const VitParams& b, int NP, int* fb_off)
{
    const FwdSmem A = fwd_smem(a.T, a.G, a.Gfull, a.sub, a.nl, NP, a.U, a.U_hi);
    const FwdSmem B = fwd_smem(b.T, b.G, b.Gfull, b.sub, b.nl, NP, b.U, b.U_hi);
    const int off = A.dp > B.dp ? A.dp : B.dp;
    const TbSmem TA = tb_smem(a.T, a.sub, a.nl, a.U, a.U_hi, a.W4, a.NB, 1);
    const TbSmem TB = tb_smem(b.T, b.sub, b.nl, b.U, b.U_hi, b.W4, b.NB, 1);
    int need = off + (TA.per_warp > TB.per_warp ? TA.per_warp : TB.per_warp);
    if (need < off + 2 * 256 * 4) need = off + 2 * 256 * 4;
    int total = A.total > B.total ? A.total : B.total;
    if (need > total) total = need;
    if (fb_off) *fb_off = off;
    return total;
}

template <class MP, int MD>
__device__ __forceinline__ void ldlq_tb(const VitParams& p, int n, int lane, unsigned char* smem, int fb_off,
                                        const float* xr)
{
    constexpr int NP = MD ? 2 : 1;
    const FwdSmem L = fwd_smem(p.T, p.G, p.Gfull, p.sub, p.nl, NP, p.U, p.U_hi);
    vit_tb_tile<MD>(p, n, lane, reinterpret_cast<const float*>(smem + L.tab),
                    reinterpret_cast<const float*>(smem + L.tabhi), reinterpret_cast<const float*>(smem + L.gain),
                    reinterpret_cast<const float*>(smem + L.gainhi), smem + fb_off, xr);
}

template <class MP, int MD>
__global__ void __launch_bounds__(256, MD == 0 ? 3 : 2) ldlq_block_kernel(const LdlqParams q)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = blockIdx.x, tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const long long row0 = 16LL * n;
    float* wsub = q.wsub + row0 * 256;
    float* xr = q.xbuf + (size_t)n * 256;
    const float* rr = q.recbuf + (size_t)n * 256;
    const int* cr = q.codebuf + (size_t)n * 256;
    float* fe = reinterpret_cast<float*>(smem + q.fb_off);  // e [16][16]
    float* ferr = fe + 256;                                 // err [16][16]

    for (int i = tid; i < 16 * 64; i += nthr) {
        const int r = i >> 6, c = (i & 63) * 4;
        *reinterpret_cast<float4*>(wsub + r * 256 + c) =
            *reinterpret_cast<const float4*>(q.wblk + (row0 + r) * q.ldw + c);
    }
    for (int ib = 0; ib < 16; ib++) {
        const int s0 = 16 * ib;
        __syncthreads();
        for (int i = tid; i < 256; i += nthr) {
            const int r = i >> 4, c = i & 15;
            const float d = fmaxf(q.d_rb[(row0 + r) * q.ldd], 1e-8f);
            xr[i] = __fmul_rn(wsub[r * 256 + s0 + c], __fdiv_rn(1.f, d));
        }
        __syncthreads();
        const float* wr = q.dwrows + (size_t)ib * 256;
        vit_fwd_tile<MP, MD, false>(q.p1, n, smem, xr, wr);
        __syncthreads();
        if (warp == 0) ldlq_tb<MP, MD>(q.p1, n, lane, smem, q.fb_off, xr);
        __syncthreads();
        vit_fwd_tile<MP, MD, false>(q.p2, n, smem, xr, wr);
        __syncthreads();
        if (warp == 0) ldlq_tb<MP, MD>(q.p2, n, lane, smem, q.fb_off, xr);
        __syncthreads();
        for (int i = tid; i < 256; i += nthr) {
            const int r = i >> 4, c = i & 15;
            const long long row = row0 + r;
            const float g = rr[i];
            const int cd = cr[i];
            q.G[row * q.ldG + s0 + c] = g;
            q.idx[row * q.ldP + s0 + c] = (int16_t)(cd & 0xffff);
            q.gi[row * q.ldP + s0 + c] = (uint8_t)(cd >> 16);
            const float d = fmaxf(q.d_rb[row * q.ldd], 1e-8f);
            fe[i] = __fsub_rn(wsub[r * 256 + s0 + c], __fmul_rn(d, g));
        }
        if (ib == 15) break;
        __syncthreads();
        for (int i = tid; i < 256; i += nthr) {
            const int r = i >> 4, k = i & 15;
            float acc = 0.f;
#pragma unroll
            for (int ii = 0; ii < 16; ii++) acc = __fmaf_rn(fe[r * 16 + ii], q.Ui[(long long)(s0 + ii) * q.ldUi + s0 + k], acc);
            ferr[i] = acc;
        }
        __syncthreads();
        const int s1 = s0 + 16, ncol = 256 - s1;
        for (int i = tid; i < 16 * ncol; i += nthr) {
            const int r = i / ncol, j = i - r * ncol;
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 16; k++) acc = __fmaf_rn(ferr[r * 16 + k], q.U[(long long)(s0 + k) * q.ldU + s1 + j], acc);
            wsub[r * 256 + s1 + j] = __fsub_rn(wsub[r * 256 + s1 + j], acc);
        }
    }
}

// weights of the 16 sub-blocks as Viterbi rows: out[ib][t] = dw[16 ib + t % 16]
static __global__ void ldlq_dwrows_kernel(const float* __restrict__ dw, float* __restrict__ out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < 16 * 256) out[i] = dw[16 * (i >> 8) + (i & 15)];
}

}  // namespace ltqb
