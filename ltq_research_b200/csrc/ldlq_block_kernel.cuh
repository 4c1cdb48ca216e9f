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
// The forward passes are vit_fwd_tile (G warps, one per gain slot), the tracebacks tb_coop (whole CTA); the feedback
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
    int fb_off;               // shared-memory offset of the feedback scratch and of the traceback region
};

// ------------------------------------------------------------------------------------------------
// Cooperative traceback of tile n by the whole CTA (the forward pass has just ended; its metric region is free).
// One thread (thread 0) walks the survivor path back, one sub-block (`chunk`) at a time, from words staged in shared
// memory; while it walks chunk c, the CTA's other warps stage chunk c - 1 — the words of every gain slot, because the
// slot of chunk c - 1 is only known once the walk reaches the start of chunk c — and the gain-merge winners of that
// boundary, into the other half of a double buffer.  The walk records per step only the code bit (bit 0 of the
// state), the parity class (D2 / D4 / EQ) and, per chunk, the gain slot; afterwards every thread rebuilds the states
//     s_t = ((s_0 << t) | sum_{q < t} c_{t-q} << q) & 1023
// and reconstructs its samples.  Same decisions, tie-breaks, states, values and codes as vit_tb_tile (the stand-alone
// traceback kernel), which the tests check bit for bit.
// Every thread waits for all of its copies (cp.async.wait_all) before every barrier, so no copy is in flight across a
// barrier.  Shared layout (from `base`): 2 x [G x (sub / 4) x W4 x 32 + 128] words, code bits (T / 32 words), slot per
// chunk (32 bytes), parity class per step (T bytes), 4 ints.
// ------------------------------------------------------------------------------------------------
// 16-byte asynchronous global -> shared copy (completion: cp_async_wait_all by the issuing thread, then a barrier)
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Drops the L2 lines [p, p + bytes) without writing them back (discard.global.L2): for data that is dead, here survivor
// words and merge winners after the traceback that consumed them.  Threads t0, t0 + ts, ... take one 128-byte line
// each in turn; p and bytes are multiples of 128.  Without it, the dirty survivor lines of every pass would be
// written to DRAM when evicted, although no one reads them again.
__device__ __forceinline__ void discard_l2(const void* p, long long bytes, int t0, int ts)
{
    const char* c = static_cast<const char*>(p);
    for (long long o = 128LL * t0; o < bytes; o += 128LL * ts)
        asm volatile("discard.global.L2 [%0], 128;\n" ::"l"(c + o) : "memory");
}

__host__ __device__ inline int tb_coop_words(const VitParams& p)
{
    return p.G * (p.sub / 4) * p.W4 * 32 + 128;
}

__host__ __device__ inline int tb_coop_bytes(const VitParams& p)
{
    return 4 * (2 * tb_coop_words(p) + MAXT / 32) + 32 + MAXT + 16;
}

template <int MD>
__device__ __forceinline__ void tb_coop(const VitParams& p, const int n, unsigned char* base, const float* s_tab,
                                        const float* s_gain, const float* xrow)
{
    constexpr bool PP = MD == 1, EQ = MD == 3;
    const int T = p.T, G = p.G, sub = p.sub, W4 = p.W4, NGRP = sub / 4, nch = T / sub, U = p.U;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int bufw = tb_coop_words(p), per_slot = NGRP * W4 * 32;
    uint32_t* buf = reinterpret_cast<uint32_t*>(base);
    uint32_t* cbits = buf + 2 * bufw;
    uint8_t* sg = reinterpret_cast<uint8_t*>(cbits + MAXT / 32);
    uint8_t* spar = sg + 32;
    int* flag = reinterpret_cast<int*>(spar + MAXT);  // [3] state at t = 0

    // stage chunk c (all slots' words — per_slot consecutive words per slot in the survivor stream — and the merge
    // winners of boundary c) into buffer b with 16-byte asynchronous copies by threads t0, t0 + ts, ...
    const int v4 = per_slot / 4;
    auto stage = [&](int c, int b, int t0, int ts) {
        uint32_t* d = buf + b * bufw;
        const uint32_t* src = p.svA + (size_t)n * G * (size_t)p.capA + (size_t)c * per_slot;
        for (int g = 0; g < G; g++, d += per_slot, src += p.capA)
            for (int r = t0; r < v4; r += ts) cp_async16(d + 4 * r, src + 4 * r);
        if (G > 1 && c > 0) {  // d now points at the merge-winner words of the buffer
            const uint32_t* gsrc = p.gsw + ((size_t)n * p.nsl + c) * (NS / 8);
            for (int k = t0; k < NS / 32; k += ts) cp_async16(d + 4 * k, gsrc + 4 * k);
        }
    };
    int wst = 0, wgs = 0;  // thread 0: the walk's state and gain slot, carried from chunk to chunk in registers
    if (tid == 0) {
        const int bi = p.best[n];
        wst = bi % NS;
        wgs = bi / NS;
    }
    // the last chunk by every thread; then, while thread 0 walks chunk c, the staging threads (the warps that do not
    // walk, or lanes 1..31 when there is one warp) copy chunk c - 1 into the other buffer
    const bool stager = G > 1 ? tid >= 32 : tid > 0;
    stage(nch - 1, (nch - 1) & 1, tid, nthr);
    cp_async_wait_all();
    __syncthreads();
    int pcur = 0, cstar = 0;  // thread 0: parity class of the current pair / quad (carried across steps)
    bool stopped = false;     // thread 0: the walk reached the first-pass middle
    for (int c = nch - 1; c >= 0; c--) {
        const int b = c & 1, lo = c * sub;
        if (stager && c > 0) stage(c - 1, b ^ 1, G > 1 ? tid - 32 : tid - 1, G > 1 ? nthr - 32 : nthr - 1);
        if (tid == 0) {
            int st = wst;
            sg[c] = (uint8_t)wgs;
            const uint32_t* B = buf + b * bufw + wgs * per_slot;
            uint32_t acc = 0;
            bool stop = false, done = false;
            for (int gl = NGRP - 1; gl >= 0 && !done; gl--) {
                // The four steps of a group read the same lane column L (bits 4..8 of the state at its last step): its
                // W4 words are loaded once and the walk runs in the register frame of the forward pass.  At step j the
                // state is register r of lane L in layout j + 1; its butterfly is r >> 1 and the decision bit h picks
                // the predecessor register (r >> 1) | h << 4 in layout j (the forward step maps (ra, ra + 16) to
                // (2 ra, 2 ra + 1)), so a step is a shift, a bit extract and an insert; the code bit is r & 1.
                constexpr int W4C = MD == 0 ? 2 : (MD == 1 ? 5 : 9);
                const int L = (st >> 4) & 31;
                int r = ((st >> 9) << 4) | (st & 15);  // the state in layout 4
                const uint32_t* Wg = B + gl * W4C * 32 + L;
                uint32_t w[W4C];
#pragma unroll
                for (int k = 0; k < W4C; k++) w[k] = Wg[32 * k];
                {
                    // a group with neither the first-pass middle nor t = 0: tb_walk_group, its code bits from the
                    // entry register
                    const int tg = lo + 4 * gl;
                    if (tg != 0 && !(p.mid_st && (unsigned)(p.mid_t - 1 - tg) < 4u)) {
                        acc |= (__brev((uint32_t)r & 15u) >> 28) << (tg - lo);
                        r = tb_walk_group<MD>(w, r, spar, tg, pcur, cstar);
                        st = L | (r << 5);
                        continue;
                    }
                }
                cfor<3, -1, -1>([&](auto JJ) {
                    constexpr int j = decltype(JJ)::value;
                    if (done) return;
                    const int t = lo + 4 * gl + j;
                    const int bi4 = r >> 1;
                    // the full state in layout j + 1 (only where the walk stops)
                    auto state = [&]() { return (r & ((2 << j) - 1)) | (L << (j + 1)) | ((r >> (j + 1)) << (j + 6)); };
                    if (PP && (j & 1)) {
                        pcur = (w[j == 1 ? 2 : 4] >> r) & 1;
                        spar[t] = spar[t - 1] = (uint8_t)pcur;
                    }
                    if (p.mid_st && t == p.mid_t - 1) {
                        st = state();
                        p.mid_st[n] = st;
                        stop = done = true;
                        return;
                    }
                    acc |= (uint32_t)(r & 1) << (t - lo);
                    if (t == 0) {
                        st = state();
                        flag[3] = st;
                        done = true;
                        return;
                    }
                    int h;
                    if constexpr (MD == 0) {
                        h = (w[j >> 1] >> ((j & 1) ? bi4 : 16 + bi4)) & 1;
                    } else if constexpr (PP) {
                        if constexpr (j & 1) h = (w[j == 1 ? 1 : 3] >> (pcur ? bi4 : 16 + bi4)) & 1;
                        else h = (w[0] >> ((j == 0) ? 16 + bi4 : bi4)) & 1;
                    } else {
                        const int ro = r;  // the output register of the state's butterfly
                        if constexpr (j == 3) {
                            cstar = (w[7] >> ro) & 1;
                            const int bb = (w[8] >> ro) & 1;
                            h = ((cstar ? w[6] : w[5]) >> (bb ? bi4 : 16 + bi4)) & 1;
                            if (EQ) {
                                spar[t] = spar[t - 1] = spar[t - 2] = spar[t - 3] = (uint8_t)cstar;
                            } else {
                                spar[t] = (uint8_t)(bb ^ cstar);
                                spar[t - 1] = (uint8_t)bb;
                            }
                        } else if constexpr (j == 2) {
                            h = (w[4] >> (cstar ? bi4 : 16 + bi4)) & 1;
                        } else if constexpr (j == 1) {
                            const int bb = ((cstar ? w[3] : w[2]) >> ro) & 1;
                            h = (w[1] >> (bb ? bi4 : 16 + bi4)) & 1;
                            if (!EQ) {
                                spar[t] = (uint8_t)(bb ^ cstar);
                                spar[t - 1] = (uint8_t)bb;
                            }
                        } else {
                            h = (w[0] >> bi4) & 1;
                        }
                    }
                    r = bi4 | (h << 4);
                });
                if (!done) st = L | (r << 5);  // the state before the group's first step, in layout 0
            }
            if (sub == 32) cbits[c] = acc;
            else reinterpret_cast<uint16_t*>(cbits)[c] = (uint16_t)acc;
            wst = st;
            stopped = stop;
            if (!stop && G > 1 && c > 0)  // the walk ended at the chunk's first step: the slot of the previous chunk
                wgs = (int)((buf[b * bufw + G * per_slot + (st >> 3)] >> (4 * (st & 7))) & 15u);
        }
        cp_async_wait_all();
        // the stop travels with the barrier (bar.red.or): a flag in shared memory read after the barrier could already
        // be overwritten by thread 0's walk of the next chunk, which no barrier separates from the read
        if (__syncthreads_or(stopped)) return;  // first tail-biting pass: only the middle state was needed
    }

    // reconstruction: every thread, from the code bits and the state at t = 0
    const unsigned st0 = (unsigned)flag[3];
    float* rn = p.rec + (size_t)n * p.ld;
    for (int t = tid; t < T; t += nthr) {
        unsigned s = t < 10 ? (st0 << t) & 1023u : 0u;
#pragma unroll
        for (int q = 0; q < 10; q++) {
            const int tq = t - q;
            if (tq >= 1) s |= ((cbits[tq >> 5] >> (tq & 31)) & 1u) << q;
        }
        const int gg = sg[t / sub];
        const int lb = label_rt((int)s, p);
        const int gi = p.cand ? (int)p.gcand[((size_t)n * p.nsl + t / sub) * G + gg] : gg;
        const float gt = s_gain[gi];
        const float* tt = s_tab + lb * U;
        const int tp = (t + p.rot) % p.ld;
        const float xt = xrow[tp];
        float bestd = BIG, val = 0.f;
        int bu = 0;
        for (int u = MD ? spar[t] : 0; u < U; u += MD ? 2 : 1) {
            const float v = __fmul_rn(gt, tt[u]);
            const float d = __fmaf_rn(-gt, tt[u], xt);
            const float dd = __fmul_rn(d, d);
            if (dd < bestd) { bestd = dd; val = v; bu = u; }
        }
        rn[tp] = val;
        if (p.code) p.code[(size_t)n * p.ld + tp] = (gi << 16) | (lb * U + bu);
    }
}

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
    const int cb = tb_coop_bytes(a) > tb_coop_bytes(b) ? tb_coop_bytes(a) : tb_coop_bytes(b);
    if (need < off + cb) need = off + cb;
    int total = A.total > B.total ? A.total : B.total;
    if (need > total) total = need;
    if (fb_off) *fb_off = off;
    return total;
}

template <class MP, int MD>
__device__ __forceinline__ void ldlq_tb(const VitParams& p, int n, unsigned char* smem, int fb_off, const float* xr)
{
    constexpr int NP = MD ? 2 : 1;
    const FwdSmem L = fwd_smem(p.T, p.G, p.Gfull, p.sub, p.nl, NP, p.U, p.U_hi);
    tb_coop<MD>(p, n, smem + fb_off, reinterpret_cast<const float*>(smem + L.tab),
                reinterpret_cast<const float*>(smem + L.gain), xr);
}

template <class MP, int MD>
// Register caps (a CTA has 32 G <= 128 threads): 128 a thread for the plain mode — at the tighter cap of 85 (3 x 256
// threads per SM) the compiler moved register data around the branch-error row loads (12 % more instructions in the
// forward pass; isolated TCQ3X block 7.20 -> 6.93 ms with 128, although fewer CTAs fit per SM; 7.33 ms at 96);
// 168 for the parity modes, whose class planes spilled at 128 (TCQ25X block 6.45 -> 6.18 ms; 6.94 ms uncapped)
__global__ void __launch_bounds__(MD == 0 ? 256 : 192, 2) ldlq_block_kernel(const __grid_constant__ LdlqParams q)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = blockIdx.x, tid = threadIdx.x, nthr = blockDim.x;
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
        // the traceback stages the survivor words and merge winners with L2 copies (cp.async.cg): each thread's
        // stores of the forward pass must reach L2 before the barrier that starts the traceback
        // both passes run the same code (one copy of the forward and traceback bodies in the instruction cache)
#pragma unroll 1
        for (int ps = 0; ps < 2; ps++) {
            const VitParams& pp = ps ? q.p2 : q.p1;
            vit_fwd_tile<MP, MD, false, true>(pp, n, smem, xr, wr);
            __threadfence();
            __syncthreads();
            ldlq_tb<MP, MD>(pp, n, smem, q.fb_off, xr);
            __syncthreads();
            // this pass's survivor words (its T / 4 groups in every slot's stream) and merge winners are dead: every
            // copy the traceback made of them completed before the barrier above.  Each slot's stream starts on a
            // 128-byte line (capA words = 64 W4 x 32), each merge-winner row is 512 bytes.
            for (int g = 0; g < pp.G; g++)
                discard_l2(pp.svA + ((size_t)n * pp.G + g) * (size_t)pp.capA, (long long)(pp.T / 4) * pp.W4 * 128, tid,
                           nthr);
            if (pp.G > 1)
                discard_l2(pp.gsw + (size_t)n * pp.nsl * (NS / 8), (long long)(pp.T / pp.sub) * 512, tid, nthr);
        }
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
        // w[:, s1:] -= err @ U[s0:s1, s1:]: a thread per column, the column's 16 values of U loaded once for all 16 rows;
        // each output is the same sequential fma chain over k = 0..15 as in the stand-alone feedback kernel
        const int s1 = s0 + 16, ncol = 256 - s1;
        for (int j = tid; j < ncol; j += nthr) {
            float u[16];
#pragma unroll
            for (int k = 0; k < 16; k++) u[k] = q.U[(long long)(s0 + k) * q.ldU + s1 + j];
#pragma unroll 2
            for (int r = 0; r < 16; r++) {
                const float4* e4 = reinterpret_cast<const float4*>(ferr + r * 16);
                float acc = 0.f;
#pragma unroll
                for (int k4 = 0; k4 < 4; k4++) {
                    const float4 e = e4[k4];
                    acc = __fmaf_rn(e.x, u[4 * k4], acc);
                    acc = __fmaf_rn(e.y, u[4 * k4 + 1], acc);
                    acc = __fmaf_rn(e.z, u[4 * k4 + 2], acc);
                    acc = __fmaf_rn(e.w, u[4 * k4 + 3], acc);
                }
                wsub[r * 256 + s1 + j] = __fsub_rn(wsub[r * 256 + s1 + j], acc);
            }
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
