// The S = 256 trellis (nu = 8) of the reference's tcq_viterbi (src/cuda/tcq_viterbi.cu:755-762: 256 states, 4 label
// subsets, no parity classes; its tcq_forward_kernel semantics :97-683 as for S = 1024).  No format table uses it;
// the reference kernel accepts it, so this entry does too.
//
// One CTA of 256 threads per tile; thread s owns state s of every gain slot (G <= 8 metrics in registers).  A step:
// every thread publishes its metrics to one half of a double-buffered shared array, one barrier, then reads the two
// predecessors s >> 1 and 128 + (s >> 1) of its state, keeps the smaller (strict <: ties keep s >> 1) and adds its
// branch error; the decision bits of a warp's 32 states become one word by ballot.  Decision words (T x G x 8) and
// gain-merge winners stay in shared memory; at a sub-block boundary each thread merges its own state's slots in
// registers (strict <, lowest slot wins).  Thread 0 walks the path back; all threads then rebuild the samples.
// Arithmetic as the reference kernel's nvcc build contracts it: branch errors w * min_u fma(-g, tab[u], x)^2, the
// candidate sums fma(err, w, e), the reconstruction distance fma(-g, tab[u], x).
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>
#include "vit_launch.cuh"

namespace ltqb {
namespace {

constexpr int S2 = 256, H2 = 128, NL2 = 4, FULLM = -1;

struct S256Smem {
    int x, w, tab, tabhi, gain, gainhi, ce, gc, err, dp, bp, gsel, st, sg, red, total;
};

__host__ __device__ inline S256Smem s256_smem(int T, int G, int Gfull, int sub, int U, int U_hi)
{
    S256Smem L;
    int o = 0;
    L.x = o; o = al16(o + 4 * T);
    L.w = o; o = al16(o + 4 * T);
    L.tab = o; o = al16(o + 4 * NL2 * U);
    L.tabhi = o; o = al16(o + 4 * NL2 * U_hi);
    L.gain = o; o = al16(o + 4 * MAXG);
    L.gainhi = o; o = al16(o + 4 * MAXG);
    L.ce = o; o = al16(o + 4 * (T / sub) * Gfull);
    L.gc = o; o = al16(o + (T / sub) * G);
    L.err = o; o = al16(o + 4 * sub * G * NL2);   // [step of the sub-block][slot][label]
    L.dp = o; o = al16(o + 4 * 2 * G * S2);       // [buffer][slot][state]
    L.bp = o; o = al16(o + 4 * T * G * (S2 / 32));  // [step][slot][warp]: decision words
    L.gsel = o; o = al16(o + (T / sub) * S2);     // [sub-block][state]: winning slot
    L.st = o; o = al16(o + 2 * T);
    L.sg = o; o = al16(o + T);
    L.red = o; o = al16(o + 8 * 8 + 16);
    L.total = o;
    return L;
}

__device__ __forceinline__ int label256(int s, int m)
{
    return (s & 1) | ((__popc((unsigned)(s >> 1) & (unsigned)m) & 1) << 1);
}

template <int G>
__global__ void __launch_bounds__(256, 1) vit256_kernel(const VitParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = blockIdx.x, s = threadIdx.x, lane = s & 31, warp = s >> 5;
    const int T = p.T, sub = p.sub, nsub = T / sub, U = p.U, U_hi = p.U_hi, mix = p.mix, Gf = p.Gfull;
    const S256Smem SL = s256_smem(T, G, Gf, sub, U, U_hi);
    float* s_x = reinterpret_cast<float*>(smem + SL.x);
    float* s_w = reinterpret_cast<float*>(smem + SL.w);
    float* s_tab = reinterpret_cast<float*>(smem + SL.tab);
    float* s_tabhi = reinterpret_cast<float*>(smem + SL.tabhi);
    float* s_gain = reinterpret_cast<float*>(smem + SL.gain);
    float* s_gainhi = reinterpret_cast<float*>(smem + SL.gainhi);
    float* s_ce = reinterpret_cast<float*>(smem + SL.ce);
    uint8_t* s_gc = smem + SL.gc;
    float* s_err = reinterpret_cast<float*>(smem + SL.err);
    float* s_dp = reinterpret_cast<float*>(smem + SL.dp);
    uint32_t* s_bp = reinterpret_cast<uint32_t*>(smem + SL.bp);
    uint8_t* s_gsel = smem + SL.gsel;
    uint16_t* s_st = reinterpret_cast<uint16_t*>(smem + SL.st);
    uint8_t* s_sg = smem + SL.sg;
    float* red_v = reinterpret_cast<float*>(smem + SL.red);
    int* red_i = reinterpret_cast<int*>(smem + SL.red + 32);
    int* flag = reinterpret_cast<int*>(smem + SL.red + 64);

    // ---- tile inputs (sample t is element (t + rot) % ld), tables, gains ----
    const float* xrow = p.x + (size_t)n * p.ld;
    const float* wrow = p.w + (size_t)n * p.ldw;
    for (int i = s; i < T; i += S2) {
        const int j = (i + p.rot) % p.ld;
        s_x[i] = xrow[j];
        s_w[i] = wrow[j];
    }
    for (int i = s; i < NL2 * U; i += S2) s_tab[i] = p.tab[i];
    for (int i = s; i < NL2 * U_hi; i += S2) s_tabhi[i] = p.tab_hi[i];
    if (s < Gf) { s_gain[s] = p.gains[s]; s_gainhi[s] = p.gains_hi[s]; }
    __syncthreads();

    // ---- gain candidates: weighted scalar error of each sub-block over the merged table, the G smallest ----
    if (p.cand) {
        for (int i = s; i < nsub * Gf; i += S2) {
            const int j = i / Gf, gi = i % Gf;
            float e = 0.f;
            for (int t = j * sub; t < (j + 1) * sub; t++) {
                const bool hi = mix > 0 && ((t / mix) & 1);
                const float be = hi ? branch_err(s_x[t], s_gainhi[gi], s_tabhi, 0, 1, NL2 * U_hi)
                                    : branch_err(s_x[t], s_gain[gi], s_tab, 0, 1, NL2 * U);
                e = __fmaf_rn(be, s_w[t], e);
            }
            s_ce[i] = e;
        }
        __syncthreads();
        if (s < nsub) {
            uint32_t used = 0;
            for (int c = 0; c < G; c++) {
                int bg = 0;
                float be = BIG;
                for (int gi = 0; gi < Gf; gi++)
                    if (!((used >> gi) & 1u) && s_ce[s * Gf + gi] < be) { be = s_ce[s * Gf + gi]; bg = gi; }
                used |= 1u << bg;
                s_gc[s * G + c] = (uint8_t)bg;
                p.gcand[((size_t)n * p.nsl + s) * G + c] = (uint8_t)bg;
            }
        }
        __syncthreads();
    }

    // ---- forward ----
    const int lab = label256(s, p.m);
    const int s0 = p.init_st ? p.init_st[n] : -1;
    float dp[G];
    for (int t0 = 0; t0 < T; t0 += sub) {
        const int sb = t0 / sub;
        if (t0 > 0 && G > 1) {  // every slot continues from this state's best slot
            float b = dp[0];
            int bg = 0;
#pragma unroll
            for (int g = 1; g < G; g++)
                if (dp[g] < b) { b = dp[g]; bg = g; }
            s_gsel[sb * S2 + s] = (uint8_t)bg;
#pragma unroll
            for (int g = 0; g < G; g++) dp[g] = b;
        }
        // branch errors of the sub-block, [step][slot][label]; the barrier before keeps the previous table until
        // every thread has read it
        __syncthreads();
        for (int i = s; i < sub * G * NL2; i += S2) {
            const int tt = i / (G * NL2), g = (i / NL2) % G, lb = i % NL2;
            const int t = t0 + tt;
            const int gi = p.cand ? (int)s_gc[sb * G + g] : g;
            const bool hi = mix > 0 && ((t / mix) & 1);
            const float e = hi ? branch_err(s_x[t], s_gainhi[gi], s_tabhi + lb * U_hi, 0, 1, U_hi)
                               : branch_err(s_x[t], s_gain[gi], s_tab + lb * U, 0, 1, U);
            s_err[i] = __fmul_rn(e, s_w[t]);
        }
        __syncthreads();
        for (int tt = 0; tt < sub; tt++) {
            const int t = t0 + tt;
            const float* er = s_err + tt * G * NL2 + lab;
            if (t == 0) {  // the tile start: states whose predecessor is the start state's successor set
                const bool ok = s0 < 0 || (s >> 1) == (s0 & (H2 - 1));
#pragma unroll
                for (int g = 0; g < G; g++) dp[g] = ok ? er[g * NL2] : BIG;
                continue;
            }
            float* buf = s_dp + (t & 1) * G * S2;
#pragma unroll
            for (int g = 0; g < G; g++) buf[g * S2 + s] = dp[g];
            __syncthreads();
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float va = buf[g * S2 + (s >> 1)], vb = buf[g * S2 + H2 + (s >> 1)];
                const bool h = vb < va;
                dp[g] = __fadd_rn(h ? vb : va, er[g * NL2]);
                const uint32_t word = __ballot_sync(FULLM, h);
                if (lane == 0) s_bp[(t * G + g) * (S2 / 32) + warp] = word;
            }
        }
    }

    // ---- argmin over (slot, state): smallest value, then smallest index g * 256 + s; tail-biting keeps s == s0 ----
    const int s_end = (p.tail && p.init_st) ? s0 : -1;
    float bv = BIG;
    int bi = 0x7fffffff;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float v = (s_end < 0 || s == s_end) ? dp[g] : BIG;
        if (v < bv) { bv = v; bi = g * S2 + s; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_down_sync(FULLM, bv, off);
        const int oi = __shfl_down_sync(FULLM, bi, off);
        if (ov < bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
    __syncthreads();
    if (s == 0) {
        for (int k = 1; k < S2 / 32; k++)
            if (red_v[k] < bv || (red_v[k] == bv && red_i[k] < bi)) { bv = red_v[k]; bi = red_i[k]; }
        // no metric below 3.4e38 (non-finite inputs): slot 0 and the required end state (or state 0), so that the
        // walk stays inside the tile's decision words
        if (bi == 0x7fffffff) bi = s_end >= 0 ? s_end : 0;
        p.best[n] = bi;
        if (p.end_st) p.end_st[n] = bi % S2;
        // ---- traceback ----
        int st = bi % S2, g = bi / S2, stop = 0;
        for (int t = T - 1; t >= 0; t--) {
            s_st[t] = (uint16_t)st;
            s_sg[t] = (uint8_t)g;
            if (p.mid_st && t == p.mid_t - 1) {
                p.mid_st[n] = st;
                stop = 1;
                break;
            }
            if (t > 0) {
                const int h = (s_bp[(t * G + g) * (S2 / 32) + (st >> 5)] >> (st & 31)) & 1;
                st = h * H2 + (st >> 1);
                if (G > 1 && (t % sub) == 0) g = s_gsel[(t / sub) * S2 + st];
            }
        }
        flag[0] = stop;
    }
    __syncthreads();
    if (flag[0]) return;  // a first tail-biting pass: only the middle state was needed

    // ---- reconstruction and codes ----
    float* rn = p.rec + (size_t)n * p.ld;
    for (int t = s; t < T; t += S2) {
        const int stt = s_st[t], gg = s_sg[t];
        const int lb = label256(stt, p.m);
        const bool hi = mix > 0 && ((t / mix) & 1);
        const int Ut = hi ? U_hi : U;
        const int gi = p.cand ? (int)s_gc[(t / sub) * G + gg] : gg;
        const float gt = hi ? s_gainhi[gi] : s_gain[gi];
        const float* tt = (hi ? s_tabhi : s_tab) + lb * Ut;
        const float xt = s_x[t];
        float bestd = BIG, val = 0.f;
        int bu = 0;
        for (int u = 0; u < Ut; u++) {
            const float v = __fmul_rn(gt, tt[u]);
            const float d = __fmaf_rn(-gt, tt[u], xt);
            const float dd = __fmul_rn(d, d);
            if (dd < bestd) { bestd = dd; val = v; bu = u; }
        }
        const int tp = (t + p.rot) % p.ld;
        rn[tp] = val;
        if (p.code) p.code[(size_t)n * p.ld + tp] = (gi << 16) | (lb * Ut + bu);
    }
}

template <int G>
int launch256(const VitParams& p, cudaStream_t st)
{
    const int smem = s256_smem(p.T, G, p.Gfull, p.sub, p.U, p.U_hi).total;
    auto k = vit256_kernel<G>;
    static std::atomic<int> done[64];
    if (ensure_smem(k, smem, done) != 0) return -1;
    k<<<p.N, S2, smem, st>>>(p);
    return 0;
}

}  // namespace

// one Viterbi pass over p.N tiles of the 256-state trellis (4 label subsets, plain mode)
int run_pass_s256(VitParams p, cudaStream_t st)
{
    if (p.nl != 4) return -1;
    p.nsl = p.T / p.sub;
    switch (p.G) {
        case 1: return launch256<1>(p, st);
        case 2: return launch256<2>(p, st);
        case 3: return launch256<3>(p, st);
        case 4: return launch256<4>(p, st);
        case 8: return launch256<8>(p, st);
        default: return -1;
    }
}

}  // namespace ltqb
