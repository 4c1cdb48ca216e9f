// B200 (sm_100a) TCQ Viterbi for the LTQ tile format.
//
// Semantics follow the reference kernel tcq_forward_kernel (lumen-inference/ltq-research,
// src/cuda/tcq_viterbi.cu:97-683) bit for bit: the same fp32 operations on the same operands (branch error
// w * min_u fma(-g, tab[u], x)^2, path metric = selected predecessor + branch error), the same strict-`<` tie-breaks,
// the same sub-block gain merge, gain candidates, D2 / D4 / EQ parity classes, tail-biting start / end constraints.
// The organisation is new; two kernels per Viterbi pass:
//
// vit_fwd_kernel — forward add-compare-select, one CTA per tile, one warp per gain slot g:
//   * each lane keeps 32 of the 1024 path metrics in registers.  In "layout j" lane L holds the states
//       s = r_lo | L << j | r_hi << (j + 5),  register r = r_hi << j | r_lo   (r_lo: j bits, r_hi: 5 - j bits)
//     so the two predecessors of a butterfly (bit 9 of the state = bit 4 of the register) sit in registers ra and
//     ra + 16 of the same lane, and one trellis step maps registers (ra, ra + 16) -> (2 ra, 2 ra + 1) for every j
//     (a perfect shuffle).  Four steps (j = 0..3) run in registers as two radix-4 passes; then the metrics go through
//     shared memory once (layout 4 -> layout 0, padded, conflict-free), i.e. one exchange per 4 trellis steps;
//   * a compare is the sign of (b - a) on the FMA pipe, the select is FMNMX, and the decision bit is packed with a
//     funnel shift: 16 decisions per lane per step become one half word, stored coalesced as survivor words;
//   * subset labels are split into a per-lane part (a branch-error table variant chosen once per step) and a
//     per-register part that is a compile-time constant when the label masks are template parameters (MaskCT), so a
//     branch error is a register operand.  MaskRT is the same kernel for arbitrary masks (errors read from shared
//     memory per butterfly);
//   * the tile start is a virtual step from metrics 0 (allowed predecessors of the start state) / 3.4e38 (others), which
//     yields exactly the reference's initial metrics (err, or 3.4e38 for states the start state cannot reach);
//   * decision bits go to global memory as a per-(tile, slot) linear word stream (SvStream), the gain-merge winners as
//     bit planes; the final argmin over (slot, state) goes to best[n].
// vit_tb_kernel — traceback, reconstruction and codes, one warp per tile: one sub-block chunk of survivor words at a
//   time is staged in shared memory and walked by lane 0; all lanes then rebuild the samples.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ltqb {

constexpr float BIG = 3.4e38f;  // the reference's "infinite" path metric (src/cuda/tcq_viterbi.cu:48, :227)
constexpr int NS = 1024;        // trellis states (10-bit memory)
constexpr int NSP = NS;         // exchange slots per gain slot
constexpr int MAXG = 16, MAXU = 128, MAXSUBS = 32, MAXT = 512;
constexpr int TB_WARPS = 8;     // tiles (warps) per traceback CTA

struct VitParams {
    const float *x, *w, *tab, *gains, *tab_hi, *gains_hi;
    float* rec;
    int* code;
    const int* init_st;
    int *end_st, *mid_st, *best;
    uint8_t* gcand;
    uint32_t *svA, *svB;   // survivor word stream: first capA words of each (tile, slot) in A, the rest in B
    uint32_t* gsw;         // gain-merge winners: [N][T/sub][128 words], 4 bits per state: word s >> 3, nibble s & 7
    long long capA, capB;  // words per (tile, slot) in A / B
    int mid_t, tail;
    int N, T, U, G, Gfull, sub, U_hi, mix, ld, ldw, rot;
    int m, m2, m3, m4, nl;
    int W4;                // survivor words per 4-step group
    int NB;                // gsel bit planes
    int cand;
    int nsl;               // row stride of gsw and gcand in sub-blocks per tile (>= T / sub)
};

// ------------------------------------------------------------------------------------------------
// compile-time loops: every register index and every label bit below is a constant expression
// ------------------------------------------------------------------------------------------------
template <int I>
struct IC {
    static constexpr int value = I;
};
// f(IC<B>), f(IC<B + S>), ... while the index has not reached E (S = +1 or -1)
template <int B, int E, int S, class F>
__device__ __forceinline__ void cfor(F&& f)
{
    if constexpr ((S > 0 && B < E) || (S < 0 && B > E)) {
        f(IC<B>{});
        cfor<B + S, E, S>(f);
    }
}

// ------------------------------------------------------------------------------------------------
// label masks
// ------------------------------------------------------------------------------------------------
__host__ __device__ constexpr int cpar(unsigned v)
{
    v ^= v >> 16; v ^= v >> 8; v ^= v >> 4; v ^= v >> 2; v ^= v >> 1;
    return (int)(v & 1u);
}

// A branch-error row of one trellis step: NL labels x NP parity classes.  Compile-time masks: permuted for this lane's
// label variant and held in registers (r).  Run-time masks: one unpermuted row per step in shared memory (ptr), the
// lane part pl of the label applied per butterfly.
template <int EW>
struct ERow {
    float r[EW];
    const float* ptr;
    int pl;
};

// Compile-time masks: label bits of every register are constants after unrolling.
template <int M0, int M1, int M2, int M3, int NL_>
struct MaskCT {
    static constexpr int NL = NL_;
    static constexpr bool RT = false;
    __device__ __forceinline__ explicit MaskCT(const VitParams&) {}
    // label bits 1.. of a state s whose (s >> 1) == v
    __host__ __device__ static constexpr int hic(unsigned v)
    {
        return cpar(v & (unsigned)M0) | (NL >= 8 ? cpar(v & (unsigned)M1) << 1 : 0) |
               (NL >= 16 ? cpar(v & (unsigned)M2) << 2 : 0) | (NL >= 32 ? cpar(v & (unsigned)M3) << 3 : 0);
    }
    __device__ __forceinline__ int hi(unsigned v) const { return hic(v); }
    // register part of the label bits of the outputs of butterfly RA at step J (a constant)
    template <int J, int RA>
    __host__ __device__ static constexpr int qc()
    {
        return hic((unsigned)((RA & ((1 << J) - 1)) | ((RA >> J) << (J + 5))));
    }
    template <int EW>
    __device__ __forceinline__ float get(const ERow<EW>& e, int i) const { return e.r[i]; }
};

// Run-time masks: same recursion, branch errors read from the shared-memory row.
template <int NL_>
struct MaskRT {
    static constexpr int NL = NL_;
    static constexpr bool RT = true;
    unsigned m0, m1, m2, m3;
    __device__ __forceinline__ explicit MaskRT(const VitParams& p)
        : m0((unsigned)p.m), m1((unsigned)p.m2), m2((unsigned)p.m3), m3((unsigned)p.m4) {}
    __device__ __forceinline__ int hi(unsigned v) const
    {
        int r = __popc(v & m0) & 1;
        if (NL >= 8) r |= (__popc(v & m1) & 1) << 1;
        if (NL >= 16) r |= (__popc(v & m2) & 1) << 2;
        if (NL >= 32) r |= (__popc(v & m3) & 1) << 3;
        return r;
    }
    template <int J, int RA>
    __device__ __forceinline__ int q() const
    {
        return hi((unsigned)((RA & ((1 << J) - 1)) | ((RA >> J) << (J + 5))));
    }
    template <int EW>
    __device__ __forceinline__ float get(const ERow<EW>& e, int i) const { return e.ptr[i]; }
};

// full label of state s for nl subsets (src/cuda/tcq_viterbi.cu:85-95), run-time masks
__device__ __forceinline__ int label_rt(int s, const VitParams& p)
{
    int lb = ((__popc((s >> 1) & p.m) & 1) << 1) | (s & 1);
    if (p.nl >= 8) lb |= (__popc((s >> 1) & p.m2) & 1) << 2;
    if (p.nl >= 16) lb |= (__popc((s >> 1) & p.m3) & 1) << 3;
    if (p.nl >= 32) lb |= (__popc((s >> 1) & p.m4) & 1) << 4;
    return lb;
}

// ------------------------------------------------------------------------------------------------
// shared memory layouts (host and device)
// ------------------------------------------------------------------------------------------------
__host__ __device__ inline int al16(int v) { return (v + 15) & ~15; }

struct FwdSmem {
    int x, w, tab, tabhi, gain, gainhi, ce, gc, dp, err, red, total;
};

__host__ __device__ inline FwdSmem fwd_smem(int T, int G, int Gfull, int sub, int NL, int NP, int U, int U_hi)
{
    FwdSmem L;
    // branch-error rows: NL / 2 label variants per step for the compiled-in mask sets (NL <= 16); one row per step for
    // run-time masks, the only kind with NL = 32 (sized for the variants below that, which the run-time kernels leave
    // partly unused)
    const int NV = NL >= 32 ? 1 : NL / 2, EW = NL * NP;
    int o = 0;
    L.x = o; o = al16(o + 4 * T);
    L.w = o; o = al16(o + 4 * T);
    L.tab = o; o = al16(o + 4 * NL * U);
    L.tabhi = o; o = al16(o + 4 * NL * U_hi);
    L.gain = o; o = al16(o + 4 * MAXG);
    L.gainhi = o; o = al16(o + 4 * MAXG);
    L.ce = o; o = al16(o + 4 * (T / sub) * Gfull);
    L.gc = o; o = al16(o + (T / sub) * G);
    L.dp = o; o = al16(o + 4 * NSP * (G + 1));  // one region per slot + the merged region
    L.err = o; o = al16(o + 4 * G * sub * NV * EW);
    L.red = o; o = al16(o + 8 * MAXG);
    L.total = o;
    return L;
}

struct TbSmem {
    int tab, tabhi, gain, gainhi, warp, tbw, tbg, st, sg, par, flag, per_warp, total;
};

__host__ __device__ inline TbSmem tb_smem(int T, int sub, int NL, int U, int U_hi, int W4, int NB, int warps)
{
    TbSmem L;
    int o = 0;
    L.tab = o; o = al16(o + 4 * NL * U);
    L.tabhi = o; o = al16(o + 4 * NL * U_hi);
    L.gain = o; o = al16(o + 4 * MAXG);
    L.gainhi = o; o = al16(o + 4 * MAXG);
    L.warp = o;
    int q = 0;  // per-warp region, relative offsets
    L.tbw = q; q = al16(q + 4 * 32 * W4 * ((sub + 3) / 4 + 1));
    L.tbg = q; q = al16(q + 4 * (NS / 8));
    L.st = q; q = al16(q + 2 * T);
    L.sg = q; q = al16(q + T);
    L.par = q; q = al16(q + T);
    L.flag = q; q = al16(q + 16);
    L.per_warp = q;
    L.total = o + q * warps;
    return L;
}

// state held by register r of lane L in layout j
__host__ __device__ __forceinline__ int state_of(int j, int L, int r)
{
    return (r & ((1 << j) - 1)) | (L << j) | ((r >> j) << (j + 5));
}
// exchange slot of state s: chunks of 4 consecutive states (16 bytes); chunk c = s >> 2 is stored at c ^ ((c >> 3) & 3).
// Reads of layout 0 (lane L, register r: state L + 32 r) hit 32 distinct banks; writes of layout 4 (lane L holds the
// chunks 4L .. 4L + 3 and 128 + 4L .. 128 + 4L + 3) are 16-byte stores whose quarter-warp phases hit distinct banks.
__host__ __device__ constexpr int swz(int s) { return ((((s >> 2) ^ ((s >> 5) & 3))) << 2) | (s & 3); }

// register index ra (0..15) of the butterfly whose outputs have (s >> 1) == b9, in layout j; lane = (b9 >> j) & 31
__device__ __forceinline__ int bfly_of(int j, int b9) { return (b9 & ((1 << j) - 1)) | ((b9 >> (j + 5)) << j); }

__device__ __forceinline__ uint32_t pushbit(float d, uint32_t acc)
{
    return __funnelshift_l(__float_as_uint(d), acc, 1);  // acc << 1 | sign(d)
}

// min_u (x - g tab[u])^2, u = u0, u0 + du, ... : the reference's contracted form d = fma(-g, tab, x)
__device__ __forceinline__ float branch_err(float x, float g, const float* tl, int u0, int du, int U)
{
    float e = BIG;
    for (int u = u0; u < U; u += du) {
        const float d = __fmaf_rn(-g, tl[u], x);
        e = fminf(e, __fmul_rn(d, d));
    }
    return e;
}

template <class MP, int EW>
__device__ __forceinline__ void load_row(ERow<EW>& e, const float* row, int pl = 0)
{
    e.ptr = row;
    e.pl = pl;
    if (!MP::RT) {
#pragma unroll
        for (int k = 0; k < EW; k += 4) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            e.r[k] = v.x; e.r[k + 1] = v.y; e.r[k + 2] = v.z; e.r[k + 3] = v.w;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// survivors
// ------------------------------------------------------------------------------------------------
struct SvStream {
    uint32_t *a, *b;
    long long capA;
    __device__ __forceinline__ void put(long long k, uint32_t v) const
    {
        if (k < capA) a[k] = v; else b[k - capA] = v;
    }
    __device__ __forceinline__ uint32_t get(long long k) const { return k < capA ? a[k] : b[k - capA]; }
};

// ------------------------------------------------------------------------------------------------
// branch error of the output with code bit C (and parity class P of NPc) of butterfly RA at step J
// ------------------------------------------------------------------------------------------------
template <class MP, int J, int RA, int C, int P, int NPc, int EW>
__device__ __forceinline__ float errv(const MP& mp, const ERow<EW>& E)
{
    if constexpr (!MP::RT) {
        constexpr int i = ((MP::template qc<J, RA>() << 1) | C) * NPc + P;
        return E.r[i];
    } else {
        const int i = (((mp.template q<J, RA>() ^ E.pl) << 1) | C) * NPc + P;
        return E.ptr[i];
    }
}

// ------------------------------------------------------------------------------------------------
// trellis pairs: steps (J, J + 1), J in {0, 2}, processed as 8 radix-4 units per lane.
// Unit u: step-J butterflies u and u + 8 -> intermediates 2u, 2u+1, 2u+16, 2u+17 -> step-(J+1) butterflies
// 2u + 1, 2u -> outputs 4u .. 4u + 3.  Units run u = 7 .. 0 so every packed bit word is built in descending order.
// ------------------------------------------------------------------------------------------------
template <int J, class MP, int EW>
__device__ __forceinline__ uint32_t pair_plain(const MP& mp, float (&cur)[32], const ERow<EW>& E0, const ERow<EW>& E1)
{
    float nx[32];
    uint32_t alo = 0, ahi = 0, a2 = 0;
    cfor<7, -1, -1>([&](auto UU) {
        constexpr int u = decltype(UU)::value;
        float iv[4];
        cfor<0, 2, 1>([&](auto HH) {
            constexpr int hh = decltype(HH)::value, ra = u + 8 * hh;
            const float va = cur[ra], vb = cur[ra + 16];
            const float d = __fsub_rn(vb, va);
            const float mn = fminf(va, vb);
            if constexpr (hh) ahi = pushbit(d, ahi); else alo = pushbit(d, alo);
            iv[2 * hh] = __fadd_rn(mn, errv<MP, J, ra, 0, 0, 1>(mp, E0));
            iv[2 * hh + 1] = __fadd_rn(mn, errv<MP, J, ra, 1, 0, 1>(mp, E0));
        });
        cfor<1, -1, -1>([&](auto CC) {
            constexpr int c = decltype(CC)::value, x = 2 * u + c;
            const float va = iv[c], vb = iv[2 + c];
            const float d = __fsub_rn(vb, va);
            const float mn = fminf(va, vb);
            a2 = pushbit(d, a2);
            nx[2 * x] = __fadd_rn(mn, errv<MP, J + 1, x, 0, 0, 1>(mp, E1));
            nx[2 * x + 1] = __fadd_rn(mn, errv<MP, J + 1, x, 1, 0, 1>(mp, E1));
        });
    });
#pragma unroll
    for (int r = 0; r < 32; r++) cur[r] = nx[r];
    return (((ahi << 8) | alo) << 16) | a2;  // step-J decisions in the high half, step-(J+1) in the low half
}

// D2: pair (J, J+1); intermediates per parity class p, the output takes the class with the smaller metric (tie p=0).
// Words: wi = step-J decisions (16 bits), wh = step-(J+1) decisions per class (p0 << 16 | p1), wc = class per output.
template <int J, class MP, int EW>
__device__ __forceinline__ void pair_d2(const MP& mp, float (&cur)[32], const ERow<EW>& E0, const ERow<EW>& E1,
                                        uint32_t& wi, uint32_t& wh, uint32_t& wc)
{
    float nx[32];
    uint32_t alo = 0, ahi = 0, h0 = 0, h1 = 0, cc = 0;
    cfor<7, -1, -1>([&](auto UU) {
        constexpr int u = decltype(UU)::value;
        float iv[2][4];
        cfor<0, 2, 1>([&](auto HH) {
            constexpr int hh = decltype(HH)::value, ra = u + 8 * hh;
            const float va = cur[ra], vb = cur[ra + 16];
            const float d = __fsub_rn(vb, va);
            const float mn = fminf(va, vb);
            if constexpr (hh) ahi = pushbit(d, ahi); else alo = pushbit(d, alo);
            iv[0][2 * hh] = __fadd_rn(mn, errv<MP, J, ra, 0, 0, 2>(mp, E0));
            iv[1][2 * hh] = __fadd_rn(mn, errv<MP, J, ra, 0, 1, 2>(mp, E0));
            iv[0][2 * hh + 1] = __fadd_rn(mn, errv<MP, J, ra, 1, 0, 2>(mp, E0));
            iv[1][2 * hh + 1] = __fadd_rn(mn, errv<MP, J, ra, 1, 1, 2>(mp, E0));
        });
        cfor<1, -1, -1>([&](auto CC) {
            constexpr int c = decltype(CC)::value, x = 2 * u + c;
            float mnp[2];
            {
                const float d0 = __fsub_rn(iv[0][2 + c], iv[0][c]);
                mnp[0] = fminf(iv[0][c], iv[0][2 + c]);
                h0 = pushbit(d0, h0);
                const float d1 = __fsub_rn(iv[1][2 + c], iv[1][c]);
                mnp[1] = fminf(iv[1][c], iv[1][2 + c]);
                h1 = pushbit(d1, h1);
            }
            cfor<1, -1, -1>([&](auto C2) {
                constexpr int c2 = decltype(C2)::value;
                const float v0 = __fadd_rn(mnp[0], errv<MP, J + 1, x, c2, 0, 2>(mp, E1));
                const float v1 = __fadd_rn(mnp[1], errv<MP, J + 1, x, c2, 1, 2>(mp, E1));
                cc = pushbit(__fsub_rn(v1, v0), cc);
                nx[2 * x + c2] = fminf(v0, v1);
            });
        });
    });
    wi = (ahi << 8) | alo;
    wh = (h0 << 16) | h1;
    wc = cc;
#pragma unroll
    for (int r = 0; r < 32; r++) cur[r] = nx[r];
}

// D4 / EQ phase A: steps (0, 1) of a group of 4.  Step 0: intermediates per low bit b of the first sample; step 1:
// outputs per class c = b0 ^ b1 (EQ: c = b0 = b1), best b per class (tie b = 0).
// Words: w0 = step-0 decisions, w1 = step-1 decisions per b (b0 << 16 | b1), w2 / w3 = chosen b of class 0 / 1.
template <bool EQ, class MP, int EW>
__device__ __forceinline__ void phase_a(const MP& mp, const float (&cur)[32], float (&o0)[32], float (&o1)[32],
                                        const ERow<EW>& E0, const ERow<EW>& E1, uint32_t (&wd)[9])
{
    uint32_t alo = 0, ahi = 0, hb0 = 0, hb1 = 0, bc0 = 0, bc1 = 0;
    cfor<7, -1, -1>([&](auto UU) {
        constexpr int u = decltype(UU)::value;
        float iv[2][4];
        cfor<0, 2, 1>([&](auto HH) {
            constexpr int hh = decltype(HH)::value, ra = u + 8 * hh;
            const float va = cur[ra], vb = cur[ra + 16];
            const float d = __fsub_rn(vb, va);
            const float mn = fminf(va, vb);
            if constexpr (hh) ahi = pushbit(d, ahi); else alo = pushbit(d, alo);
            iv[0][2 * hh] = __fadd_rn(mn, errv<MP, 0, ra, 0, 0, 2>(mp, E0));
            iv[1][2 * hh] = __fadd_rn(mn, errv<MP, 0, ra, 0, 1, 2>(mp, E0));
            iv[0][2 * hh + 1] = __fadd_rn(mn, errv<MP, 0, ra, 1, 0, 2>(mp, E0));
            iv[1][2 * hh + 1] = __fadd_rn(mn, errv<MP, 0, ra, 1, 1, 2>(mp, E0));
        });
        cfor<1, -1, -1>([&](auto CC) {
            constexpr int c = decltype(CC)::value, x = 2 * u + c;
            float mnb[2];
            {
                const float d0 = __fsub_rn(iv[0][2 + c], iv[0][c]);
                mnb[0] = fminf(iv[0][c], iv[0][2 + c]);
                hb0 = pushbit(d0, hb0);
                const float d1 = __fsub_rn(iv[1][2 + c], iv[1][c]);
                mnb[1] = fminf(iv[1][c], iv[1][2 + c]);
                hb1 = pushbit(d1, hb1);
            }
            cfor<1, -1, -1>([&](auto C2) {
                constexpr int c2 = decltype(C2)::value;
                if constexpr (EQ) {
                    o0[2 * x + c2] = __fadd_rn(mnb[0], errv<MP, 1, x, c2, 0, 2>(mp, E1));
                    o1[2 * x + c2] = __fadd_rn(mnb[1], errv<MP, 1, x, c2, 1, 2>(mp, E1));
                    bc0 = bc0 << 1;
                    bc1 = (bc1 << 1) | 1u;
                } else {
                    // class 0: b = 0 uses low bit 0, b = 1 low bit 1; class 1: b = 0 low bit 1, b = 1 low bit 0
                    const float v00 = __fadd_rn(mnb[0], errv<MP, 1, x, c2, 0, 2>(mp, E1));
                    const float v01 = __fadd_rn(mnb[1], errv<MP, 1, x, c2, 1, 2>(mp, E1));
                    bc0 = pushbit(__fsub_rn(v01, v00), bc0);
                    o0[2 * x + c2] = fminf(v00, v01);
                    const float v10 = __fadd_rn(mnb[0], errv<MP, 1, x, c2, 1, 2>(mp, E1));
                    const float v11 = __fadd_rn(mnb[1], errv<MP, 1, x, c2, 0, 2>(mp, E1));
                    bc1 = pushbit(__fsub_rn(v11, v10), bc1);
                    o1[2 * x + c2] = fminf(v10, v11);
                }
            });
        });
    });
    wd[0] = (ahi << 8) | alo;
    wd[1] = (hb0 << 16) | hb1;
    wd[2] = bc0;
    wd[3] = bc1;
}

// D4 / EQ phase B: steps (2, 3).  Step 2: intermediates per class c and low bit b; step 3: outputs over the candidates
// (c, b) = (0,0), (0,1), (1,0), (1,1) in that order with strict `<` (EQ: (0,0), (1,1)).
// Words: w4 = step-2 decisions per class (c0 << 16 | c1), w5 / w6 = step-3 decisions for class 0 / 1 per b
// (b0 << 16 | b1), w7 = chosen class per output, w8 = chosen b per output.
template <bool EQ, class MP, int EW>
__device__ __forceinline__ void phase_b(const MP& mp, const float (&o0)[32], const float (&o1)[32], float (&cur)[32],
                                        const ERow<EW>& E2, const ERow<EW>& E3, uint32_t (&wd)[9])
{
    uint32_t hlo0 = 0, hhi0 = 0, hlo1 = 0, hhi1 = 0, h00 = 0, h01 = 0, h10 = 0, h11 = 0, S1 = 0, S2 = 0, S3 = 0;
    cfor<7, -1, -1>([&](auto UU) {
        constexpr int u = decltype(UU)::value;
        float iv[2][2][4];  // [class][low bit b][intermediate]
        cfor<0, 2, 1>([&](auto CL) {
            constexpr int cl = decltype(CL)::value;
            cfor<0, 2, 1>([&](auto HH) {
                constexpr int hh = decltype(HH)::value, ra = u + 8 * hh;
                const float va = cl ? o1[ra] : o0[ra], vb = cl ? o1[ra + 16] : o0[ra + 16];
                const float d = __fsub_rn(vb, va);
                const float mn = fminf(va, vb);
                if constexpr (cl == 0) { if constexpr (hh) hhi0 = pushbit(d, hhi0); else hlo0 = pushbit(d, hlo0); }
                else { if constexpr (hh) hhi1 = pushbit(d, hhi1); else hlo1 = pushbit(d, hlo1); }
                cfor<0, 2, 1>([&](auto B) {
                    constexpr int b = decltype(B)::value;
                    if constexpr (!EQ || b == cl) {
                        iv[cl][b][2 * hh] = __fadd_rn(mn, errv<MP, 2, ra, 0, b, 2>(mp, E2));
                        iv[cl][b][2 * hh + 1] = __fadd_rn(mn, errv<MP, 2, ra, 1, b, 2>(mp, E2));
                    }
                });
            });
        });
        cfor<1, -1, -1>([&](auto CC) {
            constexpr int c = decltype(CC)::value, x = 2 * u + c;
            float mnx[2][2];
            cfor<0, 2, 1>([&](auto CL) {
                constexpr int cl = decltype(CL)::value;
                cfor<0, 2, 1>([&](auto B) {
                    constexpr int b = decltype(B)::value;
                    uint32_t& hacc = cl ? (b ? h11 : h10) : (b ? h01 : h00);
                    if constexpr (EQ && b != cl) {
                        hacc <<= 1;
                        mnx[cl][b] = BIG;
                    } else {
                        const float va = iv[cl][b][c], vb = iv[cl][b][2 + c];
                        mnx[cl][b] = fminf(va, vb);
                        hacc = pushbit(__fsub_rn(vb, va), hacc);
                    }
                });
            });
            cfor<1, -1, -1>([&](auto C2) {
                constexpr int c2 = decltype(C2)::value;
                if constexpr (EQ) {
                    const float v0 = __fadd_rn(mnx[0][0], errv<MP, 3, x, c2, 0, 2>(mp, E3));
                    const float v1 = __fadd_rn(mnx[1][1], errv<MP, 3, x, c2, 1, 2>(mp, E3));
                    S3 = pushbit(__fsub_rn(v1, v0), S3);
                    cur[2 * x + c2] = fminf(v0, v1);
                } else {
                    const float v00 = __fadd_rn(mnx[0][0], errv<MP, 3, x, c2, 0, 2>(mp, E3));
                    const float v01 = __fadd_rn(mnx[0][1], errv<MP, 3, x, c2, 1, 2>(mp, E3));
                    const float v10 = __fadd_rn(mnx[1][0], errv<MP, 3, x, c2, 1, 2>(mp, E3));
                    const float v11 = __fadd_rn(mnx[1][1], errv<MP, 3, x, c2, 0, 2>(mp, E3));
                    float best = v00;
                    S1 = pushbit(__fsub_rn(v01, best), S1);
                    best = fminf(best, v01);
                    S2 = pushbit(__fsub_rn(v10, best), S2);
                    best = fminf(best, v10);
                    S3 = pushbit(__fsub_rn(v11, best), S3);
                    best = fminf(best, v11);
                    cur[2 * x + c2] = best;
                }
            });
        });
    });
    wd[4] = (((hhi0 << 8) | hlo0) << 16) | ((hhi1 << 8) | hlo1);
    wd[5] = (h00 << 16) | (h01 & 0xffffu);
    wd[6] = (h10 << 16) | (h11 & 0xffffu);
    if (EQ) {
        wd[7] = S3;
        wd[8] = S3;
    } else {
        wd[7] = S2 | S3;
        wd[8] = S3 | (S1 & ~S2);
    }
}

// ------------------------------------------------------------------------------------------------
// sub-block gain merge (src/cuda/tcq_viterbi.cu:185-201), in state space over the exchange regions of all G slots:
// every state continues from its best slot (strict <, lowest slot wins).  The merged metrics go to one region that
// every slot reads next; the winners are 4-bit codes, 8 states per word (word s >> 3, nibble s & 7).  Thread i of the
// CTA handles states 8i .. 8i + 7 (two 16-byte chunks per region).  Inline: with the register caps of the kernels
// that call it, the out-of-line call cost 0.5 % of the fused kernel's time (measured).
// ------------------------------------------------------------------------------------------------
template <int G>
static __device__ __forceinline__ void merge_slots(const float* s_dp, float* s_mg, uint32_t* gw)
{
    for (int i = threadIdx.x; i < NS / 8; i += 32 * G) {
        const int a0 = swz(8 * i), a1 = swz(8 * i + 4);
        float v[8];
        uint32_t code = 0;
        {
            const float4 x0 = *reinterpret_cast<const float4*>(s_dp + a0);
            const float4 x1 = *reinterpret_cast<const float4*>(s_dp + a1);
            v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w; v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
        }
#pragma unroll
        for (int gg = 1; gg < G; gg++) {
            const float4 x0 = *reinterpret_cast<const float4*>(s_dp + gg * NSP + a0);
            const float4 x1 = *reinterpret_cast<const float4*>(s_dp + gg * NSP + a1);
            const float w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (w[k] < v[k]) { v[k] = w[k]; code = (code & ~(15u << (4 * k))) | ((uint32_t)gg << (4 * k)); }
        }
        *reinterpret_cast<float4*>(s_mg + a0) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(s_mg + a1) = make_float4(v[4], v[5], v[6], v[7]);
        gw[i] = code;
    }
}

static __device__ __forceinline__ void merge_any(int G, const float* s_dp, float* s_mg, uint32_t* gw)
{
    switch (G) {
        case 2: merge_slots<2>(s_dp, s_mg, gw); break;
        case 3: merge_slots<3>(s_dp, s_mg, gw); break;
        case 4: merge_slots<4>(s_dp, s_mg, gw); break;
        case 8: merge_slots<8>(s_dp, s_mg, gw); break;
        default: break;
    }
}

// branch-error table of one sub-block for one gain slot (src/cuda/tcq_viterbi.cu:202-213): for each step, label and
// parity class, w * min_u (x - g tab[u])^2, written in the NV label variants err'[P][v] = err[v ^ (P << 1)].
// UC > 0: the table width U as a compile-time constant (the minimum over u unrolled, same operations in the same
// order); UC = 0: any U and the half-integer tables (mix > 0).
template <int NL, int NP, bool MD, int UC, bool VAR>
static __device__ __forceinline__ void build_err_u(float* myerr, const float* s_x, const float* s_w, const float* s_tab,
                                                const float* s_tabhi, float gain, float gainhi, int t0, int sub, int U,
                                                int U_hi, int mix, int lane)
{
    constexpr int NV = VAR ? NL / 2 : 1, EW = NL * NP;  // label variants per step (none for run-time masks)
    __syncwarp();
    if constexpr (UC > 0 && 32 % EW == 0) {
        // EW divides 32, so every entry of this lane has the same (label, class) pair: its table values and its NV
        // destination offsets are loaded / computed once (the stores below could alias s_tab for the compiler, which
        // then reloaded the table for every entry); the arithmetic per entry is unchanged
        const int lb = (lane % EW) / NP, pc = lane % NP;
        constexpr int NU = MD ? UC / 2 : UC;
        float tv[NU];
#pragma unroll
        for (int k = 0; k < NU; k++) tv[k] = s_tab[lb * UC + (MD ? pc + 2 * k : k)];
        int doff[NV];
#pragma unroll
        for (int P = 0; P < NV; P++) doff[P] = P * EW + (lb ^ (P << 1)) * NP + pc;
        for (int tt = lane / EW; tt < sub; tt += 32 / EW) {
            const int t = t0 + tt;
            const float x = s_x[t];
            float e = BIG;
#pragma unroll
            for (int k = 0; k < NU; k++) {
                const float d = __fmaf_rn(-gain, tv[k], x);
                e = fminf(e, __fmul_rn(d, d));
            }
            e = __fmul_rn(e, s_w[t]);
            float* dst = myerr + (size_t)tt * NV * EW;
#pragma unroll
            for (int P = 0; P < NV; P++) dst[doff[P]] = e;
        }
        __syncwarp();
        return;
    }
    for (int it = lane; it < sub * NL * NP; it += 32) {
        const int tt = it / (NL * NP), lb = (it / NP) % NL, pc = it % NP;
        const int t = t0 + tt;
        const float x = s_x[t];
        float e;
        {
            const bool hi = !MD && mix > 0 && ((t / mix) & 1);
            if (MD) e = branch_err(x, gain, s_tab + lb * U, pc, 2, U);
            else if (hi) e = branch_err(x, gainhi, s_tabhi + lb * U_hi, 0, 1, U_hi);
            else e = branch_err(x, gain, s_tab + lb * U, 0, 1, U);
        }
        e = __fmul_rn(e, s_w[t]);
        float* dst = myerr + (size_t)tt * NV * EW + pc;
#pragma unroll
        for (int P = 0; P < NV; P++) dst[P * EW + (lb ^ (P << 1)) * NP] = e;
    }
    __syncwarp();
}

template <int NL, int NP, bool MD, bool VAR>
static __device__ __forceinline__ void build_err(float* myerr, const float* s_x, const float* s_w, const float* s_tab,
                                                 const float* s_tabhi, float gain, float gainhi, int t0, int sub,
                                                 int U, int U_hi, int mix, int lane)
{
    if (mix == 0) {
        switch (U) {
            case 2: build_err_u<NL, NP, MD, 2, VAR>(myerr, s_x, s_w, s_tab, s_tabhi, gain, gainhi, t0, sub, U, U_hi, mix, lane); return;
            case 4: build_err_u<NL, NP, MD, 4, VAR>(myerr, s_x, s_w, s_tab, s_tabhi, gain, gainhi, t0, sub, U, U_hi, mix, lane); return;
            case 8: build_err_u<NL, NP, MD, 8, VAR>(myerr, s_x, s_w, s_tab, s_tabhi, gain, gainhi, t0, sub, U, U_hi, mix, lane); return;
            case 16: build_err_u<NL, NP, MD, 16, VAR>(myerr, s_x, s_w, s_tab, s_tabhi, gain, gainhi, t0, sub, U, U_hi, mix, lane); return;
            default: break;
        }
    }
    build_err_u<NL, NP, MD, 0, VAR>(myerr, s_x, s_w, s_tab, s_tabhi, gain, gainhi, t0, sub, U, U_hi, mix, lane);
}

// ------------------------------------------------------------------------------------------------
// forward kernel
// SUB2: sub-block boundaries may fall in the middle of a 4-step group (sub = 2 mod 4; plain and D2 only).
// ------------------------------------------------------------------------------------------------
// One forward pass over tile n by the CTA's G warps (blockDim.x = 32 G).  The tile's samples are xrow[(t + rot) % ld]
// and its weights wrow[(t + rot) % ld].  Ends with p.best[n] written by thread 0 (no trailing barrier).
// SV1: every survivor word of the tile goes to one contiguous stream (the fused block kernel's workspace); the
// split layout for the reference ABI's caller scratch (bp, then pbits) is then compiled out, with its 64-bit index
// arithmetic (measured: the fused kernel's spills gone, 1.5 % faster)
template <class MP, int MD, bool SUB2, bool SV1 = false>
__device__ __forceinline__ void vit_fwd_tile(const VitParams& p, const int n, unsigned char* smem, const float* xrow,
                                             const float* wrow)
{
    constexpr int NL = MP::NL, NP = MD ? 2 : 1, EW = NL * NP;
    constexpr int NV = MP::RT ? 1 : NL / 2;  // branch-error row variants per step (run-time masks: one, unpermuted)
    constexpr bool PP = MD == 1, G4 = MD >= 2, EQ = MD == 3;
    const int T = p.T, G = p.G, sub = p.sub, nsub = T / sub, U = p.U, U_hi = p.U_hi, mix = p.mix, Gf = p.Gfull;
    const int tid = threadIdx.x, lane = tid & 31, g = tid >> 5, nthr = blockDim.x;
    const FwdSmem SL = fwd_smem(T, G, Gf, sub, NL, NP, U, U_hi);
    float* s_x = reinterpret_cast<float*>(smem + SL.x);
    float* s_w = reinterpret_cast<float*>(smem + SL.w);
    float* s_tab = reinterpret_cast<float*>(smem + SL.tab);
    float* s_tabhi = reinterpret_cast<float*>(smem + SL.tabhi);
    float* s_gain = reinterpret_cast<float*>(smem + SL.gain);
    float* s_gainhi = reinterpret_cast<float*>(smem + SL.gainhi);
    float* s_ce = reinterpret_cast<float*>(smem + SL.ce);
    uint8_t* s_gc = smem + SL.gc;
    float* s_dp = reinterpret_cast<float*>(smem + SL.dp);
    float* s_err = reinterpret_cast<float*>(smem + SL.err);
    float* red_v = reinterpret_cast<float*>(smem + SL.red);
    int* red_i = reinterpret_cast<int*>(smem + SL.red + 4 * MAXG);
    const MP mp(p);

    // ---- tile inputs (sample t is element (t + rot) % ld), tables, gains ----
    for (int i = tid; i < T; i += nthr) {
        const int j = (i + p.rot) % p.ld;
        s_x[i] = xrow[j];
        s_w[i] = wrow[j];
    }
    for (int i = tid; i < NL * U; i += nthr) s_tab[i] = p.tab[i];
    for (int i = tid; i < NL * U_hi; i += nthr) s_tabhi[i] = p.tab_hi[i];
    if (tid < Gf) { s_gain[tid] = p.gains[tid]; s_gainhi[tid] = p.gains_hi[tid]; }
    __syncthreads();

    // ---- gain candidates: weighted scalar error of each sub-block over the merged table (src/cuda/tcq_viterbi.cu:155-180)
    if (p.cand) {
        for (int i = tid; i < nsub * Gf; i += nthr) {
            const int j = i / Gf, gi = i % Gf;
            float e = 0.f;
            for (int t = j * sub; t < (j + 1) * sub; t++) {
                const bool hi = mix > 0 && ((t / mix) & 1);
                const float be = hi ? branch_err(s_x[t], s_gainhi[gi], s_tabhi, 0, 1, NL * U_hi)
                                    : branch_err(s_x[t], s_gain[gi], s_tab, 0, 1, NL * U);
                e = __fmaf_rn(be, s_w[t], e);
            }
            s_ce[i] = e;
        }
        __syncthreads();
        if (tid < nsub) {
            uint32_t used = 0;
            for (int c = 0; c < G; c++) {
                int bg = 0;
                float be = BIG;
                for (int gi = 0; gi < Gf; gi++)
                    if (!((used >> gi) & 1u) && s_ce[tid * Gf + gi] < be) { be = s_ce[tid * Gf + gi]; bg = gi; }
                used |= 1u << bg;
                s_gc[tid * G + c] = (uint8_t)bg;
                p.gcand[((size_t)n * p.nsl + tid) * G + c] = (uint8_t)bg;
            }
        }
        __syncthreads();
    }

    // ---- per-lane constants ----
    int PLj[4];
#pragma unroll
    for (int j = 0; j < 4; j++) PLj[j] = mp.hi((unsigned)((lane << j) & 511));
    const SvStream sv{p.svA + ((size_t)n * G + g) * (size_t)p.capA, p.svB + ((size_t)n * G + g) * (size_t)p.capB,
                      p.capA};
    float* myerr = s_err + (size_t)g * sub * NV * EW;
    float* mydp = s_dp + (size_t)g * NSP;
    float* s_mg = s_dp + (size_t)G * NSP;  // merged metrics after a sub-block boundary
    auto build = [&](int sb) {
        const int gi = p.cand ? (int)s_gc[sb * G + g] : g;
        build_err<NL, NP, MD != 0, !MP::RT>(myerr, s_x, s_w, s_tab, s_tabhi, s_gain[gi], s_gainhi[gi], sb * sub, sub, U,
                                            U_hi, mix, lane);
    };
    // per-lane exchange addresses: layout-0 reads (4 bases, by r & 3) and layout-4 chunk writes (4 bases, by chunk)
    int rbase[4], wbase[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        rbase[q] = 4 * ((lane >> 2) ^ q) + (lane & 3);
        wbase[q] = 16 * lane + 4 * (q ^ ((lane >> 1) & 3));
    }
    auto read0 = [&](float (&cur)[32], const float* src) {
        cfor<0, 32, 1>([&](auto R) { constexpr int r = decltype(R)::value; cur[r] = src[rbase[r & 3] + 32 * r]; });
    };
    auto write4 = [&](const float (&cur)[32], float* dst) {
        cfor<0, 8, 1>([&](auto K) {
            constexpr int k = decltype(K)::value, r = 4 * k;
            *reinterpret_cast<float4*>(dst + wbase[k & 3] + (k >> 2) * 512) =
                make_float4(cur[r], cur[r + 1], cur[r + 2], cur[r + 3]);
        });
    };
    // generic scalar exchange (sub-blocks that end in the middle of a group): layout jf -> layout jt through the
    // regions, with the gain merge
    auto exchange_merge = [&](float (&cur)[32], auto JF, auto JT, int sb) {
        constexpr int jf = decltype(JF)::value, jt = decltype(JT)::value;
        __syncwarp();
        cfor<0, 32, 1>([&](auto R) { constexpr int r = decltype(R)::value; mydp[swz(state_of(jf, lane, r))] = cur[r]; });
        __syncthreads();
        merge_any(G, s_dp, s_mg, p.gsw + ((size_t)n * p.nsl + sb) * (NS / 8));
        __syncthreads();
        cfor<0, 32, 1>([&](auto R) { constexpr int r = decltype(R)::value; cur[r] = s_mg[swz(state_of(jt, lane, r))]; });
    };

    // ---- virtual step before the tile start, layout 0: metric 0 for predecessors of the start state's successors,
    // written to this slot's exchange region; every group of 4 steps reads its metrics from a region (layout 0) and
    // writes them back (layout 4), so no path metric stays in registers across groups ----
    {
        const int s0 = p.init_st ? p.init_st[n] : -1;
        cfor<0, 32, 1>([&](auto R) {
            constexpr int r = decltype(R)::value;
            const int st = state_of(0, lane, r);
            mydp[rbase[r & 3] + 32 * r] = (s0 < 0 || (st & 511) == (s0 & 511)) ? 0.f : BIG;
        });
    }
    build(0);

    // ---- forward: groups of 4 steps ----
    int sb = 0, tt = 0;  // sub-block of the next step, its offset in the sub-block
    // the branch-error row of step tt + off for this lane's label part in layout j: its variant (compiled-in masks) or
    // the unpermuted row with the lane part kept beside it (run-time masks)
    auto lrow = [&](ERow<EW>& e, int off, int j) {
        if constexpr (MP::RT) load_row<MP>(e, myerr + (size_t)(tt + off) * EW, PLj[j]);
        else load_row<MP>(e, myerr + ((size_t)(tt + off) * NV + PLj[j]) * EW);
    };
    const float* src = mydp;
    // survivor words: groups that fit entirely in region A are stored through a plain pointer
    const long long gw4 = (long long)p.W4 * 32;
    const int ngA = (int)(p.capA / gw4 < (1 << 30) ? p.capA / gw4 : (1 << 30));
    uint32_t* svp = sv.a + lane;
    float cur[32];
    for (int t4 = 0, grp = 0;; t4 += 4, grp++, svp += gw4) {
        __syncwarp();
        read0(cur, src);
        // each pair's two rows load just before the pair (loading the second pair's rows with the first pair's held
        // 16 more registers over the first pair: 6 % more instructions in the plain mode, measured)
        ERow<EW> E0, E1;
        lrow(E0, 0, 0);
        lrow(E1, 1, 1);
        uint32_t wd[9];
        if constexpr (MD == 0) {
            wd[0] = pair_plain<0>(mp, cur, E0, E1);
        } else if constexpr (PP) {
            pair_d2<0>(mp, cur, E0, E1, wd[0], wd[1], wd[2]);
            wd[0] <<= 16;  // step-0 decisions in the high half, step-2 decisions in the low half
        }
        float o0[G4 ? 32 : 1], o1[G4 ? 32 : 1];
        if constexpr (G4) phase_a<EQ>(mp, cur, o0, o1, E0, E1, wd);
        tt += 2;
        const bool full = t4 + 2 < T;
        if (full) {
            if constexpr (SUB2 && !G4) {
                if (tt == sub) {  // sub-block boundary inside the group
                    sb++;
                    tt = 0;
                    if (G > 1) exchange_merge(cur, IC<2>{}, IC<2>{}, sb);
                    build(sb);
                }
            }
            ERow<EW> E2, E3;
            lrow(E2, 0, 2);
            lrow(E3, 1, 3);
            if constexpr (MD == 0) {
                wd[1] = pair_plain<2>(mp, cur, E2, E3);
            } else if constexpr (PP) {
                uint32_t wi;
                pair_d2<2>(mp, cur, E2, E3, wi, wd[3], wd[4]);
                wd[0] |= wi;
            } else {
                phase_b<EQ>(mp, o0, o1, cur, E2, E3, wd);
            }
            tt += 2;
        }
        // survivor words of this group (the last group of T = 2 mod 4 keeps only its first pair's words)
        const int nw = full ? p.W4 : (MD == 0 ? 1 : 3);
        if (SV1 || grp < ngA) {
#pragma unroll
            for (int k = 0; k < (MD == 0 ? 2 : (PP ? 5 : 9)); k++)
                if (k < nw) svp[32 * k] = wd[k];
        } else {
            const long long kb = (long long)grp * gw4 + lane;
#pragma unroll
            for (int k = 0; k < (MD == 0 ? 2 : (PP ? 5 : 9)); k++)
                if (k < nw) sv.put(kb + 32 * k, wd[k]);
        }
        if (t4 + 4 >= T) break;  // the last group's metrics stay in registers for the argmin
        // metrics (layout 4) back to this slot's region; at a sub-block boundary all slots merge first
        __syncwarp();
        write4(cur, mydp);
        src = mydp;
        if (tt == sub) {
            sb++;
            tt = 0;
            if (G > 1) {
                __syncthreads();
                merge_any(G, s_dp, s_mg, p.gsw + ((size_t)n * p.nsl + sb) * (NS / 8));
                __syncthreads();
                src = s_mg;
            }
            build(sb);
        }
    }

    // ---- final argmin over (slot, state), tail-biting keeps s == s0 (src/cuda/tcq_viterbi.cu:561-579) ----
    const int jend = ((T - 1) & 3) + 1;
    const int s_end = (p.tail && p.init_st) ? p.init_st[n] : -1;
    float bv = BIG;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < 32; r++) {
        const int s = state_of(jend, lane, r);
        const int idx = g * NS + s;
        const float v = (s_end < 0 || s == s_end) ? cur[r] : BIG;
        if (v < bv || (v == bv && idx < bi)) { bv = v; bi = idx; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, bv, off);
        const int oi = __shfl_down_sync(0xffffffffu, bi, off);
        if (ov < bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { red_v[g] = bv; red_i[g] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int k = 1; k < G; k++)
            if (red_v[k] < bv || (red_v[k] == bv && red_i[k] < bi)) { bv = red_v[k]; bi = red_i[k]; }
        // No metric compared below 3.4e38 (all NaN or +inf, i.e. non-finite inputs): there is no best path.  Take slot 0
        // and the required end state (or state 0) so that the traceback stays inside the tile's survivor rows.
        if (bi == 0x7fffffff) bi = s_end >= 0 ? s_end : 0;
        p.best[n] = bi;
        if (p.end_st) p.end_st[n] = bi % NS;
    }
}

// 128 registers a thread: the plain mode at the tighter cap of 85 (6 four-slot tiles per SM) spent 12 % more
// instructions on register moves around the branch-error row loads and ran 5 % slower than with 4 tiles per SM.
template <class MP, int MD, bool SUB2>
__global__ void __launch_bounds__(256, 2) vit_fwd_kernel(const VitParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int n = blockIdx.x;
    vit_fwd_tile<MP, MD, SUB2>(p, n, smem, p.x + (size_t)n * p.ld, p.w + (size_t)n * p.ldw);
}

// ------------------------------------------------------------------------------------------------
// One 4-step group of a traceback walk (steps tg + 3 .. tg, none of them the first pass's stop or t = 0), for both
// traceback kernels.  `w` holds the group's survivor words of lane column L (bits 4..8 of the state at step tg + 3) and
// r that state's register in layout 4, ((s >> 9) << 4) | (s & 15).  The walk runs on the butterfly index b = r >> 1:
// each step b' = (b >> 1) | (decision bit << 3), with the decision half-word pre-shifted by 3, so a plain-mode step is
// one variable shift (beside b >> 1) and one LOP3; the parity modes extract every candidate half while their class bits
// are read, then select.  Writes the parity class of the group's steps to par[tg .. tg + 3] (D2 / D4 / EQ) and returns
// the register of the state before step tg, in layout 4 of the previous group; that state is L | r << 5.  The group's
// code bits (r & 1 at steps 3, 2, 1, 0) are bits 0, 1, 2, 3 of the entry r: each step shifts r down by one.
// Same decisions as the per-step walk (the decision bit h of step j picks the predecessor register (r >> 1) | h << 4).
// ------------------------------------------------------------------------------------------------
template <int MD>
__device__ __forceinline__ int tb_walk_group(const uint32_t* w, const int r, uint8_t* par, const int tg, int& pcur,
                                             int& cstar)
{
    constexpr bool PP = MD == 1, EQ = MD == 3;
    uint32_t b = (uint32_t)r >> 1;
    if constexpr (MD == 0) {
        b = (b >> 1) | (((w[1] << 3) >> b) & 8u);
        b = (b >> 1) | ((((w[1] >> 16) << 3) >> b) & 8u);
        b = (b >> 1) | (((w[0] << 3) >> b) & 8u);
        return (int)(b | ((((w[0] >> 16) << 4) >> b) & 16u));  // step 0: high half of w[0]
    } else if constexpr (PP) {
        // step 3: class bit of the pair from w[4] at r, decision from the half of w[3] it picks
        const uint32_t c3 = (w[4] >> r) & 1u;
        const uint32_t lo3 = ((w[3] << 3) >> b) & 8u, hi3 = (((w[3] >> 16) << 3) >> b) & 8u;
        par[tg + 3] = par[tg + 2] = (uint8_t)c3;
        b = (b >> 1) | (c3 ? lo3 : hi3);
        // step 2: low half of w[0]; the full register r of step 1 for its class bit
        const uint32_t r1 = b | (((w[0] << 4) >> b) & 16u);
        b = r1 >> 1;
        // step 1: class bit from w[2] at r1, decision from the half of w[1] it picks
        const uint32_t c1 = (w[2] >> r1) & 1u;
        const uint32_t lo1 = ((w[1] << 3) >> b) & 8u, hi1 = (((w[1] >> 16) << 3) >> b) & 8u;
        par[tg + 1] = par[tg] = (uint8_t)c1;
        pcur = (int)c1;
        b = (b >> 1) | (c1 ? lo1 : hi1);
        return (int)(b | ((((w[0] >> 16) << 4) >> b) & 16u));  // step 0: high half of w[0]
    } else {
        // step 3: quad class c (w[7]) and pair bit (w[8]) at r pick the half of w[5] / w[6]
        const uint32_t c3 = (w[7] >> r) & 1u, p3 = (w[8] >> r) & 1u;
        const uint32_t wq = c3 ? w[6] : w[5];
        const uint32_t lo3 = ((wq << 3) >> b) & 8u, hi3 = (((wq >> 16) << 3) >> b) & 8u;
        cstar = (int)c3;
        if (EQ) {
            par[tg + 3] = par[tg + 2] = par[tg + 1] = par[tg] = (uint8_t)c3;
        } else {
            par[tg + 3] = (uint8_t)(p3 ^ c3);
            par[tg + 2] = (uint8_t)p3;
        }
        b = (b >> 1) | (p3 ? lo3 : hi3);
        // step 2: the half of w[4] picked by the quad class; the full register r of step 1
        const uint32_t r1 = b | ((((c3 ? w[4] : (w[4] >> 16)) << 4) >> b) & 16u);
        b = r1 >> 1;
        // step 1: pair bit from w[2] / w[3] (by the quad class) at r1 picks the half of w[1]
        const uint32_t p1 = ((c3 ? w[3] : w[2]) >> r1) & 1u;
        const uint32_t lo1 = ((w[1] << 3) >> b) & 8u, hi1 = (((w[1] >> 16) << 3) >> b) & 8u;
        if (!EQ) {
            par[tg + 1] = (uint8_t)(p1 ^ c3);
            par[tg] = (uint8_t)p1;
        }
        b = (b >> 1) | (p1 ? lo1 : hi1);
        return (int)(b | (((w[0] << 4) >> b) & 16u));  // step 0: low half of w[0]
    }
}

// ------------------------------------------------------------------------------------------------
// traceback, reconstruction and codes (src/cuda/tcq_viterbi.cu:580-682), one warp per tile
// ------------------------------------------------------------------------------------------------
// Traceback of tile n by one warp.  Tables and gains are in shared memory (s_tab ...); `wbase` is the warp's region of
// the TbSmem per-warp layout; the tile's samples are xrow[(t + rot) % ld].
template <int MD>
__device__ __forceinline__ void vit_tb_tile(const VitParams& p, const int n, const int lane, const float* s_tab,
                                            const float* s_tabhi, const float* s_gain, const float* s_gainhi,
                                            unsigned char* wbase, const float* xrow)
{
    constexpr bool PP = MD == 1, EQ = MD == 3;
    const int T = p.T, G = p.G, sub = p.sub, nsub = T / sub, U = p.U, U_hi = p.U_hi, mix = p.mix, NL = p.nl;
    const TbSmem SL = tb_smem(T, sub, NL, U, U_hi, p.W4, p.NB, 1);
    uint32_t* s_tbw = reinterpret_cast<uint32_t*>(wbase + SL.tbw);
    uint32_t* s_tbg = reinterpret_cast<uint32_t*>(wbase + SL.tbg);
    uint16_t* s_st = reinterpret_cast<uint16_t*>(wbase + SL.st);
    uint8_t* s_sg = wbase + SL.sg;
    uint8_t* s_par = wbase + SL.par;
    int* s_flag = reinterpret_cast<int*>(wbase + SL.flag);

    if (lane == 0) {
        const int bi = p.best[n];
        s_flag[0] = bi % NS;  // state
        s_flag[1] = bi / NS;  // slot
        s_flag[2] = 0;        // stopped at the first-pass middle
    }
    __syncwarp();
    for (int lo = T - sub; lo >= 0; lo -= sub) {
        const int gc = s_flag[1];
        const int grp0 = lo >> 2, grp1 = (lo + sub - 1) >> 2;
        const SvStream svg{p.svA + ((size_t)n * G + gc) * (size_t)p.capA, p.svB + ((size_t)n * G + gc) * (size_t)p.capB,
                           p.capA};
        for (int grp = grp0; grp <= grp1; grp++) {
            const int nw = (grp * 4 + 2 < T) ? p.W4 : (MD == 0 ? 1 : 3);
            for (int k = 0; k < nw; k++)
                s_tbw[((grp - grp0) * p.W4 + k) * 32 + lane] = svg.get(((long long)grp * p.W4 + k) * 32 + lane);
        }
        if (G > 1 && lo > 0)
            for (int k = lane; k < NS / 8; k += 32) s_tbg[k] = p.gsw[((size_t)n * p.nsl + lo / sub) * (NS / 8) + k];
        __syncwarp();
        if (lane == 0) {
            int st = s_flag[0], gs = s_flag[1], pcur = 0, cstar = 0;
            bool stop = false;
            for (int t = lo + sub - 1; t >= lo; t--) {
                // a whole 4-step group inside this sub-block, without the first pass's stop or t = 0: the group walk;
                // the states of its steps are the 10-bit windows of V = (state before the group) << 4 | (s_t & 15)
                if ((t & 3) == 3 && t - 3 >= lo && t != 3 && !(p.mid_st && (unsigned)(p.mid_t - 1 - (t - 3)) < 4u)) {
                    constexpr int W4C = MD == 0 ? 2 : (MD == 1 ? 5 : 9);
                    const int L = (st >> 4) & 31;
                    const uint32_t* Wg = s_tbw + ((t >> 2) - grp0) * p.W4 * 32 + L;
                    uint32_t w[W4C];
#pragma unroll
                    for (int k = 0; k < W4C; k++) w[k] = Wg[32 * k];
                    const int rn = tb_walk_group<MD>(w, ((st >> 9) << 4) | (st & 15), s_par, t - 3, pcur, cstar);
                    const int stn = L | (rn << 5);
                    const int V = (stn << 4) | (st & 15);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        s_st[t - k] = (uint16_t)((V >> k) & 1023);
                        s_sg[t - k] = (uint8_t)gs;
                    }
                    st = stn;
                    t -= 3;  // the loop's t-- moves on to the step before the group
                    if (G > 1 && t == lo) gs = (int)((s_tbg[st >> 3] >> (4 * (st & 7))) & 15u);
                    continue;
                }
                s_st[t] = (uint16_t)st;
                s_sg[t] = (uint8_t)gs;
                const int j = t & 3;
                const int b9 = st >> 1;
                const int L = (b9 >> j) & 31;
                const int bi4 = bfly_of(j, b9);
                const uint32_t* W = s_tbw + ((t >> 2) - grp0) * p.W4 * 32 + L;  // word k of this group: W[32 k]
                if (PP && (t & 1)) {
                    pcur = (W[32 * (j == 1 ? 2 : 4)] >> ((bi4 << 1) | (st & 1))) & 1;
                    s_par[t] = s_par[t - 1] = (uint8_t)pcur;
                }
                if (p.mid_st && t == p.mid_t - 1) { p.mid_st[n] = st; stop = true; break; }
                if (t == 0) break;
                int h;
                if (MD == 0) {
                    h = (W[32 * (j >> 1)] >> ((j & 1) ? bi4 : 16 + bi4)) & 1;
                } else if (PP) {
                    if (j & 1) h = (W[32 * (j == 1 ? 1 : 3)] >> (pcur ? bi4 : 16 + bi4)) & 1;
                    else h = (W[0] >> ((j == 0) ? 16 + bi4 : bi4)) & 1;
                } else {
                    const int ro = (bi4 << 1) | (st & 1);  // output register of st at steps j = 1, 3
                    if (j == 3) {
                        cstar = (W[32 * 7] >> ro) & 1;
                        const int bb = (W[32 * 8] >> ro) & 1;
                        h = (W[32 * (5 + cstar)] >> (bb ? bi4 : 16 + bi4)) & 1;
                        if (EQ) {
                            s_par[t] = s_par[t - 1] = s_par[t - 2] = s_par[t - 3] = (uint8_t)cstar;
                        } else {
                            s_par[t] = (uint8_t)(bb ^ cstar);
                            s_par[t - 1] = (uint8_t)bb;
                        }
                    } else if (j == 2) {
                        h = (W[32 * 4] >> (cstar ? bi4 : 16 + bi4)) & 1;
                    } else if (j == 1) {
                        const int bb = (W[32 * (2 + cstar)] >> ro) & 1;
                        h = (W[32 * 1] >> (bb ? bi4 : 16 + bi4)) & 1;
                        if (!EQ) {
                            s_par[t] = (uint8_t)(bb ^ cstar);
                            s_par[t - 1] = (uint8_t)bb;
                        }
                    } else {
                        h = (W[0] >> bi4) & 1;
                    }
                }
                st = (h << 9) | b9;
                if (G > 1 && t == lo) {  // sub-block boundary: slot of the previous sub-block
                    gs = (int)((s_tbg[st >> 3] >> (4 * (st & 7))) & 15u);
                }
            }
            s_flag[0] = st;
            s_flag[1] = gs;
            if (stop) s_flag[2] = 1;
        }
        __syncwarp();
        if (s_flag[2]) return;  // first tail-biting pass: only the middle state was needed
    }

    float* rn = p.rec + (size_t)n * p.ld;
    for (int t = lane; t < T; t += 32) {
        const int stt = s_st[t], gg = s_sg[t];
        const int lb = label_rt(stt, p);
        const bool hi = mix > 0 && ((t / mix) & 1);
        const int Ut = hi ? U_hi : U;
        const int gi = p.cand ? (int)p.gcand[((size_t)n * p.nsl + t / sub) * G + gg] : gg;
        const float gt = hi ? s_gainhi[gi] : s_gain[gi];
        const float* tt = (hi ? s_tabhi : s_tab) + lb * Ut;
        const int tp = (t + p.rot) % p.ld;
        const float xt = xrow[tp];
        float bestd = BIG, val = 0.f;
        int bu = 0;
        for (int u = MD ? s_par[t] : 0; u < Ut; u += MD ? 2 : 1) {
            const float v = __fmul_rn(gt, tt[u]);
            const float d = __fmaf_rn(-gt, tt[u], xt);
            const float dd = __fmul_rn(d, d);
            if (dd < bestd) { bestd = dd; val = v; bu = u; }
        }
        rn[tp] = val;
        if (p.code) p.code[(size_t)n * p.ld + tp] = (gi << 16) | (lb * Ut + bu);
    }
}

template <int MD>
__global__ void __launch_bounds__(32 * TB_WARPS) vit_tb_kernel(const VitParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    const int n = blockIdx.x * wpb + warp;
    const TbSmem SL = tb_smem(p.T, p.sub, p.nl, p.U, p.U_hi, p.W4, p.NB, wpb);
    float* s_tab = reinterpret_cast<float*>(smem + SL.tab);
    float* s_tabhi = reinterpret_cast<float*>(smem + SL.tabhi);
    float* s_gain = reinterpret_cast<float*>(smem + SL.gain);
    float* s_gainhi = reinterpret_cast<float*>(smem + SL.gainhi);
    for (int i = threadIdx.x; i < p.nl * p.U; i += blockDim.x) s_tab[i] = p.tab[i];
    for (int i = threadIdx.x; i < p.nl * p.U_hi; i += blockDim.x) s_tabhi[i] = p.tab_hi[i];
    if (threadIdx.x < p.Gfull) { s_gain[threadIdx.x] = p.gains[threadIdx.x]; s_gainhi[threadIdx.x] = p.gains_hi[threadIdx.x]; }
    __syncthreads();
    if (n >= p.N) return;
    vit_tb_tile<MD>(p, n, lane, s_tab, s_tabhi, s_gain, s_gainhi, smem + SL.warp + (size_t)warp * SL.per_warp,
                    p.x + (size_t)n * p.ld);
}

}  // namespace ltqb
