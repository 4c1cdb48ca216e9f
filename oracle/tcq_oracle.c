/*
 * TEST INFRASTRUCTURE ONLY — not part of the product.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load this library, and only as the checker or the timed CPU baseline.
 *
 * CPU restatement of the reference TCQ Viterbi (lumen-inference/ltq-research), written from the semantics of
 * src/cuda/tcq_viterbi.cu:97-683 (tcq_forward_kernel) and src/tcq_proto.py:327-419 (viterbi_ub).  One tile at a
 * time, in the plain radix-2 form of the recursion; the reference kernel's radix-4 butterfly performs the same fp32
 * operations on the same operands in the same order (an add of the selected predecessor and the branch error, a strict
 * `<` compare), so the results are identical.
 *
 * Pinned against (see tests/test_oracle_golden.py):
 *   - the reference torch Viterbi `viterbi_ub` (src/tcq_proto.py:363), imported from the reference tree and run on CPU
 *     (fixtures tests/golden/torch_viterbi_ub.npz, round_mode 0: products rounded before the subtraction, as torch does);
 *   - the reference CUDA kernel compiled for sm_100a from its own source by oracle/build_ref.sh and run on a B200
 *     (fixtures tests/golden/ref_kernel_*.npz, round_mode 7: the kernel's contracted FMAs).
 *
 * Rounding (round_mode bit flags; the reference kernel is built by nvcc with fp contraction on):
 *   bit 0: branch error d = x - g*tab as one fused multiply-add    (src/cuda/tcq_viterbi.cu:50, :79)
 *   bit 1: gain-candidate error accumulated as e = fma(err, w, e)   (src/cuda/tcq_viterbi.cu:161-162)
 *   bit 2: reconstruction distance d = x - g*tab fused              (src/cuda/tcq_viterbi.cu:675-677)
 * This file must be compiled with -ffp-contract=off so that no other operation is fused.
 *
 * Tie-breaks (src/cuda/tcq_viterbi.cu): ACS predecessor strict `<` (tie -> s' >> 1); gain merge strict `<` over g
 * ascending (:193-196); D2 class strict `<`, p ascending (:293-299, :479-483); D4 strict `<` over (c, b) (:244-250,
 * :363-367, :392-420); final argmin = smallest value then smallest flat index g*S + s (:561-579, :591-594);
 * candidates strict `<`, lowest gain index (:167-177); reconstruction level strict `<`, lowest u (:674-678).
 */
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BIG 3.4e38f
#define MAX_G 16
#define MAX_U 128
#define MAX_SUBS 32
#define MAX_T 512

typedef struct {
    const float *x, *w, *tab, *gains, *tab_hi, *gains_hi;
    float *rec;
    const int *init_st;
    int *end_st;
    uint8_t *gcand;
    int *best, *code, *mid_st;
    int mid_t, tail;
    int N, T, S, U, G, Gfull, m, sub, U_hi, mix, m2, m3, m4, nl, ld, rot, pp;
    int round_mode;
} ora_args;

typedef struct {
    float *xs, *ws, *err, *ce;
    float *dp, *nx, *i0, *i1, *c0, *c1;  /* [G * S] each */
    uint8_t *bp;      /* [T, G, S]    predecessor bit of step t per output state */
    uint8_t *pb;      /* [T/2, G, S]  D2 class of the pair's output state */
    uint8_t *pl;      /* [T/4, G, 9, S] D4 group planes (same meaning as the reference's 9 planes) */
    uint8_t *gsel;    /* [T/sub, S]  gain slot chosen at each sub-block boundary */
    uint8_t *gc;      /* [T/sub, G]  candidate gain indices */
    int *lab;         /* [S] */
    uint16_t *st;     /* [T] */
    uint8_t *sg, *par;/* [T] */
} ora_scratch;

static inline int parity32(uint32_t v) { return __builtin_popcount(v) & 1; }

/* label(s) = (s & 1) | parity((s >> 1) & m) << 1 | parity((s >> 1) & m2) << 2 | ...  (src/cuda/tcq_viterbi.cu:85-95) */
static inline int label_of(int s, const ora_args *a)
{
    int lb = (parity32((uint32_t)(s >> 1) & (uint32_t)a->m) << 1) | (s & 1);
    if (a->nl >= 8) lb |= parity32((uint32_t)(s >> 1) & (uint32_t)a->m2) << 2;
    if (a->nl >= 16) lb |= parity32((uint32_t)(s >> 1) & (uint32_t)a->m3) << 3;
    if (a->nl >= 32) lb |= parity32((uint32_t)(s >> 1) & (uint32_t)a->m4) << 4;
    return lb;
}

/* min_u (x - g * tab[u])^2 over u = u0, u0 + du, ... < U, starting from 3.4e38 (src/cuda/tcq_viterbi.cu:46-54, :75-83) */
static inline float branch_err(float xt, float g, const float *tl, int u0, int du, int U, int fused)
{
    float e = BIG;
    for (int u = u0; u < U; u += du) {
        float d;
        if (fused) d = fmaf(-g, tl[u], xt);
        else { float v = g * tl[u]; d = xt - v; }
        float dd = d * d;
        e = fminf(e, dd);
    }
    return e;
}

static int validate(const ora_args *a)
{
    /* same table as src/cuda/tcq_viterbi.cu:748-751 plus the dispatch limits :720-763 */
    if (a->G > MAX_G || a->Gfull > MAX_G || (!a->gcand && a->Gfull != a->G) || a->U > MAX_U || a->U_hi > MAX_U ||
        a->sub <= 0 || a->T % a->sub != 0 || (a->sub & 1) || a->T / a->sub > MAX_SUBS || a->T > MAX_T || a->sub > 32 ||
        a->sub * a->G * a->nl * (a->pp ? 2 : 1) > 4096 || (a->pp && (a->S != 1024 || a->mix > 0 || (a->T & 1))) ||
        (a->pp >= 2 && ((a->T & 3) || (a->sub & 3))) || a->pp > 3 || a->pp < 0 ||
        (a->nl != 4 && a->nl != 8 && a->nl != 16 && a->nl != 32) || a->ld < a->T ||
        (a->S != 1024 && a->nl != 4) || a->nl * a->U > 4 * MAX_U || a->nl * a->U_hi > 4 * MAX_U)
        return -1;
    if (a->S != 1024 && a->S != 256) return -1;
    if (!(a->G == 1 || a->G == 2 || a->G == 3 || a->G == 4 || a->G == 8)) return -1;
    return 0;
}

static int alloc_scratch(ora_scratch *s, const ora_args *a)
{
    const size_t GS = (size_t)a->G * a->S;
    memset(s, 0, sizeof(*s));
    s->xs = malloc(sizeof(float) * a->T);
    s->ws = malloc(sizeof(float) * a->T);
    s->err = malloc(sizeof(float) * (size_t)a->sub * a->G * a->nl * 2);
    s->ce = malloc(sizeof(float) * MAX_SUBS * MAX_G);
    s->dp = malloc(sizeof(float) * GS);
    s->nx = malloc(sizeof(float) * GS);
    s->i0 = malloc(sizeof(float) * GS);
    s->i1 = malloc(sizeof(float) * GS);
    s->c0 = malloc(sizeof(float) * GS);
    s->c1 = malloc(sizeof(float) * GS);
    s->bp = malloc((size_t)a->T * GS);
    s->pb = malloc((size_t)(a->T / 2 + 1) * GS);
    s->pl = malloc((size_t)(a->T / 4 + 1) * GS * 9);
    s->gsel = malloc((size_t)(a->T / a->sub) * a->S);
    s->gc = malloc((size_t)MAX_SUBS * MAX_G);
    s->lab = malloc(sizeof(int) * a->S);
    s->st = malloc(sizeof(uint16_t) * a->T);
    s->sg = malloc(a->T);
    s->par = malloc(a->T);
    return (s->xs && s->ws && s->err && s->ce && s->dp && s->nx && s->i0 && s->i1 && s->c0 && s->c1 && s->bp && s->pb &&
            s->pl && s->gsel && s->gc && s->lab && s->st && s->sg && s->par) ? 0 : -2;
}

static void free_scratch(ora_scratch *s)
{
    free(s->xs); free(s->ws); free(s->err); free(s->ce); free(s->dp); free(s->nx); free(s->i0); free(s->i1);
    free(s->c0); free(s->c1); free(s->bp); free(s->pb); free(s->pl); free(s->gsel); free(s->gc); free(s->lab);
    free(s->st); free(s->sg); free(s->par);
}

static void tile(const ora_args *a, int n, ora_scratch *sc)
{
    const int T = a->T, S = a->S, G = a->G, NL = a->nl, sub = a->sub, U = a->U, U_hi = a->U_hi, mix = a->mix;
    const int HALF = S / 2, MD = a->pp, NP = MD ? 2 : 1, nsub = T / sub, Gf = a->Gfull;
    const int PP = MD == 1, G4 = MD == 2 || MD == 3, EQ = MD == 3;
    const int cand = a->gcand != NULL;
    const int fuse_be = a->round_mode & 1, fuse_ce = (a->round_mode >> 1) & 1, fuse_rec = (a->round_mode >> 2) & 1;
    float *xs = sc->xs, *ws = sc->ws, *err = sc->err;
    float *dp = sc->dp, *nx = sc->nx;
    int *lab = sc->lab;

    for (int i = 0; i < T; i++) {
        const size_t j = (size_t)n * a->ld + (size_t)((i + a->rot) % a->ld);
        xs[i] = a->x[j];
        ws[i] = a->w[j];
    }
    for (int s = 0; s < S; s++) lab[s] = label_of(s, a);
    const int s0 = a->init_st ? a->init_st[n] : -1;

    /* gain candidates: weighted scalar error over the merged table, the G smallest (src/cuda/tcq_viterbi.cu:155-180) */
    if (cand) {
        for (int j = 0; j < nsub; j++)
            for (int gi = 0; gi < Gf; gi++) {
                float e = 0.f;
                for (int t = j * sub; t < (j + 1) * sub; t++) {
                    const int hi = mix > 0 && ((t / mix) & 1);
                    const float be = hi ? branch_err(xs[t], a->gains_hi[gi], a->tab_hi, 0, 1, NL * U_hi, fuse_be)
                                        : branch_err(xs[t], a->gains[gi], a->tab, 0, 1, NL * U, fuse_be);
                    if (fuse_ce) e = fmaf(be, ws[t], e);
                    else { float p = be * ws[t]; e = e + p; }
                }
                sc->ce[j * Gf + gi] = e;
            }
        for (int j = 0; j < nsub; j++) {
            uint32_t used = 0;
            for (int c = 0; c < G; c++) {
                int bg = 0;
                float be = BIG;
                for (int gi = 0; gi < Gf; gi++)
                    if (!((used >> gi) & 1) && sc->ce[j * Gf + gi] < be) { be = sc->ce[j * Gf + gi]; bg = gi; }
                used |= 1u << bg;
                sc->gc[j * G + c] = (uint8_t)bg;
                a->gcand[((size_t)n * nsub + j) * G + c] = (uint8_t)bg;
            }
        }
    }

#define ERR(tt, g, lb, p) err[((((tt) - t0) * G + (g)) * NL + (lb)) * NP + (p)]
#define BP(tt, g, s) sc->bp[((size_t)(tt) * G + (g)) * S + (s)]
#define PB(pi, g, s) sc->pb[((size_t)(pi) * G + (g)) * S + (s)]
#define PL(gr, g, plane, s) sc->pl[(((size_t)(gr) * G + (g)) * 9 + (plane)) * S + (s)]
    for (int t0 = 0; t0 < T; t0 += sub) {
        if (t0 > 0 && G > 1) {  /* sub-block boundary: every slot continues from the best slot (src/cuda/tcq_viterbi.cu:185-201) */
            for (int s = 0; s < S; s++) {
                float b = dp[s];
                int bg = 0;
                for (int g = 1; g < G; g++)
                    if (dp[g * S + s] < b) { b = dp[g * S + s]; bg = g; }
                sc->gsel[(size_t)(t0 / sub) * S + s] = (uint8_t)bg;
                for (int g = 0; g < G; g++) dp[g * S + s] = b;
            }
        }
        /* branch errors of the sub-block (src/cuda/tcq_viterbi.cu:202-213) */
        for (int t = t0; t < t0 + sub; t++)
            for (int g = 0; g < G; g++) {
                const int gi = cand ? sc->gc[(t0 / sub) * G + g] : g;
                const int hi = mix > 0 && ((t / mix) & 1);
                for (int lb = 0; lb < NL; lb++)
                    for (int p = 0; p < NP; p++) {
                        float e;
                        if (MD) e = branch_err(xs[t], a->gains[gi], a->tab + lb * U, p, 2, U, fuse_be);
                        else if (hi) e = branch_err(xs[t], a->gains_hi[gi], a->tab_hi + lb * U_hi, 0, 1, U_hi, fuse_be);
                        else e = branch_err(xs[t], a->gains[gi], a->tab + lb * U, 0, 1, U, fuse_be);
                        ERR(t, g, lb, p) = e * ws[t];
                    }
            }
        for (int t = t0; t < t0 + sub;) {
            if (!MD) {
                if (t == 0) {
                    for (int g = 0; g < G; g++)
                        for (int s = 0; s < S; s++) {
                            const int ok = s0 < 0 || (s >> 1) == (s0 & (HALF - 1));
                            dp[g * S + s] = ok ? ERR(0, g, lab[s], 0) : BIG;
                        }
                } else {
                    for (int g = 0; g < G; g++)
                        for (int s = 0; s < S; s++) {
                            const float va = dp[g * S + (s >> 1)], vb = dp[g * S + HALF + (s >> 1)];
                            const int h = vb < va;
                            nx[g * S + s] = (h ? vb : va) + ERR(t, g, lab[s], 0);
                            BP(t, g, s) = (uint8_t)h;
                        }
                    float *tmp = dp; dp = nx; nx = tmp;
                }
                t += 1;
            } else if (PP) {
                /* pair (t, t + 1): intermediates per parity class, output takes the best class (tie -> p = 0) */
                float *in0 = sc->i0, *in1 = sc->i1;
                for (int g = 0; g < G; g++)
                    for (int s = 0; s < S; s++) {
                        if (t == 0) {
                            const int ok = s0 < 0 || (s >> 1) == (s0 & (HALF - 1));
                            in0[g * S + s] = ok ? ERR(0, g, lab[s], 0) : BIG;
                            in1[g * S + s] = ok ? ERR(0, g, lab[s], 1) : BIG;
                        } else {
                            const float va = dp[g * S + (s >> 1)], vb = dp[g * S + HALF + (s >> 1)];
                            const int h = vb < va;
                            const float mn = h ? vb : va;
                            BP(t, g, s) = (uint8_t)h;
                            in0[g * S + s] = mn + ERR(t, g, lab[s], 0);
                            in1[g * S + s] = mn + ERR(t, g, lab[s], 1);
                        }
                    }
                for (int g = 0; g < G; g++)
                    for (int s = 0; s < S; s++) {
                        float best = BIG;
                        int bh = 0, bpar = 0;
                        for (int p = 0; p < 2; p++) {
                            const float *arr = (p ? in1 : in0) + g * S;
                            const float va = arr[s >> 1], vb = arr[HALF + (s >> 1)];
                            const int h = vb < va;
                            const float v = (h ? vb : va) + ERR(t + 1, g, lab[s], p);
                            if (v < best) { best = v; bh = h; bpar = p; }
                        }
                        nx[g * S + s] = best;
                        BP(t + 1, g, s) = (uint8_t)bh;
                        PB(t / 2, g, s) = (uint8_t)bpar;
                    }
                { float *tmp = dp; dp = nx; nx = tmp; }
                t += 2;
            } else {
                /* G4: groups of 4; phase A (t % 4 == 0) -> classes c0 / c1, phase B (t % 4 == 2) -> dp */
                const int grp = t / 4;
                float *in0 = sc->i0, *in1 = sc->i1, *c0 = sc->c0, *c1 = sc->c1;
                if ((t & 3) == 0) {
                    for (int g = 0; g < G; g++)
                        for (int s = 0; s < S; s++) {
                            if (t == 0) {
                                const int ok = s0 < 0 || (s >> 1) == (s0 & (HALF - 1));
                                in0[g * S + s] = ok ? ERR(0, g, lab[s], 0) : BIG;
                                in1[g * S + s] = ok ? ERR(0, g, lab[s], 1) : BIG;
                            } else {
                                const float va = dp[g * S + (s >> 1)], vb = dp[g * S + HALF + (s >> 1)];
                                const int h = vb < va;
                                const float mn = h ? vb : va;
                                BP(t, g, s) = (uint8_t)h;
                                in0[g * S + s] = mn + ERR(t, g, lab[s], 0);
                                in1[g * S + s] = mn + ERR(t, g, lab[s], 1);
                            }
                        }
                    for (int g = 0; g < G; g++)
                        for (int s = 0; s < S; s++)
                            for (int c = 0; c < 2; c++) {
                                float best = BIG;
                                int bh = 0, bb = 0;
                                for (int b = EQ ? c : 0; b < (EQ ? c + 1 : 2); b++) {
                                    const float *arr = (b ? in1 : in0) + g * S;
                                    const float va = arr[s >> 1], vb = arr[HALF + (s >> 1)];
                                    const int h = vb < va;
                                    const float v = (h ? vb : va) + ERR(t + 1, g, lab[s], EQ ? c : (b ^ c));
                                    if (v < best) { best = v; bh = h; bb = b; }
                                }
                                (c ? c1 : c0)[g * S + s] = best;
                                PL(grp, g, c, s) = (uint8_t)bh;
                                PL(grp, g, 2 + c, s) = (uint8_t)bb;
                            }
                } else {
                    /* outputs start at 3.4e38 with class / predecessor / low-bit planes 0 (:388-390) */
                    for (int g = 0; g < G; g++)
                        for (int s = 0; s < S; s++) {
                            nx[g * S + s] = BIG;
                            PL(grp, g, 6, s) = 0;
                            PL(grp, g, 7, s) = 0;
                            PL(grp, g, 8, s) = 0;
                        }
                    /* per output state: candidates (c = 0, b = 0), (0, 1), (1, 0), (1, 1), strict < */
                    for (int c = 0; c < 2; c++) {
                        const float *cin = c ? c1 : c0;
                        for (int g = 0; g < G; g++)
                            for (int s = 0; s < S; s++) {
                                const float va = cin[g * S + (s >> 1)], vb = cin[g * S + HALF + (s >> 1)];
                                const int h = vb < va;
                                const float mn = h ? vb : va;
                                PL(grp, g, 4 + c, s) = (uint8_t)h;
                                in0[g * S + s] = mn + ERR(t, g, lab[s], 0);
                                in1[g * S + s] = mn + ERR(t, g, lab[s], 1);
                            }
                        for (int g = 0; g < G; g++)
                            for (int s = 0; s < S; s++) {
                                for (int b = EQ ? c : 0; b < (EQ ? c + 1 : 2); b++) {
                                    const float *arr = (b ? in1 : in0) + g * S;
                                    const float va = arr[s >> 1], vb = arr[HALF + (s >> 1)];
                                    const int h = vb < va;
                                    const float v = (h ? vb : va) + ERR(t + 1, g, lab[s], EQ ? c : (b ^ c));
                                    if (v < nx[g * S + s]) {
                                        nx[g * S + s] = v;
                                        PL(grp, g, 6, s) = (uint8_t)c;
                                        PL(grp, g, 7, s) = (uint8_t)h;
                                        PL(grp, g, 8, s) = (uint8_t)b;
                                    }
                                }
                            }
                    }
                    { float *tmp = dp; dp = nx; nx = tmp; }
                }
                t += 2;
            }
        }
    }

    /* argmin over (g, s): smallest value, then smallest flat index; tail-biting keeps only s == s0 (:561-579) */
    float bv = BIG;
    int bi = 0x7fffffff;
    const int s_end = a->tail ? s0 : -1;
    for (int g = 0; g < G; g++)
        for (int s = 0; s < S; s++) {
            const int idx = g * S + s;
            const float v = (s_end < 0 || s == s_end) ? dp[idx] : BIG;
            if (v < bv || (v == bv && idx < bi)) { bv = v; bi = idx; }
        }
    a->best[n] = bi;
    if (a->end_st) a->end_st[n] = bi % S;

    /* traceback (:580-661), serial */
    int st = bi % S, g = bi / S, pcur = 0, cstar = 0;
    for (int t = T - 1; t >= 0; t--) {
        sc->st[t] = (uint16_t)st;
        sc->sg[t] = (uint8_t)g;
        if (PP) {
            if (t & 1) pcur = PB(t >> 1, g, st);
            sc->par[t] = (uint8_t)pcur;
        }
        if (a->mid_st && t == a->mid_t - 1) { a->mid_st[n] = st; return; }
        if (G4 && (t & 3)) {
            const int grp = t >> 2;
            int hh;
            if ((t & 3) == 3) {
                cstar = PL(grp, g, 6, st);
                hh = PL(grp, g, 7, st);
                if (EQ) {
                    sc->par[t] = sc->par[t - 1] = sc->par[t - 2] = sc->par[t - 3] = (uint8_t)cstar;
                } else {
                    const int bb = PL(grp, g, 8, st);
                    sc->par[t] = (uint8_t)(bb ^ cstar);
                    sc->par[t - 1] = (uint8_t)bb;
                }
            } else if ((t & 3) == 2) {
                hh = PL(grp, g, 4 + cstar, st);
            } else {
                hh = PL(grp, g, 0 + cstar, st);
                if (!EQ) {
                    const int bb = PL(grp, g, 2 + cstar, st);
                    sc->par[t] = (uint8_t)(bb ^ cstar);
                    sc->par[t - 1] = (uint8_t)bb;
                }
            }
            st = hh * HALF + (st >> 1);
        } else if (t > 0) {
            st = BP(t, g, st) * HALF + (st >> 1);
            if (G > 1 && (t % sub) == 0) g = sc->gsel[(size_t)(t / sub) * S + st];
        }
    }

    /* reconstruction and codes (:662-682) */
    float *rn = a->rec + (size_t)n * a->ld;
    for (int t = 0; t < T; t++) {
        const int stt = sc->st[t], gg = sc->sg[t];
        const int lb = label_of(stt, a);
        const int hi = mix > 0 && ((t / mix) & 1);
        const int Ut = hi ? U_hi : U;
        const int gi = cand ? (int)sc->gc[(t / sub) * G + gg] : gg;
        const float gt = hi ? a->gains_hi[gi] : a->gains[gi];
        const float *tt = (hi ? a->tab_hi : a->tab) + lb * Ut;
        const float xt = xs[t];
        float bestd = BIG, val = 0.f;
        int bu = 0;
        for (int u = MD ? sc->par[t] : 0; u < Ut; u += MD ? 2 : 1) {
            const float v = gt * tt[u];
            const float d = fuse_rec ? fmaf(-gt, tt[u], xt) : xt - v;
            const float dd = d * d;
            if (dd < bestd) { bestd = dd; val = v; bu = u; }
        }
        const int tp = (t + a->rot) % a->ld;
        rn[tp] = val;
        if (a->code) a->code[(size_t)n * a->ld + tp] = (gi << 16) | (lb * Ut + bu);
    }
#undef ERR
#undef BP
#undef PB
#undef PL
}

/* Same argument list as the reference C-ABI `tcq_viterbi` (src/cuda/tcq_viterbi.cu:743-746); the scratch pointers
 * bp / gsel / pbits are ignored (the oracle keeps its own), all other pointers are HOST memory.  Two trailing
 * arguments: round_mode (see the header) and n_threads (0 = all).  Returns 0, -1 (unsupported parameters, same table as
 * the reference) or -2 (out of host memory). */
int ora_tcq_viterbi(const float *x, const float *w, const float *tab, const float *gains, float *rec, uint32_t *bp,
                    uint8_t *gsel, const int *init_st, int *end_st, const float *tab_hi, const float *gains_hi,
                    uint8_t *gcand, int *best, int *code, int *mid_st, int mid_t, int tail, int N, int T, int S, int U,
                    int G, int Gfull, int m, int sub, int U_hi, int mix, int m2, int m3, int m4, int nl, int ld, int rot,
                    uint32_t *pbits, int pp, void *stream, int round_mode, int n_threads)
{
    (void)bp; (void)gsel; (void)pbits; (void)stream;
    ora_args a = {x, w, tab, gains, tab_hi ? tab_hi : tab, gains_hi ? gains_hi : gains, rec, init_st, end_st, gcand,
                  best, code, mid_st, mid_t, tail, N, T, S, U, G, Gfull, m, sub, U_hi, mix, m2, m3, m4, nl, ld, rot, pp,
                  round_mode};
    if (validate(&a) != 0) return -1;
    int rc = 0;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel reduction(min : rc)
#endif
    {
        ora_scratch sc;
        if (alloc_scratch(&sc, &a) != 0) {
            rc = -2;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
            for (int n = 0; n < N; n++) tile(&a, n, &sc);
        }
        free_scratch(&sc);
    }
    return rc;
}

int ora_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* DP-profile sub-block quantization through a 1-D table (src/cuda/tcq_viterbi.cu:768-804, lut_subs_kernel, as its nvcc
 * build computes it): bucket b = rint(fma(x, inv_step, half_b)) converted to int like cvt.rzi.s32 (NaN -> 0, saturating)
 * and clamped to [0, nb - 1]; err[c] = fma(d * e, e, err[c]) with e = x - lut[b][c] over j = 0..15 in order; best = the
 * first strict minimum scanned from c = 0; out[j] = lut[b_j][best]. */
static int ora_cvt_s32(float v)
{
    if (v != v) return 0;
    if (v >= 2147483648.0f) return INT_MAX;
    if (v <= -2147483648.0f) return INT_MIN;
    return (int)v;
}

void ora_lut_subs(const float* xs, const float* dh, const float* lut, float* out, int S, float inv_step, float half_b,
                  int nb)
{
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
    for (long long i = 0; i < S; i++) {
        float err[64];
        int bj[16];
        for (int c = 0; c < 64; c++) err[c] = 0.f;
        for (int j = 0; j < 16; j++) {
            const float x = xs[i * 16 + j], d = dh[i * 16 + j];
            int b = ora_cvt_s32(rintf(fmaf(x, inv_step, half_b)));
            b = b < 0 ? 0 : (b > nb - 1 ? nb - 1 : b);
            bj[j] = b;
            for (int c = 0; c < 64; c++) {
                const float e = x - lut[(long long)b * 64 + c];
                const float t = d * e;
                err[c] = fmaf(t, e, err[c]);
            }
        }
        int best = 0;
        float be = err[0];
        for (int c = 1; c < 64; c++)
            if (err[c] < be) {
                be = err[c];
                best = c;
            }
        for (int j = 0; j < 16; j++) out[i * 16 + j] = lut[(long long)bj[j] * 64 + best];
    }
}
