// Host side of the Viterbi: parameter validation, survivor-layout sizing, kernel dispatch, and the C ABI
// (include/ltq_b200.h): the reference-compatible `tcq_viterbi` and the one-call tail-biting schedule `ltq_viterbi_tb`.
#include <stdlib.h>
#include <algorithm>
#include "ltq_b200.h"
#include "vit_launch.cuh"

namespace ltqb {

// survivor words per 4-step group and for a trailing half group (T = 2 mod 4), by parity mode
static int words_per_group(int pp) { return pp == 0 ? 2 : (pp == 1 ? 5 : 9); }
static int words_half_group(int pp) { return pp == 0 ? 1 : 3; }

long long sv_words(int T, int pp)  // words per (tile, gain slot), one lane row of 32 per word
{
    return ((long long)(T / 4) * words_per_group(pp) + ((T % 4) ? words_half_group(pp) : 0)) * 32;
}
int gsel_planes(int G) { return G <= 2 ? 1 : (G <= 4 ? 2 : 4); }

// The reference's validation table (src/cuda/tcq_viterbi.cu:748-751 and the dispatch limits :720-763) plus this
// implementation's G values (1, 2, 3, 4, 8: the reference's dispatch).  S = 256 (4 subsets, plain mode, by the
// reference's table) runs the 256-state kernel.  The reference's TCQ_BLOCK switch only picks its thread-block shape.
static bool valid(int N, int T, int S, int U, int G, int Gfull, bool cand, int sub, int U_hi, int mix, int nl, int ld,
                  int pp)
{
    (void)N;
    if (sub <= 0 || T <= 0) return false;
    if (G > MAXG || Gfull > MAXG || (!cand && Gfull != G) || U > MAXU || U_hi > MAXU || T % sub != 0 || (sub & 1) ||
        T / sub > MAXSUBS || T > MAXT || sub > 32 || sub * G * nl * (pp ? 2 : 1) > 4096 ||
        (pp && (S != 1024 || mix > 0 || (T & 1))) || (pp >= 2 && ((T & 3) || (sub & 3))) || pp > 3 || pp < 0 ||
        (nl != 4 && nl != 8 && nl != 16 && nl != 32) || ld < T || (S != 1024 && nl != 4) || nl * U > 4 * MAXU ||
        nl * U_hi > 4 * MAXU)
        return false;
    if (!(G == 1 || G == 2 || G == 3 || G == 4 || G == 8)) return false;
    if ((S != 1024 && S != 256) || nl > 32 || U < 1 || U_hi < 1) return false;
    if (cand && G > Gfull) return false;
    return true;
}

static int dispatch(const VitParams& p, int pp, cudaStream_t st)
{
    const int NP = pp ? 2 : 1;
    const int smem = fwd_smem(p.T, p.G, p.Gfull, p.sub, p.nl, NP, p.U, p.U_hi).total;
    if (p.sub % 4) return launch_rt_sub2(p, pp, smem, st);
    if (p.m == 359) {
        if (p.nl == 4) return launch_ct_m359(p, pp, smem, st);
        if (p.nl == 8) {
            if (p.m2 == 241) return launch_ct_m359_241(p, pp, smem, st);
            if (p.m2 == 462) return launch_ct_m359_462(p, pp, smem, st);
            if (p.m2 == 146) return launch_ct_m359_146(p, pp, smem, st);
        }
        if (p.nl == 16) {
            if (p.m2 == 58 && p.m3 == 299) return launch_ct_m359_58_299(p, pp, smem, st);
            if (p.m2 == 211 && p.m3 == 397) return launch_ct_m359_211_397(p, pp, smem, st);
            if (p.m2 == 40 && p.m3 == 475) return launch_ct_m359_40_475(p, pp, smem, st);
        }
    }
    return launch_rt(p, pp, smem, st);
}

// one Viterbi pass over N tiles (the reference kernel's contract)
static int run_pass(VitParams p, int pp, int S, cudaStream_t st)
{
    if (S == 256) {
        if (p.N <= 0) return (int)cudaErrorInvalidConfiguration;
        return run_pass_s256(p, st);
    }
    p.W4 = words_per_group(pp);
    p.NB = gsel_planes(p.G);
    p.nsl = p.T / p.sub;
    if (p.N <= 0) return (int)cudaErrorInvalidConfiguration;  // the reference launches an empty grid: error 9
    const int rc = dispatch(p, pp, st);
    if (rc != 0) return rc;
    return launch_tb(p, pp, st);
}

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace ltqb

using namespace ltqb;

extern "C" const char* ltq_b200_version(void) { return "ltq_b200 0.1 sm_100a"; }

extern "C" int tcq_viterbi(const float* x, const float* w, const float* tab, const float* gains, float* rec, uint32_t* bp,
                           uint8_t* gsel, const int* init_st, int* end_st, const float* tab_hi, const float* gains_hi,
                           uint8_t* gcand, int* best, int* code, int* mid_st, int mid_t, int tail, int N, int T, int S,
                           int U, int G, int Gfull, int m, int sub, int U_hi, int mix, int m2, int m3, int m4, int nl,
                           int ld, int rot, uint32_t* pbits, int pp, void* stream)
{
    if (!valid(N, T, S, U, G, Gfull, gcand != nullptr, sub, U_hi, mix, nl, ld, pp)) return -1;
    // caller scratch, as the reference wrapper allocates it: bp [N, T, G, 32] words; pbits D2 [N, T/2, G, 32],
    // D4 [N, T/4, G, 9, 32]; gsel [N, T/sub, 1024] bytes
    const long long capA = (long long)T * 32;
    const long long capB = pp == 1 ? (long long)(T / 2) * 32 : (pp >= 2 ? (long long)(T / 4) * 9 * 32 : 0);
    if (sv_words(T, pp) > capA + capB) return -1;
    VitParams p{};
    p.x = x; p.w = w; p.tab = tab; p.gains = gains; p.tab_hi = tab_hi ? tab_hi : tab; p.gains_hi = gains_hi ? gains_hi : gains;
    p.rec = rec; p.code = code; p.init_st = init_st; p.end_st = end_st; p.mid_st = mid_st; p.best = best; p.gcand = gcand;
    p.svA = bp; p.svB = pbits ? pbits : bp; p.capA = capA; p.capB = capB;
    p.gsw = reinterpret_cast<uint32_t*>(gsel);
    p.mid_t = mid_t; p.tail = tail; p.N = N; p.T = T; p.U = U; p.G = G; p.Gfull = Gfull; p.sub = sub; p.U_hi = U_hi;
    p.mix = mix; p.ld = ld; p.ldw = ld; p.rot = rot; p.m = m; p.m2 = m2; p.m3 = m3; p.m4 = m4; p.nl = nl;
    p.cand = gcand != nullptr;
    // gsel bytes per tile in the reference layout: (T / sub) * 1024; ours: (T / sub) * 512 — fits
    const int rc = run_pass(p, pp, S, (cudaStream_t)stream);
    if (rc != 0) return rc;
    return (int)cudaGetLastError();
}

extern "C" size_t ltq_viterbi_tb_workspace_bytes(int N, int T, int Gfull, int n_cand, int sub, int pp, int tb_window,
                                                 int tb_cand1)
{
    if (N <= 0 || T <= 0 || sub <= 0) return 0;
    const int G = (n_cand > 0 && n_cand < Gfull) ? n_cand : Gfull;
    const int G1 = tb_cand1 > 0 ? ((tb_cand1 < Gfull) ? tb_cand1 : Gfull) : G;
    const int Gm = std::max(G, G1);
    (void)tb_window;
    size_t b = 0;
    b += al256((size_t)N * Gm * (size_t)sv_words(T, pp) * 4);           // survivors
    b += al256((size_t)N * (T / sub) * 512);                             // gain-merge winners
    b += al256((size_t)N * (T / sub) * Gm);                              // gain candidates
    b += al256((size_t)N * 4) * 2;                                       // middle state, best end
    return b;
}

extern "C" int ltq_viterbi_tb(const float* x, const float* w, int w_stride, const float* tab, const float* gains,
                              const float* tab_hi, const float* gains_hi, float* rec, int* code, int N, int T, int nu,
                              int K, int m, const int* m_extra, int n_extra, int Gfull, int n_cand, int sub, int U_hi,
                              int mix, int pp, int tb_passes, int tb_cand1, int tb_window, void* workspace,
                              size_t workspace_bytes, void* stream)
{
    if ((nu != 10 && nu != 8) || K < 1 || K > 8 || n_extra < 0 || n_extra > 3 || tb_passes < 2 || tb_window < 0 ||
        (n_extra > 0 && !m_extra))
        return -1;
    const int S = 1 << nu, U = 1 << (K - 1), nl = 4 << n_extra, h = T / 2;
    const int G = (n_cand > 0 && n_cand < Gfull) ? n_cand : Gfull;
    const int G1 = tb_cand1 > 0 ? ((tb_cand1 < Gfull) ? tb_cand1 : Gfull) : G;
    const int T1 = tb_window ? 2 * tb_window : T;
    if (tb_window && tb_window > h) return -1;
    if (!tab_hi) { tab_hi = tab; U_hi = U; mix = 0; }
    if (!gains_hi) gains_hi = gains;
    if (!valid(N, T, S, U, G, Gfull, G < Gfull, sub, U_hi, mix, nl, T, pp)) return -1;
    if (!valid(N, T1, S, U, G1, Gfull, G1 < Gfull, sub, U_hi, mix, nl, T, pp)) return -1;
    if (N <= 0) return (int)cudaErrorInvalidConfiguration;
    const size_t need = ltq_viterbi_tb_workspace_bytes(N, T, Gfull, n_cand, sub, pp, tb_window, tb_cand1);
    if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255)) return -1;
    const int Gm = std::max(G, G1);
    char* ws = static_cast<char*>(workspace);
    uint32_t* sv = reinterpret_cast<uint32_t*>(ws);
    ws += al256((size_t)N * Gm * (size_t)sv_words(T, pp) * 4);
    uint32_t* gsw = reinterpret_cast<uint32_t*>(ws);
    ws += al256((size_t)N * (T / sub) * 512);
    uint8_t* gc = reinterpret_cast<uint8_t*>(ws);
    ws += al256((size_t)N * (T / sub) * Gm);
    int* mid = reinterpret_cast<int*>(ws);
    ws += al256((size_t)N * 4);
    int* best = reinterpret_cast<int*>(ws);
    cudaStream_t st = (cudaStream_t)stream;

    VitParams p{};
    p.x = x; p.w = w; p.tab = tab; p.gains = gains; p.tab_hi = tab_hi; p.gains_hi = gains_hi;
    p.rec = rec; p.best = best; p.gsw = gsw;
    p.N = N; p.U = U; p.Gfull = Gfull; p.sub = sub; p.U_hi = U_hi; p.mix = mix; p.ld = T; p.ldw = w_stride;
    p.m = m; p.m2 = n_extra > 0 ? m_extra[0] : 0; p.m3 = n_extra > 1 ? m_extra[1] : 0;
    p.m4 = n_extra > 2 ? m_extra[2] : 0; p.nl = nl;
    p.svA = sv; p.svB = sv; p.capA = sv_words(T, pp); p.capB = 0;

    // pass 1: free start, the path state before sample h (src/tcq_proto.py:594-599)
    VitParams p1 = p;
    p1.G = G1; p1.cand = G1 < Gfull; p1.gcand = p1.cand ? gc : nullptr;
    p1.T = T1; p1.rot = tb_window ? h - tb_window : 0; p1.mid_t = tb_window ? tb_window : h; p1.mid_st = mid;
    p1.init_st = nullptr; p1.tail = 0; p1.code = nullptr;
    int rc = run_pass(p1, pp, S, st);
    if (rc != 0) return rc;
    // further passes on the tile rotated by h, start = end = the middle state (src/tcq_proto.py:600-608)
    int shift = 0;
    for (int pass = 1; pass < tb_passes; pass++) {
        shift = (shift + h) % T;
        VitParams q = p;
        q.G = G; q.cand = G < Gfull; q.gcand = q.cand ? gc : nullptr;
        q.T = T; q.rot = shift; q.init_st = mid; q.tail = 1;
        if (pass + 1 < tb_passes) { q.mid_st = mid; q.mid_t = h; q.code = nullptr; }
        else { q.mid_st = nullptr; q.mid_t = 0; q.code = code; }
        rc = run_pass(q, pp, S, st);
        if (rc != 0) return rc;
    }
    return (int)cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------
// fused LDLQ block (ldlq_block_kernel): workspace layout per tile group and the C ABI
// ------------------------------------------------------------------------------------------------
namespace ltqb {

struct LdlqWs {
    size_t sv, gsw, gc, mid, best, x, rec, code, wsub, dwr, total;
};

static LdlqWs ldlq_ws(int N, int Gm, int sub, int pp)
{
    LdlqWs L{};
    size_t o = 0;
    L.sv = o; o += al256((size_t)N * Gm * (size_t)sv_words(256, pp) * 4);
    L.gsw = o; o += al256((size_t)N * (256 / sub) * 512);
    L.gc = o; o += al256((size_t)N * (256 / sub) * Gm);
    L.mid = o; o += al256((size_t)N * 4);
    L.best = o; o += al256((size_t)N * 4);
    L.x = o; o += al256((size_t)N * 256 * 4);
    L.rec = o; o += al256((size_t)N * 256 * 4);
    L.code = o; o += al256((size_t)N * 256 * 4);
    L.wsub = o; o += al256((size_t)N * 16 * 256 * 4);
    L.dwr = o; o += al256(16 * 256 * 4);
    L.total = o;
    return L;
}

static int ldlq_dispatch(const LdlqParams& q, int pp, int smem, int grid, cudaStream_t st)
{
    const VitParams& p = q.p2;
    if (p.m == 359) {
        if (p.nl == 4) return ldlq_ct_m359(q, pp, smem, grid, st);
        if (p.nl == 8) {
            if (p.m2 == 241) return ldlq_ct_m359_241(q, pp, smem, grid, st);
            if (p.m2 == 462) return ldlq_ct_m359_462(q, pp, smem, grid, st);
            if (p.m2 == 146) return ldlq_ct_m359_146(q, pp, smem, grid, st);
        }
        if (p.nl == 16) {
            if (p.m2 == 58 && p.m3 == 299) return ldlq_ct_m359_58_299(q, pp, smem, grid, st);
            if (p.m2 == 211 && p.m3 == 397) return ldlq_ct_m359_211_397(q, pp, smem, grid, st);
            if (p.m2 == 40 && p.m3 == 475) return ldlq_ct_m359_40_475(q, pp, smem, grid, st);
        }
    }
    return ldlq_rt(q, pp, smem, grid, st);
}

}  // namespace ltqb

extern "C" size_t ltq_ldlq_block_workspace_bytes(int M, int Gfull, int n_cand, int sub, int pp, int tb_window)
{
    (void)tb_window;
    if (M <= 0 || M % 16 || sub <= 0 || Gfull <= 0) return 0;
    const int G = (n_cand > 0 && n_cand < Gfull) ? n_cand : Gfull;
    return ldlq_ws(M / 16, G, sub, pp).total;
}

extern "C" int ltq_ldlq_block(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* dw,
                              const float* U, long long ldU, const float* Uinv, long long ldUi, float* G, long long ldG,
                              int16_t* idx, uint8_t* gi, long long ldP, int M, const float* tab, const float* gains,
                              int K, int m, const int* m_extra, int n_extra, int Gfull, int n_cand, int sub, int pp,
                              int tb_window, void* workspace, size_t workspace_bytes, void* stream)
{
    constexpr int T = 256, h = T / 2;
    if (M < 0 || M % 16 || K < 1 || K > 8 || n_extra < 0 || n_extra > 2 || (n_extra > 0 && !m_extra) ||
        tb_window < 0 || tb_window > h || !w_blk || !d_rb || !dw || !U || !Uinv || !G || !idx || !gi || !tab ||
        !gains || ld_w < T || ld_d < 1 || ldU < T || ldUi < T || ldG < T || ldP < T || ((uintptr_t)w_blk & 15) ||
        (ld_w % 4) || sub % 4)
        return -1;
    const int U_ = 1 << (K - 1), nl = 4 << n_extra;
    const int Gr = (n_cand > 0 && n_cand < Gfull) ? n_cand : Gfull;
    const int T1 = tb_window ? 2 * tb_window : T;
    if (Gr > 4) return -1;  // one CTA of at most 4 warps per tile group
    if (!valid(1, T, 1024, U_, Gr, Gfull, Gr < Gfull, sub, U_, 0, nl, T, pp)) return -1;
    if (!valid(1, T1, 1024, U_, Gr, Gfull, Gr < Gfull, sub, U_, 0, nl, T, pp)) return -1;
    if (M == 0) return 0;
    const int N = M / 16;
    const LdlqWs L = ldlq_ws(N, Gr, sub, pp);
    if (!workspace || workspace_bytes < L.total || ((uintptr_t)workspace & 255)) return -1;
    char* ws = static_cast<char*>(workspace);
    cudaStream_t st = (cudaStream_t)stream;

    VitParams p{};
    p.tab = tab; p.gains = gains; p.tab_hi = tab; p.gains_hi = gains;
    p.best = reinterpret_cast<int*>(ws + L.best);
    p.gsw = reinterpret_cast<uint32_t*>(ws + L.gsw);
    p.N = N; p.T = T; p.U = U_; p.Gfull = Gfull; p.sub = sub; p.U_hi = U_; p.mix = 0; p.ld = T; p.ldw = 0;
    p.m = m; p.m2 = n_extra > 0 ? m_extra[0] : 0; p.m3 = n_extra > 1 ? m_extra[1] : 0; p.m4 = 0; p.nl = nl;
    p.svA = reinterpret_cast<uint32_t*>(ws + L.sv); p.svB = p.svA; p.capA = sv_words(T, pp); p.capB = 0;
    p.W4 = words_per_group(pp); p.NB = gsel_planes(Gr);
    p.nsl = T / sub;  // both passes index gsw / gcand rows with the full tile's stride
    p.G = Gr; p.cand = Gr < Gfull; p.gcand = p.cand ? reinterpret_cast<uint8_t*>(ws + L.gc) : nullptr;
    p.x = reinterpret_cast<float*>(ws + L.x);
    p.rec = reinterpret_cast<float*>(ws + L.rec);
    int* mid = reinterpret_cast<int*>(ws + L.mid);

    LdlqParams q{};
    q.p1 = p;  // free start; the window [h - W, h + W), or the whole tile when W = 0
    q.p1.T = T1; q.p1.rot = tb_window ? h - tb_window : 0; q.p1.mid_t = tb_window ? tb_window : h; q.p1.mid_st = mid;
    q.p1.init_st = nullptr; q.p1.tail = 0; q.p1.code = nullptr;
    q.p2 = p;  // rotated by h, start = end = the middle state
    q.p2.rot = h; q.p2.init_st = mid; q.p2.tail = 1; q.p2.mid_st = nullptr; q.p2.mid_t = 0;
    q.p2.code = reinterpret_cast<int*>(ws + L.code);
    q.wblk = w_blk; q.ldw = ld_w; q.wsub = reinterpret_cast<float*>(ws + L.wsub);
    q.d_rb = d_rb; q.ldd = ld_d; q.dwrows = reinterpret_cast<float*>(ws + L.dwr);
    q.U = U; q.ldU = ldU; q.Ui = Uinv; q.ldUi = ldUi; q.G = G; q.ldG = ldG; q.idx = idx; q.gi = gi; q.ldP = ldP;
    q.xbuf = reinterpret_cast<float*>(ws + L.x); q.recbuf = reinterpret_cast<float*>(ws + L.rec);
    q.codebuf = reinterpret_cast<int*>(ws + L.code);
    const int smem = ldlq_smem(q.p1, q.p2, pp ? 2 : 1, &q.fb_off);

    ldlq_dwrows_kernel<<<16, 256, 0, st>>>(dw, const_cast<float*>(q.dwrows));
    const int rc = ldlq_dispatch(q, pp, smem, N, st);
    if (rc != 0) return rc;
    return (int)cudaGetLastError();
}
