/*
 * ltq_b200 — C ABI of the B200 (sm_100a) LTQ / TCQ quantizer kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed as void*), runs
 * asynchronously on that stream and returns an int status:
 *     0   success (launch errors of the queued kernels are reported as positive cudaError_t codes),
 *    -1   unsupported or invalid parameters (the same validation table as the reference, plus the limits named below),
 *    >0   a cudaError_t from the launch.
 * No entry point allocates device memory: outputs and scratch are passed in by the caller.  All entry points are
 * re-entrant; calls on different streams may run concurrently.  One exception, ltq_viterbi_tb_noalloc (end of this
 * file): its scratch is one array inside the library shared by all its calls on a device, so calls of it that overlap
 * on the GPU must be serialised by the caller, and it returns -2 for a problem larger than that array.
 *
 * Reference: lumen-inference/ltq-research (paths below are relative to its root).
 */
#ifndef LTQ_B200_H
#define LTQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version string, e.g. "ltq_b200 0.1 sm_100a". */
const char* ltq_b200_version(void);

/*
 * Drop-in replacement for the reference C-ABI `tcq_viterbi` (src/cuda/tcq_viterbi.cu:743-746), bound by ctypes in
 * src/tcq_proto.py:529 as 15 pointers, 18 ints, pointer, int, pointer.  Same argument list, same meaning, same
 * validation (returns -1 where the reference returns -1, src/cuda/tcq_viterbi.cu:748-751), same outputs:
 *   rec [N, ld], code [N, ld] ((gain index << 16) | (label * U + u), optional), gcand [N, T/sub, G] (when G < Gfull),
 *   best [N] (g * S + s), end_st [N] (optional), mid_st [N] (first tail-biting pass, optional).
 * bp [N, T, G, S/32] u32, gsel [N, T/sub, S] u8 and pbits (pp = 1: [N, T/2, G, S/32]; pp >= 2: [N, T/4, G, 9, S/32])
 * are caller-allocated scratch of the sizes the reference's Python wrapper allocates (src/tcq_proto.py:623-637);
 * this implementation stores its own survivor layout in them.
 * S = 1024 (nu = 10) or 256 (nu = 8; 4 subsets and plain mode, the reference's table); nl = 32 (m2, m3, m4 all used)
 * runs the run-time-mask kernel.  Limit beyond the reference: with pp = 1 and T < 10 the caller's scratch is too small
 * for the survivor layout (returns -1).
 */
int tcq_viterbi(const float* x, const float* w, const float* tab, const float* gains, float* rec, uint32_t* bp,
                uint8_t* gsel, const int* init_st, int* end_st, const float* tab_hi, const float* gains_hi,
                uint8_t* gcand, int* best, int* code, int* mid_st, int mid_t, int tail, int N, int T, int S, int U,
                int G, int Gfull, int m, int sub, int U_hi, int mix, int m2, int m3, int m4, int nl, int ld, int rot,
                uint32_t* pbits, int pp, void* stream);

/*
 * The whole tail-biting schedule of `viterbi_ub_cuda(..., tail_biting=True)` (src/tcq_proto.py:584-609) in one
 * call: pass 1 (free start; over the window [T/2 - tb_window, T/2 + tb_window) when tb_window > 0, over tb_cand1 gain
 * candidates when tb_cand1 > 0) finds the path state before sample T/2; tb_passes - 1 further passes run on the tile
 * rotated by T/2 with that state as start and end.  The last pass writes rec [N, T] and code [N, T] (optional) at the
 * original positions.
 *   x [N, T] fp32; w: per-position weights, row stride w_stride (0 = one row [T] shared by all tiles);
 *   tab [nl * 2^(K-1)], gains [Gfull]; tab_hi / gains_hi / mix: half-integer mode (NULL / 0 when unused);
 *   nu: 10 (1024 states) or 8 (256 states, no extra masks, pp = 0);
 *   m: primary label mask, m_extra[n_extra]: extra label masks (n_extra <= 3, nl = 4 << n_extra);
 *   n_cand: Viterbi over n_cand gain candidates per sub-block (0 = all Gfull); pp: 0 none, 1 D2, 2 D4, 3 EQ.
 * workspace: device memory of at least ltq_viterbi_tb_workspace_bytes(...) bytes, 256-byte aligned.
 */
size_t ltq_viterbi_tb_workspace_bytes(int N, int T, int Gfull, int n_cand, int sub, int pp, int tb_window,
                                      int tb_cand1);
int ltq_viterbi_tb(const float* x, const float* w, int w_stride, const float* tab, const float* gains,
                   const float* tab_hi, const float* gains_hi, float* rec, int* code, int N, int T, int nu, int K,
                   int m, const int* m_extra, int n_extra, int Gfull, int n_cand, int sub, int U_hi, int mix, int pp,
                   int tb_passes, int tb_cand1, int tb_window, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * Matrix-level kernels of the quantizer path (src/liqk_v2.py).  No single C entry in the reference: each replaces a
 * few torch operations of the function cited.  Device pointers, row strides in elements, asynchronous on `stream`.
 *
 * ltq_fwht256: normalized block FWHT-256 along rows, out[r, :] = H256(x[r, :]) / 16 per 256-column block, with
 *   x = in (mode 0), in / scale[col] (mode 1, as W / suh), in * scale[col] (mode 2, as H * suh); `in` is fp32 or
 *   (in_bf16 = 1) bf16.  Replaces fwht_inplace (src/iqk_format.py:153-170) in compute_optimal_suh
 *   (src/liqk_v2.py:436-440) and _fwht_rows (:1024-1026); same butterfly order, bit-identical results.
 * ltq_scale_fit: per-(row, 256-block) scale of the row-scale formats (src/liqk_v2.py:938-946): fp16 d_row (bits in
 *   d_row_h, value in d_row), 5-bit exponent e and d_rb = d_row * 2^(e_step * e).  Any output may be NULL.
 * ltq_ldlq_gather: Viterbi input tiles of one 16-column sub-block, x[n][16 r + c] = w[16 n + r][c] * inv_d[16 n + r]
 *   (src/liqk_v2.py:914, :963).
 * ltq_ldlq_feedback: after the sub-block at columns [s0, s0 + 16) of a 256-column block (src/liqk_v2.py:964-971):
 *   G[:, s0:s0+16] = rec (tile layout [M/16][256]); with code, idx = label * U + u and gi = gain index;
 *   w[:, s0+16:256] -= ((w[:, s0:s0+16] - d_rb * rec) @ Uinv[s0:s0+16, s0:s0+16]) @ U[s0:s0+16, s0+16:256].
 */
int ltq_fwht256(const void* in, int in_bf16, long long ld_in, float* out, long long ld_out, const float* scale, int mode,
                int rows, int cols, void* stream);
int ltq_scale_fit(const float* W, long long ld, int M, int K, float scale, float e_step, int e_bits, uint16_t* d_row_h,
                  float* d_row, int8_t* e, float* d_rb, void* stream);
int ltq_ldlq_gather(const float* w, long long ld, const float* inv_d, int M, float* x, void* stream);
int ltq_ldlq_feedback(float* w, long long ld, int M, int s0, const float* d_rb, const float* rec, const int* code,
                      const float* U, long long ldU, const float* Uinv, long long ldUi, float* G, long long ldG,
                      int16_t* idx, uint8_t* gi, long long ldP, void* stream);

/*
 * One 256-column block of the row-scale TCQ LDLQ quantizer in one launch (src/liqk_v2.py:956-971 with quant_sub
 * :913-936): for each of the block's 16 sub-blocks, the gather, the two-pass tail-biting Viterbi of
 * viterbi_ub_cuda(..., tail_biting=True, tb_window=W) (src/tcq_proto.py:584-609) on the M/16 tiles, and the intra-block
 * feedback — the same results, bit for bit, as ltq_ldlq_gather + ltq_viterbi_tb + ltq_ldlq_feedback per sub-block.
 *   w_blk [M, 256] (row stride ld_w): the block of the working matrix at the block's start (read only);
 *   d_rb: the rows' block scale at d_rb[row * ld_d] (clamped to 1e-8 inside); dw [256]: diag_w of the block's columns;
 *   U / Uinv: U[c0:c0+256, c0:c0+256] and its inverse, row strides ldU / ldUi;
 *   out: G [M, 256] (stride ldG) reconstruction levels, idx (label * U + u) and gi (gain index) [M, 256] (stride ldP);
 *   the table, gains, masks, K, Gfull, n_cand, sub and pp of the format as for ltq_viterbi_tb (nu = 10, T = 256).
 * workspace: at least ltq_ldlq_block_workspace_bytes(M, ...) bytes, 256-byte aligned.  The inter-block update after the
 * block (src/liqk_v2.py:972-979) stays with the caller (a GEMM).  Limits: M % 16 == 0, sub % 4 == 0, at most 4 gain
 * slots in the search (n_cand <= 4 or Gfull <= 4).
 */
size_t ltq_ldlq_block_workspace_bytes(int M, int Gfull, int n_cand, int sub, int pp, int tb_window);
/*
 * The inter-block update after a block (src/liqk_v2.py:972-979),
 *     W_work[:, c1:] -= ((w_blk - d_rb * G) @ Uinv_blk) @ U[c0:c1, c1:],
 * as one fp32-accurate tensor-core GEMM acat @ bcat_b of bf16 operands (the three-way split x = x0 + x1 + x2,
 * x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1), and the six products a0 b0 + a0 b1 + a1 b0 + a0 b2 + a1 b1 + a2 b0):
 * ltq_ldlq_bcat, once per matrix: for every block b < K/256 - 1 (c0 = 256 b, c1 = c0 + 256) the [1536, K - c1] matrix
 *   [u0; u1; u0; u2; u1; u0] of U[c0:c1, c1:K], contiguous, at element offset 1536 * sum_{b' < b} (K - 256 (b' + 1));
 *   ltq_ldlq_bcat_elems(K) elements in all (bf16 bits).  U 16-byte aligned, ldU a multiple of 4.
 * ltq_ldlq_inter, per block after ltq_ldlq_block: what = d * G and d_h = fp16(d) (d = max(d_rb, 1e-8)) — the
 *   reference's own operations; with acat (else NULL, e.g. for the last block): err = (w_blk - what) @ Uinv (fp32
 *   sequential fma chains, Uinv upper triangular) as acat [M, 1536] = [e0 e0 e1 e0 e1 e2] (bf16 bits, row stride 1536).
 *   d_h may be NULL.  M % 16 == 0.
 */
/*
 * ltq_bf16x6_split: one operand of that six-product form for a general fp32 product (the refits' products with H,
 *   src/liqk_v2.py:1136-1170): order 0 the left slots [x0 x0 x1 x0 x1 x2], order 1 the right slots
 *   [x0 x1 x0 x2 x1 x0]; side 0 concatenates them along the columns (out [rows, 6 cols]), side 1 along the rows
 *   (out [6 rows, cols]); row strides ld / ld_out.  cols, ld, ld_out multiples of 4; x 16-byte, out 8-byte aligned.
 */
int ltq_bf16x6_split(const float* x, long long ld, int rows, int cols, int order, int side, uint16_t* out,
                     long long ld_out, void* stream);
/* the same for `batch` matrices at x + z * xbs -> out + z * obs (z < 65536); neg splits -x. */
int ltq_bf16x6_split_batched(const float* x, long long ld, long long xbs, int rows, int cols, int batch, int order,
                             int side, int neg, uint16_t* out, long long ld_out, long long obs, void* stream);
/*
 * Hessian factorization (src/liqk_v2.py:1074-1088, U = flip(L^-1) for L = chol(flip(H_reg))), the leaves of the
 * triangular inverse: the inverses of the nb lower-triangular 256 x 256 diagonal blocks of L (row-major, row stride ldL)
 * into the diagonal blocks of X (row stride ldX; each block's strictly upper part written as 0), by forward
 * substitution in fp32.  The blocks above the leaves are merged by GEMMs on the caller's side.
 */
int ltq_trtri256_lower(const float* L, long long ldL, int nb, float* X, long long ldX, void* stream);
/*
 * Blocked Cholesky of the damped Hessian (src/liqk_v2.py:1078 torch.linalg.cholesky of flip(H_reg); :1163 the refit
 * system's solve), the diagonal step: the 256 x 256 block at (c0, c0) of A (row-major fp32, row stride ld, lower
 * triangle read, trailing updates of the earlier panels already applied) is factored in place (L, zeros above its
 * diagonal) and its factor inverted; xt3 [256][768] (bf16) receives the compact right operand of the panel product
 * below the block for ltq_gemm_bf16x3p_tn (row n = the three-way bf16 split [x0 x1 x2] of row n of X = L_blk^-1), and X
 * (optional, row stride ldx) the inverse itself at (c0, c0).  The first pivot that is not positive sets
 * *info = c0 + j + 1 when *info is 0 (LAPACK's convention).  The panel and trailing updates are tensor-core GEMMs.
 */
int ltq_chol256_diag(float* A, long long ld, int c0, uint16_t* xt3, float* X, long long ldx, int* info, void* stream);
/*   (ldx = 256 with c0 > 0: X is the 256 x 256 inverse alone, the compact form ltq_chol_solve reads.) */
/*
 * The refit system's solve (src/liqk_v2.py:1161-1163, A_in suh = b_in with A_in = L L^T): x = L^-T L^-1 b for the
 * blocked factor L [K, K] (row-major, row stride ld, K a multiple of 256) and the inverses Dinv [K/256][256][256] of
 * its diagonal blocks (lower triangles, from ltq_chol256_diag).  2 K / 256 launches on `stream`; work: 2 K floats.
 */
int ltq_chol_solve(const float* L, long long ld, int K, const float* Dinv, const float* b, float* x, float* work,
                   void* stream);
/*
 * Tensor-core GEMM of the fast mode's fp32-accurate products (tcgen05.mma, accumulator in tensor memory, operands by
 * TMA): C[M, N] = beta * C + alpha * A[M, Kd] B[N, Kd]^T with A, B bf16 (K contiguous, row strides lda / ldb) and C
 * fp32 (row stride ldc).  Replaces the library GEMM (torch.addmm / torch.mm on cuBLAS) that ran the six-product bf16
 * form of the LDLQ inter-block update W_work[:, c1:] -= ((w_blk - what) @ U_blk_inv) @ U[c0:c1, c1:]
 * (src/liqk_v2.py:972-979).  Limits: N % 16 == 0, Kd a positive multiple of 64, lda and ldb multiples of 8, ldc of 4,
 * A / B / C 16-byte aligned.  err (optional, device int): set to 1 if a pipeline wait ran out (the result is then
 * not valid); the caller clears it.
 */
int ltq_gemm_bf16_tn(const uint16_t* A, long long lda, const uint16_t* B, long long ldb, float* C, long long ldc,
                     int M, int N, int Kd, float alpha, float beta, int* err, void* stream);
/*
 * Self-test of the GEMMs' bounded pipeline waits (device pointers err, done): one thread waits on an mbarrier that
 * expects one arrival.  arrive = 1: the arrival is made first, the wait completes, *done = 1.  arrive = 0: nothing
 * arrives, the wait gives up after `limit` polls (1 .. 2^26), sets *err = 1 and returns, *done = 2 — the path a lost
 * TMA or MMA completion takes inside the GEMMs, run without a fault or a hang.
 */
int ltq_gemm_wait_selftest(int arrive, unsigned int limit, int* err, int* done, void* stream);
/*
 * The same product in the six-product form from compact three-part operands A3 = [a0 a1 a2] [M, 3 Kp] and
 * B3 = [b0 b1 b2] [N, 3 Kp] (x = x0 + x1 + x2 the three-way bf16 split of an fp32 operand):
 *     C = beta C + alpha (a0 b0^T + a0 b1^T + a1 b0^T + a0 b2^T + a1 b1^T + a2 b0^T),
 * each A part of a K chunk loaded once for the three B parts it meets — half the operand bytes of the concatenated form
 * [a0 a0 a1 a0 a1 a2] [b0 b1 b0 b2 b1 b0]^T.  Limits as ltq_gemm_bf16_tn with Kp a positive multiple of 64 and
 * lda, ldb >= 3 Kp.  This is the LDLQ inter-block update's GEMM (A3 from ltq_ldlq_inter3, B3 from ltq_ldlq_bcat_t).
 */
int ltq_gemm_bf16x6_tn(const uint16_t* A3, long long lda, const uint16_t* B3, long long ldb, float* C, long long ldc,
                       int M, int N, int Kp, float alpha, float beta, int* err, void* stream);
/*
 * The general part-operand form, batched: for z < batch (A3 + z abs, B3 + z bbs, C + z cbs, elements),
 *     C_z = beta C_z + alpha sum_{p + q < nq} a_p b_q^T,
 * nq = 3 the six products above, nq = 2 the three a0 b0 + a1 b0 + a0 b1 (A3 / B3 then need only their first 2 Kp
 * columns).  The fast mode's products with H, the refit's Gram matrix, the Cholesky panel and trailing updates and the
 * triangular-inverse merges (src/liqk_v2.py:1074-1088, :1139-1180) run on it.  Limits as ltq_gemm_bf16x6_tn;
 * batch <= 65535; batched strides multiples of 8 (A, B) / 4 (C) elements.  beta 0 and 1 write C by TMA store /
 * reduce-add (no read of C; one rounding of beta C + alpha acc), other beta by a read-modify-write.  One launch per
 * call: with beta 0 / 1 and more 128 x 256 tiles (over all batches) than the device has SMs, a persistent kernel of one
 * CTA per SM with two accumulators in tensor memory, bit-identical to the one-tile kernel used otherwise.
 */
int ltq_gemm_bf16x3p_tn(const uint16_t* A3, long long lda, long long abs, const uint16_t* B3, long long ldb,
                        long long bbs, float* C, long long ldc, long long cbs, int M, int N, int Kp, int nq, int batch,
                        float alpha, float beta, int* err, void* stream);
/*
 * The compact part operand of `batch` fp32 matrices x_z = x + z xbs (rows x cols, row stride ld): trans 0 writes
 * out_z[r][p Kp + c] = part_p(s x_z[r][c]) (Kp >= cols), trans 1 writes out_z[c][p Kp + r] = part_p(s x_z[r][c])
 * (Kp >= rows), zero-padded up to Kp (a multiple of 32); s = -1 when neg.  part_p: x0 = bf16(x), x1 = bf16(x - x0),
 * x2 = bf16(x - x0 - x1).  out row stride ld_out >= 3 Kp (multiple of 4), batch stride obs; 8-byte aligned.
 */
int ltq_bf16x3_split(const float* x, long long ld, long long xbs, int rows, int cols, int batch, int trans, int neg,
                     int Kp, uint16_t* out, long long ld_out, long long obs, void* stream);
size_t ltq_ldlq_bcat_elems(int K);
int ltq_ldlq_bcat(const float* U, long long ldU, int K, uint16_t* bcat, void* stream);
/* the right operands in the compact three-part form of ltq_gemm_bf16x6_tn (K contiguous): block b's
 * [K - 256 (b + 1), 768] matrix whose row n is [u0 u1 u2], the three-way split of column 256 (b + 1) + n of
 * U[256 b : 256 b + 256, :], at element offset 768 * sum_{b' < b} (K - 256 (b' + 1)), ltq_ldlq_bcat_elems(K) / 2 elements
 * in all (K >= 512; bcat 16-byte aligned). */
int ltq_ldlq_bcat_t(const float* U, long long ldU, int K, uint16_t* bcat, void* stream);
int ltq_ldlq_inter(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* G, long long ldG,
                   const float* Uinv, long long ldUi, int M, float* what, long long ld_what, uint16_t* d_h,
                   long long ld_dh, uint16_t* acat, void* stream);
/* ltq_ldlq_inter with err's split in the compact form acat3 [M, 768] = [e0 e1 e2] (row stride 768) for
 * ltq_gemm_bf16x6_tn. */
int ltq_ldlq_inter3(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* G,
                    long long ldG, const float* Uinv, long long ldUi, int M, float* what, long long ld_what,
                    uint16_t* d_h, long long ld_dh, uint16_t* acat3, void* stream);
int ltq_ldlq_block(const float* w_blk, long long ld_w, const float* d_rb, long long ld_d, const float* dw,
                   const float* U, long long ldU, const float* Uinv, long long ldUi, float* G, long long ldG,
                   int16_t* idx, uint8_t* gi, long long ldP, int M, const float* tab, const float* gains, int K, int m,
                   const int* m_extra, int n_extra, int Gfull, int n_cand, int sub, int pp, int tb_window,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * DP-profile sub-block quantization through a 1-D table — the reference's own export, same signature
 * (src/cuda/tcq_viterbi.cu:806-811, bound at src/tcq_proto.py:530-532): for each of S sub-blocks of 16 values xs with
 * weights dh, bucket b = clamp(rint(fma(x, inv_step, half_b)), 0, nb - 1), the column c < 64 of lut [nb, 64] with the
 * smallest sum_j fma(d e, e, .) (e = x - lut[b][c], lowest c on ties), out = lut[b_j][c].  lut 8-byte aligned.
 */
int lut_subs_quant(const float* xs, const float* dh, const float* lut, float* out, int S, float inv_step, float half_b,
                   int nb, void* stream);

/*
 * int8 ring format of the row tables, the comparison baseline of the ring quantizer (replaces int8_rows,
 * src/ple_quant.py:68-77): per ring of 256 consecutive values, d = max(fp16(max |x| / 127), 1e-10) and
 * out = clamp(round_half_even(x / d), -127, 127) * d, in the input's dtype (bf16 = 1: bf16, else fp32); NaN propagates
 * as in the reference's torch operations.  in / out hold n_rings * 256 values, 16-byte aligned.
 */
int ltq_int8_rings(const void* in, void* out, long long n_rings, int bf16, void* stream);

/*
 * .ltq tile packing and spec decode (src/ltq_file.py:54-148; tile fields src/ltq_format.py:104-147).  A row slice
 * [R, K] (R, K multiples of 16) is (R/16)(K/16) tiles of 16 x 16; the packed slice is four structure-of-arrays regions
 * (codes, planes, lsb, gains), each at a multiple of 64 bytes — byte for byte what the reference's pack_slice writes.
 *   kbits: K of the format (2..8); frac: 0 none, 1 D2, 2 D4; h: gain-index bits (0..4); sub: weights per gain (16/32).
 * ltq_slice_bytes: bytes of a packed slice (0 for unsupported parameters).
 * ltq_pack_slice (replaces pack_slice, src/ltq_file.py:79-102): idx (label * U + u) int16 and gi uint8, [R, K] with row
 *   stride ld (multiple of 8; idx 16-byte and gi 8-byte aligned) -> out (64-byte aligned, >= ltq_slice_bytes bytes).
 * ltq_decode_slice (replaces decode_slice, src/ltq_file.py:119-148): the spec decode of a packed slice, value
 *   gain_tab[g] * lut[label * U + u] with labels from the tail-biting code-bit states and the format's masks
 *   (masks[0 .. n_masks-1], the primary mask first).  out [R, K] (stride ld_out) may be NULL; with ref (stride ld_ref),
 *   adds to *mismatches the number of positions whose value differs from ref (the verify of LtqWriter.add_matrix,
 *   src/ltq_file.py:204-207).
 */
size_t ltq_slice_bytes(int R, int K, int kbits, int frac, int h, int sub);
int ltq_pack_slice(const int16_t* idx, const uint8_t* gi, long long ld, int R, int K, int kbits, int frac, int h,
                   int sub, uint8_t* out, size_t out_bytes, void* stream);
int ltq_decode_slice(const uint8_t* data, int R, int K, int kbits, int frac, int h, int sub, const int* masks,
                     int n_masks, const float* lut, const float* gain_tab, float* out, long long ld_out,
                     const float* ref, long long ld_ref, unsigned long long* mismatches, void* stream);
/*
 * Batch-1 product y = W x straight from a packed slice (the inference-side decode; the reference prototypes it in
 * src/cuda/ltq_matvec_bench.cu:77-150): y[r] = sum_b d[r][b] sum_{k in block b} val(r, k) x_rot[k] for the slice's R
 * rows, with val the spec-decoded tile value, d[r][b] = fp16 d_row[r] * 2^(e[r][b] / 4) (d_row as fp16 bits, e int8 with
 * row stride ld_e) and x_rot = H256(suh * x) (ltq_fwht256 mode 2), so y = W x for W = H256(d val) * suh.  K % 256 == 0,
 * kbits <= 6, data 64-byte and x_rot 16-byte aligned.  Deterministic (fixed summation order).
 */
int ltq_matvec_slice(const uint8_t* data, int R, int K, int kbits, int frac, int h, int sub, const int* masks,
                     int n_masks, const float* lut, const float* gain_tab, const uint16_t* d_row, const int8_t* e,
                     long long ld_e, const float* x_rot, float* y, void* stream);

/*
 * Allocation-free tail-biting Viterbi.  No counterpart in the reference (the reference's Python wrapper allocates all
 * scratch with torch); added for callers that cannot allocate device memory while they quantize — an engine that plans
 * its device memory at start-up and forbids allocation afterwards, or a binding (cgo / JNI / N-API / ctypes) that only
 * holds device pointers to its inputs and outputs.  Same arguments and results as ltq_viterbi_tb without the
 * workspace: the scratch is a 64 MiB array inside the library's device memory (ltq_viterbi_tb_noalloc_capacity()),
 * held on every GPU that loads the library until the process exits.  Returns -2 when
 * ltq_viterbi_tb_workspace_bytes(...) exceeds that capacity.  Every call on a device shares the array: calls that
 * overlap on the GPU race and must be serialised.  The first call on a device looks up the array's address (make it
 * before any stream capture) and keeps it for the life of the process: after cudaDeviceReset on that device the kept
 * address is stale, so a process that resets a device must not call this entry on it again.  Calls no allocator.
 * Errors: -1 invalid parameters, -2 too large for the array, >0 the cudaError_t of the address lookup or the launch.
 */
size_t ltq_viterbi_tb_noalloc_capacity(void);
int ltq_viterbi_tb_noalloc(const float* x, const float* w, int w_stride, const float* tab, const float* gains,
                           const float* tab_hi, const float* gains_hi, float* rec, int* code, int N, int T, int nu,
                           int K, int m, const int* m_extra, int n_extra, int Gfull, int n_cand, int sub, int U_hi,
                           int mix, int pp, int tb_passes, int tb_cand1, int tb_window, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LTQ_B200_H */
